// bw_probe.cu - measures the machine parameters the KVForge cost model reads
// (src/machine.cpp keys: bw_peak_gbs, bw_sm_gbs, lat_ns, bw_l2_gbs, f32_gflops,
// launch_us, ...) on a B200, and prints them as a `.gpu` machine file.
//
// Replaces bench/bw_probe.cu (kernels :42-98, main :140-265) with probes that
// match how the sm_100a decode kernels move data: besides the plain 16-byte
// streaming load it times a cp.async.bulk (TMA) read stream into a shared-memory
// ring, and the legacy f16 tensor-core MMA rate the decode kernels rely on.
//
//   kvf_bw_probe [--device 0] [--mb 2048] [--name b200]
#include "ptx.cuh"

#include <cuda.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#define PROBE_CHECK(call)                                                               \
  do {                                                                                  \
    cudaError_t e__ = (call);                                                           \
    if (e__ != cudaSuccess) {                                                           \
      std::fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e__), __FILE__, \
                   __LINE__);                                                           \
      std::exit(1);                                                                     \
    }                                                                                   \
  } while (0)

using namespace kvfb;

__device__ unsigned long long g_probe_sink;
__device__ unsigned g_probe_err;

// Grid-stride 16-byte streaming loads, four in flight per thread.
__global__ void __launch_bounds__(512) ldg_stream(const uint4 *p, size_t n16) {
  uint32_t acc = 0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = __ldcs(p + i), b = __ldcs(p + i + stride), c = __ldcs(p + i + 2 * stride),
                d = __ldcs(p + i + 3 * stride);
    acc ^= a.x ^ b.y ^ c.z ^ d.w;
  }
  for (; i < n16; i += stride) acc ^= __ldcs(p + i).x;
  if (acc == 0x9e3779b9u) atomicAdd(&g_probe_sink, 1ull);
}

// One thread per CTA keeps `stages` bulk copies of `chunk` bytes in flight over
// the CTA's contiguous share of the buffer. Nothing consumes the data: this is
// the TMA engine's read rate.
__global__ void __launch_bounds__(32) bulk_stream(const uint8_t *p, size_t bytes, int chunk,
                                                  int stages) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[16];
  if (threadIdx.x != 0) return;
  for (int s = 0; s < stages; ++s) ptx::mbar_init(ptx::smem_u32(&bars[s]), 1);
  ptx::fence_barrier_init();
  const size_t per = (bytes / gridDim.x) & ~(size_t)(chunk - 1);
  const uint8_t *base = p + per * blockIdx.x;
  const int n = (int)(per / chunk);
  const uint64_t pol = ptx::policy_evict_first();
  uint32_t phase = 0;
  int issued = 0;
  for (; issued < stages && issued < n; ++issued) {
    const uint32_t bar = ptx::smem_u32(&bars[issued]);
    ptx::mbar_arrive_expect_tx(bar, chunk);
    ptx::bulk_g2s(ptx::smem_u32(smem + (size_t)issued * chunk), base + (size_t)issued * chunk,
                  chunk, bar, pol);
  }
  for (int done = 0; done < n; ++done) {
    const int s = done % stages;
    const uint32_t bar = ptx::smem_u32(&bars[s]);
    if (!ptx::mbar_wait(bar, (phase >> s) & 1u)) {
      atomicExch(&g_probe_err, 1u);
      // Drain what is still in flight (bounded) before leaving.
      for (int k = done; k < issued; ++k) {
        const int s2 = k % stages;
        ptx::mbar_wait(ptx::smem_u32(&bars[s2]), (phase >> s2) & 1u);
        phase ^= 1u << s2;
      }
      return;
    }
    phase ^= 1u << s;
    if (issued < n) {
      ptx::mbar_arrive_expect_tx(bar, chunk);
      ptx::bulk_g2s(ptx::smem_u32(smem + (size_t)s * chunk), base + (size_t)issued * chunk,
                    chunk, bar, pol);
      ++issued;
    }
  }
}

// One thread per CTA streams a token range of one head group through a ring
// of `stages` stages; each stage is `nxb` tiled TMA copies of [128 B,
// box_rows tokens, 4 heads] (the decode kernels' box shape) from a 4-D view
// (x, token, head, 1) of a cache with 8 KV heads. CTA pairs take head groups
// 0-3 and 4-7 of the same tokens.
__global__ void __launch_bounds__(32) tma_tile_stream(const __grid_constant__ CUtensorMap tm, int nxb,
                                                      int box_rows, int stages, int rows_per_block) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[16];
  if (threadIdx.x != 0) return;
  uint8_t *buf = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem) + 1023) & ~uintptr_t(1023));
  for (int s = 0; s < stages; ++s) ptx::mbar_init(ptx::smem_u32(&bars[s]), 1);
  ptx::fence_barrier_init();
  const uint64_t pol = ptx::policy_evict_first();
  const uint32_t box_bytes = 128u * (uint32_t)box_rows * 4u;
  const int n = rows_per_block / box_rows;
  const int h0 = (blockIdx.x & 1) * 4;
  const int row0 = (blockIdx.x >> 1) * rows_per_block;
  uint32_t phase = 0;
  int issued = 0;
  auto issue = [&](int k, int s) {
    const uint32_t bar = ptx::smem_u32(&bars[s]);
    ptx::mbar_arrive_expect_tx(bar, box_bytes * (uint32_t)nxb);
    for (int xb = 0; xb < nxb; ++xb)
      ptx::tma_g2s_4d(ptx::smem_u32(buf + ((size_t)s * nxb + xb) * box_bytes), &tm, xb * 128,
                      row0 + k * box_rows, h0, 0, bar, pol);
  };
  for (; issued < stages && issued < n; ++issued) issue(issued, issued);
  for (int done = 0; done < n; ++done) {
    const int s = done % stages;
    if (!ptx::mbar_wait(ptx::smem_u32(&bars[s]), (phase >> s) & 1u)) {
      atomicExch(&g_probe_err, 1u);
      for (int k = done; k < issued; ++k) {
        const int s2 = k % stages;
        ptx::mbar_wait(ptx::smem_u32(&bars[s2]), (phase >> s2) & 1u);
        phase ^= 1u << s2;
      }
      return;
    }
    phase ^= 1u << s;
    if (issued < n) issue(issued++, s);
  }
}

// Dependent pointer chase for the idle DRAM latency. Each run continues the
// cycle where the previous one stopped (`pos`), so repeated runs never touch
// a line twice and every access misses L2.
__global__ void chase(const unsigned *next, int steps, unsigned *pos) {
  unsigned j = *pos;
  for (int i = 0; i < steps; ++i) j = __ldcg(next + j);
  *pos = j;
}

// L2-resident re-reads.
__global__ void l2_read(const uint4 *p, size_t n16, int reps) {
  uint32_t acc = 0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (int r = 0; r < reps; ++r)
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride)
      acc ^= __ldcg(p + i).x;
  if (acc == 0x9e3779b9u) atomicAdd(&g_probe_sink, 1ull);
}

// FP32 FMA issue rate: eight independent chains per thread.
__global__ void fma_rate(float seed, int iters, float *out) {
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = seed + k + threadIdx.x;
  for (int i = 0; i < iters; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = fmaf(a[k], 0.999999f, 1e-7f);
  float s = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) s += a[k];
  if (s == 12345.f) *out = s;
}

// mma.sync m16n8k16 f16 -> f32 rate: eight independent accumulators per warp.
__global__ void mma_rate(int iters, float *out) {
  uint32_t a[4] = {0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u};
  const uint32_t b0 = 0x3c00u + threadIdx.x, b1 = 0x3c00u;
  float c[8][4] = {};
  for (int i = 0; i < iters; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) ptx::mma_f16(c[k], a, b0, b1);
  float s = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) s += c[k][0] + c[k][1] + c[k][2] + c[k][3];
  if (s == 12345.f) *out = s;
}

__global__ void empty_kernel() {}

struct Timer {
  cudaEvent_t e0, e1;
  Timer() {
    PROBE_CHECK(cudaEventCreate(&e0));
    PROBE_CHECK(cudaEventCreate(&e1));
  }
  ~Timer() {
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  }
  template <class F> float best_ms(F &&f, int reps, void *flush = nullptr, size_t flush_bytes = 0) {
    float best = 1e30f;
    for (int r = 0; r < reps; ++r) {
      if (flush) PROBE_CHECK(cudaMemsetAsync(flush, r & 0xFF, flush_bytes));
      PROBE_CHECK(cudaEventRecord(e0));
      f();
      PROBE_CHECK(cudaEventRecord(e1));
      PROBE_CHECK(cudaEventSynchronize(e1));
      PROBE_CHECK(cudaGetLastError());
      float ms = 0;
      PROBE_CHECK(cudaEventElapsedTime(&ms, e0, e1));
      best = std::min(best, ms);
    }
    return best;
  }
};

int main(int argc, char **argv) {
  int dev = 0;
  size_t mb = 2048;
  std::string name = "b200";
  for (int i = 1; i + 1 < argc; i += 2) {
    const std::string a = argv[i];
    if (a == "--device") dev = std::atoi(argv[i + 1]);
    else if (a == "--mb") mb = std::strtoull(argv[i + 1], nullptr, 10);
    else if (a == "--name") name = argv[i + 1];
  }
  PROBE_CHECK(cudaSetDevice(dev));
  cudaDeviceProp prop;
  PROBE_CHECK(cudaGetDeviceProperties(&prop, dev));
  const int sms = prop.multiProcessorCount;
  int clk_khz = 0;
  PROBE_CHECK(cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, dev));
  const size_t bytes = mb << 20;
  uint8_t *buf = nullptr;
  PROBE_CHECK(cudaMalloc(&buf, bytes));
  PROBE_CHECK(cudaMemset(buf, 1, bytes));
  Timer tm;
  std::printf("# Measured by kvf_bw_probe on %s (cc %d.%d, %d SMs)\n", prop.name, prop.major,
              prop.minor, sms);

  // Streaming read, 16-byte loads: sweep the launch shape, keep the best.
  double bw_ldg = 0;
  int best_ldg_blocks = 0, best_ldg_threads = 0;
  for (int per_sm : {2, 4, 8})
    for (int thr : {256, 512}) {
      const int blocks = sms * per_sm;
      const float ms = tm.best_ms(
          [&] { ldg_stream<<<blocks, thr>>>(reinterpret_cast<const uint4 *>(buf), bytes / 16); },
          5);
      const double gbs = bytes / (ms * 1e6);
      std::printf("# ldg_stream %dx%d: %.1f GB/s\n", blocks, thr, gbs);
      if (gbs > bw_ldg) { bw_ldg = gbs; best_ldg_blocks = blocks; best_ldg_threads = thr; }
    }
  // One SM alone.
  const size_t one_bytes = 64u << 20;
  const float ms1 = tm.best_ms(
      [&] { ldg_stream<<<1, 512>>>(reinterpret_cast<const uint4 *>(buf), one_bytes / 16); }, 3);
  const double bw_sm = one_bytes / (ms1 * 1e6);

  // TMA bulk read stream: chunk size x stages x CTAs per SM.
  double bw_bulk = 0;
  int best_chunk = 0, best_stages = 0, best_ctas = 0;
  for (int chunk : {8192, 16384, 32768})
    for (int stages : {4, 6})
      for (int per_sm : {1, 2}) {
        const int smem = chunk * stages;
        if (smem * per_sm > 200 * 1024) continue;
        PROBE_CHECK(cudaFuncSetAttribute(bulk_stream, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem));
        const int blocks = sms * per_sm;
        const float ms = tm.best_ms(
            [&] { bulk_stream<<<blocks, 32, smem>>>(buf, bytes, chunk, stages); }, 5);
        const size_t moved = ((bytes / blocks) & ~(size_t)(chunk - 1)) * blocks;
        const double gbs = moved / (ms * 1e6);
        std::printf("# bulk_stream chunk=%d stages=%d ctas/sm=%d: %.1f GB/s\n", chunk, stages,
                    per_sm, gbs);
        if (gbs > bw_bulk) { bw_bulk = gbs; best_chunk = chunk; best_stages = stages; best_ctas = per_sm; }
      }
  // Tiled TMA stream with the decode kernels' box shapes: a [n_tok][8 heads]
  // x row_bytes token-major tensor (rows of one head strided by 8 rows), box
  // [128 B, box_rows tokens, 4 heads] (token-major) or a head-major tensor
  // [8 heads][n_tok] x row_bytes with box [128 B, box_rows, 4 heads].
  typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                    const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                    const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  void *encp = nullptr;
  cudaDriverEntryPointQueryResult qres;
  PROBE_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &encp, cudaEnableDefault, &qres));
  EncodeTiledFn enc = reinterpret_cast<EncodeTiledFn>(encp);
  double bw_tile = 0;
  for (int tm_layout : {1, 0})
    for (int rb : {128, 256})
      for (int box_rows : {16, 32, 64})
        for (int stages : {2, 4, 6})
          for (int per_sm : {1, 2}) {
            const int heads = 8;
            const size_t tokens = bytes / ((size_t)heads * rb);
            cuuint64_t dims[4] = {(cuuint64_t)rb, (cuuint64_t)tokens, (cuuint64_t)heads, 1};
            cuuint64_t strides[3];
            strides[0] = tm_layout ? (cuuint64_t)heads * rb : (cuuint64_t)rb;
            strides[1] = tm_layout ? (cuuint64_t)rb : (cuuint64_t)tokens * rb;
            strides[2] = (cuuint64_t)tokens * heads * rb;
            const cuuint32_t box[4] = {128u, (cuuint32_t)box_rows, 4u, 1u};
            const cuuint32_t es[4] = {1, 1, 1, 1};
            CUtensorMap tmap;
            if (enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, buf, dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
              std::printf("# tma_tile_stream encode failed (tm=%d rb=%d)\n", tm_layout, rb);
              continue;
            }
            const int nxb = rb / 128;
            const int stage_bytes = 128 * box_rows * 4 * nxb;
            const int smem = stage_bytes * stages + 1024;
            if (smem * per_sm > 220 * 1024 || smem > 227 * 1024) continue;
            PROBE_CHECK(cudaFuncSetAttribute(tma_tile_stream, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            const int ctas = (sms * per_sm) & ~1;
            const int rows_per_block = (int)(tokens / (ctas / 2)) / box_rows * box_rows;
            const float ms = tm.best_ms(
                [&] { tma_tile_stream<<<ctas, 32, smem>>>(tmap, nxb, box_rows, stages, rows_per_block); }, 3);
            const double moved = (double)ctas * rows_per_block * 4 * rb;
            const double gbs = moved / (ms * 1e6);
            std::printf("# tma_tile_stream %s row=%dB box=[128B x %d tok x 4 heads] x%d stage=%dKB stages=%d "
                        "ctas/sm=%d: %.1f GB/s\n",
                        tm_layout ? "token-major" : "head-major", rb, box_rows, nxb, stage_bytes / 1024, stages,
                        per_sm, gbs);
            bw_tile = std::max(bw_tile, gbs);
          }

  unsigned perr = 0;
  PROBE_CHECK(cudaMemcpyFromSymbol(&perr, g_probe_err, 4));
  if (perr) std::printf("# WARNING: bulk_stream barrier wait timed out\n");

  // DRAM latency: a random cycle over 256 MB.
  const size_t nidx = (256u << 20) / 4;
  std::vector<unsigned> nxt(nidx);
  {
    std::vector<unsigned> perm(nidx / 32);
    for (size_t i = 0; i < perm.size(); ++i) perm[i] = (unsigned)i;
    uint64_t s = 88172645463325252ull;
    for (size_t i = perm.size() - 1; i > 0; --i) {
      s ^= s << 13; s ^= s >> 7; s ^= s << 17;
      std::swap(perm[i], perm[s % (i + 1)]);
    }
    for (size_t i = 0; i < perm.size(); ++i)
      nxt[(size_t)perm[i] * 32] = perm[(i + 1) % perm.size()] * 32;
  }
  unsigned *dnext = nullptr, *dout = nullptr;
  PROBE_CHECK(cudaMalloc(&dnext, nidx * 4));
  PROBE_CHECK(cudaMalloc(&dout, 4));
  PROBE_CHECK(cudaMemcpy(dnext, nxt.data(), nidx * 4, cudaMemcpyHostToDevice));
  PROBE_CHECK(cudaMemset(dout, 0, 4));
  {
    // Evict the freshly written chase lines from L2 before timing.
    void *scratch = nullptr;
    const size_t sb = (size_t)4 * (size_t)prop.l2CacheSize;
    PROBE_CHECK(cudaMalloc(&scratch, sb));
    PROBE_CHECK(cudaMemset(scratch, 1, sb));
    PROBE_CHECK(cudaDeviceSynchronize());
    PROBE_CHECK(cudaFree(scratch));
  }
  const int steps = 20000;
  const float msl = tm.best_ms([&] { chase<<<1, 1>>>(dnext, steps, dout); }, 3);
  const double lat_ns = msl * 1e6 / steps;

  // L2 bandwidth over a quarter of L2.
  const size_t l2b = (size_t)prop.l2CacheSize / 4;
  const int l2reps = 50;
  const float msl2 = tm.best_ms(
      [&] { l2_read<<<sms * 4, 512>>>(reinterpret_cast<const uint4 *>(buf), l2b / 16, l2reps); },
      5);
  const double bw_l2 = (double)l2b * l2reps / (msl2 * 1e6);

  // FP32 and tensor-core issue rates.
  float *fout = nullptr;
  PROBE_CHECK(cudaMalloc(&fout, 4));
  const int fiters = 4096;
  const float msf = tm.best_ms([&] { fma_rate<<<sms * 8, 256>>>(1.f, fiters, fout); }, 5);
  const double gflops = 2.0 * 8 * fiters * (double)sms * 8 * 256 / (msf * 1e6);
  const int miters = 2048;
  double mma_tflops = 0;
  int best_mma_warps = 0;
  for (int warps : {4, 8, 16, 32}) {
    const float msm = tm.best_ms([&] { mma_rate<<<sms, warps * 32>>>(miters, fout); }, 5);
    const double fl = 2.0 * 16 * 8 * 16 * 8 * (double)miters * sms * warps;
    const double tf = fl / (msm * 1e9);
    std::printf("# mma.sync m16n8k16 f16->f32, %d warps/SM: %.1f TFLOP/s (%.3f MMA/clk/SM at %d MHz)\n",
                warps, tf, fl / 4096.0 / sms / (msm * 1e-3) / (clk_khz * 1e3), clk_khz / 1000);
    if (tf > mma_tflops) { mma_tflops = tf; best_mma_warps = warps; }
  }

  // Launch overhead: back-to-back empty kernels.
  const int nl = 1000;
  const float msk = tm.best_ms([&] { for (int i = 0; i < nl; ++i) empty_kernel<<<1, 32>>>(); }, 3);

  std::printf("# ldg_stream best launch %dx%d; bulk best chunk=%d stages=%d ctas/sm=%d\n",
              best_ldg_blocks, best_ldg_threads, best_chunk, best_stages, best_ctas);
  std::printf("# bw_ldg_gbs = %.1f   bw_bulk_gbs = %.1f   mma_f16_tflops = %.1f (%d warps/SM)\n",
              bw_ldg, bw_bulk, mma_tflops, best_mma_warps);
  std::printf("name = %s\n", name.c_str());
  std::printf("compute_capability = %d.%d\n", prop.major, prop.minor);
  std::printf("dram_gb = %.1f\n", prop.totalGlobalMem / 1e9);
  std::printf("sms = %d\n", sms);
  std::printf("bw_peak_gbs = %.1f\n", std::max(bw_ldg, bw_bulk));
  std::printf("bw_sm_gbs = %.2f\n", bw_sm);
  std::printf("lat_ns = %.0f\n", lat_ns);
  std::printf("bw_l2_gbs = %.0f\n", bw_l2);
  std::printf("l2_bytes = %d\n", prop.l2CacheSize);
  std::printf("sector_bytes = 32\n");
  std::printf("line_bytes = 128\n");
  std::printf("f32_gflops = %.0f\n", gflops);
  std::printf("launch_us = %.2f\n", msk * 1e3 / nl);
  std::printf("max_warps_per_sm = %d\n", prop.maxThreadsPerMultiProcessor / 32);
  std::printf("max_blocks_per_sm = %d\n", prop.maxBlocksPerMultiProcessor);
  std::printf("regs_per_sm = %d\n", prop.regsPerMultiprocessor);
  cudaFree(buf);
  cudaFree(dnext);
  cudaFree(dout);
  cudaFree(fout);
  return perr ? 3 : 0;
}
