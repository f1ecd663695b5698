// decode.cu - host side of the sm_100a decode-attention kernels: argument
// checks, launch planning (heads per block, stage depth, split chunking), TMA
// tensor-map encoding and the C-ABI entry points declared in kvforge_b200.h.
//
// The reference launcher this replaces is kvf::launch<> in
// runtime/kvf_kernels.cuh:309-320 (grid (splits, G>1 ? Hkv : H, B), the partial
// kernel, then decode_merge when splits > 1).
#include "kvforge_b200.h"

#include "decode_kernel.cuh"
#include "decode_tc.cuh"

#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

namespace kvfb {
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    cudaGetLastError();
  });
  return fn;
}

int ilog2(int v) {
  int s = 0;
  while ((1 << s) < v) ++s;
  return s;
}

struct Shape {
  int fmt, d, ord, paged, bt, gpr;
};

// Validates the arguments the way the reference's preconditions state them
// (runtime/kvf_kernels.cuh:131-132, src/ir.cpp:122-133, src/format.cpp:90-102,
// src/layout.cpp:62-78).
cudaError_t check_args(const kvf_args *a, int fmt, int d, int g, int ord, int paged, Shape &sh) {
  if (!a) return cudaErrorInvalidValue;
  if (fmt < 0 || fmt > 2 || (d != 64 && d != 128) || (ord != 0 && ord != 1)) return cudaErrorInvalidValue;
  if (a->B < 0 || a->H <= 0 || a->Hkv <= 0 || a->H % a->Hkv || a->n < 0 || a->splits < 1)
    return cudaErrorInvalidValue;
  const int gq = a->H / a->Hkv;
  if (gq > 8) return cudaErrorInvalidValue;
  if (g != 1 && g != gq) return cudaErrorInvalidValue;
  sh.fmt = fmt;
  sh.d = d;
  sh.ord = ord;
  sh.paged = paged ? 1 : 0;
  sh.gpr = 0;
  sh.bt = 0;
  if (fmt != 0) {
    if (a->group_shift < 5 || a->group_shift > 7) return cudaErrorInvalidValue;
    const int group = 1 << a->group_shift;
    if (group > d || (fmt == 1 && group < 64)) return cudaErrorInvalidValue;
    sh.gpr = d / group;
    if (!a->k_meta || !a->v_meta) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a->k_meta) | reinterpret_cast<uintptr_t>(a->v_meta)) &
        (uintptr_t)(4 * sh.gpr - 1))
      return cudaErrorMisalignedAddress;
  }
  if (sh.paged) {
    if (a->block_shift < 4 || a->block_shift > 7) return cudaErrorInvalidValue;
    sh.bt = 1 << a->block_shift;
    if (!a->block_table || a->max_blocks < (a->n + sh.bt - 1) / sh.bt) return cudaErrorInvalidValue;
  }
  if (a->B == 0 || a->H == 0) return cudaSuccess;
  if (!a->q || !a->k || !a->v || !a->out) return cudaErrorInvalidValue;
  if (a->splits > 1 && (!a->part_o || !a->part_ml)) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a->k) | reinterpret_cast<uintptr_t>(a->v)) & 15u)
    return cudaErrorMisalignedAddress;
  if ((reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->out)) & 3u)
    return cudaErrorMisalignedAddress;
  return cudaSuccess;
}

bool group_ok(int fmt, int d, int group) {
  if (fmt == 0) return true;
  if (group != 32 && group != 64 && group != 128) return false;
  return group <= d && !(fmt == 1 && group < 64);
}

int heads_per_block(int Hkv, int fmt, int d) {
  // Four KV heads (consumer warps) per block keep a stage near 32 KB and let
  // two blocks share an SM, each with its own barriers, so one block's
  // dependent softmax chain overlaps the other's.
  (void)fmt;
  (void)d;
  for (int h = 4; h > 1; h >>= 1)
    if (Hkv % h == 0) return h;
  return 1;
}

template <int FMT, int D, int GPR, int NT, bool LEAN> struct K {
  static void *fn() { return reinterpret_cast<void *>(&decode_kernel<FMT, D, GPR, NT, LEAN>); }
};

// Kernel for (fmt, d, gpr, nt, lean); nullptr for an unsupported combination.
void *kernel_for(int fmt, int d, int gpr, int nt, bool lean) {
#define KVFB_CASE(F, DD, G, N)                                                     \
  if (fmt == F && d == DD && gpr == G && nt == N)                                  \
    return lean ? K<F, DD, G, N, true>::fn() : K<F, DD, G, N, false>::fn();
#define KVFB_NT(F, DD, G) KVFB_CASE(F, DD, G, 1) KVFB_CASE(F, DD, G, 2)
  KVFB_NT(0, 128, 0) KVFB_NT(0, 64, 0)
  KVFB_NT(1, 128, 1) KVFB_NT(1, 128, 2) KVFB_NT(1, 64, 1)
  KVFB_NT(2, 128, 1) KVFB_NT(2, 128, 2) KVFB_NT(2, 128, 4) KVFB_NT(2, 64, 1) KVFB_NT(2, 64, 2)
#undef KVFB_NT
#undef KVFB_CASE
  return nullptr;
}

struct KernelInfo {
  int regs = 0;
  int static_smem = 0;
  bool ok = false;
};

KernelInfo info_for(void *fn) {
  static std::mutex mu;
  static void *keys[64];
  static KernelInfo vals[64];
  static int count = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < count; ++i)
    if (keys[i] == fn) return vals[i];
  KernelInfo ki;
  cudaFuncAttributes at;
  if (cudaFuncGetAttributes(&at, fn) == cudaSuccess) {
    ki.regs = at.numRegs;
    ki.static_smem = (int)at.sharedSizeBytes;
    ki.ok = true;
  } else {
    cudaGetLastError();
  }
  if (count < 64) {
    keys[count] = fn;
    vals[count++] = ki;
  }
  return ki;
}

constexpr int kSmemPerSM = 228 * 1024;
constexpr int kSmemPerBlockMax = 227 * 1024;
constexpr int kReservedPerBlock = 1024;

struct Launch {
  Plan p;
  void *fn = nullptr;
  int threads = 0;
  int blocks = 0;
  int occupancy = 0;
};

cudaError_t plan_launch(const kvf_args *a, const Shape &sh, Launch &L, bool lean) {
  Plan &p = L.p;
  std::memset(&p, 0, sizeof(p));
  const int gq = a->H / a->Hkv;
  const int nt = gq <= 4 ? 1 : 2;
  L.fn = kernel_for(sh.fmt, sh.d, sh.gpr, nt, lean);
  if (!L.fn) return cudaErrorInvalidValue;
  p.gq = gq;
  p.gpr = sh.gpr;
  p.hh = heads_per_block(a->Hkv, sh.fmt, sh.d);
  p.hg = a->Hkv / p.hh;
  const int rb = row_bytes(sh.fmt, sh.d);
  p.rb = rb;
  p.tb = 16 * stage_mtiles(sh.fmt, sh.d);
  p.paged = sh.paged;
  p.tm = sh.ord;
  p.bt_shift = sh.paged ? ilog2(sh.bt) : 0;
  p.tbox = sh.paged ? std::min(p.tb, sh.bt) : p.tb;
  p.tbox_shift = ilog2(p.tbox);
  p.npg = p.tb / p.tbox;
  p.boxx = std::min(rb, 128);
  p.nxb = rb / p.boxx;
  p.swz = p.boxx == 128 ? 0x70u : p.boxx == 64 ? 0x30u : 0x10u;
  p.box_bytes = (uint32_t)(p.boxx * p.tbox * p.hh);
  p.kv_bytes = (uint32_t)(p.tb * p.hh * rb);
  p.meta_bytes = (uint32_t)(p.tb * p.hh * sh.gpr * 4);
  p.tx_bytes = 2u * p.kv_bytes;
  // Metadata by TMA for contiguous caches whose layout gives rows of >= 16
  // bytes in a 3-D view (see decode_kernel.cuh); cp.async otherwise.
  p.meta_tma = 0;
  p.meta_ts = (uint32_t)(sh.gpr * 4);
  p.meta_hs = (uint32_t)(p.tb * sh.gpr * 4);
  if (sh.gpr > 0 && !sh.paged && (p.meta_bytes % 128u) == 0 &&
      (reinterpret_cast<uintptr_t>(a->k_meta) & 15u) == 0 && (reinterpret_cast<uintptr_t>(a->v_meta) & 15u) == 0) {
    const long long g4 = (long long)sh.gpr * 4;
    const bool ok = sh.ord ? ((a->Hkv * g4) % 16 == 0 && (p.hh * g4) % 16 == 0)
                           : (((long long)a->n * g4) % 16 == 0 && p.tb * sh.gpr <= 256 && (p.tb * g4) % 16 == 0);
    if (ok) {
      p.meta_tma = 1;
      p.tx_bytes += 2u * p.meta_bytes;
      if (sh.ord) {
        p.meta_ts = (uint32_t)(p.hh * g4);
        p.meta_hs = (uint32_t)g4;
      }
    }
  }
  const uint32_t meta_al = (p.meta_bytes + 127u) & ~127u;
  p.stage_bytes = (2u * p.kv_bytes + 2u * meta_al + 1023u) & ~1023u;
  const int ng = sh.gpr > 0 ? sh.gpr : 1;
  p.pscr_warp = (uint32_t)(ng * nt * 384);
  L.threads = (p.hh + 1) * 32;

  const KernelInfo ki = info_for(L.fn);
  if (!ki.ok) return cudaErrorInvalidDeviceFunction;
  // Blocks per SM the registers allow (at most 2), then as many stages as the
  // shared memory of that many blocks holds.
  const int regs_per_block = ((ki.regs + 7) / 8 * 8) * L.threads;
  int occ = std::max(1, std::min(2, 65536 / std::max(1, regs_per_block)));
  const uint32_t fixed = 1024u + 16u * 8u + p.pscr_warp * p.hh + (uint32_t)ki.static_smem;
  int stages = 0;
  for (; occ >= 1; --occ) {
    const int budget = std::min(kSmemPerBlockMax, kSmemPerSM / occ - kReservedPerBlock) - (int)fixed;
    stages = std::min(8, budget / (int)p.stage_bytes);
    if (stages >= 2) break;
  }
  if (stages < 2) return cudaErrorInvalidValue;
  L.occupancy = occ;
  p.stages = stages;
  p.off_bars = (uint32_t)stages * p.stage_bytes;
  p.off_pscr = p.off_bars + 16u * (uint32_t)stages;
  p.off_pscr = (p.off_pscr + 127u) & ~127u;
  p.smem_total = 1024u + p.off_pscr + p.pscr_warp * (uint32_t)p.hh;

  p.splits = a->splits;
  p.final_out = a->splits == 1;
  const int per = (a->n + a->splits - 1) / std::max(1, a->splits);
  p.chunk = std::max(p.tb, (per + p.tb - 1) / p.tb * p.tb);
  if (sh.paged && sh.bt > p.tb) p.chunk = (p.chunk + sh.bt - 1) / sh.bt * sh.bt;
  L.blocks = a->B * p.hg * a->splits;
  return cudaSuccess;
}

cudaError_t encode_maps_box(const kvf_args *a, const Shape &sh, int rbytes, int boxx, int tbox, int heads,
                            CUtensorMap &tk, CUtensorMap &tv);

cudaError_t encode_maps(const kvf_args *a, const Shape &sh, const Plan &p, CUtensorMap &tk,
                        CUtensorMap &tv) {
  return encode_maps_box(a, sh, p.rb, p.boxx, p.tbox, p.hh, tk, tv);
}

// Tensor maps over the K and V metadata (32-bit words) of a contiguous cache:
// token-major [B][n][Hkv * groups] with boxes of (hh * groups, tb, 1),
// head-major [B][Hkv][n * groups] with boxes of (tb * groups, hh, 1).
cudaError_t encode_meta_maps(const kvf_args *a, const Shape &sh, const Plan &p, CUtensorMap &tkm,
                             CUtensorMap &tvm) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t g = (cuuint64_t)sh.gpr, n = (cuuint64_t)std::max(a->n, 1), H = (cuuint64_t)a->Hkv;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  if (sh.ord) {
    dims[0] = H * g;
    dims[1] = n;
    strides[0] = H * g * 4;
    box[0] = (cuuint32_t)(p.hh * sh.gpr);
    box[1] = (cuuint32_t)p.tb;
  } else {
    dims[0] = n * g;
    dims[1] = H;
    strides[0] = n * g * 4;
    box[0] = (cuuint32_t)(p.tb * sh.gpr);
    box[1] = (cuuint32_t)p.hh;
  }
  dims[2] = (cuuint64_t)std::max(a->B, 1);
  strides[1] = n * H * g * 4;
  box[2] = 1u;
  const cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = enc(&tkm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void *>(a->k_meta), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  r = enc(&tvm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void *>(a->v_meta), dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t encode_maps_box(const kvf_args *a, const Shape &sh, int rbytes, int boxx, int tbox, int heads,
                            CUtensorMap &tk, CUtensorMap &tv) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t rb = (cuuint64_t)rbytes;
  cuuint64_t dims[4], strides[3];
  dims[0] = rb;
  dims[2] = (cuuint64_t)a->Hkv;
  if (sh.paged) {
    const cuuint64_t bt = (cuuint64_t)sh.bt;
    const cuuint64_t page = bt * a->Hkv * rb;
    dims[1] = bt;
    dims[3] = std::min<cuuint64_t>((1ull << 31) - 1, ((1ull << 40) - 1) / page);
    strides[0] = sh.ord ? a->Hkv * rb : rb;
    strides[1] = sh.ord ? rb : bt * rb;
    strides[2] = page;
  } else {
    const cuuint64_t n = (cuuint64_t)std::max(a->n, 1);
    dims[1] = n;
    dims[3] = (cuuint64_t)std::max(a->B, 1);
    strides[0] = sh.ord ? a->Hkv * rb : rb;
    strides[1] = sh.ord ? rb : n * rb;
    strides[2] = n * a->Hkv * rb;
  }
  const cuuint32_t box[4] = {(cuuint32_t)boxx, (cuuint32_t)tbox, (cuuint32_t)heads, 1u};
  const cuuint32_t es[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapSwizzle swz = boxx == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : boxx == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                              : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = enc(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<unsigned char *>(a->k), dims,
                   strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  r = enc(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<unsigned char *>(a->v), dims, strides,
          box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  return cudaSuccess;
}

// Streaming multiprocessors of the current device (148 when it cannot be asked).
int sm_count() {
  static std::atomic<int> cache[16];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 148;
  }
  if (dev >= 0 && dev < 16) {
    const int v = cache[dev].load(std::memory_order_relaxed);
    if (v > 0) return v;
  }
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
    cudaGetLastError();
    v = 148;
  }
  if (dev >= 0 && dev < 16) cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

// Blocks of merge_kernel resident per SM (at least 1).
int merge_blocks_per_sm() {
  static std::atomic<int> v{0};
  int r = v.load(std::memory_order_relaxed);
  if (r > 0) return r;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, merge_kernel, kMergeWarps * 32, 0) != cudaSuccess || r < 1) {
    cudaGetLastError();
    r = 1;
  }
  v.store(r, std::memory_order_relaxed);
  return r;
}

cudaError_t launch_merge(const kvf_args *a, int d, cudaStream_t st, bool pdl, const kvf_exchange *x = nullptr,
                         MergeBalance bal = MergeBalance{0, 0, 0}) {
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  const long long slices = (long long)a->H * a->B * ((d + 31) / 32);
  if (x)
    cfg.gridDim = dim3((unsigned)a->H, (unsigned)a->B, (unsigned)((d + 31) / 32));
  else
    cfg.gridDim = dim3((unsigned)std::min<long long>(slices, (long long)sm_count() * merge_blocks_per_sm()), 1, 1);
  cfg.blockDim = dim3(kMergeWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const kvf_args args = *a;
  if (x) {
    const kvf_exchange xc = *x;
    return cudaLaunchKernelEx(&cfg, merge_exchange_kernel, args, d, xc);
  }
  return cudaLaunchKernelEx(&cfg, merge_kernel, args, d, bal);
}


// ---------------------------------------------------------------------------
// Tensor-core (tcgen05) path: int8 rows of 128 dimensions.

template <int GPR, int NH> struct TK {
  static void *fn() { return reinterpret_cast<void *>(&decode_tc_kernel<GPR, NH>); }
};

void *tc_kernel_for(int gpr, int nh) {
#define KVFB_TC(G, N) \
  if (gpr == G && nh == N) return TK<G, N>::fn();
  KVFB_TC(1, 4) KVFB_TC(1, 8) KVFB_TC(2, 4) KVFB_TC(2, 8)
#undef KVFB_TC
  return nullptr;
}

uint32_t tc_misc_bytes(int gpr, int nh) {
  size_t n = 0;
  if (gpr == 1) n = nh == 4 ? sizeof(TcMisc<1, 4>) : sizeof(TcMisc<1, 8>);
  else n = nh == 4 ? sizeof(TcMisc<2, 4>) : sizeof(TcMisc<2, 8>);
  return (uint32_t)((n + 127) & ~(size_t)127);
}

// The tensor-core kernel takes one KV head per block; it wins once there are
// enough (sequence, KV head) units to fill the GPU without many splits. The
// B200 sweep (machines/b200-sxm.sweep.csv) puts the crossover between 8 units
// (mma.sync 25.6 us vs 30.8 us) and 32 units (tcgen05 43.1 us vs 45.9 us).
// KVF_PATH_TC forces it for every shape it supports, KVF_PATH_MMA never.
constexpr int kTcMinUnits = 32;

bool tc_supported(const Shape &sh) { return sh.fmt == 1 && sh.d == 128 && (sh.gpr == 1 || sh.gpr == 2); }

bool tc_applies(const Shape &sh, int units) { return tc_supported(sh) && units >= kTcMinUnits; }

constexpr int kPathMask = 0xFF;
constexpr int kFlagMask = KVF_FLAG_MERGE_KERNEL | KVF_FLAG_GRID_MERGE | KVF_FLAG_NO_BALANCE;

// The kernel a launch on `path` runs: 1 = mma.sync, 2 = tcgen05; an error
// status for a path value that does not exist, contradictory or unknown
// flags, or a tcgen05 request the shape does not allow.
cudaError_t resolve_path(const Shape &sh, int units, int path, int &kernel) {
  const int flags = path & ~kPathMask;
  if ((flags & ~kFlagMask) ||
      ((flags & KVF_FLAG_MERGE_KERNEL) && (flags & KVF_FLAG_GRID_MERGE)))
    return cudaErrorInvalidValue;
  switch (path & kPathMask) {
  case KVF_PATH_AUTO:
    kernel = tc_applies(sh, units) ? 2 : 1;
    return cudaSuccess;
  case KVF_PATH_MMA:
    kernel = 1;
    return cudaSuccess;
  case KVF_PATH_TC:
    if (!tc_supported(sh)) return cudaErrorNotSupported;
    kernel = 2;
    return cudaSuccess;
  default:
    return cudaErrorInvalidValue;
  }
}

struct TcLaunch {
  TcPlan p;
  void *fn = nullptr;
  int blocks = 0;
  int occupancy = 0;
  int nh = 4;
};

cudaError_t plan_tc(const kvf_args *a, const Shape &sh, TcLaunch &L) {
  TcPlan &p = L.p;
  std::memset(&p, 0, sizeof(p));
  p.gq = a->H / a->Hkv;
  L.nh = p.gq <= 4 ? 4 : 8;
  L.fn = tc_kernel_for(sh.gpr, L.nh);
  if (!L.fn) return cudaErrorInvalidValue;
  const int ns = L.nh == 4 ? 16 : 32;
  const int np = sh.gpr * ns;
  p.paged = sh.paged;
  p.tm = sh.ord;
  p.bt_shift = sh.paged ? ilog2(sh.bt) : 0;
  p.tbox = sh.paged ? std::min(kTcTokens, sh.bt) : kTcTokens;
  p.tbox_shift = ilog2(p.tbox);
  p.npg = kTcTokens / p.tbox;
  p.meta_bytes = (uint32_t)((kTcTokens * sh.gpr * 4 + 127) & ~127);
  p.stage_bytes = (2u * kTcTokens * 128u + 2u * p.meta_bytes + 1023u) & ~1023u;
  p.ptile_bytes = (uint32_t)(np * kTcTokens);
  const uint32_t qtile = (uint32_t)(ns * 128);
  const uint32_t misc = tc_misc_bytes(sh.gpr, L.nh);
  // 1024 bytes of slack for aligning the dynamic shared-memory base.
  // The P' tile of a stage is written over its K tile (dead after the score
  // MMAs), so it takes no shared memory of its own.
  const uint32_t fixed = 1024u + ((qtile + 1023u) & ~1023u) + misc;
  int occ = 2, stages = 0;
  for (; occ >= 1; --occ) {
    const int budget = std::min(kSmemPerBlockMax, kSmemPerSM / occ - kReservedPerBlock) - (int)fixed;
    stages = std::min(8, budget / (int)p.stage_bytes);
    if (stages >= 2) break;
  }
  if (stages < 2) return cudaErrorInvalidValue;
  L.occupancy = occ;
  p.stages = stages;
  p.off_q = (uint32_t)stages * p.stage_bytes;
  p.off_misc = p.off_q + ((qtile + 1023u) & ~1023u);
  p.smem_total = 1024u + p.off_misc + misc;
  uint32_t cols = (uint32_t)(2 * sh.gpr * ns + np);  // two score buffers and the value accumulator
  uint32_t alloc = 32;
  while (alloc < cols) alloc <<= 1;
  p.tmem_cols = alloc;
  p.splits = a->splits;
  p.final_out = a->splits == 1;
  const int per = (a->n + a->splits - 1) / std::max(1, a->splits);
  p.chunk = std::max(kTcTokens, (per + kTcTokens - 1) / kTcTokens * kTcTokens);
  if (sh.paged && sh.bt > kTcTokens) p.chunk = (p.chunk + sh.bt - 1) / sh.bt * sh.bt;
  L.blocks = a->B * a->Hkv * a->splits;
  // The last block of a head merges in-kernel when counters are given and its
  // scratch (a weight per split and query-head slot) fits in the idle ring.
  p.merge_in_kernel = (a->split_sem && a->splits > 1 &&
                       (size_t)(8 * a->splits + 8) * sizeof(float) <= (size_t)stages * p.stage_bytes)
                          ? 1
                          : 0;
  return cudaSuccess;
}

// Launches `fn` with its parameter array; with `pdl` as the programmatic
// dependent of the previous kernel on the stream (the kernels wait for it with
// griddepcontrol.wait before reading the queries).
cudaError_t launch_params(void *fn, int blocks, int threads, void **params, uint32_t smem, cudaStream_t stream,
                          bool pdl, bool coop = false) {
  if (!pdl && !coop) return cudaLaunchKernel(fn, dim3((unsigned)blocks), dim3((unsigned)threads), params, smem, stream);
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (coop) {
    attr[na].id = cudaLaunchAttributeCooperative;
    attr[na].val.cooperative = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelExC(&cfg, fn, params);
}

// Identifier of the current CUDA context (cuCtxGetId), 0 when there is none
// yet or the driver cannot tell. Per-context caches key on it, so a context
// that replaced another (after cudaDeviceReset) never sees stale entries.
unsigned long long context_id() {
  typedef CUresult (*GetCurrentFn)(CUcontext *);
  typedef CUresult (*GetIdFn)(CUcontext, unsigned long long *);
  static std::once_flag once;
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(p);
    cudaGetLastError();
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Per-context facts about a kernel: the dynamic shared memory it may use
// (cudaFuncSetAttribute is called only when a launch needs more than was set)
// and its resident blocks per SM for one (threads, shared memory) pair, so a
// decode step does not pay these driver queries on every call.
struct KernelCtxEntry {
  void *fn;
  unsigned long long ctx;
  uint32_t smem_set;
  int occ_threads;
  uint32_t occ_smem;
  int occ_blocks;
};
std::mutex g_kctx_mu;
KernelCtxEntry g_kctx[128];
int g_kctx_n = 0;

KernelCtxEntry *kctx_find(void *fn, unsigned long long ctx) {
  for (int i = 0; i < g_kctx_n; ++i)
    if (g_kctx[i].fn == fn && g_kctx[i].ctx == ctx) return &g_kctx[i];
  return nullptr;
}

KernelCtxEntry *kctx_add(void *fn, unsigned long long ctx) {
  if (ctx == 0) return nullptr;
  if (KernelCtxEntry *e = kctx_find(fn, ctx)) return e;
  if (g_kctx_n == 128) return nullptr;  // full: no caching, every call asks the driver
  g_kctx[g_kctx_n] = KernelCtxEntry{fn, ctx, 0u, 0, 0u, 0};
  return &g_kctx[g_kctx_n++];
}

// Lets `fn` use `smem` bytes of dynamic shared memory.
cudaError_t ensure_smem(void *fn, uint32_t smem) {
  std::lock_guard<std::mutex> lock(g_kctx_mu);
  const unsigned long long ctx = context_id();
  if (ctx) {
    KernelCtxEntry *e = kctx_find(fn, ctx);
    if (e && e->smem_set >= smem) return cudaSuccess;
  }
  const cudaError_t r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (r != cudaSuccess) return r;
  if (KernelCtxEntry *e = kctx_add(fn, context_id())) e->smem_set = std::max(e->smem_set, smem);
  return cudaSuccess;
}

// Whether every block of the launch can be resident at once (required by a
// cooperative launch).
bool coop_fits(void *fn, int blocks, int threads, uint32_t smem) {
  // The occupancy of a block with this much dynamic shared memory counts only
  // once the kernel may use it (set here too, so describing agrees with launching).
  if (ensure_smem(fn, smem) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int per_sm = -1;
  {
    std::lock_guard<std::mutex> lock(g_kctx_mu);
    const KernelCtxEntry *e = kctx_find(fn, context_id());
    if (e && e->occ_threads == threads && e->occ_smem == smem) per_sm = e->occ_blocks;
  }
  if (per_sm < 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    std::lock_guard<std::mutex> lock(g_kctx_mu);
    if (KernelCtxEntry *e = kctx_add(fn, context_id())) {
      e->occ_threads = threads;
      e->occ_smem = smem;
      e->occ_blocks = per_sm;
    }
  }
  return blocks <= per_sm * sm_count();
}

// Whether a decode launch should merge its splits itself (cooperative launch,
// grid barrier): partials to merge, split counters with room for the barrier
// words (two or more (sequence, KV head) units); behind a programmatic
// dependency too (the zero-copy step's staging kernel), falling back to the
// merge kernel where the runtime refuses that pair. It pays once the
// separate merge kernel is large:
// measured on B200, 8 sequences with 1024 merge slices (query head x 32
// columns) for 288 decode blocks step in 53.7 us instead of 57.2, while
// single sequences with 128 slices for ~295 blocks lose 1.4-2.5 us (the
// cooperative launch costs more than the merge kernel it replaces). So by
// default it is used from two slices per decode block; KVF_FLAG_GRID_MERGE
// asks for it wherever possible, KVF_FLAG_MERGE_KERNEL never.
// Split counts up to which the last finishers merge: 64 for f16; for int8
// and int4 the most for which the tail merge's narrower loads give the merge
// kernel's bits (kMergeWarps x kTailMergeUnroll = 160). Measured below, at
// the plan_mma call.
constexpr int kTailMergeMaxSplits = 64;
constexpr int kTailMergeMaxSplitsInt = kMergeWarps * kTailMergeUnroll;

bool coop_wanted(const kvf_args *a, int d, long long blocks, int flags) {
  if (a->splits <= 1 || !a->split_sem || (long long)a->B * a->Hkv < 2) return false;
  if (flags & KVF_FLAG_MERGE_KERNEL) return false;
  if (flags & KVF_FLAG_GRID_MERGE) return true;
  const long long slices = (long long)a->B * a->H * ((d + 31) / 32);
  return slices >= 2LL * blocks;
}


// The mma.sync launch: plan, token-balanced splits, in-launch merge.
//
// When seq_lens is given (sequences may differ in length) and every
// (sequence, head group) fits in one wave of blocks, the grid is one wave
// (blocks per SM x SMs, or fewer when the splits need fewer) and the blocks
// share the tokens evenly (balanced_chunk in decode_kernel.cuh). Measured on
// B200 (8 sequences, f16, pages of 16): one sequence of 32768 tokens among
// seven of 1024 steps in 46.4 us instead of 91.6 (with one split count for
// all, the long sequence had 36 of 296 blocks); 2k-8k tokens each, which
// already streams at the batch's aggregate rate, 52.1 instead of 50.1. The
// in-launch merge and the balanced splits need the general kernel;
// contiguous caches without either run the lean one. flags: KVF_FLAG_* bits.
cudaError_t plan_mma(const kvf_args *a, const Shape &sh, int d, const kvf_exchange *x, int flags, Launch &L,
                     bool &want_coop) {
  const int hh = heads_per_block(a->Hkv, sh.fmt, sh.d);
  const bool bal_wanted = !x && a->seq_lens && a->splits > 1 && !(flags & KVF_FLAG_NO_BALANCE);
  want_coop = !x && coop_wanted(a, d, (long long)a->B * (a->Hkv / hh) * a->splits, flags);
  cudaError_t e = plan_launch(a, sh, L, !sh.paged && !want_coop && !bal_wanted);
  if (e != cudaSuccess) return e;
  const long long slots = (long long)L.occupancy * sm_count();
  if (bal_wanted && (long long)a->B * L.p.hg <= slots) {
    L.p.bal_gran = (sh.paged && sh.bt > L.p.tb) ? sh.bt : L.p.tb;
    L.blocks = (int)std::min<long long>(slots, L.blocks);
    want_coop = !x && coop_wanted(a, d, L.blocks, flags);
  }
  // Without the grid merge, the last finishers of each (sequence, head
  // group) merge its splits in the same launch, where the grid fits in one
  // wave (their bounded wait is for blocks that are already running or
  // about to) and the splits are few; the merge kernel otherwise, or when
  // asked for. A tail merger reads each slice's partials with its block's
  // consumer warps, two rounds of loads for 4 warps where the merge kernel's
  // 8 warps need one: measured on B200 at B = 1, 37 splits (mha, 32 heads)
  // step in 24.2 us instead of 25.6 with the merge kernel, 147 splits (8 KV
  // heads, int8:64) in the same 27.6 us (one launch instead of two, so ~4 us
  // less host time per call), 147 splits of int4:32 in 40.9 instead of 37.9.
  const int tail_max = sh.fmt != 0 ? kTailMergeMaxSplitsInt : kTailMergeMaxSplits;
  L.p.tail_merge = (!x && !want_coop && a->split_sem && a->splits > 1 && a->splits <= tail_max &&
                    L.p.bal_gran == 0 && !(flags & KVF_FLAG_MERGE_KERNEL) && (long long)L.blocks <= slots)
                       ? 1
                       : 0;
  return cudaSuccess;
}

cudaError_t launch_tc(const kvf_args *a, const Shape &sh, cudaStream_t stream, const kvf_exchange *x = nullptr,
                      bool pdl = false) {
  TcLaunch L;
  cudaError_t e = plan_tc(a, sh, L);
  if (e != cudaSuccess) return e;
  if (x) L.p.merge_in_kernel = 0;  // the exchange runs in the separate merge
  CUtensorMap tk, tv;
  e = encode_maps_box(a, sh, 128, 128, L.p.tbox, 1, tk, tv);
  if (e != cudaSuccess) return e;
  e = ensure_smem(L.fn, L.p.smem_total);
  if (e != cudaSuccess) return e;
  const kvf_args args = *a;
  const TcPlan plan = L.p;
  void *params[4] = {const_cast<kvf_args *>(&args), const_cast<TcPlan *>(&plan), &tk, &tv};
  e = launch_params(L.fn, L.blocks, kTcThreads, params, L.p.smem_total, stream, pdl);
  if (e != cudaSuccess) return e;
  if (!L.p.final_out && !L.p.merge_in_kernel) e = launch_merge(a, sh.d, stream, true, x);
  return e != cudaSuccess ? e : cudaGetLastError();
}

} // namespace
} // namespace kvfb

using namespace kvfb;

namespace kvfb {
namespace {

cudaError_t decode_impl(const kvf_args *a, int fmt, int d, int g, int ord, int paged, int path, cudaStream_t stream,
                        const kvf_exchange *x, bool pdl = false) {
  Shape sh;
  cudaError_t e = check_args(a, fmt, d, g, ord, paged, sh);
  if (e != cudaSuccess) return e;
  int kernel = 1;
  e = resolve_path(sh, a->B * a->Hkv, path, kernel);
  if (e != cudaSuccess) return e;
  if (a->B == 0) return cudaSuccess;
  if (kernel == 2) return launch_tc(a, sh, stream, x, pdl);
  Launch L;
  bool want_coop = false;
  e = plan_mma(a, sh, d, x, path & ~kPathMask, L, want_coop);
  if (e != cudaSuccess) return e;
  CUtensorMap tk, tv, tkm, tvm;
  e = encode_maps(a, sh, L.p, tk, tv);
  if (e != cudaSuccess) return e;
  std::memset(&tkm, 0, sizeof(tkm));
  std::memset(&tvm, 0, sizeof(tvm));
  if (L.p.meta_tma && encode_meta_maps(a, sh, L.p, tkm, tvm) != cudaSuccess) {
    // The metadata goes by cp.async after all.
    L.p.meta_tma = 0;
    L.p.tx_bytes = 2u * L.p.kv_bytes;
    L.p.meta_ts = (uint32_t)(sh.gpr * 4);
    L.p.meta_hs = (uint32_t)(L.p.tb * sh.gpr * 4);
  }
  e = ensure_smem(L.fn, L.p.smem_total);
  if (e != cudaSuccess) return e;
  L.p.coop_merge = (want_coop && !L.p.final_out && coop_fits(L.fn, L.blocks, L.threads, L.p.smem_total)) ? 1 : 0;
  const kvf_args args = *a;
  Plan plan = L.p;
  void *params[6] = {const_cast<kvf_args *>(&args), &plan, &tk, &tv, &tkm, &tvm};
  e = launch_params(L.fn, L.blocks, L.threads, params, L.p.smem_total, stream, pdl, L.p.coop_merge != 0);
  if (e != cudaSuccess && L.p.coop_merge && pdl) {
    // Not taken as a cooperative launch behind a programmatic dependency:
    // the merge goes to its own kernel instead.
    cudaGetLastError();
    L.p.coop_merge = 0;
    plan.coop_merge = 0;
    e = launch_params(L.fn, L.blocks, L.threads, params, L.p.smem_total, stream, pdl, false);
  }
  if (e != cudaSuccess) return e;
  if (!L.p.final_out && !L.p.coop_merge && !L.p.tail_merge)
    e = launch_merge(a, d, stream, true, x,
                     L.p.bal_gran > 0 ? MergeBalance{L.p.hg, L.blocks, L.p.bal_gran} : MergeBalance{0, 0, 0});
  return e != cudaSuccess ? e : cudaGetLastError();
}

} // namespace
} // namespace kvfb

extern "C" cudaError_t kvf_b200_decode(const kvf_args *a, int fmt, int d, int g, int ord, int paged,
                                       cudaStream_t stream) {
  return decode_impl(a, fmt, d, g, ord, paged, KVF_PATH_AUTO, stream, nullptr);
}

extern "C" cudaError_t kvf_b200_decode_path(const kvf_args *a, int fmt, int d, int g, int ord, int paged, int path,
                                            cudaStream_t stream) {
  return decode_impl(a, fmt, d, g, ord, paged, path, stream, nullptr);
}

namespace kvfb {
namespace {

// Copies the queries from host memory the device can address into a->q:
// one 16-byte load and store per thread (the host reads go over PCIe). The
// decode grid that follows may start at once; it reads the queries after
// griddepcontrol.wait.
__global__ void __launch_bounds__(256) stage_in_kernel(float4 *dst, const float4 *src, long long n4) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n4) dst[i] = src[i];
}

// Host memory the kernels may read or write directly: pinned and mapped at
// the same address (cudaHostAlloc under unified addressing), or device memory.
bool device_addressable(const void *p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) return true;
  return at.type == cudaMemoryTypeHost && at.devicePointer == p;
}

// Copies n4 float4 from host memory with 128-thread blocks of at most 32
// registers a thread, so that one block fits beside two resident tcgen05
// decode blocks on an SM (they leave 4096 registers); each thread keeps
// several loads in flight. Launched as the programmatic dependent of a decode
// grid whose data it does not touch, it starts at once and lets its own
// dependent launch.
__global__ void __launch_bounds__(128, 16) stage_in_narrow_kernel(float4 *dst, const float4 *src, int n4) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int stride = gridDim.x * blockDim.x;
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n4; i += 4 * stride) {
    const float4 v0 = src[i], v1 = src[i + stride], v2 = src[i + 2 * stride], v3 = src[i + 3 * stride];
    dst[i] = v0;
    dst[i + stride] = v1;
    dst[i + 2 * stride] = v2;
    dst[i + 3 * stride] = v3;
  }
  for (; i < n4; i += stride) dst[i] = src[i];
}

// Arguments of sequences [b0, b0 + nb) of a batch.
kvf_args sub_batch(const kvf_args *a, const Shape &sh, int d, int b0, int nb) {
  kvf_args s = *a;
  const long long qo = (long long)b0 * a->H * d;
  s.q = a->q + qo;
  s.out = a->out + qo;
  if (a->lse) s.lse = a->lse + (long long)b0 * a->H;
  if (a->seq_lens) s.seq_lens = a->seq_lens + b0;
  if (a->part_o) s.part_o = a->part_o + (long long)b0 * a->H * a->splits * d;
  if (a->part_ml) s.part_ml = a->part_ml + (long long)b0 * a->H * a->splits * 2;
  if (a->split_sem) s.split_sem = a->split_sem + 2LL * b0 * a->Hkv;  // two words per (sequence, KV head)
  if (sh.paged) {
    s.block_table = a->block_table + (long long)b0 * a->max_blocks;
  } else {
    const long long rows = (long long)b0 * a->n * a->Hkv;  // a sequence's rows are contiguous in both orders
    s.k = a->k + rows * row_bytes(sh.fmt, sh.d);
    s.v = a->v + rows * row_bytes(sh.fmt, sh.d);
    if (sh.gpr > 0) {
      s.k_meta = static_cast<const uint32_t *>(a->k_meta) + rows * sh.gpr;
      s.v_meta = static_cast<const uint32_t *>(a->v_meta) + rows * sh.gpr;
    }
  }
  s.B = nb;
  return s;
}

// Host-query steps of large batches on the tcgen05 path. With one staging
// kernel for the whole batch every decode block waits for all of the queries
// (config 5: 2 MB, ~40 us over PCIe). Instead the sequences whose blocks fit
// one wave are staged and decoded first; the rest are staged by a narrow copy
// kernel that runs beside that decode, and decoded after it, each launch the
// programmatic dependent of the one before. Returns the number of sequences
// of the first part, B for no split (one wave holds everything, or the rest
// of the queries is small).
constexpr long long kSplitStageMinBytes = 256 * 1024;

int first_wave_sequences(const kvf_args *a, const Shape &sh, int d) {
  if (a->B < 2) return a->B;
  TcLaunch L;
  if (plan_tc(a, sh, L) != cudaSuccess) {
    cudaGetLastError();
    return a->B;
  }
  const long long per_seq = (long long)a->Hkv * std::max(1, a->splits);
  const long long s1 = (long long)L.occupancy * sm_count() / per_seq;  // every block of part 1 resident at once
  if (s1 < 1 || s1 >= a->B) return a->B;
  const long long rest = (a->B - s1) * (long long)a->H * d * 4;
  // (the narrow kernel indexes float4 with 32-bit integers, i + 3 x its grid)
  return rest >= kSplitStageMinBytes && rest / 16 <= (1LL << 30) ? (int)s1 : a->B;
}

} // namespace
} // namespace kvfb

extern "C" cudaError_t kvf_b200_decode_from_host(const kvf_args *a, int fmt, int d, int g, int ord, int paged,
                                                 int path, const float *q_host, cudaStream_t stream) {
  Shape sh;
  cudaError_t e = check_args(a, fmt, d, g, ord, paged, sh);
  if (e != cudaSuccess) return e;
  if (a->B == 0) return cudaSuccess;
  const long long n = (long long)a->B * a->H * d;
  if (!q_host || (reinterpret_cast<uintptr_t>(q_host) & 15u) || (reinterpret_cast<uintptr_t>(a->q) & 15u) ||
      (n & 3))
    return cudaErrorInvalidValue;
  if (!device_addressable(q_host) || !device_addressable(a->q) || !device_addressable(a->out) ||
      (a->lse && !device_addressable(a->lse)))
    return cudaErrorInvalidValue;
  int kernel = 1;
  e = resolve_path(sh, a->B * a->Hkv, path, kernel);
  if (e != cudaSuccess) return e;
  const int s1 = kernel == 2 ? first_wave_sequences(a, sh, d) : a->B;
  const long long h1 = (long long)s1 * a->H * d;
  stage_in_kernel<<<(unsigned)((h1 / 4 + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<float4 *>(const_cast<float *>(a->q)), reinterpret_cast<const float4 *>(q_host), h1 / 4);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (s1 == a->B) return decode_impl(a, fmt, d, g, ord, paged, path, stream, nullptr, true);
  // Both parts on the tcgen05 kernel (the launcher's unit rule would see each
  // part's smaller batch), with the same flags.
  const int ptc = KVF_PATH_TC | (path & ~kPathMask);
  const kvf_args a1 = sub_batch(a, sh, d, 0, s1), a2 = sub_batch(a, sh, d, s1, a->B - s1);
  e = decode_impl(&a1, fmt, d, g, ord, paged, ptc, stream, nullptr, true);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)sm_count());
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, stage_in_narrow_kernel, reinterpret_cast<float4 *>(const_cast<float *>(a2.q)),
                         reinterpret_cast<const float4 *>(q_host + h1), (int)((n - h1) / 4));
  if (e != cudaSuccess) return e;
  return decode_impl(&a2, fmt, d, g, ord, paged, ptc, stream, nullptr, true);
}

extern "C" cudaError_t kvf_b200_decode_exchange(const kvf_args *a, int fmt, int d, int g, int ord, int paged,
                                                const kvf_exchange *x, cudaStream_t stream) {
  if (!a || !x || a->splits <= 1 || x->P < 1 || x->P > 8 || x->rank < 0 || x->rank >= x->P || !x->gather ||
      x->timeout_ms == 0 || x->epoch < 1)
    return cudaErrorInvalidValue;
  for (int p = 0; p < x->P; ++p)
    if (!x->peer_gather[p]) return cudaErrorInvalidValue;
  return decode_impl(a, fmt, d, g, ord, paged, KVF_PATH_AUTO, stream, x);
}

extern "C" cudaError_t kvf_b200_merge(const kvf_args *a, int d, cudaStream_t stream) {
  if (!a || (d != 64 && d != 128) || a->splits < 1 || a->H <= 0 || a->B < 0) return cudaErrorInvalidValue;
  if (a->B == 0) return cudaSuccess;
  if (!a->part_o || !a->part_ml || !a->out) return cudaErrorInvalidValue;
  const cudaError_t e = launch_merge(a, d, stream, false);
  return e != cudaSuccess ? e : cudaGetLastError();
}

extern "C" cudaError_t kvf_b200_merge_states(const float *o, const float *lse, int P, int rows, int d,
                                             long long o_stride, long long lse_stride, float *out, float *lse_out,
                                             cudaStream_t stream) {
  if (P < 1 || rows < 0 || d < 1 || d > 1024 || !o || !lse || !out) return cudaErrorInvalidValue;
  if (o_stride < (long long)rows * d || lse_stride < rows) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  const int threads = (d + 31) / 32 * 32;
  merge_states_kernel<<<rows, threads, 0, stream>>>(o, lse, P, rows, d, o_stride, lse_stride, out, lse_out);
  return cudaGetLastError();
}

extern "C" cudaError_t kvf_b200_describe_path(const kvf_args *a, int fmt, int d, int ord, int paged, int path,
                                              char *buf, int buf_len) {
  Shape sh;
  cudaError_t e = check_args(a, fmt, d, 1, ord, paged, sh);
  if (e != cudaSuccess) return e;
  int kernel = 1;
  e = resolve_path(sh, a->B * a->Hkv, path, kernel);
  if (e != cudaSuccess) return e;
  if (kernel == 2) {
    TcLaunch T;
    e = plan_tc(a, sh, T);
    if (e != cudaSuccess) return e;
    if (buf && buf_len > 0) {
      const KernelInfo ki = info_for(T.fn);
      std::snprintf(buf, (size_t)buf_len,
                    "kernel=tcgen05 grid=%d block=%d heads/block=1 tokens/stage=%d stages=%d stage_bytes=%u "
                    "smem=%u tmem_cols=%u chunk=%d splits=%d blocks/sm=%d regs=%d final=%d merge=%s",
                    T.blocks, kTcThreads, kTcTokens, T.p.stages, T.p.stage_bytes, T.p.smem_total, T.p.tmem_cols,
                    T.p.chunk, T.p.splits, T.occupancy, ki.regs, T.p.final_out,
                    T.p.final_out ? "none" : T.p.merge_in_kernel ? "in-kernel" : "kernel");
    }
    return cudaSuccess;
  }
  Launch L;
  bool want_coop = false;
  e = plan_mma(a, sh, d, nullptr, path & ~kPathMask, L, want_coop);
  if (e != cudaSuccess) return e;
  if (buf && buf_len > 0) {
    const KernelInfo ki = info_for(L.fn);
    char chunk[48];
    if (L.p.bal_gran > 0)
      std::snprintf(chunk, sizeof(chunk), "balanced(gran=%d)", L.p.bal_gran);
    else
      std::snprintf(chunk, sizeof(chunk), "%d", L.p.chunk);
    std::snprintf(buf, (size_t)buf_len,
                  "kernel=mma.sync grid=%d block=%d heads/block=%d tokens/stage=%d stages=%d stage_bytes=%u "
                  "smem=%u chunk=%s splits=%d blocks/sm=%d regs=%d final=%d meta=%s merge=%s",
                  L.blocks, L.threads, L.p.hh, L.p.tb, L.p.stages, L.p.stage_bytes, L.p.smem_total,
                  chunk, L.p.splits, L.occupancy, ki.regs, L.p.final_out,
                  sh.gpr == 0 ? "none" : L.p.meta_tma ? "tma" : "cp.async",
                  L.p.final_out ? "none"
                  : want_coop && coop_fits(L.fn, L.blocks, L.threads, L.p.smem_total) ? "in-kernel(grid)"
                  : L.p.tail_merge ? "in-kernel(tail)" : "kernel");
  }
  return cudaSuccess;
}

extern "C" cudaError_t kvf_b200_describe(const kvf_args *a, int fmt, int d, int ord, int paged, char *buf,
                                         int buf_len) {
  return kvf_b200_describe_path(a, fmt, d, ord, paged, KVF_PATH_AUTO, buf, buf_len);
}

namespace kvfb {
namespace {

int suggest_splits(int B, int H, int Hkv, int n, int fmt, int d, int group, int paged, int block_tokens,
                   bool ragged) {
  if (B <= 0 || H <= 0 || Hkv <= 0 || H % Hkv || n <= 0 || (d != 64 && d != 128) || fmt < 0 || fmt > 2)
    return 1;
  const int sms = sm_count();
  Shape shq;
  shq.fmt = fmt;
  shq.d = d;
  shq.ord = 0;
  shq.paged = paged ? 1 : 0;
  shq.bt = paged ? block_tokens : 0;
  shq.gpr = fmt ? d / std::max(group, 1) : 0;
  const bool tc = group_ok(fmt, d, group) && H / Hkv <= 8 && tc_applies(shq, B * Hkv);
  // Work units (blocks per split) and tokens per stage of the kernel that runs.
  const int hh = tc ? 1 : heads_per_block(Hkv, fmt, d);
  const int units = B * (Hkv / hh);
  const int tb = tc ? kTcTokens : 16 * stage_mtiles(fmt, d);
  int gran = tb;
  if (paged && block_tokens > tb) gran = block_tokens;
  // Blocks per SM from the launch plan (registers and shared memory); 1 when
  // the kernel cannot be inspected (no device).
  int occ = 1;
  {
    kvf_args a;
    std::memset(&a, 0, sizeof(a));
    a.B = B;
    a.H = H;
    a.Hkv = Hkv;
    a.n = n;
    a.splits = 1;
    a.group_shift = fmt ? ilog2(std::max(group, 1)) : 0;
    a.block_shift = paged ? ilog2(std::max(block_tokens, 1)) : 0;
    Shape sh;
    sh.fmt = fmt;
    sh.d = d;
    sh.ord = 0;
    sh.paged = paged ? 1 : 0;
    sh.bt = paged ? block_tokens : 0;
    sh.gpr = fmt ? d / std::max(group, 1) : 0;
    if (tc) {
      TcLaunch T;
      if (plan_tc(&a, sh, T) == cudaSuccess) occ = T.occupancy;
    } else {
      Launch L;
      if (group_ok(fmt, d, group) && H / Hkv <= 8 && plan_launch(&a, sh, L, !paged) == cudaSuccess) occ = L.occupancy;
    }
    cudaGetLastError();
  }
  const int slots = sms * occ;
  const int smax = std::max(1, std::min(1024, (n + gran - 1) / gran));
  // Cost model in stage times: every wave of blocks pays a fixed fill and
  // drain of about three stages plus its share of the stages; a split count
  // that leaves the last wave nearly empty, or that makes many short waves,
  // loses. Ties go to fewer splits (less merge work).
  const double stages_per_unit = std::ceil((double)n / tb);
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= smax; ++s) {
    const int chunk = ((n + s - 1) / s + gran - 1) / gran * gran;
    const int used = (n + chunk - 1) / chunk;  // non-empty splits
    if (used < s) continue;
    const double waves = std::ceil((double)units * s / slots);
    const double cost = waves * (3.0 + std::ceil(stages_per_unit / s)) * (1.0 + 0.002 * s);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  if (ragged && !tc && units <= slots && best > 1) {
    // Balanced launches (plan_mma) choose the chunk themselves; the split
    // count is the workspace's capacity per sequence. One sequence may use
    // up to slots / head-groups splits (when the others are short); the
    // capacity allows that while the partials stay within 64 MiB.
    const int per = slots / (Hkv / hh);
    const long long per_split = (long long)B * H * (d + 2) * 4;
    const int by_bytes = (int)std::min<long long>(1024, (64ll << 20) / per_split);
    return std::max(best, std::min({per, smax, by_bytes}));
  }
  return best;
}

} // namespace
} // namespace kvfb

extern "C" int kvf_b200_suggest_splits(int B, int H, int Hkv, int n, int fmt, int d, int group,
                                       int paged, int block_tokens) {
  return suggest_splits(B, H, Hkv, n, fmt, d, group, paged, block_tokens, false);
}

extern "C" int kvf_b200_balanced_chunk(const int *seq_lens, int B, int n, int splits, int units, int grid,
                                       int gran) {
  if (!seq_lens || B <= 0 || n < 0 || splits < 1 || units < 1 || gran < 1 || grid < 1 ||
      (long long)units * B > grid)
    return -1;
  auto len_of = [&](int b) { return std::min(std::max(seq_lens[b], 0), n); };
  long long T = 0;
  int nz = 0;
  for (int b = 0; b < B; ++b) {
    T += len_of(b);
    nz += len_of(b) > 0;
  }
  return balance_search(T, nz, n, splits, grid / units, gran, [&](int c) {
    long long cnt = 0;
    for (int b = 0; b < B; ++b) cnt += (len_of(b) + c - 1) / c;
    return cnt;
  });
}

extern "C" int kvf_b200_suggest_splits_ragged(int B, int H, int Hkv, int n, int fmt, int d, int group,
                                              int paged, int block_tokens) {
  return suggest_splits(B, H, Hkv, n, fmt, d, group, paged, block_tokens, true);
}

namespace kvfb {
unsigned take_append_errors();  // quantize.cu
}

extern "C" unsigned kvf_b200_device_errors(void) {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_kvfb_error, sizeof(v)) != cudaSuccess) {
    cudaGetLastError();
    return 0xFFFFFFFFu;
  }
  if (v) cudaMemcpyToSymbol(g_kvfb_error, &zero, sizeof(zero));
  if (kvfb::take_append_errors()) v |= 4u;  // an appended row fell outside the cache
  return v;
}

extern "C" const char *kvf_b200_version(void) { return "kvforge_b200 0.1 (sm_100a)"; }

// ---------------------------------------------------------------------------
// Decode without any allocation by the caller or by this library.
//
// Some callers cannot call cudaMalloc: a serving engine that reserved all of
// device memory for its KV page pool at start-up (any later allocation can
// fail, and cudaMalloc may synchronise the device in the middle of a decode
// step), or a plugin whose host framework owns and accounts for every device
// allocation and hands it nothing but the tensors of the call. For them the
// split partials live in this file-scope device array, which every GPU that
// loads the library holds until the process exits.
namespace kvfb {
namespace {

constexpr size_t kNoAllocScratchBytes = KVF_B200_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array, looked up once per device with that
// device current (and again if the device's context was replaced, e.g. after
// cudaDeviceReset, which reloads the module). In host code the array's name is
// only a host-side stand-in, never a device address, so it is never passed to
// a kernel directly.
void *noalloc_scratch_address(cudaError_t &err) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static void *addr[kMaxDevices] = {};
  static unsigned long long ctx_of[kMaxDevices] = {};
  int dev = 0;
  err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= kMaxDevices) {
    err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev] || ctx_of[dev] != context_id()) {
    void *p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess) return nullptr;
    addr[dev] = p;
    ctx_of[dev] = context_id();
  }
  err = cudaSuccess;
  return addr[dev];
}

} // namespace
} // namespace kvfb

extern "C" cudaError_t kvf_b200_decode_noalloc(const kvf_args *a, int fmt, int d, int g, int ord,
                                               int paged, cudaStream_t stream) {
  if (!a) return cudaErrorInvalidValue;
  if (a->splits <= 1 || a->B == 0) return kvf_b200_decode(a, fmt, d, g, ord, paged, stream);
  if (a->B < 0 || a->H <= 0 || (d != 64 && d != 128)) return cudaErrorInvalidValue;
  // part_ml [B][H][splits][2] then part_o [B][H][splits][D], both fp32.
  const size_t heads = (size_t)a->B * (size_t)a->H * (size_t)a->splits;
  const size_t ml_bytes = (heads * 2 * sizeof(float) + 255) & ~(size_t)255;
  const size_t o_bytes = heads * (size_t)d * sizeof(float);
  if (heads > kvfb::kNoAllocScratchBytes || ml_bytes + o_bytes > kvfb::kNoAllocScratchBytes)
    return cudaErrorInvalidValue;  // partials exceed KVF_B200_NOALLOC_SCRATCH_BYTES
  cudaError_t err;
  unsigned char *base = static_cast<unsigned char *>(kvfb::noalloc_scratch_address(err));
  if (!base) return err;
  kvf_args b = *a;
  b.part_ml = reinterpret_cast<float *>(base);
  b.part_o = reinterpret_cast<float *>(base + ml_bytes);
  return kvf_b200_decode(&b, fmt, d, g, ord, paged, stream);
}
