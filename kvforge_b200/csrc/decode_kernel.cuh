// decode_kernel.cuh - the sm_100a split-KV decode-attention kernel.
//
// Counterpart of decode_partial<FMT,D,G,U,ORD,PAGED,FINAL> in the reference
// (runtime/kvf_kernels.cuh:124-285): one block owns a chunk of one sequence's
// tokens for `hh` KV heads and all of their query heads, streams the chunk's
// K/V rows once, and produces either the normalised output (one split) or an
// unnormalised partial plus (max, sum) in log2 units for the split merge.
//
// Structure (B200-first, not a translation of the reference's SIMT loop):
//
//  * Producer warp. Lane 0 moves each stage's K and V tiles with tiled TMA
//    (cp.async.bulk.tensor, 4-D tensor maps that express all four placements:
//    head/token major x contiguous/paged) into a ring of shared-memory stages
//    guarded by full/empty mbarriers. The tiles land swizzled (128/64/32-byte
//    swizzle matching the row size) so the ldmatrix reads below are free of
//    bank conflicts. Per-row quantization metadata (4-16 bytes per row) of
//    contiguous caches comes by TMA as well, one box per stage and K/V: a
//    3-D view whose inner dimension folds the KV heads (token-major rows:
//    the block's heads of one token are adjacent) or the tokens (head-major
//    rows: one head's tokens are adjacent), so a box row is >= 16 bytes. Paged
//    caches fetch it with cp.async from all 32 lanes, counted on the same
//    full barrier.
//
//  * One consumer warp per KV head. Scores and the value product run on the
//    tensor cores with mma.sync m16n8k16 (f16 in, fp32 accumulate), with the
//    cached tokens as the M dimension:
//        S^T[16 tokens x 8] = K[16 x D]   * Q^T[D x 8]
//        O^T[16 dims   x 8] = V^T[16 x 16] * P^T[16 tokens x 8]
//    The 8 columns are (query head, part) pairs: every fp32 query is split into
//    fp16 hi + lo parts (q = hi + lo to ~2^-22), and so is every probability,
//    so the products carry fp32-level accuracy although the tensor-core inputs
//    are fp16. Integer codes (0..255, 0..15) and fp16 K/V are exact in fp16.
//    Packed G <= 4 query heads fill one 8-column tile, G <= 8 two.
//
//  * Quantized rows are dequantised algebraically as the reference does
//    (runtime/kvf_kernels.cuh:211,237-240): codes go to fp16 with the
//    0x6400 magic-exponent trick (exact), each quantization group accumulates
//    its own dot product, and
//        s   = sum_g scale_g * dot_g + zero_g * sum(q in g)
//        acc = sum_t (p_t * scale_t,g) * code_t + sum_t p_t * zero_t,g
//    where the second term of acc is a rank-1 correction kept in fp32.
//
//  * Online softmax in the log2 domain with one rescale per stage.
#pragma once

#include "ptx.cuh"
#include "kvforge_b200.h"

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <type_traits>

namespace kvfb {

// Per-launch constants computed by the host launcher (decode.cu) and shared by
// both sides. All byte offsets are relative to the 1024-aligned dynamic
// shared-memory base.
struct Plan {
  int gq;          // query heads per KV head (<= 8)
  int gpr;         // quantization groups per row (0 for f16)
  int hh;          // KV heads per block (one consumer warp each)
  int hg;          // head groups: Hkv / hh
  int tb;          // tokens per stage (multiple of 16)
  int tbox;        // tokens per TMA box (tb, or the page size when smaller)
  int tbox_shift;  // log2(tbox)
  int npg;         // boxes along tokens per stage: tb / tbox
  int nxb;         // boxes along the row: row_bytes / boxx
  int boxx;        // inner box bytes (<= 128)
  int rb;          // row bytes
  int stages;      // ring depth
  int chunk;       // tokens per split (multiple of tb)
  int splits;      // splits per sequence
  int paged;       // page addressing
  int tm;          // token-major rows (else head-major)
  int bt_shift;    // log2(tokens per page)
  int final_out;   // 1: write normalised out; 0: write partials
  int coop_merge;  // cooperative launch: the blocks merge the splits after a grid barrier
  int tail_merge;  // the last finishers of each (sequence, head group) merge its splits
  int bal_gran;    // > 0: token-balanced splits (see balanced_chunk), chunk granularity
  uint32_t swz;    // swizzle mask for the K/V tiles (0x70, 0x30, 0x10)
  uint32_t box_bytes;   // one TMA box
  uint32_t kv_bytes;    // K (or V) bytes in one stage
  uint32_t meta_bytes;  // K (or V) metadata bytes in one stage
  uint32_t stage_bytes; // one stage, 1024-aligned
  uint32_t tx_bytes;    // TMA bytes expected per stage (K + V, and their metadata by TMA)
  int meta_tma;         // metadata by TMA (contiguous caches) instead of cp.async
  uint32_t meta_ts;     // bytes between a head's consecutive tokens in a stage's metadata area
  uint32_t meta_hs;     // bytes between the heads' first tokens there
  uint32_t off_bars;    // full[stages], empty[stages]
  uint32_t off_pscr;    // P^T scratch, pscr_warp bytes per consumer warp
  uint32_t pscr_warp;
  uint32_t smem_total;
};

__device__ unsigned g_kvfb_error;
enum : unsigned { KVFB_ERR_TIMEOUT = 1u, KVFB_ERR_EXCHANGE = 2u };

// (scale, zero) of an fp16 half2 metadata word.
__device__ __forceinline__ float2 meta_sz(uint32_t w) { return ptx::unpack_f16x2(w); }

// ---------------------------------------------------------------------------
// Token-balanced splits for a batch of unequal sequences (seq_lens given).
//
// With one split count for every sequence, the blocks of the longest sequence
// set the launch time while the short sequences' blocks finish early or have
// nothing to do. Balanced, the launch has `grid` blocks for `units` head
// groups per sequence, and all sequences share one chunk c: the smallest
// multiple of `gran` with c >= ceil(n / S) (so no sequence needs more than
// the workspace's S splits) for which the work items
// units * sum_b ceil(len_b / c) fit in the grid. Sequence b then has
// s_b = ceil(len_b / c) splits, its partials in split slots [0, s_b), and
// no block reads more than c tokens. The chunk depends on seq_lens only, so
// the decode blocks and the merge compute it on the device and agree, and
// the host never reads the lengths.

// The chunk search, shared by the device (warp-parallel counts) and the host
// (plain loops): T tokens in nz non-empty sequences, per = grid / units items
// per head group, count(c) = sum_b ceil(len_b / c), non-increasing in c.
template <class Count>
__host__ __device__ __forceinline__ int balance_search(long long T, int nz, int n, int S, int per, int gran,
                                                       Count count) {
  const long long g = gran;
  auto up = [g](long long x) { return (x + g - 1) / g * g; };
  const long long by_s = (n + S - 1) / S, by_t = (T + per - 1) / per;
  long long lo = up(by_s > by_t ? by_s : by_t);
  if (lo < g) lo = g;
  // count(c) <= T / c + nz, so c >= T / (per - nz) is enough; a chunk of n
  // (one split per sequence, nz <= per items) always is.
  const long long whole = up(n > 1 ? n : 1);
  long long hi = per > nz ? up((T + (per - nz) - 1) / (per - nz)) : whole;
  if (hi > whole) hi = whole;
  if (hi <= lo || count((int)lo) <= per) return (int)lo;  // the usual case: the lower bound fits
  lo += g;
  while (lo < hi) {
    const long long mid = lo + (hi - lo) / g / 2 * g;
    if (count((int)mid) <= per) hi = mid;
    else lo = mid + g;
  }
  return (int)lo;
}

__device__ __forceinline__ int seq_len_of(const kvf_args &a, int b) {
  return min(max(__ldg(a.seq_lens + b), 0), a.n);
}

// Lane i's first length, seq_lens[i] (0 past the batch): kept in a register
// so that batches of up to 32 sequences read seq_lens once.
__device__ __forceinline__ int first_len(const kvf_args &a) {
  const int lane = threadIdx.x & 31;
  return lane < a.B ? seq_len_of(a, lane) : 0;
}

// The balanced chunk; every lane of the calling warp takes part and gets it.
__device__ __forceinline__ int balanced_chunk(const kvf_args &a, int len0, int units, int grid, int gran) {
  const int lane = threadIdx.x & 31;
  long long T = 0;
  int nz = 0;
  for (int b0 = 0; b0 < a.B; b0 += 32) {
    const int len = b0 == 0 ? len0 : b0 + lane < a.B ? seq_len_of(a, b0 + lane) : 0;
    T += len;
    nz += len > 0;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) T += __shfl_xor_sync(0xffffffffu, T, off);
  nz = __reduce_add_sync(0xffffffffu, (unsigned)nz);
  return balance_search(T, nz, a.n, a.splits, grid / units, gran, [&](int c) {
    unsigned cnt = 0;
    for (int b0 = 0; b0 < a.B; b0 += 32) {
      const int len = b0 == 0 ? len0 : b0 + lane < a.B ? seq_len_of(a, b0 + lane) : 0;
      cnt += (unsigned)((len + c - 1) / c);
    }
    return (long long)__reduce_add_sync(0xffffffffu, cnt);
  });
}

// (sequence b, split) of work item j (items ordered by sequence, then split)
// under chunk c; b = -1 when j is past the last item. Warp-collective.
__device__ __forceinline__ void balanced_item(const kvf_args &a, int len0, int c, int j, int &b, int &split) {
  const int lane = threadIdx.x & 31;
  b = -1;
  split = 0;
  int carry = 0;
  for (int b0 = 0; b0 < a.B; b0 += 32) {
    const int len = b0 == 0 ? len0 : b0 + lane < a.B ? seq_len_of(a, b0 + lane) : 0;
    const int s = (len + c - 1) / c;
    int incl = s;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += y;
    }
    incl += carry;
    const unsigned hit = __ballot_sync(0xffffffffu, incl > j);
    if (hit) {
      const int f = __ffs(hit) - 1;
      const int excl = __shfl_sync(0xffffffffu, incl - s, f);
      b = b0 + f;
      split = j - excl;
      return;
    }
    carry = __shfl_sync(0xffffffffu, incl, 31);
  }
}

// Integer codes go to the tensor cores centred: int8 code - 128 in [-128, 127],
// int4 code - 8 in [-8, 7], exact in fp16. The dequantised value is then
// x = scale * (code - c) + (zero + c * scale), so the code term and the zero
// term are both small and their sum does not cancel (with raw codes and the
// group minimum as zero point both terms are several times the result).
constexpr float kCentre8 = 128.f, kCentre4 = 8.f;

// int8 codes: 4 bytes -> two f16x2 words of centred codes (fp16 1024 + code,
// minus 1152).
__device__ __forceinline__ uint32_t u8pair(uint32_t r, uint32_t sel) {
  return ptx::hsub2_u32(ptx::prmt(r, 0x64646464u, sel), 0x64806480u);
}
// int4 codes: nibble pairs (bits 0-3, 16-19) / (bits 4-7, 20-23) -> f16x2.
__device__ __forceinline__ uint32_t u4lo(uint32_t x) {
  // (1024 + n) - 1032 = n - 8
  return ptx::hsub2_u32(ptx::lop3_and_or(x, 0x000F000Fu, 0x64006400u), 0x64086408u);
}
__device__ __forceinline__ uint32_t u4hi(uint32_t x) {
  // (1024 + 16 n) / 16 - 72 = n - 8, all exact in fp16.
  return ptx::hfma2_u32(ptx::lop3_and_or(x, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD480D480u);
}

__device__ __forceinline__ void stsm_x2_t(uint32_t addr, uint32_t r0, uint32_t r1) {
  asm volatile("stmatrix.sync.aligned.m8n8.x2.trans.shared.b16 [%0], {%1, %2};" ::"r"(addr),
               "r"(r0), "r"(r1)
               : "memory");
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t &r0, uint32_t &r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

// fp32 -> (hi, lo) fp16 pair packed as one word, hi in bits 0-15.
__device__ __forceinline__ uint32_t split_hi_lo(float x) {
  const __half h = __float2half_rn(x);
  const float r = x - __half2float(h);
  return ptx::pack_f16x2(__half2float(h), r);
}

// Element (column d) of one query row used by a B fragment.
template <int FMT>
__device__ __forceinline__ int q_dim(int ks, int c, int j) {
  // j in 0..3 enumerates b0.lo, b0.hi, b1.lo, b1.hi of k-step ks.
  if (FMT == 0) return 16 * ks + ((j & 2) ? 8 : 0) + 2 * c + (j & 1);
  if (FMT == 1) return 16 * ks + 4 * c + j;
  // int4: two k-steps per 32-column chunk; pairs (0,4) (1,5) | (2,6) (3,7).
  const int ch = ks >> 1, sub = ks & 1;
  const int off = (j & 1) ? 4 : 0;
  const int base = (j & 2) ? 1 : 0;
  return 32 * ch + 8 * c + 2 * sub + base + off;
}

// Output column of row r (0..15) of value d-tile md.
template <int FMT>
__device__ __forceinline__ int v_dim(int md, int r) {
  if (FMT == 0) return 16 * md + r;
  if (FMT == 1) return r < 8 ? 16 * md + 2 * r : 16 * md + 2 * (r - 8) + 1;
  const int ch = md >> 1, pi = md & 1;
  return r < 8 ? 32 * ch + 4 * r + 2 * pi : 32 * ch + 4 * (r - 8) + 2 * pi + 1;
}

// First column of k-step ks (the group it belongs to).
template <int FMT> __host__ __device__ constexpr int k_dim0(int ks) {
  return FMT == 2 ? 32 * (ks >> 1) : 16 * ks;
}
// First column of value d-tile md.
template <int FMT> __host__ __device__ constexpr int v_dim0(int md) {
  return FMT == 2 ? 32 * (md >> 1) : 16 * md;
}

// Row bytes and 16-token m-tiles per stage, fixed per (format, head dim):
// one stage moves about 4 KB of K (and of V) per KV head, in up to four
// independent m-tiles per warp (instruction-level parallelism for the
// consumer's dependent ldmatrix -> MMA -> softmax chain).
__host__ __device__ constexpr int row_bytes(int fmt, int d) {
  return fmt == 0 ? 2 * d : fmt == 1 ? d : d / 2;
}
__host__ __device__ constexpr int stage_mtiles(int fmt, int d) {
  return row_bytes(fmt, d) >= 256 ? 1 : row_bytes(fmt, d) >= 128 ? 2 : 4;
}

// Waits on an mbarrier phase, giving up when the block has been told to abort
// or the wait runs out of time; the result is uniform across the warp.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag) {
  bool ok = true;
  if (!ptx::mbar_try_wait(bar, parity)) {
    const uint64_t t0 = ptx::globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
      if (ptx::mbar_try_wait(bar, parity)) break;
      if ((it & 63u) == 0) {
        if (*abort_flag || ptx::globaltimer_ns() - t0 > 2000000000ull) {
          ok = false;
          break;
        }
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// warp_wait for one thread (an MMA issuer): mbarrier.try_wait sleeps in
// hardware between checks, so the waiting thread takes few issue slots.
__device__ __forceinline__ bool thread_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0 && (*abort_flag || ptx::globaltimer_ns() - t0 > 2000000000ull)) return false;
  }
}

// Two fp32 operations in one instruction (sm_100a packed f32x2), each lane
// rounded to nearest exactly as fmaf / __fmul_rn / __fsub_rn round.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

// 2^x by the hardware approximation (flush-to-zero; 2^-inf = 0). Its error,
// a few ulp, lies far inside the output tolerance; it replaces exp2f in the
// softmax of both decode kernels.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^e as a float, for e in [-126, 127].
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// Exponent that brings a positive magnitude m into [2^(top-1), 2^top):
// top - ceil(log2(m)), or `top` when m is zero.
__device__ __forceinline__ int norm_exp(float m, int top) {
  const uint32_t u = __float_as_uint(m);
  if (m <= 0.f) return top;
  int e = (int)((u >> 23) & 0xFFu) - 127;
  if (u & 0x7FFFFFu) e += 1;
  return top - e;
}

// Log-sum-exp merge of the split partials (runtime/kvf_kernels.cuh:288-306):
//   M = max_s m_s,  L = sum_s l_s 2^(m_s - M),  out = sum_s o_s 2^(m_s - M) / L
// (splits with m_s = -inf contribute nothing; L = 0 gives 0). One block per
// (query head, sequence, 32 output columns); warp w takes splits w, w+8, ...,
// issuing all of its loads before using any (one L2 round trip for up to
// 256 splits), and the warps' partial (M, L, O) are combined the same way.
constexpr int kMergeWarps = 8;
constexpr int kMergeUnroll = 32;
// The decode kernel's tail merge loads 20 splits per warp and round (fewer
// live registers beside the decode's own); for at most kMergeWarps x 20 =
// 160 splits both take one round, in which the extra slots of the wider one
// add exact zeros, so the two give the same bits.
constexpr int kTailMergeUnroll = 20;

// Merged (M, L, O) of one (query head, 32-column slice) over all splits, for
// warp 0 (lane = column); warps 0 .. nw-1 of the caller's block take part (a
// block of kMergeWarps warps, or the consumer warps of a decode block, which
// then synchronise on named barrier 1).
struct MergeSmem {
  float m[kMergeWarps], l[kMergeWarps];
  float o[kMergeWarps][32];
};

template <int U = kMergeUnroll>
__device__ __forceinline__ void merge_splits(const kvf_args &a, int d, long long head, int col, bool colok,
                                             MergeSmem &sm, float &Mt, float &Lt, float &Ot, int nw = kMergeWarps,
                                             int nsp = -1) {
  // kMergeWarps partial states, each over splits w, w + kMergeWarps, ...;
  // warp i of the nw warps computes states i, i + nw, ..., so the arithmetic
  // (and the result, bit for bit) is the same for any nw. Only split slots
  // [0, nsp) hold partials (all S of them when nsp < 0).
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int S = a.splits;
  const int NS = nsp < 0 ? S : min(nsp, S);
  const float *ml = a.part_ml + head * S * 2;
  const float *po = a.part_o + head * (long long)S * d;

  for (int vw = warp; vw < kMergeWarps; vw += nw) {
    float M = -INFINITY, L = 0.f, O = 0.f;
    for (int base = vw; base < NS; base += kMergeWarps * U) {
      float ms[U], ls[U], os[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int sp = base + k * kMergeWarps;
        const bool v = sp < NS;
        ms[k] = v ? __ldcg(ml + 2 * sp) : -INFINITY;
        ls[k] = v ? __ldcg(ml + 2 * sp + 1) : 0.f;
        os[k] = (v && colok) ? __ldcg(po + (long long)sp * d + col) : 0.f;
      }
      float mx = M;
#pragma unroll
      for (int k = 0; k < U; ++k) mx = fmaxf(mx, ms[k]);
      if (mx == -INFINITY) continue;
      const float r = exp2f(M - mx);  // 0 when M is -inf
      L *= r;
      O *= r;
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const float w = ms[k] == -INFINITY ? 0.f : exp2f(ms[k] - mx);
        L = fmaf(ls[k], w, L);
        O = fmaf(os[k], w, O);
      }
      M = mx;
    }
    if (lane == 0) {
      sm.m[vw] = M;
      sm.l[vw] = L;
    }
    sm.o[vw][lane] = O;
  }
  if (nw == kMergeWarps) __syncthreads();
  else asm volatile("bar.sync 1, %0;" ::"r"(nw * 32) : "memory");
  Mt = -INFINITY;
  Lt = 0.f;
  Ot = 0.f;
  if (warp == 0) {
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) Mt = fmaxf(Mt, sm.m[w]);
    if (Mt != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kMergeWarps; ++w) {
        const float wt = sm.m[w] == -INFINITY ? 0.f : exp2f(sm.m[w] - Mt);
        Lt = fmaf(sm.l[w], wt, Lt);
        Ot = fmaf(sm.o[w][lane], wt, Ot);
      }
    }
  }
}

// LEAN: a contiguous cache without the in-launch split merge; the block-table
// and grid-barrier code is compiled out (it costs the contiguous launches
// 1-3 % even when it does not run).
template <int FMT, int D, int GPR, int NT, bool LEAN>
// At most 4 KV heads (4 consumer warps + 1 producer warp) per block, two
// blocks per SM.
__global__ void __launch_bounds__(160, 2)
decode_kernel(const kvf_args a, const Plan p, const __grid_constant__ CUtensorMap tmk,
              const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmkm,
              const __grid_constant__ CUtensorMap tmvm) {
  constexpr int RB = row_bytes(FMT, D);
  constexpr int NCH = RB / 16;          // 16-byte chunks per row
  constexpr int KSTEPS = D / 16;        // MMA k-steps per row
  constexpr int MD = D / 16;            // value d-tiles
  constexpr int MT = stage_mtiles(FMT, D);
  constexpr int TB = 16 * MT;           // tokens per stage
  constexpr int NG = GPR > 0 ? GPR : 1; // accumulator groups
  constexpr int BOXX = RB < 128 ? RB : 128;
  constexpr int CPB = BOXX / 16;        // chunks per box row
  constexpr uint32_t SWZ = BOXX == 128 ? 0x70u : BOXX == 64 ? 0x30u : 0x10u;
  static_assert(D == 64 || D == 128, "head dimension");
  static_assert(NT == 1 || NT == 2, "column tiles");
  static_assert(NCH % 2 == 0 && CPB % 2 == 0, "ldmatrix.x4 covers two chunks of one box");

  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t bar_full = sbase + p.off_bars;
  const uint32_t bar_empty = bar_full + 8u * p.stages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Work item: (sequence b, head group hgi, split), split fastest so that a
  // sequence's blocks run together; balanced, head group fastest over the
  // items of balanced_item, and a block past the last item (idle) reads and
  // writes nothing.
  // The epilogue reads a balanced item back from s_item (sequence or -1,
  // split, chunk) rather than holding it in registers through the stages.
  __shared__ int s_item[3];
  int split, hgi, b, chunk = p.chunk;
  bool idle = false;
  if (!LEAN && p.bal_gran > 0) {
    const int len0 = first_len(a);
    chunk = balanced_chunk(a, len0, p.hg, gridDim.x, p.bal_gran);
    hgi = blockIdx.x % p.hg;
    balanced_item(a, len0, chunk, blockIdx.x / p.hg, b, split);
    idle = b < 0;
    if (threadIdx.x == 0) {
      s_item[0] = b;
      s_item[1] = split;
      s_item[2] = chunk;
    }
    if (idle) b = 0;
  } else {
    split = blockIdx.x % p.splits;
    const int rest = blockIdx.x / p.splits;
    hgi = rest % p.hg;
    b = rest / p.hg;
  }
  int nb = a.n;
  if (a.seq_lens) nb = min(max(a.seq_lens[b], 0), a.n);
  const int t0 = idle ? 0 : split * chunk;
  const int t1 = idle ? 0 : min(nb, t0 + chunk);
  const int tbs = p.tbox_shift;

  __shared__ int s_abort;
  __shared__ int s_tag[8];  // first token of the stage in each ring slot, -1 = no more work
  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < p.stages; ++s) {
      ptx::mbar_init(bar_full + 8u * s, (GPR > 0 && !p.meta_tma) ? 33u : 1u);
      ptx::mbar_init(bar_empty + 8u * s, (uint32_t)p.hh);
    }
    ptx::fence_barrier_init();
  }
  __syncthreads();
  // The merge kernel (if any) may be scheduled now; it waits for this grid.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == p.hh) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      ptx::prefetch_tmap(&tmk);
      ptx::prefetch_tmap(&tmv);
      if (GPR > 0 && p.meta_tma) {
        ptx::prefetch_tmap(&tmkm);
        ptx::prefetch_tmap(&tmvm);
      }
    }
    const uint64_t pol = ptx::policy_evict_first();
    const int bmask = (1 << p.bt_shift) - 1;
    const int nblk_valid = p.paged ? min(a.max_blocks, (nb + bmask) >> p.bt_shift) : 0;
    const long long tab0 = (long long)b * a.max_blocks;
    const int h0 = hgi * p.hh;
    const uint32_t *kmeta = reinterpret_cast<const uint32_t *>(a.k_meta);
    const uint32_t *vmeta = reinterpret_cast<const uint32_t *>(a.v_meta);
    // Block-table window: pages of blocks [win, win + 96) in three registers
    // per lane, loaded one window ahead of use, so a stage's page lookup is
    // two shuffles and never waits for memory.
    int win = 0;
    int pg_cur = 0, pg_nxt = 0, pg_nn = 0;
    if constexpr (!LEAN) {
      if (p.paged) {
        win = t0 >> p.bt_shift;
        if (win + lane < nblk_valid) pg_cur = __ldg(a.block_table + tab0 + win + lane);
        if (win + 32 + lane < nblk_valid) pg_nxt = __ldg(a.block_table + tab0 + win + 32 + lane);
        if (win + 64 + lane < nblk_valid) pg_nn = __ldg(a.block_table + tab0 + win + 64 + lane);
      }
    }
    // Stages to load: the chunk [t0, t1) in TB steps; each ring slot is tagged
    // with its first token, and a slot tagged -1 tells the consumers to stop.
    int tt = t0;
    bool ok = true;
    bool ended = false;
    int issued = 0;
    int s = 0;
    uint32_t phase = 0;
    for (int i = 0;; ++i) {
      const int cur = tt < t1 ? tt : -1;  // first token of stage i, -1 when done
      if (i >= p.stages && !warp_wait(bar_empty + 8u * s, phase ^ 1u, &s_abort)) {
        ok = false;
        break;
      }
      if (cur < 0) {
        // No more work: a slot tagged -1, completed by plain arrivals.
        if (lane == 0) *reinterpret_cast<volatile int *>(&s_tag[s]) = -1;
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar_full + 8u * s);
        if (GPR > 0 && !p.meta_tma) ptx::mbar_arrive(bar_full + 8u * s);  // 32 more: the cp.async share
        ended = true;
        break;
      }
      if (lane == 0) *reinterpret_cast<volatile int *>(&s_tag[s]) = cur;
      const uint32_t sk = sbase + s * p.stage_bytes;
      const uint32_t sv = sk + p.kv_bytes;
      // Page of TMA box `lane` of this stage (paged): box j lies in block
      // blk0 + j (several boxes per stage only when a page is shorter than
      // a stage, one box per page).
      int lanepage = 0;
      if (!LEAN && p.paged) {
        const int blk0 = cur >> p.bt_shift;
        while (blk0 >= win + 32) {
          win += 32;
          pg_cur = pg_nxt;
          pg_nxt = pg_nn;
          pg_nn = (win + 64 + lane < nblk_valid) ? __ldg(a.block_table + tab0 + win + 64 + lane) : 0;
        }
        const int idx = blk0 - win + (lane < p.npg ? lane : 0);  // < 32 + 4
        const int from_cur = __shfl_sync(0xffffffffu, pg_cur, idx & 31);
        const int from_nxt = __shfl_sync(0xffffffffu, pg_nxt, idx & 31);
        lanepage = idx < 32 ? from_cur : from_nxt;
      }
      if (lane == 0) ptx::mbar_arrive_expect_tx(bar_full + 8u * s, p.tx_bytes);
#pragma unroll
      for (int j = 0; j < MT; ++j) {
        if (j < p.npg) {
          const int pg = __shfl_sync(0xffffffffu, lanepage, j);
          if (lane == 0) {
            const int tok = cur + (j << tbs);
            const int c1 = p.paged ? (tok & bmask) : tok;
            const int c3 = p.paged ? pg : b;
#pragma unroll
            for (int xb = 0; xb < RB / BOXX; ++xb) {
              const uint32_t off = (uint32_t)(xb * p.npg + j) * p.box_bytes;
              ptx::tma_g2s_4d(sk + off, &tmk, xb * BOXX, c1, h0, c3, bar_full + 8u * s, pol);
              ptx::tma_g2s_4d(sv + off, &tmv, xb * BOXX, c1, h0, c3, bar_full + 8u * s, pol);
            }
          }
        }
      }
      if (GPR > 0 && p.meta_tma) {
        // Metadata of the stage by TMA, counted in tx_bytes: token-major
        // (group words of the block's heads, token, sequence) lands as
        // [token][head][group]; head-major (token x group words, head,
        // sequence) as [head][token][group].
        if (lane == 0) {
          const uint32_t smk = sv + p.kv_bytes;
          const uint32_t smv = smk + p.meta_bytes;
          const int x = p.tm ? h0 * GPR : cur * GPR;
          const int y = p.tm ? cur : h0;
          ptx::tma_g2s_3d(smk, &tmkm, x, y, b, bar_full + 8u * s, pol);
          ptx::tma_g2s_3d(smv, &tmvm, x, y, b, bar_full + 8u * s, pol);
        }
      } else if (GPR > 0) {
        // Metadata rows (hh heads x TB tokens) of the stage's tokens.
        const uint32_t smk = sv + p.kv_bytes;
        const uint32_t smv = smk + p.meta_bytes;
        const int rows = p.hh * TB;
        for (int r0 = 0; r0 < rows; r0 += 32) {
          const int r = r0 + lane;
          const int hl = r / TB, t = r - hl * TB;
          const int tok = cur + t;
          const int pg = p.paged ? __shfl_sync(0xffffffffu, lanepage, (t >> tbs) & 31) : 0;
          if (r >= rows || tok >= nb) continue;
          const int h = h0 + hl;
          long long row;
          if (p.paged) {
            const int tl = tok & bmask;
            const long long base = ((long long)pg * a.Hkv) << p.bt_shift;
            row = p.tm ? base + (long long)tl * a.Hkv + h : base + ((long long)h << p.bt_shift) + tl;
          } else {
            row = p.tm ? ((long long)b * a.n + tok) * a.Hkv + h : ((long long)b * a.Hkv + h) * a.n + tok;
          }
          const uint32_t dst = (uint32_t)(r * GPR * 4);
          if (GPR == 1) {
            ptx::cp_async_4(smk + dst, kmeta + row);
            ptx::cp_async_4(smv + dst, vmeta + row);
          } else if (GPR == 2) {
            ptx::cp_async_8(smk + dst, kmeta + row * 2);
            ptx::cp_async_8(smv + dst, vmeta + row * 2);
          } else {
            ptx::cp_async_16(smk + dst, kmeta + row * 4);
            ptx::cp_async_16(smv + dst, vmeta + row * 4);
          }
        }
        ptx::cp_async_arrive(bar_full + 8u * s);
      }
      issued = i + 1;
      tt += TB;
      if (++s == p.stages) {
        s = 0;
        phase ^= 1u;
      }
      if (s_abort) break;
    }
    if (!ok) {
      if (lane == 0) atomicOr(&g_kvfb_error, KVFB_ERR_TIMEOUT);
      s_abort = 1;
    }
    // Never leave with copies in flight: wait (bounded) for the last stages.
    // The end-of-work slot reused the barrier of stage issued - stages, which
    // was consumed (and so landed) before the slot was reused; its old parity
    // must not be waited on again.
    for (int i = max(0, issued - p.stages + (ended ? 1 : 0)); i < issued; ++i) {
      const int s = i % p.stages;
      volatile int never = 0;
      if (!warp_wait(bar_full + 8u * s, (i / p.stages) & 1, &never) && lane == 0)
        atomicOr(&g_kvfb_error, KVFB_ERR_TIMEOUT);
    }
    return;
  }

  // -------------------------------------------------------------- consumer
  const int h = hgi * p.hh + warp;  // KV head of this warp
  const int g8 = lane >> 2;         // fragment row group
  const int c4 = lane & 3;          // thread in group
  // When launched as the programmatic dependent of a kernel that stages the
  // queries (kvf_b200_decode_from_host), the K/V stream above has already
  // started; the queries are read only once that kernel has completed. A
  // launch without that dependency returns here at once.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float *qbase = a.q + ((long long)b * a.H + (long long)h * p.gq) * D;
  constexpr float CENTRE = FMT == 1 ? kCentre8 : kCentre4;

  // Q^T fragments: column n = g8 holds (query head nt*4 + g8/2, part g8&1).
  // Each head is pre-scaled by a power of two 2^eq (max |q| in [2^13, 2^14))
  // before the fp16 hi/lo split, so the lo part never drops into fp16's
  // subnormal range; scores are scaled back by 2^-eq in fp32.
  uint32_t qf[KSTEPS][NT][2];
  float qinv[NT];     // 2^-eq of head nt*4 + c4
  float qs[NG][NT];   // group sums of the scaled query of head nt*4 + c4
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int hq = nt * 4 + (g8 >> 1);
    const bool live = hq < p.gq;
    const float *qh = qbase + (long long)(live ? hq : 0) * D;
    float x[KSTEPS][4];
    float mx = 0.f;
    float gs[NG];
#pragma unroll
    for (int gi = 0; gi < NG; ++gi) gs[gi] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float v = live ? __ldg(qh + q_dim<FMT>(ks, c4, j)) * a.scale_log2 : 0.f;
        x[ks][j] = v;
        mx = fmaxf(mx, fabsf(v));
        gs[(k_dim0<FMT>(ks) * NG) / D] += v;
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const int eq = min(norm_exp(mx, 14), 100);
    const float fq = exp2i(max(eq, -126));
#pragma unroll
    for (int gi = 0; gi < NG; ++gi) {
      gs[gi] += __shfl_xor_sync(0xffffffffu, gs[gi], 1);
      gs[gi] += __shfl_xor_sync(0xffffffffu, gs[gi], 2);
    }
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float xs = x[ks][j] * fq;
        const float hi = __half2float(__float2half_rn(xs));
        v[j] = (g8 & 1) ? xs - hi : hi;
      }
      qf[ks][nt][0] = ptx::pack_f16x2(v[0], v[1]);
      qf[ks][nt][1] = ptx::pack_f16x2(v[2], v[3]);
    }
    // Row group 2*c4 holds head nt*4 + c4.
    qinv[nt] = __shfl_sync(0xffffffffu, exp2i(max(-eq, -126)), 8 * c4);
#pragma unroll
    for (int gi = 0; gi < NG; ++gi) qs[gi][nt] = __shfl_sync(0xffffffffu, gs[gi], 8 * c4);
  }

  float o[MD][NT][4];
#pragma unroll
  for (int md = 0; md < MD; ++md)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[md][nt][e] = 0.f;
  float m_run[NT], l_run[NT], z_run[NG][NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt] = -INFINITY;
    l_run[nt] = 0.f;
#pragma unroll
    for (int gi = 0; gi < NG; ++gi) z_run[gi][nt] = 0.f;
  }
  // O accumulates sum_t (p_t * scale_t * 2^ev) * code_t; ev is re-chosen per
  // stage (exactly, by powers of two) so the fp16 hi/lo parts keep full
  // precision.
  int ev_run = 14;

  const uint32_t pscr = sbase + p.off_pscr + warp * p.pscr_warp;
  const int st_row = lane & 7, st_mat = (lane >> 3) & 1;
  // ldmatrix lane roles: token row within a 16-token m-tile, chunk within a
  // pair. Offsets of this lane's rows inside a stage, per m-tile and per
  // chunk pair, computed once (rows start at multiples of 8, so the swizzle
  // term depends on the lane only).
  uint32_t off_mt[MT], off_xi[NCH / 2];
  {
    const int ld_tok = (lane & 7) + ((lane >> 3) & 1) * 8;
    const int ld_chp = lane >> 4;
    const uint32_t xorv = BOXX == 128 ? (uint32_t)((ld_tok & 7) << 4)
                          : BOXX == 64 ? (uint32_t)(((ld_tok & 7) >> 1) << 4)
                                       : (uint32_t)(((ld_tok & 7) >> 2) << 4);
    const uint32_t tbox_mask = (1u << tbs) - 1u;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const uint32_t t16 = (uint32_t)mt * 16u;
      off_mt[mt] = (t16 >> tbs) * p.box_bytes + (uint32_t)((warp << tbs) + ld_tok) * BOXX +
                   (t16 & tbox_mask) * BOXX;
    }
#pragma unroll
    for (int xi = 0; xi < NCH / 2; ++xi) {
      const int ch = 2 * xi + ld_chp;
      off_xi[xi] = (uint32_t)((2 * xi) / CPB) * (uint32_t)p.npg * p.box_bytes +
                   (((uint32_t)(ch % CPB) * 16u) ^ xorv);
    }
  }
  // Metadata of (this warp's head, token t): words at meta + warp*hs + t*ts
  // (hs = TB*GPR*4, ts = GPR*4 when [head][token][group]; hs = GPR*4,
  // ts = hh*GPR*4 when [token][head][group]).
  const uint32_t meta_ts = p.meta_ts;
  const uint32_t meta_lane = (uint32_t)warp * p.meta_hs + (uint32_t)g8 * meta_ts;

  int s = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (;;) {
    if (!warp_wait(bar_full + 8u * s, phase, &s_abort)) {
      ok = false;
      break;
    }
    const int tt = *reinterpret_cast<volatile int *>(&s_tag[s]);  // first token of the stage
    if (tt < 0) break;                                               // no more work
    const int vt = min(TB, nb - tt);  // valid tokens in this stage
    const uint32_t sk = sbase + s * p.stage_bytes;
    const uint32_t sv = sk + p.kv_bytes;
    const uint32_t smk = sv + p.kv_bytes;
    const uint32_t smv = smk + p.meta_bytes;

    // One stage; FULL (every token valid) drops the masking.
    auto stage = [&](auto full_tag) {
      constexpr bool FULL = decltype(full_tag)::value;
      const int nmt = FULL ? MT : (vt + 15) >> 4;

      // f16 rows past the sequence end may hold any bits (NaN); zero this
      // warp's V rows there so 0 * NaN never reaches the accumulators.
      if (!FULL && FMT == 0 && vt < nmt * 16) {
        const uint32_t tbox_mask = (1u << tbs) - 1u;
        for (int t = vt; t < nmt * 16; ++t) {
          const uint32_t pg = (uint32_t)(t >> tbs), tl = (uint32_t)t & tbox_mask;
          for (int ch = lane; ch < NCH; ch += 32) {
            const uint32_t xb = (uint32_t)(ch / CPB);
            const uint32_t lin = (((uint32_t)warp << tbs) + tl) * BOXX + (uint32_t)(ch % CPB) * 16u;
            const uint32_t ad = sv + (xb * (uint32_t)p.npg + pg) * p.box_bytes + (lin ^ ((lin >> 3) & SWZ));
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(ad), "r"(0) : "memory");
          }
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
      }

      // Metadata words of this thread's tokens (rows g8, g8 + 8 of m-tile mt).
      auto load_meta = [&](uint32_t base, int mt, int rr, uint32_t (&w)[NG]) {
        const uint32_t ad = base + meta_lane + (uint32_t)(mt * 16 + rr * 8) * meta_ts;
        if (GPR == 1) {
          asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w[0]) : "r"(ad));
        } else if (GPR == 2) {
          asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(w[0]), "=r"(w[NG > 1 ? 1 : 0]) : "r"(ad));
        } else if (GPR == 4) {
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(w[0]), "=r"(w[NG > 1 ? 1 : 0]), "=r"(w[NG > 2 ? 2 : 0]), "=r"(w[NG > 3 ? 3 : 0])
                       : "r"(ad));
        }
      };

      // ---- scores of every 16-token m-tile of the stage
      float sc[MT][NT][2];
      float tmax[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) tmax[nt] = -INFINITY;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) sc[mt][nt][0] = sc[mt][nt][1] = -INFINITY;
        if (FULL || mt < nmt) {
          float acc[NG][NT][4];
#pragma unroll
          for (int gi = 0; gi < NG; ++gi)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[gi][nt][e] = 0.f;
#pragma unroll
          for (int xi = 0; xi < NCH / 2; ++xi) {
            uint32_t r0, r1, r2, r3;
            ptx::ldsm_x4(sk + off_mt[mt] + off_xi[xi], r0, r1, r2, r3);
            if (FMT == 0) {
              const uint32_t af[4] = {r0, r1, r2, r3};
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) ptx::mma_f16(acc[0][nt], af, qf[xi][nt][0], qf[xi][nt][1]);
            } else if (FMT == 1) {
#pragma unroll
              for (int hf = 0; hf < 2; ++hf) {
                const uint32_t ra = hf ? r2 : r0, rb = hf ? r3 : r1;
                const uint32_t af[4] = {u8pair(ra, 0x4140u), u8pair(rb, 0x4140u), u8pair(ra, 0x4342u),
                                        u8pair(rb, 0x4342u)};
                const int ks = 2 * xi + hf;
                const int gi = (k_dim0<FMT>(ks) * NG) / D;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) ptx::mma_f16(acc[gi][nt], af, qf[ks][nt][0], qf[ks][nt][1]);
              }
            } else {
#pragma unroll
              for (int hf = 0; hf < 2; ++hf) {
                const uint32_t ra = hf ? r2 : r0, rb = hf ? r3 : r1;
                const uint32_t ra8 = ra >> 8, rb8 = rb >> 8;
                const uint32_t afa[4] = {u4lo(ra), u4lo(rb), u4hi(ra), u4hi(rb)};
                const uint32_t afb[4] = {u4lo(ra8), u4lo(rb8), u4hi(ra8), u4hi(rb8)};
                const int ksa = 4 * xi + 2 * hf;
                const int gi = (k_dim0<FMT>(ksa) * NG) / D;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                  ptx::mma_f16(acc[gi][nt], afa, qf[ksa][nt][0], qf[ksa][nt][1]);
                  ptx::mma_f16(acc[gi][nt], afb, qf[ksa + 1][nt][0], qf[ksa + 1][nt][1]);
                }
              }
            }
          }
          // Combine parts and groups for rows g8 and g8 + 8 of the m-tile, the
          // two rows as one packed f32x2 pair:
          // s = 2^-eq * sum_g scale_g * dot_g + sum_g zero'_g * qsum_g.
          float2 ksc[NG], kz[NG];
          if (GPR > 0) {
            uint32_t w0[NG], w1[NG];
            load_meta(smk, mt, 0, w0);
            load_meta(smk, mt, 1, w1);
#pragma unroll
            for (int gi = 0; gi < NG; ++gi) {
              const float2 f0 = meta_sz(w0[gi]), f1 = meta_sz(w1[gi]);
              ksc[gi] = make_float2(f0.x, f1.x);
              kz[gi] = fma2(make_float2(CENTRE, CENTRE), ksc[gi], make_float2(f0.y, f1.y));
            }
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            float2 v;
            if (GPR > 0) {
              float2 dsum = make_float2(0.f, 0.f), zq = make_float2(0.f, 0.f);
#pragma unroll
              for (int gi = 0; gi < NG; ++gi) {
                const float2 d = add2(make_float2(acc[gi][nt][0], acc[gi][nt][2]),
                                      make_float2(acc[gi][nt][1], acc[gi][nt][3]));
                dsum = fma2(ksc[gi], d, dsum);
                zq = fma2(kz[gi], make_float2(qs[gi][nt], qs[gi][nt]), zq);
              }
              v = fma2(dsum, make_float2(qinv[nt], qinv[nt]), zq);
            } else {
              v = mul2(add2(make_float2(acc[0][nt][0], acc[0][nt][2]), make_float2(acc[0][nt][1], acc[0][nt][3])),
                       make_float2(qinv[nt], qinv[nt]));
            }
            if (!FULL && mt * 16 + g8 >= vt) v.x = -INFINITY;
            if (!FULL && mt * 16 + g8 + 8 >= vt) v.y = -INFINITY;
            sc[mt][nt][0] = v.x;
            sc[mt][nt][1] = v.y;
            tmax[nt] = fmaxf(tmax[nt], fmaxf(v.x, v.y));
          }
        }
      }

      // ---- value pre-scale for this stage: 2^ev * max(V scale) in [2^13, 2^14)
      int ev = 14;
      if (GPR > 0) {
        uint32_t vbits = 0;  // fp16 bits of positive scales order like the values
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int rr = 0; rr < 2; ++rr)
            if (FULL || mt * 16 + g8 + rr * 8 < vt) {
              uint32_t w[NG];
              load_meta(smv, mt, rr, w);
#pragma unroll
              for (int gi = 0; gi < NG; ++gi) vbits = max(vbits, w[gi] & 0x7FFFu);
            }
        vbits = max(vbits, __shfl_xor_sync(0xffffffffu, vbits, 4));
        vbits = max(vbits, __shfl_xor_sync(0xffffffffu, vbits, 8));
        vbits = max(vbits, __shfl_xor_sync(0xffffffffu, vbits, 16));
        ev = max(min(norm_exp(__half2float(__ushort_as_half((unsigned short)vbits)), 14), 100), -100);
      }
      const float fv = exp2i(max(min(ev, 127), -126));
      const float fratio = exp2i(max(min(ev - ev_run, 127), -126));
      ev_run = ev;

      // ---- online softmax, one rescale per stage (O is rescaled when the
      // stage's value product is folded in below)
      float ao[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float mx = tmax[nt];
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run[nt], mx);
        const float alpha = ex2_approx(m_run[nt] - m_new);  // 0 on the first stage
        m_run[nt] = m_new;
        l_run[nt] *= alpha;
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) z_run[gi][nt] *= alpha;
        ao[nt] = alpha * fratio;
      }

      // ---- probabilities: P'^T fragments of every m-tile, per value group,
      // through a stmatrix.trans/ldmatrix round trip (C layout of S^T -> B
      // layout of P^T)
      uint32_t pb[MT][NG][NT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        if (FULL || mt < nmt) {
          // Probabilities of this thread's two tokens (rows g8, g8 + 8) as a
          // packed pair; 0 for masked rows.
          float2 pr[NT];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const float2 d = sub2(make_float2(sc[mt][nt][0], sc[mt][nt][1]), make_float2(m_run[nt], m_run[nt]));
            pr[nt] = make_float2(ex2_approx(d.x), ex2_approx(d.y));
            l_run[nt] += pr[nt].x;
            l_run[nt] += pr[nt].y;
          }
          // Value scale (times 2^ev) and centred zero of the two tokens; 0 for
          // masked rows so stale bits never leak in.
          float2 vsc[NG], vz[NG];
          const bool valid0 = FULL || mt * 16 + g8 < vt, valid1 = FULL || mt * 16 + g8 + 8 < vt;
          if (GPR > 0) {
            uint32_t w0[NG], w1[NG];
            load_meta(smv, mt, 0, w0);
            load_meta(smv, mt, 1, w1);
#pragma unroll
            for (int gi = 0; gi < NG; ++gi) {
              const float2 f0 = meta_sz(w0[gi]), f1 = meta_sz(w1[gi]);
              const float2 sv = make_float2(f0.x, f1.x);
              vsc[gi] = mul2(sv, make_float2(fv, fv));
              vz[gi] = fma2(make_float2(CENTRE, CENTRE), sv, make_float2(f0.y, f1.y));
              if (!valid0) vsc[gi].x = vz[gi].x = 0.f;
              if (!valid1) vsc[gi].y = vz[gi].y = 0.f;
            }
          } else {
            vsc[0] = make_float2(valid0 ? fv : 0.f, valid1 ? fv : 0.f);
            vz[0] = make_float2(0.f, 0.f);
          }
#pragma unroll
          for (int gi = 0; gi < NG; ++gi)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const float2 pp = mul2(pr[nt], vsc[gi]);
              const uint32_t w0 = split_hi_lo(pp.x);
              const uint32_t w1 = split_hi_lo(pp.y);
              if (GPR > 0) {
                z_run[gi][nt] = fmaf(pr[nt].x, vz[gi].x, z_run[gi][nt]);
                z_run[gi][nt] = fmaf(pr[nt].y, vz[gi].y, z_run[gi][nt]);
              }
              stsm_x2_t(pscr + (uint32_t)((gi * NT + nt) * 384 + st_row * 48 + st_mat * 16), w0, w1);
            }
          __syncwarp();
#pragma unroll
          for (int gi = 0; gi < NG; ++gi)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              ldsm_x2(pscr + (uint32_t)((gi * NT + nt) * 384 + st_row * 48 + st_mat * 16),
                      pb[mt][gi][nt][0], pb[mt][gi][nt][1]);
          __syncwarp();
        }
      }

      // ---- value product. Each chunk pair's d-tiles accumulate this stage's
      // tokens in fresh tensor-core accumulators (a handful of MMA additions),
      // then fold into the running fp32 O with one round-to-nearest FFMA that
      // also applies the stage's rescale: tensor-core accumulation truncates,
      // so long runs of MMA additions into one register would bias the sum.
      constexpr int DT = FMT == 0 ? 1 : FMT == 1 ? 2 : 4;  // d-tiles per chunk pair
#pragma unroll
      for (int xi = 0; xi < NCH / 2; ++xi) {
        float tacc[DT][NT][4];
#pragma unroll
        for (int k = 0; k < DT; ++k)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) tacc[k][nt][e] = 0.f;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          if (FULL || mt < nmt) {
            uint32_t r0, r1, r2, r3;
            ptx::ldsm_x4_t(sv + off_mt[mt] + off_xi[xi], r0, r1, r2, r3);
            if (FMT == 0) {
              const uint32_t af[4] = {r0, r2, r1, r3};
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) ptx::mma_f16(tacc[0][nt], af, pb[mt][0][nt][0], pb[mt][0][nt][1]);
            } else if (FMT == 1) {
#pragma unroll
              for (int hf = 0; hf < 2; ++hf) {
                const uint32_t ra = hf ? r2 : r0, rb = hf ? r3 : r1;
                const uint32_t af[4] = {u8pair(ra, 0x4240u), u8pair(ra, 0x4341u), u8pair(rb, 0x4240u),
                                        u8pair(rb, 0x4341u)};
                const int gi = (v_dim0<FMT>(2 * xi + hf) * NG) / D;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                  ptx::mma_f16(tacc[hf][nt], af, pb[mt][gi][nt][0], pb[mt][gi][nt][1]);
              }
            } else {
#pragma unroll
              for (int hf = 0; hf < 2; ++hf) {
                const uint32_t ra = hf ? r2 : r0, rb = hf ? r3 : r1;
                const uint32_t ra8 = ra >> 8, rb8 = rb >> 8;
                const int ch = 2 * xi + hf;
                const int gi = (v_dim0<FMT>(2 * ch) * NG) / D;
                const uint32_t af0[4] = {u4lo(ra), u4hi(ra), u4lo(rb), u4hi(rb)};
                const uint32_t af1[4] = {u4lo(ra8), u4hi(ra8), u4lo(rb8), u4hi(rb8)};
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                  ptx::mma_f16(tacc[2 * hf][nt], af0, pb[mt][gi][nt][0], pb[mt][gi][nt][1]);
                  ptx::mma_f16(tacc[2 * hf + 1][nt], af1, pb[mt][gi][nt][0], pb[mt][gi][nt][1]);
                }
              }
            }
          }
        }
#pragma unroll
        for (int k = 0; k < DT; ++k)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
              const float2 r = fma2(make_float2(o[DT * xi + k][nt][e], o[DT * xi + k][nt][e + 1]),
                                    make_float2(ao[nt], ao[nt]), make_float2(tacc[k][nt][e], tacc[k][nt][e + 1]));
              o[DT * xi + k][nt][e] = r.x;
              o[DT * xi + k][nt][e + 1] = r.y;
            }
      }
    };
    if (vt == TB)
      stage(std::true_type{});
    else
      stage(std::false_type{});

    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(bar_empty + 8u * s);
    if (++s == p.stages) {
      s = 0;
      phase ^= 1u;
    }
  }

  // ---------------------------------------------------------------- epilogue
  if (!ok) {
    if (lane == 0) atomicOr(&g_kvfb_error, KVFB_ERR_TIMEOUT);
    s_abort = 1;
  }
  // With an in-launch merge every consumer warp takes part in the barriers
  // below; a warp that gave up only skips its writes.
  if (!ok && !p.tail_merge && (LEAN || !p.coop_merge)) return;
  // Reduce the per-thread sums over the 8 row groups.
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l_run[nt] += __shfl_xor_sync(0xffffffffu, l_run[nt], off);
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) z_run[gi][nt] += __shfl_xor_sync(0xffffffffu, z_run[gi][nt], off);
    }
  }
  const float finv = exp2i(max(min(-ev_run, 127), -126));
  int eb, esplit;
  if (!LEAN && p.bal_gran > 0) {
    eb = s_item[0];
    esplit = s_item[1];
  } else {
    esplit = blockIdx.x % p.splits;
    eb = blockIdx.x / p.splits / p.hg;
  }
  // O = (O_hi + O_lo) * 2^-ev + zero term; one query head per (n-tile, c4).
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int hq = nt * 4 + c4;
    if (ok && eb >= 0 && hq < p.gq) {
      const long long head = (long long)eb * a.H + (long long)h * p.gq + hq;
      const float L = l_run[nt];
      const float inv = L > 0.f ? 1.f / L : 0.f;
      float *dst;
      if (p.final_out) {
        dst = a.out + head * D;
        if (g8 == 0 && a.lse) a.lse[head] = L > 0.f ? m_run[nt] + log2f(L) : -INFINITY;
      } else {
        dst = a.part_o + (head * p.splits + esplit) * D;
        if (g8 == 0) {
          a.part_ml[(head * p.splits + esplit) * 2] = m_run[nt];
          a.part_ml[(head * p.splits + esplit) * 2 + 1] = L;
        }
      }
#pragma unroll
      for (int md = 0; md < MD; ++md) {
        const int gi = (v_dim0<FMT>(md) * NG) / D;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int d = v_dim<FMT>(md, g8 + rr * 8);
          float val = (o[md][nt][2 * rr] + o[md][nt][2 * rr + 1]) * finv;
          if (GPR > 0) val += z_run[gi][nt];
          dst[d] = p.final_out ? val * inv : val;
        }
      }
    }
  }

  if constexpr (!LEAN) {
  if (p.coop_merge) {
    // ---- the split merge inside this launch. A cooperative launch keeps
    // every block resident, so the blocks may wait for each other: a grid
    // barrier (arrival count, bounded wait; the last block to leave resets
    // both counters to zero for the next launch), then block i merges the
    // (query head, 32-column) slices i, i + grid, ... as merge_kernel does.
    const int nthr = p.hh * 32;
    __threadfence();
    asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    __shared__ int s_pass;
    if (threadIdx.x == 0) {
      unsigned *arrived = a.split_sem + 1, *departed = a.split_sem + 3;
      const unsigned nblk = gridDim.x;
      atomicAdd(arrived, 1u);
      const uint64_t tw = ptx::globaltimer_ns();
      int pass = 1;
      for (;;) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(arrived) : "memory");
        if (v >= nblk) break;
        if (ptx::globaltimer_ns() - tw > 2000000000ull) {
          pass = 0;
          break;
        }
        __nanosleep(64);
      }
      if (!pass) atomicOr(&g_kvfb_error, KVFB_ERR_TIMEOUT);
      if (atomicAdd(departed, 1u) == nblk - 1) {
        *reinterpret_cast<volatile unsigned *>(arrived) = 0u;
        *reinterpret_cast<volatile unsigned *>(departed) = 0u;
      }
      s_pass = pass && !s_abort;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    if (!s_pass) return;
    __threadfence();
    __shared__ MergeSmem msm;
    const int nz = (D + 31) / 32;
    const long long items = (long long)a.B * a.H * nz;
    for (long long it = blockIdx.x; it < items; it += gridDim.x) {
      const long long head = it / nz;
      const int zc = (int)(it - head * nz);
      const int col = zc * 32 + lane;
      const bool colok = col < D;
      float Mt, Lt, Ot;
      const int nsp = p.bal_gran > 0 ? (seq_len_of(a, (int)(head / a.H)) + s_item[2] - 1) / s_item[2] : p.splits;
      merge_splits(a, D, head, col, colok, msm, Mt, Lt, Ot, p.hh, nsp);
      if (warp == 0) {
        if (colok) a.out[head * D + col] = Lt > 0.f ? Ot / Lt : 0.f;
        if (lane == 0 && zc == 0 && a.lse) a.lse[head] = Lt > 0.f ? Mt + log2f(Lt) : -INFINITY;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");  // msm is reused by the next slice
    }
  }
  }

  if (p.tail_merge) {
    // ---- the split merge by the last finishers of this (sequence, head
    // group). Each block takes a ticket when its partials are written; the
    // holders of the last K tickets (K = min(splits, merge slices of the
    // group)) wait, bounded, until every split's ticket is taken, then merge
    // the group's (query head, 32-column) slices part, part + K, ... as
    // merge_kernel does. The host enables this only when the grid fits in one
    // wave, so the blocks a merger waits for are running or about to. The
    // last merger out resets both counters for the next launch.
    const int nthr = p.hh * 32;
    const int S = p.splits;
    const int nz = (D + 31) / 32;
    const int items = p.hh * p.gq * nz;
    const int K = min(S, items);
    unsigned *cnt = a.split_sem + 2 * ((long long)b * p.hg + hgi);
    __threadfence();
    asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    __shared__ int s_part;
    if (threadIdx.x == 0) {
      int part = -1;
      if (!s_abort) {
        const int t = (int)atomicAdd(cnt, 1u);
        if (t >= S - K) {
          const uint64_t tw = ptx::globaltimer_ns();
          for (;;) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
            if ((int)v >= S) {
              part = t - (S - K);
              break;
            }
            if (ptx::globaltimer_ns() - tw > 2000000000ull) {
              atomicOr(&g_kvfb_error, KVFB_ERR_TIMEOUT);
              break;
            }
            __nanosleep(32);
          }
        }
      }
      s_part = part;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    const int part = s_part;
    if (part >= 0) {
      __threadfence();
      // Scratch in the stage ring, idle now: every stage was consumed and the
      // producer has seen all of its copies land.
      MergeSmem &tsm = *reinterpret_cast<MergeSmem *>(smem);
      for (int it = part; it < items; it += K) {
        const int hq = it / nz;  // query head of the group: KV head hgi*hh + hq / gq
        const int zc = it - hq * nz;
        const long long head = (long long)b * a.H + (long long)hgi * p.hh * p.gq + hq;
        const int col = zc * 32 + lane;
        const bool colok = col < D;
        float Mt, Lt, Ot;
        merge_splits<kTailMergeUnroll>(a, D, head, col, colok, tsm, Mt, Lt, Ot, p.hh, S);
        if (warp == 0) {
          if (colok) a.out[head * D + col] = Lt > 0.f ? Ot / Lt : 0.f;
          if (lane == 0 && zc == 0 && a.lse) a.lse[head] = Lt > 0.f ? Mt + log2f(Lt) : -INFINITY;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");  // tsm is reused by the next slice
      }
      if (threadIdx.x == 0 && atomicAdd(cnt + 1, 1u) == (unsigned)(K - 1)) {
        *reinterpret_cast<volatile unsigned *>(cnt) = 0u;
        *reinterpret_cast<volatile unsigned *>(cnt + 1) = 0u;
      }
    }
  }
}

// bal: the decode's (units, grid, gran) when its splits were token-balanced
// (units = 0 otherwise); each sequence's split count then follows from
// seq_lens and the chunk, which the block works out before waiting for the
// decode grid.
struct MergeBalance {
  int units, grid, gran;
};

// A persistent grid (at most one wave): block i merges the (query head,
// 32-column) slices i, i + grid, ... in the order of the reference's
// (head, sequence, slice) grid, so that a block pays its start-up once.
__global__ void __launch_bounds__(kMergeWarps * 32, 2) merge_kernel(const kvf_args a, int d, const MergeBalance bal) {
  int c = 0;
  if (bal.units > 0) c = balanced_chunk(a, first_len(a), bal.units, bal.grid, bal.gran);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ MergeSmem sm;
  const int lane = threadIdx.x & 31;
  const int nz = (d + 31) / 32;
  const long long items = (long long)a.B * a.H * nz;
  for (long long it = blockIdx.x; it < items; it += gridDim.x) {
    const long long head = it / nz;  // sequence * H + query head
    const int zc = (int)(it - head * nz);
    const int col = zc * 32 + lane;
    const bool colok = col < d;
    const int nsp = c > 0 ? (seq_len_of(a, (int)(head / a.H)) + c - 1) / c : -1;
    float Mt, Lt, Ot;
    merge_splits(a, d, head, col, colok, sm, Mt, Lt, Ot, kMergeWarps, nsp);
    if ((threadIdx.x >> 5) == 0) {
      if (colok) a.out[head * d + col] = Lt > 0.f ? Ot / Lt : 0.f;
      if (lane == 0 && zc == 0 && a.lse) a.lse[head] = Lt > 0.f ? Mt + log2f(Lt) : -INFINITY;
    }
    __syncthreads();  // sm is reused by the next slice
  }
}

// The split merge of one rank of a split-KV decode across GPUs, fused with
// the cross-GPU exchange (see kvf_b200_decode_exchange): this rank's
// (output slice, lse) goes into every rank's gather cells, and once all P
// parts of the slice carry this step's epoch (bounded wait) they are combined
// into out. A cell is one 64-bit store (value bits, epoch), single-copy
// atomic over NVLink, so a reader that sees the epoch sees the value: the
// step needs no system-scope fence and no counter.
__global__ void __launch_bounds__(kMergeWarps * 32) merge_exchange_kernel(const kvf_args a, int d,
                                                                         const kvf_exchange x) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ MergeSmem sm;
  const long long head = (long long)blockIdx.y * a.H + blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int col = blockIdx.z * 32 + lane;
  const bool colok = col < d;
  float Mt, Lt, Ot;
  merge_splits(a, d, head, col, colok, sm, Mt, Lt, Ot);
  if ((threadIdx.x >> 5) != 0) return;
  const long long rows = (long long)a.B * a.H;
  const long long stride = d + 1;                 // cells per (rank, row): output then lse
  const long long par = (long long)(x.epoch & 1) * x.P;
  const unsigned long long tag = (unsigned long long)(unsigned)x.epoch << 32;
  const float val = Lt > 0.f ? Ot / Lt : 0.f;
  const float lse = Lt > 0.f ? Mt + log2f(Lt) : -INFINITY;
  const unsigned long long cv = tag | __float_as_uint(val), cl = tag | __float_as_uint(lse);
  for (int p = 0; p < x.P; ++p) {
    unsigned long long *g = x.peer_gather[p] + ((par + x.rank) * rows + head) * stride;
    if (colok) asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(g + col), "l"(cv) : "memory");
    if (lane == 0) asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(g + d), "l"(cl) : "memory");
  }
  // Each lane waits for its own column of every part, lane 0 also for the
  // lse cells; then the warp agrees.
  const unsigned long long *base = x.gather + par * rows * stride + head * stride;
  const uint64_t limit = (uint64_t)x.timeout_ms * 1000000ull;
  const uint64_t t0 = ptx::globaltimer_ns();
  // Waits (bounded) for the cell at c to carry this step's epoch; its value.
  auto wait_cell = [&](const unsigned long long *c, int &ok) -> float {
    for (uint32_t it = 0; ok; ++it) {
      unsigned long long v;
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(c) : "memory");
      if ((v >> 32) == (unsigned long long)(unsigned)x.epoch) return __uint_as_float((unsigned)v);
      if ((it & 15u) == 15u && ptx::globaltimer_ns() - t0 > limit) ok = 0;
    }
    return 0.f;
  };
  float lp[8], op[8];
  int ok = 1;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    lp[p] = -INFINITY;
    op[p] = 0.f;
    if (p < x.P) {
      const unsigned long long *cp = base + p * rows * stride;
      if (colok) op[p] = wait_cell(cp + col, ok);
      if (lane == 0) lp[p] = wait_cell(cp + d, ok);
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && lane == 0) atomicOr(&g_kvfb_error, KVFB_ERR_EXCHANGE);
  float M = -INFINITY;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    lp[p] = __shfl_sync(0xffffffffu, lp[p], 0);
    if (p < x.P) M = fmaxf(M, lp[p]);
  }
  float W = 0.f, O = 0.f;
  if (M != -INFINITY && ok) {
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      if (p >= x.P) break;
      const float w = lp[p] == -INFINITY ? 0.f : exp2f(lp[p] - M);
      W += w;
      if (colok && w > 0.f) O = fmaf(w, op[p], O);
    }
  }
  if (colok) a.out[head * d + col] = W > 0.f ? O / W : 0.f;
  if (lane == 0 && blockIdx.z == 0 && a.lse) a.lse[head] = W > 0.f ? M + log2f(W) : -INFINITY;
}

// Combination of attention states over disjoint token ranges (no reference
// counterpart): one block per output row, one thread per column; P is small
// (one part per GPU).
__global__ void merge_states_kernel(const float *o, const float *lse, int P, int rows, int d, long long o_stride,
                                    long long lse_stride, float *out, float *lse_out) {
  const int r = blockIdx.x;
  const int c = threadIdx.x;
  float M = -INFINITY;
  for (int k = 0; k < P; ++k) M = fmaxf(M, __ldg(lse + k * lse_stride + r));
  float W = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int k = 0; k < P; ++k) {
      const float lk = __ldg(lse + k * lse_stride + r);
      const float w = lk == -INFINITY ? 0.f : exp2f(lk - M);
      W += w;
      if (c < d && w > 0.f) O = fmaf(w, __ldg(o + k * o_stride + (long long)r * d + c), O);
    }
  }
  if (c < d) out[(long long)r * d + c] = W > 0.f ? O / W : 0.f;
  if (c == 0 && lse_out) lse_out[r] = W > 0.f ? M + log2f(W) : -INFINITY;
}

} // namespace kvfb
