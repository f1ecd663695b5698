// quantize.cu - KV cache quantization on the GPU, bit-exact with the
// reference's host quantizer kvf::quantize (runtime/kvf_host.h:72-120).
//
// Per group of `group` channels of one row (asymmetric, unsigned codes):
//   lo, hi   = min, max of the group (first-wins comparisons, as std::min/max)
//   zero_h   = fp16(lo), round to nearest even
//   scale    = (hi - lo) / levels   (levels 255 or 15; 1 when <= 0)
//   scale_h  = fp16(scale)
//   code     = clamp(round_half_away((x - zero) / sc), 0, levels)
// with zero, sc the fp16 values widened back to fp32, every operation in
// IEEE single precision with round-to-nearest (no contraction). The metadata
// word is scale_h | zero_h << 16. int4 puts column c in byte c/2, odd columns
// in the high nibble. f16 rows are the fp16 (round to nearest even) values.
#include "kvforge_b200.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace kvfb {

// Rows of an append that fell outside the cache (bit 0; read and cleared by
// take_append_errors, reported as bit 2 of kvf_b200_device_errors).
__device__ unsigned g_kvfb_append_error;

namespace {

__device__ __forceinline__ uint16_t h_bits(__half h) { return __half_as_ushort(h); }

// Destination row of source row r: the same row (kvf_b200_quantize), or the
// physical cache row of an appended token (kvf_b200_append); < 0 = not written.
struct RowsSame {
  __device__ __forceinline__ long long operator()(long long r) const { return r; }
};

// Source rows are the new tokens in logical order [B][Hkv][t_new]; token j of
// sequence b is token pos[b] + j of the cache, at the physical row of
// runtime/kvf_kernels.cuh:51-64 (kvf_host.h:124-135).
struct RowsAppend {
  const int *pos;
  const int *table;
  int Hkv, t_new, n, head_major, paged, bt_shift, max_blocks;
  __device__ __forceinline__ long long operator()(long long r) const {
    const long long bh = r / t_new;
    const int j = (int)(r - bh * t_new);
    const int h = (int)(bh % Hkv);
    const int b = (int)(bh / Hkv);
    const int p0 = pos[b];
    const long long t = (long long)p0 + j;
    if (p0 < 0 || t >= n) return -1;
    if (!paged) return head_major ? ((long long)b * Hkv + h) * n + t : ((long long)b * n + t) * Hkv + h;
    const int blk = (int)(t >> bt_shift);
    if (blk >= max_blocks) return -1;
    const long long bt = 1ll << bt_shift, tl = t & (bt - 1);
    const long long base = (long long)table[(long long)b * max_blocks + blk] * Hkv * bt;
    return head_major ? base + (long long)h * bt + tl : base + tl * Hkv + h;
  }
};

// clamp(lround((x - zero) / sc), 0, levels) with the host's behaviour at the
// edges: lround of a NaN, an infinity or a value of magnitude >= 2^63 yields
// LONG_MIN on x86-64, which the clamp turns into 0 (this happens when a group
// exceeds the fp16 range and zero becomes -inf).
__device__ __forceinline__ int code(float x, float zero, float sc, int levels) {
  const float t = __fdiv_rn(__fsub_rn(x, zero), sc);
  if (!(t < 9.223372036854775808e18f && t > -9.223372036854775808e18f)) return 0;
  const long long q = llroundf(t);
  return q < 0 ? 0 : (q > levels ? levels : (int)q);
}

// One thread per (row, group).
template <int FMT, class Dst>
__global__ void quantize_groups(const float *__restrict__ x, long long rows, int d, int group,
                                uint8_t *__restrict__ data, uint32_t *__restrict__ meta, const Dst dst) {
  const int gpr = d / group;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * gpr) return;
  const long long r = idx / gpr;
  const int gi = (int)(idx - r * gpr);
  const long long dr = dst(r);
  if (dr < 0) {
    if (gi == 0) atomicOr(&g_kvfb_append_error, 1u);
    return;
  }
  const float *xg = x + r * d + (long long)gi * group;
  float lo = xg[0], hi = xg[0];
  for (int i = 1; i < group; ++i) {
    const float v = xg[i];
    lo = (v < lo) ? v : lo;
    hi = (hi < v) ? v : hi;
  }
  const int levels = FMT == KVF_FMT_INT8 ? 255 : 15;
  const __half zero_h = __float2half_rn(lo);
  float scale = __fdiv_rn(__fsub_rn(hi, lo), (float)levels);
  if (scale <= 0.f) scale = 1.f;
  const __half scale_h = __float2half_rn(scale);
  const float zero = __half2float(zero_h);
  const float sc = __half2float(scale_h);
  meta[dr * gpr + gi] = (uint32_t)h_bits(scale_h) | ((uint32_t)h_bits(zero_h) << 16);
  if (FMT == KVF_FMT_INT8) {
    uint8_t *out = data + dr * d + (long long)gi * group;
    for (int i = 0; i < group; ++i) out[i] = (uint8_t)code(xg[i], zero, sc, levels);
  } else {
    uint8_t *out = data + dr * (d / 2) + (long long)gi * (group / 2);
    for (int i = 0; i < group; i += 2)
      out[i / 2] = (uint8_t)(code(xg[i], zero, sc, levels) | (code(xg[i + 1], zero, sc, levels) << 4));
  }
}

// Coalesced form of quantize_groups for groups of 4..D channels (powers of
// two): lane li of a row holds channels 4 li .. 4 li + 3 (one 16-byte load),
// a group spans group / 4 lanes, and its min and max are combined across them
// with shuffles. The combination keeps the host loop's results bit for bit:
// a lane that does not hold the group's first element folds its values into
// +inf / -inf (NaNs never replace a running value in the host loop, which
// starts from the first element), the first lane starts from that element
// (a NaN there stays NaN), and two adjacent ranges combine as the loop
// would have met them, earlier range first (ties keep the earlier value).
template <int FMT, int D, class Dst>
__global__ void __launch_bounds__(256) quantize_rows(const float *__restrict__ x, long long rows, int group,
                                                     uint8_t *__restrict__ data, uint32_t *__restrict__ meta,
                                                     const Dst dst) {
  constexpr int LPR = D / 4;     // lanes per row
  constexpr int RPW = 32 / LPR;  // rows per warp
  const int lane = threadIdx.x & 31;
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long r = wid * RPW + lane / LPR;
  const int li = lane % LPR;
  const bool valid = r < rows;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (valid) v = __ldcs(reinterpret_cast<const float4 *>(x + r * D) + li);
  const int lpg = group >> 2;  // lanes per group
  const bool first = (li & (lpg - 1)) == 0;
  float lo = first ? v.x : INFINITY, hi = first ? v.x : -INFINITY;
  const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (k == 0 && first) continue;
    lo = (e[k] < lo) ? e[k] : lo;
    hi = (hi < e[k]) ? e[k] : hi;
  }
  for (int off = 1; off < lpg; off <<= 1) {
    const float plo = __shfl_xor_sync(0xffffffffu, lo, off);
    const float phi = __shfl_xor_sync(0xffffffffu, hi, off);
    const bool earlier = (li & off) == 0;
    const float alo = earlier ? lo : plo, blo = earlier ? plo : lo;
    const float ahi = earlier ? hi : phi, bhi = earlier ? phi : hi;
    lo = (blo < alo) ? blo : alo;
    hi = (ahi < bhi) ? bhi : ahi;
  }
  const int levels = FMT == KVF_FMT_INT8 ? 255 : 15;
  const __half zero_h = __float2half_rn(lo);
  float scale = __fdiv_rn(__fsub_rn(hi, lo), (float)levels);
  if (scale <= 0.f) scale = 1.f;
  const __half scale_h = __float2half_rn(scale);
  const float zero = __half2float(zero_h);
  const float sc = __half2float(scale_h);
  if (!valid) return;
  const long long dr = dst(r);
  if (dr < 0) {
    if (li == 0) atomicOr(&g_kvfb_append_error, 1u);
    return;
  }
  const int gpr = D / group;
  if (first) meta[dr * gpr + li / lpg] = (uint32_t)h_bits(scale_h) | ((uint32_t)h_bits(zero_h) << 16);
  uint32_t c[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) c[k] = (uint32_t)code(e[k], zero, sc, levels);
  if (FMT == KVF_FMT_INT8) {
    reinterpret_cast<uint32_t *>(data + dr * D)[li] = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
  } else {
    reinterpret_cast<uint16_t *>(data + dr * (D / 2))[li] = (uint16_t)(c[0] | (c[1] << 4) | (c[2] << 8) | (c[3] << 12));
  }
}

// code() without the division in the common case. With a = x - zero (fp32,
// as the host computes it) and r = 1/sc rounded to nearest, t' = a * r is
// within 3 * 2^-24 |t| of the host's t = a / sc (both correctly rounded), so
// for |t'| < 1024 the two differ by less than 2^-12. When t' is further than
// that from every half-integer, t lies strictly between the same two
// half-integers as t', and round-half-away(t) = rint(t'); otherwise (and for
// |t'| >= 1024, NaN or infinities, including sc = 0) the exact code() decides.
__device__ __forceinline__ int code_fast(float x, float zero, float sc, float rsc, int levels) {
  const float a = __fsub_rn(x, zero);
  const float t = __fmul_rn(a, rsc);
  if (fabsf(t) < 1024.f) {
    const float q = rintf(t);
    if (fabsf(__fsub_rn(t, q)) < 0.5f - 0x1p-12f) {
      const int qi = (int)q;
      return qi < 0 ? 0 : (qi > levels ? levels : qi);
    }
  }
  return code(x, zero, sc, levels);
}

// quantize_rows with eight channels per lane (two 16-byte loads in flight,
// one combining round fewer) and division-free codes, for groups of 8..D
// channels (powers of two). Same bit-exact rules as quantize_rows.
template <int FMT, int D, class Dst>
__global__ void __launch_bounds__(256) quantize_rows8(const float *__restrict__ x, long long rows, int group,
                                                      uint8_t *__restrict__ data, uint32_t *__restrict__ meta,
                                                      const Dst dst) {
  constexpr int LPR = D / 8;     // lanes per row
  constexpr int RPW = 32 / LPR;  // rows per warp
  const int lane = threadIdx.x & 31;
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long r = wid * RPW + lane / LPR;
  const int li = lane % LPR;
  const bool valid = r < rows;
  float e[8];
  {
    float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
    if (valid) {
      const float4 *src = reinterpret_cast<const float4 *>(x + r * D) + 2 * li;
      v0 = __ldcs(src);
      v1 = __ldcs(src + 1);
    }
    e[0] = v0.x; e[1] = v0.y; e[2] = v0.z; e[3] = v0.w;
    e[4] = v1.x; e[5] = v1.y; e[6] = v1.z; e[7] = v1.w;
  }
  const int lpg = group >> 3;  // lanes per group
  const bool first = (li & (lpg - 1)) == 0;
  float lo = first ? e[0] : INFINITY, hi = first ? e[0] : -INFINITY;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (k == 0 && first) continue;
    lo = (e[k] < lo) ? e[k] : lo;
    hi = (hi < e[k]) ? e[k] : hi;
  }
  for (int off = 1; off < lpg; off <<= 1) {
    const float plo = __shfl_xor_sync(0xffffffffu, lo, off);
    const float phi = __shfl_xor_sync(0xffffffffu, hi, off);
    const bool earlier = (li & off) == 0;
    const float alo = earlier ? lo : plo, blo = earlier ? plo : lo;
    const float ahi = earlier ? hi : phi, bhi = earlier ? phi : hi;
    lo = (blo < alo) ? blo : alo;
    hi = (ahi < bhi) ? bhi : ahi;
  }
  const int levels = FMT == KVF_FMT_INT8 ? 255 : 15;
  const __half zero_h = __float2half_rn(lo);
  float scale = __fdiv_rn(__fsub_rn(hi, lo), (float)levels);
  if (scale <= 0.f) scale = 1.f;
  const __half scale_h = __float2half_rn(scale);
  const float zero = __half2float(zero_h);
  const float sc = __half2float(scale_h);
  const float rsc = __frcp_rn(sc);
  if (!valid) return;
  const long long dr = dst(r);
  if (dr < 0) {
    if (li == 0) atomicOr(&g_kvfb_append_error, 1u);
    return;
  }
  const int gpr = D / group;
  if (first) meta[dr * gpr + li / lpg] = (uint32_t)h_bits(scale_h) | ((uint32_t)h_bits(zero_h) << 16);
  uint32_t c[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) c[k] = (uint32_t)code_fast(e[k], zero, sc, rsc, levels);
  if (FMT == KVF_FMT_INT8) {
    const uint2 w = make_uint2(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24),
                               c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24));
    reinterpret_cast<uint2 *>(data + dr * D)[li] = w;
  } else {
    reinterpret_cast<uint32_t *>(data + dr * (D / 2))[li] =
        c[0] | (c[1] << 4) | (c[2] << 8) | (c[3] << 12) | (c[4] << 16) | (c[5] << 20) | (c[6] << 24) | (c[7] << 28);
  }
}

template <class Dst>
__global__ void to_f16(const float *__restrict__ x, long long count, int d, __half *__restrict__ out, const Dst dst) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const long long r = i / d;
  const long long dr = dst(r);
  if (dr < 0) {
    if (i == r * d) atomicOr(&g_kvfb_append_error, 1u);
    return;
  }
  out[dr * d + (i - r * d)] = __float2half_rn(x[i]);
}

// Quantizes `rows` rows of d channels from x into the rows dst(r) of data and
// meta, with the fastest kernel the group and the alignment allow.
template <class Dst>
cudaError_t quantize_into(int fmt, int d, int group, const float *x, long long rows, unsigned char *data,
                          void *meta, const Dst &dst, cudaStream_t stream) {
  if (fmt == KVF_FMT_F16) {
    const long long count = rows * d;
    to_f16<<<(unsigned)((count + 255) / 256), 256, 0, stream>>>(x, count, d, reinterpret_cast<__half *>(data),
                                                                dst);
    return cudaGetLastError();
  }
  uint32_t *m = reinterpret_cast<uint32_t *>(meta);
  const bool pow2 = (group & (group - 1)) == 0;
  if (group >= 8 && pow2 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
      (reinterpret_cast<uintptr_t>(data) & (fmt == KVF_FMT_INT8 ? 7u : 3u)) == 0) {
    // Eight channels per lane: 16 lanes per row (D = 128) or 8 (D = 64).
    const long long warps = (rows * d / 8 + 31) / 32;
    const unsigned blocks = (unsigned)((warps + 7) / 8);
    if (fmt == KVF_FMT_INT8 && d == 128)
      quantize_rows8<KVF_FMT_INT8, 128><<<blocks, 256, 0, stream>>>(x, rows, group, data, m, dst);
    else if (fmt == KVF_FMT_INT8)
      quantize_rows8<KVF_FMT_INT8, 64><<<blocks, 256, 0, stream>>>(x, rows, group, data, m, dst);
    else if (d == 128)
      quantize_rows8<KVF_FMT_INT4, 128><<<blocks, 256, 0, stream>>>(x, rows, group, data, m, dst);
    else
      quantize_rows8<KVF_FMT_INT4, 64><<<blocks, 256, 0, stream>>>(x, rows, group, data, m, dst);
    return cudaGetLastError();
  }
  const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(data) & (fmt == KVF_FMT_INT8 ? 3u : 1u)) == 0;
  if (group >= 4 && pow2 && aligned) {
    // One warp per row (D = 128) or two (D = 64), 8 warps per block.
    const long long warps = (rows * d / 4 + 31) / 32;
    const unsigned blocks = (unsigned)((warps + 7) / 8);
    if (fmt == KVF_FMT_INT8 && d == 128)
      quantize_rows<KVF_FMT_INT8, 128><<<blocks, 256, 0, stream>>>(x, rows, group, data, m, dst);
    else if (fmt == KVF_FMT_INT8)
      quantize_rows<KVF_FMT_INT8, 64><<<blocks, 256, 0, stream>>>(x, rows, group, data, m, dst);
    else if (d == 128)
      quantize_rows<KVF_FMT_INT4, 128><<<blocks, 256, 0, stream>>>(x, rows, group, data, m, dst);
    else
      quantize_rows<KVF_FMT_INT4, 64><<<blocks, 256, 0, stream>>>(x, rows, group, data, m, dst);
    return cudaGetLastError();
  }
  const long long threads = rows * (d / group);
  const unsigned blocks = (unsigned)((threads + 127) / 128);
  if (fmt == KVF_FMT_INT8)
    quantize_groups<KVF_FMT_INT8><<<blocks, 128, 0, stream>>>(x, rows, d, group, data, m, dst);
  else
    quantize_groups<KVF_FMT_INT4><<<blocks, 128, 0, stream>>>(x, rows, d, group, data, m, dst);
  return cudaGetLastError();
}

} // namespace

// Nonzero if an append met a row outside the cache since the last call (then
// cleared).
unsigned take_append_errors() {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_kvfb_append_error, sizeof(v)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (v) cudaMemcpyToSymbol(g_kvfb_append_error, &zero, sizeof(zero));
  return v;
}

} // namespace kvfb

// Quantizes `rows` rows of d fp32 channels (device memory, logical row order)
// into `data` (rows * row_bytes) and, for int8/int4, `meta` (rows * d/group
// 32-bit words). Bit-exact with kvf::quantize (runtime/kvf_host.h:72-120).
extern "C" cudaError_t kvf_b200_quantize(int fmt, int d, int group, const float *x, long long rows,
                                         unsigned char *data, void *meta, cudaStream_t stream) {
  if (rows < 0 || (d != 64 && d != 128) || fmt < 0 || fmt > 2) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  if (!x || !data) return cudaErrorInvalidValue;
  if (fmt != KVF_FMT_F16 && (group <= 0 || d % group || !meta || (fmt == KVF_FMT_INT4 && (group & 1))))
    return cudaErrorInvalidValue;
  return kvfb::quantize_into(fmt, d, group, x, rows, data, meta, kvfb::RowsSame{}, stream);
}

// Appends t_new tokens per sequence (see kvforge_b200.h).
extern "C" cudaError_t kvf_b200_append(const kvf_args *a, int fmt, int d, int ord, int paged, const float *k_new,
                                       const float *v_new, int t_new, const int *pos, cudaStream_t stream) {
  if (!a || (d != 64 && d != 128) || fmt < 0 || fmt > 2 || (ord != KVF_ORD_HEAD && ord != KVF_ORD_TOKEN) ||
      (paged != 0 && paged != 1) || t_new < 0 || a->B < 0 || a->Hkv <= 0 || a->n <= 0)
    return cudaErrorInvalidValue;
  if (t_new == 0 || a->B == 0) return cudaSuccess;
  if (!k_new || !v_new || !pos || !a->k || !a->v) return cudaErrorInvalidValue;
  int group = 0;
  if (fmt != KVF_FMT_F16) {
    if (a->group_shift < 0 || a->group_shift > 7 || !a->k_meta || !a->v_meta) return cudaErrorInvalidValue;
    group = 1 << a->group_shift;
    if (d % group || (fmt == KVF_FMT_INT4 && (group & 1))) return cudaErrorInvalidValue;
  }
  if (paged && (!a->block_table || a->max_blocks <= 0 || a->block_shift < 0 || a->block_shift > 20))
    return cudaErrorInvalidValue;
  const kvfb::RowsAppend dst{pos, a->block_table, a->Hkv, t_new, a->n, ord == KVF_ORD_HEAD ? 1 : 0, paged,
                             paged ? a->block_shift : 0, paged ? a->max_blocks : 0};
  const long long rows = (long long)a->B * a->Hkv * t_new;
  cudaError_t e = kvfb::quantize_into(fmt, d, group, k_new, rows, const_cast<unsigned char *>(a->k),
                                      const_cast<void *>(a->k_meta), dst, stream);
  if (e != cudaSuccess) return e;
  return kvfb::quantize_into(fmt, d, group, v_new, rows, const_cast<unsigned char *>(a->v),
                             const_cast<void *>(a->v_meta), dst, stream);
}
