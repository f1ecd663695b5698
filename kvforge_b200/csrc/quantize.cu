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
namespace {

__device__ __forceinline__ uint16_t h_bits(__half h) { return __half_as_ushort(h); }

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
template <int FMT>
__global__ void quantize_groups(const float *__restrict__ x, long long rows, int d, int group,
                                uint8_t *__restrict__ data, uint32_t *__restrict__ meta) {
  const int gpr = d / group;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * gpr) return;
  const long long r = idx / gpr;
  const int gi = (int)(idx - r * gpr);
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
  meta[r * gpr + gi] = (uint32_t)h_bits(scale_h) | ((uint32_t)h_bits(zero_h) << 16);
  if (FMT == KVF_FMT_INT8) {
    uint8_t *out = data + r * d + (long long)gi * group;
    for (int i = 0; i < group; ++i) out[i] = (uint8_t)code(xg[i], zero, sc, levels);
  } else {
    uint8_t *out = data + r * (d / 2) + (long long)gi * (group / 2);
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
template <int FMT, int D>
__global__ void __launch_bounds__(256) quantize_rows(const float *__restrict__ x, long long rows, int group,
                                                     uint8_t *__restrict__ data, uint32_t *__restrict__ meta) {
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
  const int gpr = D / group;
  if (first) meta[r * gpr + li / lpg] = (uint32_t)h_bits(scale_h) | ((uint32_t)h_bits(zero_h) << 16);
  uint32_t c[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) c[k] = (uint32_t)code(e[k], zero, sc, levels);
  if (FMT == KVF_FMT_INT8) {
    reinterpret_cast<uint32_t *>(data + r * D)[li] = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
  } else {
    reinterpret_cast<uint16_t *>(data + r * (D / 2))[li] = (uint16_t)(c[0] | (c[1] << 4) | (c[2] << 8) | (c[3] << 12));
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
template <int FMT, int D>
__global__ void __launch_bounds__(256) quantize_rows8(const float *__restrict__ x, long long rows, int group,
                                                      uint8_t *__restrict__ data, uint32_t *__restrict__ meta) {
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
  const int gpr = D / group;
  if (first) meta[r * gpr + li / lpg] = (uint32_t)h_bits(scale_h) | ((uint32_t)h_bits(zero_h) << 16);
  uint32_t c[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) c[k] = (uint32_t)code_fast(e[k], zero, sc, rsc, levels);
  if (FMT == KVF_FMT_INT8) {
    const uint2 w = make_uint2(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24),
                               c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24));
    reinterpret_cast<uint2 *>(data + r * D)[li] = w;
  } else {
    reinterpret_cast<uint32_t *>(data + r * (D / 2))[li] =
        c[0] | (c[1] << 4) | (c[2] << 8) | (c[3] << 12) | (c[4] << 16) | (c[5] << 20) | (c[6] << 24) | (c[7] << 28);
  }
}

__global__ void to_f16(const float *__restrict__ x, long long count, __half *__restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) out[i] = __float2half_rn(x[i]);
}

} // namespace
} // namespace kvfb

// Quantizes `rows` rows of d fp32 channels (device memory, logical row order)
// into `data` (rows * row_bytes) and, for int8/int4, `meta` (rows * d/group
// 32-bit words). Bit-exact with kvf::quantize (runtime/kvf_host.h:72-120).
extern "C" cudaError_t kvf_b200_quantize(int fmt, int d, int group, const float *x, long long rows,
                                         unsigned char *data, void *meta, cudaStream_t stream) {
  if (rows < 0 || (d != 64 && d != 128) || fmt < 0 || fmt > 2) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  if (!x || !data) return cudaErrorInvalidValue;
  if (fmt == KVF_FMT_F16) {
    const long long count = rows * d;
    kvfb::to_f16<<<(unsigned)((count + 255) / 256), 256, 0, stream>>>(x, count,
                                                                      reinterpret_cast<__half *>(data));
    return cudaGetLastError();
  }
  if (group <= 0 || d % group || !meta) return cudaErrorInvalidValue;
  if ((fmt == KVF_FMT_INT4 && (group & 1))) return cudaErrorInvalidValue;
  const bool pow2 = (group & (group - 1)) == 0;
  if (group >= 8 && pow2 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
      (reinterpret_cast<uintptr_t>(data) & (fmt == KVF_FMT_INT8 ? 7u : 3u)) == 0) {
    // Eight channels per lane: 16 lanes per row (D = 128) or 8 (D = 64).
    const long long warps = (rows * d / 8 + 31) / 32;
    const unsigned blocks = (unsigned)((warps + 7) / 8);
    uint32_t *m = reinterpret_cast<uint32_t *>(meta);
    if (fmt == KVF_FMT_INT8 && d == 128)
      kvfb::quantize_rows8<KVF_FMT_INT8, 128><<<blocks, 256, 0, stream>>>(x, rows, group, data, m);
    else if (fmt == KVF_FMT_INT8)
      kvfb::quantize_rows8<KVF_FMT_INT8, 64><<<blocks, 256, 0, stream>>>(x, rows, group, data, m);
    else if (d == 128)
      kvfb::quantize_rows8<KVF_FMT_INT4, 128><<<blocks, 256, 0, stream>>>(x, rows, group, data, m);
    else
      kvfb::quantize_rows8<KVF_FMT_INT4, 64><<<blocks, 256, 0, stream>>>(x, rows, group, data, m);
    return cudaGetLastError();
  }
  const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(data) & (fmt == KVF_FMT_INT8 ? 3u : 1u)) == 0;
  if (group >= 4 && pow2 && aligned) {
    // One warp per row (D = 128) or two (D = 64), 8 warps per block.
    const long long warps = (rows * d / 4 + 31) / 32;
    const unsigned blocks = (unsigned)((warps + 7) / 8);
    if (fmt == KVF_FMT_INT8 && d == 128)
      kvfb::quantize_rows<KVF_FMT_INT8, 128><<<blocks, 256, 0, stream>>>(x, rows, group, data,
                                                                        reinterpret_cast<uint32_t *>(meta));
    else if (fmt == KVF_FMT_INT8)
      kvfb::quantize_rows<KVF_FMT_INT8, 64><<<blocks, 256, 0, stream>>>(x, rows, group, data,
                                                                       reinterpret_cast<uint32_t *>(meta));
    else if (d == 128)
      kvfb::quantize_rows<KVF_FMT_INT4, 128><<<blocks, 256, 0, stream>>>(x, rows, group, data,
                                                                        reinterpret_cast<uint32_t *>(meta));
    else
      kvfb::quantize_rows<KVF_FMT_INT4, 64><<<blocks, 256, 0, stream>>>(x, rows, group, data,
                                                                       reinterpret_cast<uint32_t *>(meta));
    return cudaGetLastError();
  }
  const long long threads = rows * (d / group);
  const unsigned blocks = (unsigned)((threads + 127) / 128);
  if (fmt == KVF_FMT_INT8)
    kvfb::quantize_groups<KVF_FMT_INT8><<<blocks, 128, 0, stream>>>(
        x, rows, d, group, data, reinterpret_cast<uint32_t *>(meta));
  else
    kvfb::quantize_groups<KVF_FMT_INT4><<<blocks, 128, 0, stream>>>(
        x, rows, d, group, data, reinterpret_cast<uint32_t *>(meta));
  return cudaGetLastError();
}
