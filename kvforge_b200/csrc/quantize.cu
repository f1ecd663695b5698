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
