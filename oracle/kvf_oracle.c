/* kvf_oracle.c - CPU restatement of KVForge's decode-attention semantics.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the sm_100a kernels:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 * The product (kvforge_b200/) never links or calls it.
 *
 * It restates, in plain C, the reference's host-side oracle in
 * runtime/kvf_host.h:
 *   kvfo_quantize    <- kvf::quantize            runtime/kvf_host.h:72-120
 *   kvfo_row_of      <- kvf::host_row_of         runtime/kvf_host.h:124-135
 *   kvfo_attention   <- kvf::reference_attention runtime/kvf_host.h:202-234
 *   kvfo_rel_l2      <- kvf::rel_l2              runtime/kvf_host.h:236-245
 * and the fp16 conversion the reference gets from cuda_fp16.h (__float2half,
 * round to nearest even; __half2float, exact).
 *
 * Pinning: tests/golden/ holds outputs of the reference's own functions
 * (compiled from the reference sources into oracle/_ref by oracle/build.py)
 * and tests/test_oracle.py checks this file against them bit for bit.
 *
 * Build with -ffp-contract=off so that a*b+c is never fused: the reference's
 * host code is compiled for x86-64 without FMA, and the quantizer's
 * dequantised values depend on that rounding.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { KVFO_F16 = 0, KVFO_INT8 = 1, KVFO_INT4 = 2 };
enum { KVFO_HEAD = 0, KVFO_TOKEN = 1 };

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary32 -> binary16, round to nearest, ties to even. Every NaN
 * becomes 0x7fff whatever its sign and payload, as the reference's host
 * conversion gives (checked against oracle/_ref in tests/test_oracle.py). */
uint16_t kvfo_f2h(float f) {
  const uint32_t x = f2u(f);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return 0x7fffu; /* nan */
  if (ax == 0x7f800000u) return (uint16_t)(sign | 0x7c00u); /* inf */
  const int e = (int)(ax >> 23);
  if (e >= 143) return (uint16_t)(sign | 0x7c00u); /* >= 2^16: overflow */
  if (e >= 113) { /* normal half: biased half exponent e - 112 in [1, 30] */
    const uint32_t mant = ax & 0x7fffffu;
    uint32_t h = ((uint32_t)(e - 112) << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h; /* may carry to inf */
    return (uint16_t)(sign | h);
  }
  if (e == 0) return sign; /* float subnormal: far below half's range */
  { /* half subnormal: value = m * 2^-24 */
    const uint32_t M = (ax & 0x7fffffu) | 0x800000u;
    const int shift = 126 - e; /* >= 14 */
    if (shift > 25) return sign;
    uint32_t q = M >> shift;
    const uint32_t rem = M & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
  }
}

/* binary16 -> binary32, exact; a NaN becomes 0x7fffffff, as the reference's
 * host conversion gives. */
float kvfo_h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  if (e == 0x1f) return m ? u2f(0x7fffffffu) : u2f(sign | 0x7f800000u);
  if (e == 0) {
    if (m == 0) return u2f(sign);
    /* subnormal: normalise */
    int k = 0;
    while (!(m & 0x400u)) { m <<= 1; ++k; }
    m &= 0x3ffu;
    return u2f(sign | ((uint32_t)(113 - k) << 23) | (m << 13));
  }
  return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

void kvfo_f2h_array(const float *x, uint16_t *h, int64_t n) {
  for (int64_t i = 0; i < n; ++i) h[i] = kvfo_f2h(x[i]);
}

void kvfo_h2f_array(const uint16_t *h, float *x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] = kvfo_h2f(h[i]);
}

static float fmin_ref(float a, float b) { return (b < a) ? b : a; } /* std::min */
static float fmax_ref(float a, float b) { return (a < b) ? b : a; } /* std::max */

/* Quantize `rows` logical rows of D channels (runtime/kvf_host.h:72-120).
 *   f16:  data = fp16 bits of X (2 B per element), deq = those values.
 *   int8/int4: per group of `group` channels, asymmetric min/max:
 *     zero_h = half(lo); scale = (hi - lo) / levels, 1 when <= 0;
 *     scale_h = half(scale); q = clamp(lround((x - zero) / sc), 0, levels);
 *     meta word = scale_h | zero_h << 16 (a __half2 with .x = scale);
 *     int4 packs column c into byte c/2, odd columns in the high nibble.
 * `meta` may be NULL for f16. Returns 0, or -1 on bad arguments. */
int kvfo_quantize(int fmt, int D, int group, const float *X, int64_t rows, uint8_t *data,
                  uint32_t *meta, float *deq) {
  if (fmt == KVFO_F16) {
    for (int64_t i = 0; i < rows * D; ++i) {
      const uint16_t h = kvfo_f2h(X[i]);
      memcpy(data + i * 2, &h, 2);
      deq[i] = kvfo_h2f(h);
    }
    return 0;
  }
  if ((fmt != KVFO_INT8 && fmt != KVFO_INT4) || group <= 0 || D % group) return -1;
  const int rb = fmt == KVFO_INT8 ? D : D / 2;
  const int gpr = D / group;
  const int levels = fmt == KVFO_INT8 ? 255 : 15;
  memset(data, 0, (size_t)(rows * rb));
  for (int64_t r = 0; r < rows; ++r) {
    for (int gi = 0; gi < gpr; ++gi) {
      const float *x = X + r * D + (int64_t)gi * group;
      float lo = x[0], hi = x[0];
      for (int i = 1; i < group; ++i) {
        lo = fmin_ref(lo, x[i]);
        hi = fmax_ref(hi, x[i]);
      }
      const uint16_t zero_h = kvfo_f2h(lo);
      float scale = (hi - lo) / (float)levels;
      if (scale <= 0.f) scale = 1.f;
      const uint16_t scale_h = kvfo_f2h(scale);
      const float zero = kvfo_h2f(zero_h);
      const float sc = kvfo_h2f(scale_h);
      meta[r * gpr + gi] = (uint32_t)scale_h | ((uint32_t)zero_h << 16);
      for (int i = 0; i < group; ++i) {
        const int col = gi * group + i;
        const float t = (x[i] - zero) / sc;
        long qv = lroundf(t);
        if (qv < 0) qv = 0;
        if (qv > levels) qv = levels;
        const float qf = (float)qv * sc;
        deq[r * D + col] = qf + zero;
        if (fmt == KVFO_INT8) {
          data[r * rb + col] = (uint8_t)qv;
        } else {
          uint8_t *byte = &data[r * rb + col / 2];
          *byte = (col & 1) ? (uint8_t)((*byte & 0x0F) | (qv << 4))
                            : (uint8_t)((*byte & 0xF0) | qv);
        }
      }
    }
  }
  return 0;
}

/* Physical row of (sequence b, KV head h, token t) (runtime/kvf_host.h:124-135).
 * bt = 0 selects the contiguous layouts. */
int64_t kvfo_row_of(int order, int bt, int Hkv, int n, const int32_t *table, int max_blocks,
                    int b, int h, int t) {
  if (bt == 0)
    return order == KVFO_HEAD ? ((int64_t)b * Hkv + h) * n + t
                              : ((int64_t)b * n + t) * Hkv + h;
  const int blk = t / bt, tl = t % bt;
  const int64_t page = table[(int64_t)b * max_blocks + blk];
  const int64_t base = page * Hkv * bt;
  return order == KVFO_HEAD ? base + (int64_t)h * bt + tl : base + (int64_t)tl * Hkv + h;
}

/* fp64 attention over logical, already dequantised K and V
 * (runtime/kvf_host.h:202-234). Layout: q, out [B][H][D]; K, V
 * [B][Hkv][n_stride][D]. seq_lens (nullable) gives sequence b's length
 * (<= n_stride); NULL means every sequence has n_stride tokens. Per sequence
 * this is the reference function called with Shape{B=1, n=seq_lens[b]}.
 * A sequence of length 0 yields zeros, the reference kernel's L == 0 rule
 * (runtime/kvf_kernels.cuh:275,305). `threads` > 1 splits the (b, h) pairs
 * across OpenMP threads; each pair's arithmetic is unchanged. */
int kvfo_attention(int B, int H, int Hkv, int D, int n_stride, const int32_t *seq_lens,
                   const float *q, const float *K, const float *V, float scale, float *out,
                   int threads) {
  if (B < 0 || H <= 0 || Hkv <= 0 || H % Hkv || D <= 0 || n_stride < 0) return -1;
  const int gq = H / Hkv;
  const int64_t pairs = (int64_t)B * H;
  int err = 0;
#ifdef _OPENMP
  if (threads < 1) threads = 1;
#pragma omp parallel num_threads(threads)
#endif
  {
    double *sc = (double *)malloc(sizeof(double) * (size_t)(n_stride > 0 ? n_stride : 1));
    double *acc = (double *)malloc(sizeof(double) * (size_t)D);
    if (!sc || !acc) {
      err = -2;
    } else {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
      for (int64_t pi = 0; pi < pairs; ++pi) {
        const int b = (int)(pi / H), h = (int)(pi % H);
        const int n = seq_lens ? seq_lens[b] : n_stride;
        const int hk = h / gq;
        const float *qh = q + ((int64_t)b * H + h) * D;
        float *o = out + ((int64_t)b * H + h) * D;
        if (n <= 0) {
          for (int c = 0; c < D; ++c) o[c] = 0.f;
          continue;
        }
        double mx = -1e300;
        for (int t = 0; t < n; ++t) {
          const float *k = K + (((int64_t)b * Hkv + hk) * n_stride + t) * D;
          double d = 0;
          for (int c = 0; c < D; ++c) d += (double)qh[c] * k[c];
          sc[t] = d * scale;
          if (mx < sc[t]) mx = sc[t];
        }
        double sum = 0;
        for (int c = 0; c < D; ++c) acc[c] = 0.0;
        for (int t = 0; t < n; ++t) {
          const double p = exp(sc[t] - mx);
          sum += p;
          const float *v = V + (((int64_t)b * Hkv + hk) * n_stride + t) * D;
          for (int c = 0; c < D; ++c) acc[c] += p * v[c];
        }
        for (int c = 0; c < D; ++c) o[c] = (float)(acc[c] / sum);
      }
    }
    free(sc);
    free(acc);
  }
  return err;
}

/* Relative L2 error (runtime/kvf_host.h:236-245). */
double kvfo_rel_l2(const float *a, const float *ref, int64_t n) {
  double num = 0, den = 0;
  for (int64_t i = 0; i < n; ++i) {
    const double d = (double)a[i] - ref[i];
    num += d * d;
    den += (double)ref[i] * ref[i];
  }
  return den > 0 ? sqrt(num / den) : 0;
}

int kvfo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
