// ref_shim.cu - C entry points onto the reference's OWN host functions.
//
// TEST INFRASTRUCTURE ONLY (the checker, never the product). Compiled by
// oracle/build.py with -I<reference>/runtime so that it includes the
// unmodified reference header runtime/kvf_host.h; the output goes to
// oracle/_ref/libkvf_ref.so, which is never committed. Nothing here touches
// a GPU: the wrapped functions are host code.
//
//   kvfr_quantize   -> kvf::quantize            runtime/kvf_host.h:72-120
//   kvfr_attention  -> kvf::reference_attention runtime/kvf_host.h:202-234
//   kvfr_row_of     -> kvf::host_row_of         runtime/kvf_host.h:124-135
//   kvfr_rel_l2     -> kvf::rel_l2              runtime/kvf_host.h:236-245
//   kvfr_scale_log2 -> kvf::make_args           runtime/kvf_host.h:273-293
//   kvfr_make_data  -> kvf::make_data           runtime/kvf_host.h:51-60
#include "kvf_host.h"

#include <cstring>
#include <vector>

extern "C" {

int kvfr_quantize(int fmt, int D, int group, const float *X, long long rows, unsigned char *data,
                  unsigned *meta, float *deq) {
  kvf::FormatSel f;
  f.fmt = fmt;
  f.group = group;
  const std::vector<float> xv(X, X + rows * D);
  const kvf::Quantized q = kvf::quantize(f, D, xv, rows);
  std::memcpy(data, q.data.data(), q.data.size());
  if (meta && !q.meta.empty()) std::memcpy(meta, q.meta.data(), q.meta.size() * 4);
  std::memcpy(deq, q.deq.data(), q.deq.size() * 4);
  return 0;
}

int kvfr_attention(int B, int H, int Hkv, int D, int n, const float *q, const float *K,
                   const float *V, float scale, float *out) {
  kvf::Shape s;
  s.B = B;
  s.H = H;
  s.Hkv = Hkv;
  s.D = D;
  s.n = n;
  const std::vector<float> qv(q, q + (size_t)B * H * D);
  const std::vector<float> kv(K, K + (size_t)s.rows() * D);
  const std::vector<float> vv(V, V + (size_t)s.rows() * D);
  const std::vector<float> o = kvf::reference_attention(s, qv, kv, vv, scale);
  std::memcpy(out, o.data(), o.size() * 4);
  return 0;
}

long long kvfr_row_of(int order, int paged, int bt, int Hkv, int n, const int *table,
                      int max_blocks, int b, int h, int t) {
  kvf::Shape s;
  s.Hkv = Hkv;
  s.n = n;
  kvf::LayoutSel l;
  l.order = order;
  l.paged = paged != 0;
  l.bt = bt;
  return kvf::host_row_of(s, l, table, max_blocks, b, h, t);
}

double kvfr_rel_l2(const float *a, const float *ref, long long n) {
  const std::vector<float> av(a, a + n), rv(ref, ref + n);
  return kvf::rel_l2(av, rv);
}

float kvfr_scale_log2(int D) {
  kvf::Shape s;
  s.D = D;
  kvf::FormatSel f;
  kvf::LayoutSel l;
  kvf::Cache c;
  kvf::DeviceBuffers d;
  return kvf::make_args(s, f, l, c, d, 1, 4).scale_log2;
}

void kvfr_make_data(int B, int H, int Hkv, int D, int n, unsigned long long seed, float *q,
                    float *K, float *V) {
  kvf::Shape s;
  s.B = B;
  s.H = H;
  s.Hkv = Hkv;
  s.D = D;
  s.n = n;
  std::vector<float> qv, kv, vv;
  kvf::make_data(s, seed, qv, kv, vv);
  std::memcpy(q, qv.data(), qv.size() * 4);
  std::memcpy(K, kv.data(), kv.size() * 4);
  std::memcpy(V, vv.data(), vv.size() * 4);
}

} // extern "C"
