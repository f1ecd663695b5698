// registry.cu - variant-id dispatch for the C ABI.
//
// The reference names every kernel instantiation by an id of the form
// fmt_{hm,tm}_{c,p}_g{G}_u{U}_d{D} (src/codegen.cpp:59-65) and looks launchers
// up by that id (runtime/kvf_registry.h:15-29, bench/sweep.cu:180-184). C++
// callers keep using that registry through include/kvf_registry.h; this file
// gives FFI callers the same lookup through kvf_b200_launch_variant. On
// sm_100a an id may carry a kernel-path suffix, "_mma" (mma.sync kernel) or
// "_tc" (tcgen05 kernel, int8 rows of 128 only); the bare id lets the
// launcher choose.
#include "kvforge_b200.h"

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace {

struct VariantId {
  int fmt, ord, paged, g, u, d, path;
};

bool parse_id(const char *id, VariantId &v) {
  if (!id) return false;
  char fmt[8] = {0}, ord[4] = {0}, res[4] = {0};
  int g = 0, u = 0, d = 0, used = 0;
  if (std::sscanf(id, "%7[a-z0-9]_%3[a-z]_%3[a-z]_g%d_u%d_d%d%n", fmt, ord, res, &g, &u, &d, &used) != 6)
    return false;
  v.path = KVF_PATH_AUTO;
  if (!std::strcmp(id + used, "_mma")) v.path = KVF_PATH_MMA;
  else if (!std::strcmp(id + used, "_tc")) v.path = KVF_PATH_TC;
  else if (id[used] != '\0') return false;
  if (!std::strcmp(fmt, "f16")) v.fmt = KVF_FMT_F16;
  else if (!std::strcmp(fmt, "int8")) v.fmt = KVF_FMT_INT8;
  else if (!std::strcmp(fmt, "int4")) v.fmt = KVF_FMT_INT4;
  else return false;
  if (!std::strcmp(ord, "hm")) v.ord = KVF_ORD_HEAD;
  else if (!std::strcmp(ord, "tm")) v.ord = KVF_ORD_TOKEN;
  else return false;
  if (!std::strcmp(res, "c")) v.paged = 0;
  else if (!std::strcmp(res, "p")) v.paged = 1;
  else return false;
  if (g != 1 && g != 2 && g != 4 && g != 8) return false;
  if (u != 2 && u != 4) return false;
  if (d != 64 && d != 128) return false;
  if (v.path == KVF_PATH_TC && (v.fmt != KVF_FMT_INT8 || d != 128)) return false;
  v.g = g;
  v.u = u;
  v.d = d;
  return true;
}

const std::vector<std::string> &all_ids() {
  static const std::vector<std::string> ids = [] {
    std::vector<std::string> out;
    const char *fmts[3] = {"f16", "int8", "int4"};
    for (const char *f : fmts)
      for (const char *o : {"hm", "tm"})
        for (const char *r : {"c", "p"})
          for (int d : {128, 64})
            for (int g : {1, 2, 4, 8})
              for (int u : {2, 4}) {
                char buf[64];
                std::snprintf(buf, sizeof(buf), "%s_%s_%s_g%d_u%d_d%d", f, o, r, g, u, d);
                out.emplace_back(buf);
              }
    // Path-pinned ids: every variant on mma.sync, int8 rows of 128 on tcgen05.
    const size_t base = out.size();
    for (size_t i = 0; i < base; ++i) out.push_back(out[i] + "_mma");
    for (size_t i = 0; i < base; ++i)
      if (out[i].rfind("int8_", 0) == 0 && out[i].size() > 5 && out[i].compare(out[i].size() - 5, 5, "_d128") == 0)
        out.push_back(out[i] + "_tc");
    return out;
  }();
  return ids;
}

} // namespace

extern "C" cudaError_t kvf_b200_launch_variant(const char *variant_id, const kvf_args *a,
                                               cudaStream_t stream) {
  VariantId v;
  if (!parse_id(variant_id, v)) return cudaErrorInvalidDeviceFunction;
  return kvf_b200_decode_path(a, v.fmt, v.d, v.g, v.ord, v.paged, v.path, stream);
}

extern "C" int kvf_b200_variant_count(void) { return (int)all_ids().size(); }

extern "C" const char *kvf_b200_variant_name(int i) {
  const auto &ids = all_ids();
  return (i >= 0 && i < (int)ids.size()) ? ids[(size_t)i].c_str() : nullptr;
}
