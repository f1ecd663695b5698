// kvf_registry.h - drop-in replacement for the reference's
// runtime/kvf_registry.h (:15-29): maps a variant id to its launcher.
//
// The generated dispatch sources (gen/kvf_dispatch_*.cu, emitted by
// src/codegen.cpp:119-172) register `&kvf::launch<...>` instantiations here;
// with include/kvf_kernels.cuh those instantiations forward to the sm_100a
// kernels. FFI callers without C++ use kvf_b200_launch_variant instead.
#pragma once

#include "kvf_kernels.cuh"

#include <string>
#include <unordered_map>

namespace kvf {

using LaunchFn = cudaError_t (*)(const Args &, cudaStream_t);

struct Registry {
  std::unordered_map<std::string, LaunchFn> fn;
  void add(const char *id, LaunchFn f) { fn[id] = f; }
  LaunchFn find(const std::string &id) const {
    const auto it = fn.find(id);
    return it == fn.end() ? nullptr : it->second;
  }
};

} // namespace kvf

// Defined by the generated kvf_dispatch.cu.
void kvf_register_all(kvf::Registry &r);
