// kvf_kernels.cuh - drop-in replacement for the reference's
// runtime/kvf_kernels.cuh on sm_100a.
//
// Keeps the names generated code and the host runtime use:
//   kvf::Fmt / kvf::Ord enums            (runtime/kvf_kernels.cuh:26-27)
//   kvf::Args                            (runtime/kvf_kernels.cuh:29-46), same
//                                        field order, plus trailing seq_lens, split_sem, lse
//   kvf::launch<FMT, D, G, U, ORD, PAGED>(const Args &, cudaStream_t)
//                                        (runtime/kvf_kernels.cuh:309-320)
// so that the launchers src/codegen.cpp emits (`kvf_launch_<name>`), the
// dispatch tables in gen/kvf_dispatch_*.cu and runtime/kvf_host.h compile
// unchanged. launch<> forwards to the C ABI in kvforge_b200.h; the kernels
// themselves live in libkvforge_b200.so. U (unroll) and `warps` were tuning
// knobs of the reference's SIMT kernel and have no effect here.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "kvforge_b200.h"

namespace kvf {

enum Fmt { FMT_F16 = KVF_FMT_F16, FMT_INT8 = KVF_FMT_INT8, FMT_INT4 = KVF_FMT_INT4 };
enum Ord { ORD_HEAD = KVF_ORD_HEAD, ORD_TOKEN = KVF_ORD_TOKEN };

struct Args {
  const float *q;              // [B][H][D], fp32
  const unsigned char *k;      // K payload
  const unsigned char *v;      // V payload
  const __half2 *k_meta;       // [rows][D/group] (scale, zero), quantized only
  const __half2 *v_meta;
  const int *block_table;      // [B][max_blocks] page ids, paged layouts only
  float *out;                  // [B][H][D], fp32
  float *part_o;               // [B][H][splits][D] unnormalised partial output
  float *part_ml;              // [B][H][splits][2] running max (log2) and sum
  int B, H, Hkv, n;
  int splits;                  // chunks of the KV length per head
  int warps;                   // accepted, unused on sm_100a
  int group_shift;             // log2(quantization group), quantized only
  int block_shift;             // log2(tokens per page), paged only
  int max_blocks;              // pages per sequence in the block table
  float scale_log2;            // softmax scale * log2(e)
  const int *seq_lens;         // [B] tokens per sequence; nullptr = n for all
  unsigned *split_sem;         // [B][Hkv][2] zeroed counters for the in-kernel merge; nullptr = two launches
  float *lse;                  // [B][H] log2 softmax denominators, optional
};

static_assert(sizeof(Args) == sizeof(kvf_args), "kvf::Args must mirror kvf_args");
static_assert(offsetof(Args, scale_log2) == offsetof(kvf_args, scale_log2), "layout");
static_assert(offsetof(Args, seq_lens) == offsetof(kvf_args, seq_lens), "layout");
static_assert(offsetof(Args, split_sem) == offsetof(kvf_args, split_sem), "layout");
static_assert(offsetof(Args, lse) == offsetof(kvf_args, lse), "layout");

inline const kvf_args *c_args(const Args &a) { return reinterpret_cast<const kvf_args *>(&a); }

// One decode step on `st`: the sm_100a kernel plus the split merge when
// a.splits > 1. Returns the launch status; never synchronises.
template <int FMT, int D, int G, int U, int ORD, bool PAGED>
cudaError_t launch(const Args &a, cudaStream_t st) {
  static_assert(FMT == FMT_F16 || FMT == FMT_INT8 || FMT == FMT_INT4, "format");
  static_assert(D == 64 || D == 128, "head dimension");
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "GQA pack size");
  static_assert(U == 2 || U == 4, "unroll");
  return kvf_b200_decode(c_args(a), FMT, D, G, ORD, PAGED ? 1 : 0, st);
}

// launch<> pinned to one sm_100a kernel path (KVF_PATH_MMA or KVF_PATH_TC),
// the extra template parameter the sm_100a dispatch tables
// (kvforge_b200/codegen.py) instantiate for "_mma" / "_tc" variant ids.
template <int FMT, int D, int G, int U, int ORD, bool PAGED, int PATH>
cudaError_t launch_path(const Args &a, cudaStream_t st) {
  static_assert(FMT == FMT_F16 || FMT == FMT_INT8 || FMT == FMT_INT4, "format");
  static_assert(D == 64 || D == 128, "head dimension");
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "GQA pack size");
  static_assert(U == 2 || U == 4, "unroll");
  static_assert(PATH == KVF_PATH_AUTO || PATH == KVF_PATH_MMA || PATH == KVF_PATH_TC, "kernel path");
  static_assert(PATH != KVF_PATH_TC || (FMT == FMT_INT8 && D == 128), "the tcgen05 kernel takes int8 rows of 128");
  return kvf_b200_decode_path(c_args(a), FMT, D, G, ORD, PAGED ? 1 : 0, PATH, st);
}

} // namespace kvf
