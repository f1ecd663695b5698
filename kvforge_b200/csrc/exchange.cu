// exchange.cu - cross-GPU combination of split-KV decode states over NVLink
// peer memory (no reference counterpart: the reference decodes on one GPU).
//
// Each rank decodes its own token range and holds a packed state (normalised
// output [rows][d] followed by lse [rows]). Instead of a collective, the
// producing rank stores its state straight into its slot of every peer's
// gather buffer (peer pointers of a symmetric allocation, NVLink stores),
// fences at system scope and raises an epoch flag in each peer's flag array.
// The consuming kernel on every rank waits (bounded) until all P flags carry
// the current epoch (or a later one) and merges the P states as
// kvf_b200_merge_states does. Epochs increase by one per step and the caller
// alternates two gather buffers by epoch parity: a peer can run at most one
// step ahead (its next wait needs this rank's next push, which follows this
// rank's merge), so it never overwrites the buffer being read.
#include "kvforge_b200.h"

#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>

namespace kvfb {

__device__ unsigned g_xchg_error;

namespace {

constexpr int kMaxPeers = 8;

struct PeerPtrs {
  float *slot[kMaxPeers];  // this rank's slot in peer p's gather buffer
  int *flag[kMaxPeers];    // this rank's flag word in peer p's flag array
};

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One block: the state goes to every peer (16-byte stores when aligned),
// then a system-scope fence and the epoch flag per peer.
__global__ void __launch_bounds__(1024) push_state_kernel(const float *state, int floats, PeerPtrs pp, int P,
                                                          int epoch) {
  const bool v4 = (floats & 3) == 0 && ((reinterpret_cast<uintptr_t>(state) & 15u) == 0);
  for (int p = 0; p < P; ++p) {
    float *dst = pp.slot[p];
    if (v4 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
      const float4 *s4 = reinterpret_cast<const float4 *>(state);
      float4 *d4 = reinterpret_cast<float4 *>(dst);
      for (int i = threadIdx.x; i < floats / 4; i += blockDim.x) d4[i] = __ldg(s4 + i);
    } else {
      for (int i = threadIdx.x; i < floats; i += blockDim.x) dst[i] = __ldg(state + i);
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < P) {
    int *f = pp.flag[threadIdx.x];
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
  }
}

// One block per output row: wait (bounded) for every part of this epoch, then
// the lse-weighted combination.
__global__ void wait_merge_kernel(const float *gathered, const int *flags, int P, int epoch, int rows, int d,
                                  long long part_stride, long long lse_off, float *out, float *lse_out,
                                  unsigned timeout_ms) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const uint64_t t0 = now_ns();
    const uint64_t limit = (uint64_t)timeout_ms * 1000000ull;
    int ok = 1;
    for (int p = 0; p < P && ok; ++p) {
      for (;;) {
        int v;
        asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flags + p) : "memory");
        if (v - epoch >= 0) break;  // this epoch or a later one (wrap-safe)
        if (now_ns() - t0 > limit) {
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    if (!ok) atomicOr(&g_xchg_error, 1u);
    s_ok = ok;
  }
  __syncthreads();
  const int r = blockIdx.x;
  const int c = threadIdx.x;
  if (!s_ok) {
    if (c < d) out[(long long)r * d + c] = 0.f;
    return;
  }
  float M = -INFINITY;
  for (int k = 0; k < P; ++k) M = fmaxf(M, __ldcg(gathered + k * part_stride + lse_off + r));
  float W = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int k = 0; k < P; ++k) {
      const float lk = __ldcg(gathered + k * part_stride + lse_off + r);
      const float w = lk == -INFINITY ? 0.f : exp2f(lk - M);
      W += w;
      if (c < d && w > 0.f) O = fmaf(w, __ldcg(gathered + k * part_stride + (long long)r * d + c), O);
    }
  }
  if (c < d) out[(long long)r * d + c] = W > 0.f ? O / W : 0.f;
  if (c == 0 && lse_out) lse_out[r] = W > 0.f ? M + log2f(W) : -INFINITY;
}

} // namespace
} // namespace kvfb

using namespace kvfb;

extern "C" cudaError_t kvf_b200_push_state(const float *state, int floats, float *const *peer_slots,
                                           int *const *peer_flags, int P, int epoch, cudaStream_t stream) {
  if (!state || floats <= 0 || !peer_slots || !peer_flags || P < 1 || P > kMaxPeers) return cudaErrorInvalidValue;
  PeerPtrs pp{};
  for (int p = 0; p < P; ++p) {
    if (!peer_slots[p] || !peer_flags[p]) return cudaErrorInvalidValue;
    pp.slot[p] = peer_slots[p];
    pp.flag[p] = peer_flags[p];
  }
  push_state_kernel<<<1, 1024, 0, stream>>>(state, floats, pp, P, epoch);
  return cudaGetLastError();
}

extern "C" cudaError_t kvf_b200_wait_merge_states(const float *gathered, const int *flags, int P, int epoch,
                                                  int rows, int d, long long part_stride, long long lse_off,
                                                  float *out, float *lse_out, unsigned timeout_ms,
                                                  cudaStream_t stream) {
  if (!gathered || !flags || !out || P < 1 || P > kMaxPeers || rows < 0 || d < 1 || d > 1024) return cudaErrorInvalidValue;
  if (lse_off < (long long)rows * d || part_stride < lse_off + rows || timeout_ms == 0) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  wait_merge_kernel<<<rows, (d + 31) / 32 * 32, 0, stream>>>(gathered, flags, P, epoch, rows, d, part_stride, lse_off,
                                                           out, lse_out, timeout_ms);
  return cudaGetLastError();
}

// Device buffers shared across processes of one node through CUDA IPC (plain
// peer mappings only). The exporting process allocates
// (zeroed) and passes the 64-byte handle to the others, which open it.
extern "C" cudaError_t kvf_b200_ipc_alloc(size_t bytes, void **ptr, void *handle64) {
  if (!ptr || !handle64 || bytes == 0) return cudaErrorInvalidValue;
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return e;
  e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return e;
  }
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(handle64, &h, sizeof(h));
  return cudaSuccess;
}

extern "C" cudaError_t kvf_b200_ipc_open(const void *handle64, void **ptr) {
  if (!handle64 || !ptr) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

extern "C" cudaError_t kvf_b200_ipc_close(void *ptr) { return cudaIpcCloseMemHandle(ptr); }

extern "C" cudaError_t kvf_b200_ipc_free(void *ptr) { return cudaFree(ptr); }

extern "C" unsigned kvf_b200_exchange_errors(void) {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_xchg_error, sizeof(v)) != cudaSuccess) {
    cudaGetLastError();
    return 0xFFFFFFFFu;
  }
  if (v) cudaMemcpyToSymbol(g_xchg_error, &zero, sizeof(zero));
  return v;
}
