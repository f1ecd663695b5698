/* kvforge_b200.h - C ABI of the B200 (sm_100a) decode-attention kernels.
 *
 * One decode step of one attention layer: every query head attends to the
 * n cached tokens of its sequence, over a KV cache stored as f16, int8:G or
 * int4:G (asymmetric per-group scale and zero point), head-major or
 * token-major, contiguous or paged. Results are written to `out`.
 *
 * This header is plain C (plain pointers and sizes, no C++ or torch types) so
 * it can be bound from ctypes, cgo or JNI. The C++ drop-in for the reference's
 * `kvf::launch<>` / `kvf::Args` (runtime/kvf_kernels.cuh) is kvf_kernels.cuh in
 * this directory; it forwards to the functions below.
 *
 * Error behaviour follows the reference launcher (runtime/kvf_kernels.cuh:309-320):
 * every entry point returns a cudaError_t, never throws, never synchronises
 * and never exits. Launches are stream-ordered; the library holds no state
 * between calls apart from caches of driver facts: driver entry points, SM
 * counts, and per CUDA context each kernel's shared-memory attribute and
 * occupancy (a context that replaces another, after cudaDeviceReset, starts
 * with empty caches).
 */
#ifndef KVFORGE_B200_H
#define KVFORGE_B200_H

#include <cuda_runtime_api.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Storage formats and placements: same values as kvf::Fmt / kvf::Ord
 * (runtime/kvf_kernels.cuh:26-27). */
enum { KVF_FMT_F16 = 0, KVF_FMT_INT8 = 1, KVF_FMT_INT4 = 2 };
enum { KVF_ORD_HEAD = 0, KVF_ORD_TOKEN = 1 };

/* Kernel argument block. Field order and types are those of kvf::Args
 * (runtime/kvf_kernels.cuh:29-46), so a pointer to a reference kvf::Args is a
 * valid kvf_args pointer. Fields after scale_log2 are additions; callers that
 * zero-initialise the struct (`kvf::Args a{}`) get the reference behaviour.
 *
 *   q            [B][H][D] fp32
 *   k, v         cache payload; row r holds one token's D channels of one KV
 *                head: f16 2*D bytes, int8 D bytes, int4 D/2 bytes (column c in
 *                byte c/2, odd columns in the high nibble)
 *   k_meta,v_meta [rows][D/group] words, each (scale | zero << 16) as fp16
 *                (a __half2 with .x = scale); quantized formats only
 *   block_table  [B][max_blocks] page ids, paged layouts only
 *   out          [B][H][D] fp32
 *   part_o       [B][H][splits][D] fp32 workspace, used when splits > 1
 *   part_ml      [B][H][splits][2] fp32 workspace (running max in log2 units,
 *                running sum), used when splits > 1
 *   splits       partitions of each sequence's tokens (>= 1). With seq_lens
 *                given, the mma.sync path balances the tokens over one wave
 *                of blocks: every sequence uses the same chunk of tokens, so
 *                a long sequence gets more splits than a short one, and
 *                splits is then the most any sequence may use (the
 *                workspace's capacity; kvf_b200_suggest_splits_ragged).
 *   warps        reference tuning knob; accepted and ignored on sm_100a
 *   group_shift  log2(quantization group), quantized formats
 *   block_shift  log2(tokens per page), paged layouts
 *   scale_log2   softmax scale * log2(e)
 *   seq_lens     [B] tokens of each sequence (each <= n); NULL = all n.
 *   split_sem    [B][Hkv][2] unsigned counters, zero before the first call
 *                and left zero by every call. When given (and splits > 1)
 *                the split merge runs inside the decode launch instead of a
 *                second kernel (part_o/part_ml are still written and read):
 *                on the tensor-core path the last block of each (sequence,
 *                KV head) merges (counter word 2u of unit u); on the mma.sync
 *                path, for batches with at least two merge slices per block,
 *                a cooperative launch merges after a grid barrier (words 1
 *                and 3), and for grids of one wave with at most 160
 *                splits (int8, int4) or 64 (f16) the last
 *                finishers of each (sequence, head group) g share
 *                its merge (words 2g and 2g + 1). NULL = the reference's
 *                two-launch scheme. Calls sharing one array must not overlap
 *                on the GPU.
 *   lse          [B][H] fp32, optional (NULL = not written): log2 of the
 *                softmax denominator of each query head, in the same units as
 *                part_ml (max + log2(sum)); -inf for a head with no tokens.
 *                It lets outputs computed on different token ranges (e.g. on
 *                different GPUs) be combined with kvf_b200_merge_states.
 */
typedef struct kvf_args {
  const float *q;
  const unsigned char *k;
  const unsigned char *v;
  const void *k_meta;
  const void *v_meta;
  const int *block_table;
  float *out;
  float *part_o;
  float *part_ml;
  int B, H, Hkv, n;
  int splits;
  int warps;
  int group_shift;
  int block_shift;
  int max_blocks;
  float scale_log2;
  /* ---- additions (zero = reference behaviour) ---- */
  const int *seq_lens;
  unsigned *split_sem;
  float *lse;
} kvf_args;

/* One decode step: the sm_100a counterpart of
 * kvf::launch<FMT, D, G, U, ORD, PAGED>(a, st) (runtime/kvf_kernels.cuh:309-320),
 * i.e. decode_partial (:124-285) plus, when a->splits > 1, the log-sum-exp
 * merge decode_merge (:288-306).
 *   fmt    KVF_FMT_*;  d  64 or 128;  ord  KVF_ORD_*;  paged  0/1
 *   g      query heads per KV head the caller packed (1, or H/Hkv). The
 *          sm_100a kernels always pack every query head of a KV head into one
 *          block, so 1 and H/Hkv give the same result; other values are
 *          rejected with cudaErrorInvalidValue.
 * Returns cudaSuccess, cudaErrorInvalidValue (bad shape, format, group, page
 * size or null pointer), cudaErrorMisalignedAddress (k or v not 16-byte
 * aligned, meta not 4-byte aligned), or the launch error. */
cudaError_t kvf_b200_decode(const kvf_args *a, int fmt, int d, int g, int ord, int paged,
                            cudaStream_t stream);

/* Kernel paths of the sm_100a decode (the B200 counterpart of the plan's
 * "mma on/off" choice):
 *   KVF_PATH_AUTO  by shape: the tcgen05 kernel for int8 rows of 128
 *                  dimensions with one or two quantization groups once there
 *                  are >= 32 (sequence, KV head) units, else mma.sync;
 *   KVF_PATH_MMA   always the mma.sync kernel (every format);
 *   KVF_PATH_TC    always the tcgen05 kernel; shapes it does not cover return
 *                  cudaErrorNotSupported without launching. */
enum { KVF_PATH_AUTO = 0, KVF_PATH_MMA = 1, KVF_PATH_TC = 2 };

/* Scheduling flags, OR'ed into a path value. They choose how the mma.sync
 * launch is organised, not what it computes: every combination gives the
 * same output (the three merge schemes bit for bit).
 *   KVF_FLAG_MERGE_KERNEL  the split merge runs as its own kernel, even where
 *                          the launch would merge in-kernel (after a grid
 *                          barrier, or by its last finishers);
 *   KVF_FLAG_GRID_MERGE    the grid-barrier merge wherever it is possible
 *                          (split_sem given, at least two (sequence, KV head)
 *                          units, every block resident), not only where it
 *                          measured faster (two or more merge slices per
 *                          decode block);
 *   KVF_FLAG_NO_BALANCE    one split count for every sequence even when
 *                          seq_lens is given (the reference's schedule).
 * MERGE_KERNEL and GRID_MERGE together, or any other bit, is
 * cudaErrorInvalidValue. */
enum { KVF_FLAG_MERGE_KERNEL = 0x100, KVF_FLAG_GRID_MERGE = 0x200, KVF_FLAG_NO_BALANCE = 0x400 };

/* kvf_b200_decode on an explicit kernel path: path is KVF_PATH_*, optionally
 * OR'ed with KVF_FLAG_* bits; any other value returns cudaErrorInvalidValue.
 * kvf_b200_decode is path AUTO with no flags. */
cudaError_t kvf_b200_decode_path(const kvf_args *a, int fmt, int d, int g, int ord, int paged, int path,
                                 cudaStream_t stream);

/* One decode step whose queries come from host memory, with no copy-engine
 * transfer: a small kernel reads q_host (B*H*d floats, 16-byte aligned, in
 * pinned host memory the device addresses at the same pointer, e.g. from
 * cudaHostAlloc) into a->q, and the decode (on `path`, as kvf_b200_decode_path
 * takes it) is launched
 * as its programmatic dependent, so the K/V stream starts while the queries
 * are still in flight; the decode reads them only once the copy kernel has
 * completed. On the tcgen05 path, when the grid is more than one wave and the
 * other sequences' queries are 256 KB or more, the sequences whose blocks fit
 * one wave are copied and decoded first, and the rest are copied by a narrow
 * kernel running beside that decode and decoded after it (four launches on
 * `stream`, each the programmatic dependent of the one before; the output is
 * the same bit for bit). a->out (and a->lse) may likewise point at such host memory: the
 * kernels then write the result there directly. Host buffers the device cannot
 * address (pageable memory) are rejected with cudaErrorInvalidValue before
 * anything launches. Otherwise as kvf_b200_decode_path. */
cudaError_t kvf_b200_decode_from_host(const kvf_args *a, int fmt, int d, int g, int ord, int paged, int path,
                                      const float *q_host, cudaStream_t stream);

/* The split merge alone (decode_merge<D>, runtime/kvf_kernels.cuh:288-306):
 * out[b][h] = sum_s part_o[s] * 2^(m_s - M) / sum_s l_s * 2^(m_s - M). */
cudaError_t kvf_b200_merge(const kvf_args *a, int d, cudaStream_t stream);

/* Combines attention outputs of the same query heads computed over disjoint
 * token ranges (e.g. one range per GPU when the KV cache is split across
 * GPUs along the tokens):
 *   out[i][x] = sum_p 2^(lse_p[i] - LSE) * o_p[i][x],   LSE = log2 sum_p 2^lse_p[i]
 * Part p's normalised output o_p [rows][d] starts at o + p * o_stride and its
 * lse_p [rows] (as written by kvf_b200_decode through kvf_args::lse) at
 * lse + p * lse_stride (strides in floats), so parts gathered into one packed
 * buffer per rank need no copy. out [rows][d]; lse_out [rows] (NULL = not
 * written) receives LSE. A row whose parts all have lse = -inf gets zeros.
 * No reference counterpart: the reference runs on one GPU. */
cudaError_t kvf_b200_merge_states(const float *o, const float *lse, int P, int rows, int d, long long o_stride,
                                  long long lse_stride, float *out, float *lse_out, cudaStream_t stream);

/* Split-KV across GPUs, fused into the decode's split merge: each rank
 * decodes its own token range, and the merge kernel that combines its splits
 * also stores the result (normalised output and lse of every query head, in
 * 32-column slices) straight into the gather buffer of every rank over NVLink,
 * waits (bounded) until all P parts of its slice are there and writes their
 * combination (the same arithmetic as kvf_b200_merge_states) to out. Every
 * value travels in one 64-bit cell together with the epoch that wrote it, so
 * a cell that holds the current epoch is complete by itself: no fence and no
 * counter sit between the stores and the reads. One decode launch plus one
 * merge launch per step, no collective library.
 *   gather       this rank's cells, [2][P][B*H][D+1] x 64 bits, zero
 *                initially: low word the float's bits, high word the epoch
 *                (two halves alternate by epoch parity; a rank runs at most
 *                one step ahead)
 *   peer_gather  the same buffer of rank p, mapped on this GPU (p = rank
 *                included); epoch: 1, 2, 3, ... one per step. */
typedef struct kvf_exchange {
  int P, rank, epoch;
  unsigned timeout_ms;
  unsigned long long *gather;
  unsigned long long *peer_gather[8];
} kvf_exchange;

/* kvf_b200_decode over this rank's tokens with the cross-GPU combination
 * fused into the split merge (a->splits must be > 1; split_sem is ignored).
 * A wait that runs out of time zeroes its slice and sets bit 1 (value 2) of
 * kvf_b200_device_errors(). */
cudaError_t kvf_b200_decode_exchange(const kvf_args *a, int fmt, int d, int g, int ord, int paged,
                                     const kvf_exchange *x, cudaStream_t stream);

/* Cross-GPU exchange of split-KV states over NVLink peer memory, without a
 * collective library (no reference counterpart). A rank's packed state
 * (`floats` floats: output then lse) is stored into its slot of each of the P
 * ranks' gather buffers (peer_slots[p], device pointers valid on this GPU,
 * e.g. from a symmetric allocation), followed by a system-scope fence and
 * `epoch` written to peer_flags[p] (this rank's flag word on rank p). One
 * block; at most 8 ranks. */
cudaError_t kvf_b200_push_state(const float *state, int floats, float *const *peer_slots, int *const *peer_flags,
                                int P, int epoch, cudaStream_t stream);

/* Waits until flags[0..P) all hold `epoch` or later (bounded by timeout_ms;
 * on timeout the rows are zeroed and kvf_b200_exchange_errors() reports it),
 * then combines the P gathered states (part p at gathered + p * part_stride:
 * output [rows][d], lse at + lse_off) like kvf_b200_merge_states. */
cudaError_t kvf_b200_wait_merge_states(const float *gathered, const int *flags, int P, int epoch, int rows, int d,
                                       long long part_stride, long long lse_off, float *out, float *lse_out,
                                       unsigned timeout_ms, cudaStream_t stream);

/* Nonzero if a wait of kvf_b200_wait_merge_states ran out of time since the
 * last call (then cleared). */
unsigned kvf_b200_exchange_errors(void);

/* Zeroed device buffer shareable with other processes of the node:
 * *ptr receives the device pointer, handle64 the 64-byte CUDA IPC handle. */
cudaError_t kvf_b200_ipc_alloc(size_t bytes, void **ptr, void *handle64);
/* Maps another process's buffer (peer access enabled); release with
 * kvf_b200_ipc_close. */
cudaError_t kvf_b200_ipc_open(const void *handle64, void **ptr);
cudaError_t kvf_b200_ipc_close(void *ptr);
/* Frees a buffer from kvf_b200_ipc_alloc. */
cudaError_t kvf_b200_ipc_free(void *ptr);

/* Launch by variant id, e.g. "int8_tm_p_g4_u2_d128": the registry lookup plus
 * call of bench/sweep.cu:180-184 (id format of src/codegen.cpp:59-65,
 * fmt_{hm,tm}_{c,p}_g{1,2,4,8}_u{2,4}_d{64,128}). Unknown ids return
 * cudaErrorInvalidDeviceFunction. */
cudaError_t kvf_b200_launch_variant(const char *variant_id, const kvf_args *a,
                                    cudaStream_t stream);

/* Variant ids may end in "_mma" or "_tc" to pin the kernel path
 * (KVF_PATH_MMA / KVF_PATH_TC); without a suffix the path is AUTO. "_tc" ids
 * exist for int8 rows of 128 dimensions only.
 *
 * Number of variant ids this library registers, and the i-th id (NULL when i
 * is out of range). Mirrors kvf_register_all (gen/kvf_dispatch.cu, and the
 * sm_100a tables kvforge_b200/codegen.py emits). */
int kvf_b200_variant_count(void);
const char *kvf_b200_variant_name(int i);

/* Split count the sm_100a kernels run best with for this shape: the
 * B200 counterpart of the planner's `splits` choice (src/plan.cpp:25-35).
 * n is the longest sequence. Always >= 1. */
int kvf_b200_suggest_splits(int B, int H, int Hkv, int n, int fmt, int d, int group, int paged,
                            int block_tokens);
/* The split count (workspace capacity per sequence) for a batch whose
 * sequences may differ in length (seq_lens given): as many splits as one
 * sequence can use under balanced splits, within 64 MiB of partials; the
 * same as kvf_b200_suggest_splits where the launch does not balance
 * (tensor-core path, or more (sequence, head group) units than one wave of
 * blocks). */
int kvf_b200_suggest_splits_ragged(int B, int H, int Hkv, int n, int fmt, int d, int group, int paged,
                                   int block_tokens);
/* The chunk (tokens per split) a balanced launch uses, computed on the host
 * from host seq_lens exactly as the kernels compute it on the device: the
 * smallest multiple of gran, at least ceil(n / splits), for which
 * units * sum_b ceil(seq_lens[b] / chunk) <= grid (units: head groups per
 * sequence; grid: blocks launched, as kvf_b200_describe reports them). -1
 * for invalid arguments or units * B > grid. For sizing and tests; the
 * launch itself never reads seq_lens on the host. */
int kvf_b200_balanced_chunk(const int *seq_lens, int B, int n, int splits, int units, int grid, int gran);

/* Writes a one-line description of the launch kvf_b200_decode would make
 * (grid, block, stages, tokens per stage, shared memory) into buf. Returns
 * the same status kvf_b200_decode would return for these arguments, without
 * launching anything. */
cudaError_t kvf_b200_describe(const kvf_args *a, int fmt, int d, int ord, int paged, char *buf,
                              int buf_len);
/* kvf_b200_describe for an explicit kernel path (KVF_PATH_* with optional
 * KVF_FLAG_* bits, as kvf_b200_decode_path takes it). */
cudaError_t kvf_b200_describe_path(const kvf_args *a, int fmt, int d, int ord, int paged, int path, char *buf,
                                   int buf_len);

/* Device-side error word of the current device, then cleared. Bit 0: a
 * shared-memory barrier wait in a decode kernel ran out of time (the kernel
 * abandoned the step and its output is not valid). Bit 1: a cross-GPU wait
 * of kvf_b200_decode_exchange ran out of time (the affected output slices are
 * zero). Bit 2: kvf_b200_append met a token outside the cache (not written).
 * 0 = no error. This call synchronises with the device. */
unsigned kvf_b200_device_errors(void);

/* Quantizes `rows` logical rows of d fp32 channels (device memory) into the
 * cache format: the device counterpart of kvf::quantize
 * (runtime/kvf_host.h:72-120), bit-exact with it. `data` receives
 * rows * row_bytes bytes; for int8/int4 `meta` receives rows * (d / group)
 * words (scale | zero << 16, fp16). f16 ignores group and meta. */
cudaError_t kvf_b200_quantize(int fmt, int d, int group, const float *x, long long rows,
                              unsigned char *data, void *meta, cudaStream_t stream);

/* Appends t_new tokens to every sequence of a cache on the device: the new
 * rows k_new, v_new (fp32 [B][Hkv][t_new][d], device memory, logical order)
 * are quantized exactly as kvf_b200_quantize does (kvf::quantize,
 * runtime/kvf_host.h:72-120) and their codes and (scale, zero) words written
 * at the physical rows of tokens pos[b] .. pos[b] + t_new - 1 in the cache
 * `a` describes (row formula of runtime/kvf_kernels.cuh:51-64 and
 * kvf_host.h:124-135 for `ord` and `paged`; read: k, v, k_meta, v_meta,
 * block_table, max_blocks, block_shift, group_shift, B, Hkv, n; the cache
 * buffers are written through). pos: device int[B], the first new token of
 * each sequence, usually its length so far; the caller then raises its
 * seq_lens by t_new. For a paged cache the block table must already map every
 * block the new tokens fall in. A token at or past n, or in a block past
 * max_blocks, is skipped and sets bit 2 of kvf_b200_device_errors(). No
 * reference counterpart: the reference places a whole cache on the host
 * (upload_cache, kvf_host.h:149-195). */
cudaError_t kvf_b200_append(const kvf_args *a, int fmt, int d, int ord, int paged, const float *k_new,
                            const float *v_new, int t_new, const int *pos, cudaStream_t stream);

/* Bytes of device scratch behind kvf_b200_decode_noalloc (8 MiB). */
#define KVF_B200_NOALLOC_SCRATCH_BYTES (8u << 20)

/* kvf_b200_decode for callers that cannot allocate device memory. It has no
 * counterpart in the reference, whose harnesses always allocate the split
 * workspace themselves (alloc_buffers).
 *
 * Callers such as a serving engine that reserved all device memory for its
 * KV pool at start-up, or a plugin whose framework owns every allocation,
 * cannot cudaMalloc the part_o / part_ml workspace that splits > 1 needs.
 * This entry point ignores a->part_o and a->part_ml and keeps the partials in
 * a static device array of KVF_B200_NOALLOC_SCRATCH_BYTES inside the library
 * (held by every GPU that loads the library until the process exits); it
 * calls no allocator. The caller still passes q, the cache, out and the
 * other inputs. Limits and rules:
 *   - B * H * splits * (d + 2) * 4 bytes (plus alignment) must fit the
 *     scratch; larger requests return cudaErrorInvalidValue (use fewer
 *     splits, or kvf_b200_decode with your own workspace);
 *   - all calls on a device share the one array: calls that overlap on the
 *     GPU (concurrent streams) race and corrupt each other's partials.
 *     Nothing needs clearing between calls: every call writes each partial
 *     it later reads;
 *   - the first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current), and looks it up
 *     again if the device's context was replaced (cudaDeviceReset); make
 *     that first call before any stream capture.
 * splits <= 1 needs no scratch and behaves exactly like kvf_b200_decode. */
cudaError_t kvf_b200_decode_noalloc(const kvf_args *a, int fmt, int d, int g, int ord, int paged,
                                    cudaStream_t stream);

/* Library version string. */
const char *kvf_b200_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KVFORGE_B200_H */
