// decode_tc.cuh - the tcgen05 (5th-generation tensor core) decode kernel for
// int8 K/V rows of 128 dimensions.
//
// Counterpart of decode_partial<FMT_INT8, 128, G, U, ORD, PAGED, FINAL> in the
// reference (runtime/kvf_kernels.cuh:124-285). One block owns a chunk of one
// sequence's tokens for one KV head and all of its query heads; stages of 128
// tokens stream through a TMA-fed shared-memory ring.
//
// Both products run on the tensor cores as exact integer MMAs
// (tcgen05.mma kind::i8, s32 accumulators in tensor memory):
//
//   scores  S^T[128 tokens x cols] = K codes (u8, K-major, the TMA tile as it
//           landed) * Q planes (s8). The query row of each head is scaled by a
//           power of two 2^eq and rounded to a 22-bit integer Qi, written as
//           three balanced base-256 digits (Qi = b0 + 256 b1 + 65536 b2); each
//           digit plane is one column, and each quantization group of the row
//           accumulates into its own columns. A token's score is then
//             s = 2^-eq sum_g scale_g (D0 + 256 D1 + 65536 D2)_g + sum_g zero_g qsum_g
//           with every D exact in int32 (runtime/kvf_kernels.cuh:211 dequantises
//           the same way: scale * code + zero).
//
//   values  O^T[128 dims x cols] = V codes (u8, read MN-major from the same
//           tile) * P' planes (u8, written over the stage's K tile, which is
//           dead once the score MMAs completed), where P'_t = rint(p_t * vscale_t * 2^ev) is a
//           23-bit integer per (token, head, group) split into byte planes;
//           ev puts the stage's largest V scale in [2^22, 2^23). Each stage's
//           exact product is folded into fp32 registers with the stage's
//           rescale. The zero term sum_t p_t * vzero_t stays on the CUDA cores.
//
// Warp roles (384 threads, two blocks per SM):
//   warps 0-7  warp w serves tensor-memory lanes 32(w%4) .. 32(w%4)+31 and half
//              w/4 of the query heads: each thread owns one token (scores) and
//              one dimension (output) for its heads. It reads the stage's
//              scores from tensor memory, runs the online softmax in the log2
//              domain with one rescale per stage, writes P' planes, and folds
//              each stage's value product into fp32;
//   warps 8-9  producers, both on every stage: warp 8 the K tile (TMA) and K
//              metadata rows (cp.async), warp 9 the same for V, all counted
//              on the stage's full barrier. A ring slot is held from the
//              first copy instruction to the value MMAs, and with small pages
//              a stage takes 16 TMA boxes and 256 metadata rows: issuing them
//              from two warps, with every address worked out before the slot
//              is free, keeps that time short;
//   warp 10    score-MMA issuer (one thread): a stage's score MMAs as soon as
//              its tiles land and its score buffer is free; also allocates
//              and frees tensor memory;
//   warp 11    value-MMA issuer (one thread): a stage's value MMAs as soon as
//              its P' planes are written, then hands the slot back.
// Score columns of a quantization group g are ordered g*NS + half*NS/2 +
// plane*NH/2 + head-in-half, value (P') columns g*NS + half*NS/2 +
// 4*head-in-half + plane (planes 0-2 of P'; the fourth byte of a head's word
// is not part of it and its column is never read), so each warp reads and
// writes only its own columns.
// With a split-counter array (kvf_args::split_sem) the last block to finish a
// (sequence, KV head) merges that head's split partials itself
// (decode_merge, runtime/kvf_kernels.cuh:288-306), so no second kernel runs.
// Every wait is bounded in time; tensor memory is released before exit.
#pragma once

#include "decode_kernel.cuh"
#include "tc.cuh"

namespace kvfb {

// Host-computed constants of a tensor-core launch; byte offsets relative to
// the 1024-aligned dynamic shared-memory base.
struct TcPlan {
  int gq;          // query heads per KV head (<= 8)
  int tbox;        // tokens per TMA box (128, or the page size)
  int tbox_shift;
  int npg;         // TMA boxes per stage: 128 / tbox
  int stages;      // ring depth (<= 8)
  int chunk;       // tokens per split (multiple of 128)
  int splits;
  int paged, tm, bt_shift;
  int final_out;
  int merge_in_kernel;   // split_sem given and the merge scratch fits in the ring
  uint32_t stage_bytes;  // K tile, V tile (128 x 128 bytes each), K meta, V meta; 1024-aligned
  uint32_t meta_bytes;   // one metadata area: 128 rows x groups x 4 bytes, 128-aligned
  uint32_t off_q;        // Q plane tile: NS rows x 128 bytes, 128-byte swizzle
  uint32_t ptile_bytes;  // P' tile bytes (<= the K tile)
  uint32_t off_misc;     // scalars, exchange areas, barriers
  uint32_t tmem_cols;    // allocated tensor-memory columns
  uint32_t smem_total;
};

constexpr int kTcTokens = 128;  // tokens per stage (M of the score MMA)
constexpr int kTcThreads = 384;     // 8 softmax warps, 2 producers, 2 MMA issuers
constexpr int kTcProducerWarp = 8;  // and 9
constexpr int kTcProducers = 2;
constexpr int kTcMmaWarp = 10;      // score MMAs; allocates tensor memory
constexpr int kTcValueWarp = 11;    // value MMAs

// Scalars, exchange areas and barriers in the misc region.
template <int GPR, int NH> struct TcMisc {
  float qinv[NH];             // 2^-eq per query head
  float qsum[NH][GPR];        // 2^-eq * sum of Qi over each group
  // Stage maxima (+ V-scale bits) per half, double-buffered: high word the
  // stage number + 1, low word the order-mapped value.
  unsigned long long redx[2][2][NH / 2 + 1];
  float xl[8][NH / 2];        // epilogue: per-warp sums of p
  float xz[8][NH / 2][GPR];   // epilogue: per-warp sums of p * vzero
  uint32_t tmem_base;
  int abort_flag;             // set by any warp that gave up; the others stop waiting
  int last;                   // this block is the last of its (sequence, KV head)
  int slot_last[8];           // last stage whose copies went into each ring slot (-1: none)
  // full[8], empty[8], sfull[2], sfree[2], pready, ofull, red[2 parities][2 halves], done[2]
  uint64_t bars[32];
};

// Start of a running maximum: the most negative finite float, so the
// maximum stays finite, 2^(m_old - m_new) never meets inf - inf (a finite
// score against it gives -inf or 0 in the exponent), and a head that saw
// only masked rows keeps it (reported as -inf).
constexpr float kTcMinusBig = -3.402823466e38f;

template <int GPR, int NH>
__global__ void __launch_bounds__(kTcThreads, 2)
decode_tc_kernel(const kvf_args a, const TcPlan p, const __grid_constant__ CUtensorMap tmk,
                 const __grid_constant__ CUtensorMap tmv) {
  constexpr int D = 128;
  constexpr int TB = kTcTokens;
  constexpr int NS = NH == 4 ? 16 : 32;  // columns per group: 3 planes x NH heads, padded
  constexpr int SC = GPR * NS;           // score columns per S buffer
  constexpr int NP = GPR * NS;           // value columns
  constexpr int KPG = (D / 32) / GPR;    // 32-byte k-steps per quantization group
  constexpr int HT = NH / 2;             // query heads per thread
  constexpr int CH = NS / 2;             // columns per half of a group
  static_assert(NH == 4 || NH == 8, "head slots");
  static_assert(GPR == 1 || GPR == 2, "groups per row");

  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  TcMisc<GPR, NH> &ms = *reinterpret_cast<TcMisc<GPR, NH> *>(smem + p.off_misc);
  volatile int *abort_flag = &ms.abort_flag;
  const uint32_t bars = ptx::smem_u32(&ms.bars[0]);
  const uint32_t bar_full = bars, bar_empty = bars + 64, bar_sfull = bars + 128, bar_sfree = bars + 144,
                 bar_pready = bars + 160, bar_ofull = bars + 168, bar_red = bars + 176, bar_done = bars + 208;
  const uint32_t sq = sbase + p.off_q;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;

  const int split = blockIdx.x % p.splits;
  const int rest = blockIdx.x / p.splits;
  const int h = rest % a.Hkv;
  const int b = rest / a.Hkv;
  int nb = a.n;
  if (a.seq_lens) nb = min(max(a.seq_lens[b], 0), a.n);
  const int t0 = split * p.chunk;
  const int t1 = min(nb, t0 + p.chunk);
  const int ntiles = t1 > t0 ? (t1 - t0 + TB - 1) / TB : 0;

  if (tid == 0) {
    ms.abort_flag = 0;
    for (int s = 0; s < 8; ++s) ms.slot_last[s] = -1;
    for (int e = 0; e < 2 * 2 * (NH / 2 + 1); ++e) (&ms.redx[0][0][0])[e] = 0ull;
    for (int s = 0; s < p.stages; ++s) {
      ptx::mbar_init(bar_full + 8u * s, 66u);  // per producer: expect_tx arrival + 32 cp.async arrivals
      ptx::mbar_init(bar_empty + 8u * s, 1u);
    }
    for (int j = 0; j < 2; ++j) {
      ptx::mbar_init(bar_sfull + 8u * j, 1u);
      ptx::mbar_init(bar_sfree + 8u * j, 8u);
      // Each half's four warps cover all 128 tokens of a stage, so a half
      // exchanges its maxima (and the stage's V-scale maximum) on its own.
      for (int hf = 0; hf < 2; ++hf) ptx::mbar_init(bar_red + 8u * (2 * j + hf), 4u);
    }
    ptx::mbar_init(bar_pready, 8u);
    ptx::mbar_init(bar_ofull, 1u);
    ptx::mbar_init(bar_done, 1u);
    ptx::mbar_init(bar_done + 8u, 1u);
    ptx::fence_barrier_init();
  }
  if (warp == kTcMmaWarp) {
    tc::alloc(ptx::smem_u32(&ms.tmem_base), p.tmem_cols);
    tc::relinquish();
  }

  // Q planes (warps 0-7): warp w builds head w; lane i covers dimensions
  // 4i .. 4i+3.
  if (warp < 8) {
    for (int r = tid; r < NS * 8; r += 256)  // zero the whole tile (padding rows)
      asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(sq + 16u * r), "r"(0) : "memory");
  }
  __syncthreads();
  if (warp < NH) {
    // Queries staged by a preceding kernel (kvf_b200_decode_from_host) are
    // read only after it completed; without that dependency this returns at once.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    {
      const int hq = warp;
      const bool live = hq < p.gq;
      float x[4];
      float mx = 0.f;
      const float *qh = a.q + ((long long)b * a.H + (long long)h * p.gq + (live ? hq : 0)) * D + 4 * lane;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[j] = live ? __ldg(qh + j) * a.scale_log2 : 0.f;
        mx = fmaxf(mx, fabsf(x[j]));
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const int eq = max(min(norm_exp(mx, 22), 120), -120);
      const float fq = eq >= 0 ? exp2i(min(eq, 127)) : exp2i(max(eq, -126));
      uint32_t w0 = 0, w1 = 0, w2 = 0;
      int qsum = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int qi = __float2int_rn(x[j] * fq);
        qsum += qi;
        const int b0 = (qi << 24) >> 24;
        const int r1 = (qi - b0) >> 8;
        const int b1 = (r1 << 24) >> 24;
        const int b2 = (r1 - b1) >> 8;
        w0 |= (uint32_t)(b0 & 255) << (8 * j);
        w1 |= (uint32_t)(b1 & 255) << (8 * j);
        w2 |= (uint32_t)(b2 & 255) << (8 * j);
      }
      // Row r of the tile at r*128 + (byte ^ ((r & 7) << 4)) (128-byte swizzle).
      const uint32_t byte = 4u * lane;
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) {
        const uint32_t r = (uint32_t)((hq / HT) * CH + pl * HT + (hq % HT));
        const uint32_t ad = sq + r * 128u + (byte ^ ((r & 7u) << 4));
        asm volatile("st.shared.u32 [%0], %1;" ::"r"(ad), "r"(pl == 0 ? w0 : pl == 1 ? w1 : w2) : "memory");
      }
      // Group sums: GPR groups of 128/GPR dimensions = 32/GPR lanes each.
      float gs = (float)qsum;
#pragma unroll
      for (int off = 1; off < 32 / GPR; off <<= 1) gs += __shfl_xor_sync(0xffffffffu, gs, off);
      const float qinv = eq <= 0 ? exp2i(min(-eq, 127)) : exp2i(max(-eq, -126));
      if ((lane & (32 / GPR - 1)) == 0) ms.qsum[hq][lane / (32 / GPR)] = live ? gs * qinv : 0.f;
      if (lane == 0) ms.qinv[hq] = live ? qinv : 0.f;
    }
    ptx::fence_proxy_async_smem();  // the tile is read by the tensor cores
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tbase = ms.tmem_base;
  // The separate merge kernel (if any) may be scheduled now; it waits for this grid.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp >= kTcProducerWarp && warp < kTcProducerWarp + kTcProducers) {
    // ----------------------------------------------------------- producers
    // Both producers work on every stage, side by side: warp 8 copies the K
    // tile and K metadata, warp 9 the V tile and V metadata. Block-table and
    // metadata addresses of a stage are worked out before its slot is free,
    // so the slot waits only for the copy instructions themselves.
    const int pw = warp - kTcProducerWarp;
    const CUtensorMap *tmap = pw ? &tmv : &tmk;
    const uint32_t *meta = reinterpret_cast<const uint32_t *>(pw ? a.v_meta : a.k_meta);
    if (lane == 0) ptx::prefetch_tmap(tmap);
    const uint64_t pol = ptx::policy_evict_first();
    const int tbs = p.tbox_shift;
    const int bmask = (1 << p.bt_shift) - 1;
    const int nblk_valid = p.paged ? min(a.max_blocks, (nb + bmask) >> p.bt_shift) : 0;
    const long long tab0 = (long long)b * a.max_blocks;
    // Block-table window: pages of blocks [win, win + 96) in three registers
    // per lane, loaded one window ahead of use.
    int win = p.paged ? (t0 >> p.bt_shift) : 0;
    int pg_cur = 0, pg_nxt = 0, pg_nn = 0;
    if (p.paged) {
      if (win + lane < nblk_valid) pg_cur = __ldg(a.block_table + tab0 + win + lane);
      if (win + 32 + lane < nblk_valid) pg_nxt = __ldg(a.block_table + tab0 + win + 32 + lane);
      if (win + 64 + lane < nblk_valid) pg_nn = __ldg(a.block_table + tab0 + win + 64 + lane);
    }
    bool ok = true;
    int s = 0;
    uint32_t phase = 0;  // parity of the slot's current use
    for (int i = 0; i < ntiles; ++i, s = (s + 1 == p.stages) ? (phase ^= 1u, 0) : s + 1) {
      const int tt = t0 + i * TB;
      int lanepage = 0;  // page of TMA box `lane` of this stage (lanes < npg)
      if (p.paged) {
        // Box j of the stage lies in block blk0 + j (several boxes per stage
        // only when a page holds at most 128 tokens, one box per page).
        const int blk0 = tt >> p.bt_shift;
        while (blk0 >= win + 32) {
          win += 32;
          pg_cur = pg_nxt;
          pg_nxt = pg_nn;
          pg_nn = (win + 64 + lane < nblk_valid) ? __ldg(a.block_table + tab0 + win + 64 + lane) : 0;
        }
        const int idx = blk0 - win + (lane < p.npg ? lane : 0);  // < 32 + 8
        const int from_cur = __shfl_sync(0xffffffffu, pg_cur, idx & 31);
        const int from_nxt = __shfl_sync(0xffffffffu, pg_nxt, idx & 31);
        lanepage = idx < 32 ? from_cur : from_nxt;
      }
      // Metadata rows of tokens lane + 32k of the stage (null past the chunk,
      // where the row is zero-filled instead).
      const uint32_t *msrc[TB / 32];
#pragma unroll
      for (int k = 0; k < TB / 32; ++k) {
        const int r = lane + 32 * k;
        const int tok = tt + r;
        const int pg = p.paged ? __shfl_sync(0xffffffffu, lanepage, r >> tbs) : 0;
        long long row;
        if (p.paged) {
          const int tl = tok & bmask;
          const long long base = ((long long)pg * a.Hkv) << p.bt_shift;
          row = p.tm ? base + (long long)tl * a.Hkv + h : base + ((long long)h << p.bt_shift) + tl;
        } else {
          row = p.tm ? ((long long)b * a.n + tok) * a.Hkv + h : ((long long)b * a.Hkv + h) * a.n + tok;
        }
        msrc[k] = tok < t1 ? meta + row * GPR : nullptr;
      }
      const int c1 = p.paged ? ((tt + (lane << tbs)) & bmask) : tt + (lane << tbs);
      const int c3 = p.paged ? lanepage : b;

      if (i >= p.stages && !warp_wait(bar_empty + 8u * s, phase ^ 1u, abort_flag)) {
        ok = false;
        break;
      }
      const uint32_t sk = sbase + s * p.stage_bytes;
      ptx::mbar_arrive_expect_tx_if(bar_full + 8u * s, TB * 128u, lane == 0);
      __syncwarp();
      // lane j issues box j of the tile
      ptx::tma_g2s_4d_if(sk + (uint32_t)pw * (TB * 128u) + (uint32_t)lane * (uint32_t)(p.tbox * 128), tmap, 0, c1,
                         h, c3, bar_full + 8u * s, pol, lane < p.npg);
      const uint32_t smeta = sk + 2u * TB * 128u + (uint32_t)pw * p.meta_bytes;
#pragma unroll
      for (int k = 0; k < TB / 32; ++k) {
        const uint32_t dst = smeta + (uint32_t)((lane + 32 * k) * GPR * 4);
        const bool live = msrc[k] != nullptr;
        if (GPR == 1)
          ptx::cp_async_4_zfill(dst, live ? msrc[k] : meta, live ? 4u : 0u);
        else
          ptx::cp_async_8_zfill(dst, live ? msrc[k] : meta, live ? 8u : 0u);
      }
      ptx::cp_async_arrive(bar_full + 8u * s);
      if (lane == 0) *reinterpret_cast<volatile int *>(&ms.slot_last[s]) = i;
      if (*abort_flag) break;
    }
    if (!ok) {
      if (lane == 0) atomicOr(&g_kvfb_error, KVFB_ERR_TIMEOUT);
      *abort_flag = 1;
    }
    // Never leave with copies in flight: once both producers are done, wait
    // (bounded) for the last stage put into each slot (no later stage reused
    // the slot, so its barrier parity is current).
    asm volatile("bar.sync 3, 64;" ::: "memory");
    if (pw == 0) {
      for (int s = 0; s < p.stages; ++s) {
        const int last = *reinterpret_cast<volatile int *>(&ms.slot_last[s]);
        volatile int never = 0;
        if (last >= 0 && !warp_wait(bar_full + 8u * s, (uint32_t)(last / p.stages) & 1u, &never) && lane == 0)
          atomicOr(&g_kvfb_error, KVFB_ERR_TIMEOUT);
      }
    }
  } else if (warp == kTcMmaWarp || warp == kTcValueWarp) {
    // --------------------------------------------------------- MMA issuers
    // One thread each: warp 10 issues a stage's score MMAs once its tiles
    // landed and its score buffer is free; warp 11 its value MMAs once all
    // softmax warps handed over the stage's P' planes (which they write
    // only after the stage's score MMAs completed).
    if (lane == 0) {
      bool ok = true;
      if (warp == kTcMmaWarp) {
        constexpr uint32_t ID_S = tc::idesc_i8(false, true, false, false, 128, NS);
        int s = 0;
        uint32_t ph = 0;
        for (int ns = 0; ns < ntiles; ++ns, s = (s + 1 == p.stages) ? (ph ^= 1u, 0) : s + 1) {
          const int j = ns & 1;
          if (!thread_wait(bar_full + 8u * s, ph, abort_flag) ||
              (ns >= 2 && !thread_wait(bar_sfree + 8u * j, (uint32_t)(((ns >> 1) - 1) & 1), abort_flag))) {
            ok = false;
            break;
          }
          tc::fence_after();
          const uint32_t sk = sbase + (uint32_t)s * p.stage_bytes;
#pragma unroll
          for (int g = 0; g < GPR; ++g)
#pragma unroll
            for (int kk = 0; kk < KPG; ++kk) {
              const int ks = g * KPG + kk;
              tc::mma_i8(tbase + (uint32_t)(j * SC + g * NS),
                         tc::smem_desc(sk + ks * 32u, 16u, 1024u, tc::kSwizzle128),
                         tc::smem_desc(sq + ks * 32u, 16u, 1024u, tc::kSwizzle128), ID_S, kk > 0);
            }
          tc::commit(bar_sfull + 8u * j);
        }
      } else {
        constexpr uint32_t ID_V = tc::idesc_i8(false, false, true, true, 128, NP);
        int s = 0;
        for (int npv = 0; npv < ntiles; ++npv, s = (s + 1 == p.stages) ? 0 : s + 1) {
          if (!thread_wait(bar_pready, (uint32_t)(npv & 1), abort_flag)) {
            ok = false;
            break;
          }
          tc::fence_after();
          const uint32_t sk = sbase + (uint32_t)s * p.stage_bytes;  // P' tile of the stage
          const uint32_t sv = sk + TB * 128u;
#pragma unroll
          for (int ks = 0; ks < TB / 32; ++ks)
            tc::mma_i8(tbase + 2u * SC, tc::smem_desc(sv + ks * 4096u, 16384u, 1024u, tc::kSwizzle128),
                       tc::smem_desc(sk + ks * 512u, 128u, 2048u, tc::kSwizzleNone), ID_V, ks > 0);
          tc::commit(bar_ofull);
          tc::commit(bar_empty + 8u * s);
        }
      }
      if (!ok) {
        atomicOr(&g_kvfb_error, KVFB_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      // Tensor memory is freed below only after every MMA issued here completed.
      const uint32_t bd = bar_done + 8u * (uint32_t)(warp - kTcMmaWarp);
      tc::commit(bd);
      if (!ptx::mbar_wait(bd, 0u, 1000000000ull)) atomicOr(&g_kvfb_error, KVFB_ERR_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax / fold warps
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;  // token of the stage / output dimension
    const uint32_t lane_base = tbase + ((uint32_t)(32 * quarter) << 16);
    const int gd = (row * GPR) / D;       // quantization group of this thread's dimension
    float mrun[HT], lrun[HT], zrun[HT][GPR], ocur[HT], aocur[HT], aoprev[HT];
#pragma unroll
    for (int e = 0; e < HT; ++e) {
      mrun[e] = kTcMinusBig;
      lrun[e] = 0.f;
      ocur[e] = 0.f;
      aocur[e] = aoprev[e] = 1.f;
#pragma unroll
      for (int g = 0; g < GPR; ++g) zrun[e][g] = 0.f;
    }
    float qinv[HT], qsum[HT][GPR];
#pragma unroll
    for (int e = 0; e < HT; ++e) {
      qinv[e] = ms.qinv[half * HT + e];
#pragma unroll
      for (int g = 0; g < GPR; ++g) qsum[e][g] = ms.qsum[half * HT + e][g];
    }
    int ev_run = 22;
    float finv_run = exp2i(-22);
    bool ok = true;

    // Loads this half's CH columns of each group from tensor memory.
    auto ld_cols = [&](uint32_t col0, uint32_t (&r)[GPR * CH]) {
#pragma unroll
      for (int g = 0; g < GPR; ++g) {
        const uint32_t ad = lane_base + col0 + (uint32_t)(g * NS + half * CH);
        if (CH == 8) {
          uint32_t t8[8];
          tc::ld8(ad, t8);
#pragma unroll
          for (int e = 0; e < 8; ++e) r[g * CH + e] = t8[e];
        } else {
          uint32_t t16[16];
          tc::ld16(ad, t16);
#pragma unroll
          for (int e = 0; e < 16; ++e) r[g * CH + e] = t16[e];
        }
      }
    };
    // Folds stage k's exact value product into the fp32 accumulators.
    auto fold = [&](int k, const float (&ao)[HT]) -> bool {
      if (!warp_wait(bar_ofull, (uint32_t)(k & 1), abort_flag)) return false;
      tc::fence_after();
      uint32_t r[CH];
      {
        const uint32_t ad = lane_base + 2u * SC + (uint32_t)(gd * NS + half * CH);
        if (CH == 8) {
          uint32_t t8[8];
          tc::ld8(ad, t8);
#pragma unroll
          for (int e = 0; e < 8; ++e) r[e] = t8[e];
        } else {
          uint32_t t16[16];
          tc::ld16(ad, t16);
#pragma unroll
          for (int e = 0; e < 16; ++e) r[e] = t16[e];
        }
      }
      tc::wait_ld();
      tc::fence_before();
      // Heads in pairs: planes 0 and 1 summed exactly in 32 bits (each
      // < 2^23), then one rounding, as fmaf(256, D1, D0) gives.
#pragma unroll
      for (int e = 0; e < HT; e += 2) {
        const uint32_t d0 = r[4 * e] + (r[4 * e + 1] << 8), d1 = r[4 * e + 4] + (r[4 * e + 5] << 8);
        const float2 v = fma2(make_float2(65536.f, 65536.f),
                              make_float2(__uint2float_rn(r[4 * e + 2]), __uint2float_rn(r[4 * e + 6])),
                              make_float2(__uint2float_rn(d0), __uint2float_rn(d1)));
        const float2 o = fma2(make_float2(ocur[e], ocur[e + 1]), make_float2(ao[e], ao[e + 1]), v);
        ocur[e] = o.x;
        ocur[e + 1] = o.y;
      }
      return true;
    };

    int s = 0;  // ring slot of stage i
    for (int i = 0; i < ntiles; ++i, s = (s + 1 == p.stages) ? 0 : s + 1) {
      const int j = i & 1;
      const int tok = t0 + i * TB + row;
      const bool valid = tok < t1;

      // ---- scores of this thread's token
      if (!warp_wait(bar_sfull + 8u * j, (uint32_t)((i >> 1) & 1), abort_flag)) {
        ok = false;
        break;
      }
      tc::fence_after();
      uint32_t sr[GPR * CH];
      ld_cols((uint32_t)(j * SC), sr);
      tc::wait_ld();
      tc::fence_before();
      __syncwarp();
      ptx::mbar_arrive_if(bar_sfree + 8u * j, lane == 0);

      // Metadata of this thread's token (rows past the chunk end were
      // zero-filled by the producers: zero scales and zero points).
      const uint32_t smk = sbase + (uint32_t)s * p.stage_bytes + 2u * TB * 128u;
      const uint32_t smv = smk + p.meta_bytes;
      uint32_t kw[GPR], vw[GPR];
      if (GPR == 1) {
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(kw[0]) : "r"(smk + 4u * row));
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(vw[0]) : "r"(smv + 4u * row));
      } else {
        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(kw[0]), "=r"(kw[GPR - 1]) : "r"(smk + 8u * row));
        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(vw[0]), "=r"(vw[GPR - 1]) : "r"(smv + 8u * row));
      }
      float ks[GPR], kz[GPR], vs[GPR], vz[GPR];
      uint32_t vbits = 0;
#pragma unroll
      for (int g = 0; g < GPR; ++g) {
        const float2 kf = meta_sz(kw[g]), vf = meta_sz(vw[g]);
        ks[g] = kf.x;
        kz[g] = kf.y;
        vs[g] = vf.x;
        vz[g] = vf.y;
        vbits = max(vbits, vw[g] & 0x7FFFu);  // fp16 bits of a positive scale order like the values
      }
      float sc[HT];
      float red[HT];
      // A row past the chunk end has zero scales, so its code term is 0; its
      // zero-point sum starts at -inf instead of 0, so its score is -inf
      // (valid rows: the same arithmetic as a sum started at 0).
      const float bias = valid ? 0.f : -INFINITY;
      // Heads in pairs (packed f32x2 arithmetic).
#pragma unroll
      for (int e = 0; e < HT; e += 2) {
        float2 acc = make_float2(0.f, 0.f), zq = make_float2(bias, bias);
#pragma unroll
        for (int g = 0; g < GPR; ++g) {
          const uint32_t *c = sr + g * CH;
          // |D0|, |D1| < 2^22: exact 32-bit sums, then one rounding.
          const int d0 = (int)c[e] + (int)(c[HT + e] << 8), d1 = (int)c[e + 1] + (int)(c[HT + e + 1] << 8);
          const float2 dg = fma2(make_float2(65536.f, 65536.f),
                                 make_float2(__int2float_rn((int)c[2 * HT + e]), __int2float_rn((int)c[2 * HT + e + 1])),
                                 make_float2(__int2float_rn(d0), __int2float_rn(d1)));
          acc = fma2(make_float2(ks[g], ks[g]), dg, acc);
          zq = fma2(make_float2(kz[g], kz[g]), make_float2(qsum[e][g], qsum[e + 1][g]), zq);
        }
        const float2 s2 = fma2(acc, make_float2(qinv[e], qinv[e + 1]), zq);
        sc[e] = s2.x;
        sc[e + 1] = s2.y;
        red[e] = sc[e];
        red[e + 1] = sc[e + 1];
      }
      // Warp maxima in one redux.sync each (scores as floats, the V-scale
      // bits as integers). Lane e then folds value e into its half's slot
      // with one 64-bit atomicMax whose high word is the stage number + 1, so
      // the slot (reused every second stage) needs no clearing: a stale
      // stage's entry always compares lower; a score goes in through an
      // order-preserving map of floats to unsigned integers (sign bit set for
      // >= 0, all bits flipped for < 0). A warp writes stage i + 2 only after
      // all four warps of its half arrived for stage i + 1, i.e. after they
      // read stage i.
      const uint32_t vbmax = __reduce_max_sync(0xffffffffu, vbits);
      float vsel = 0.f;
#pragma unroll
      for (int e = 0; e < HT; ++e) {
        float v;
        asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(v) : "f"(red[e]));
        vsel = (e == 0 || lane == e) ? v : vsel;
      }
      // the map: u | 2^31 for u >= 0, ~u for u < 0
      const uint32_t us = __float_as_uint(vsel);
      const uint32_t mine = lane < HT ? us ^ ((uint32_t)((int)us >> 31) | 0x80000000u) : vbmax;
      ptx::atom_max_u64_if(ptx::smem_u32(&ms.redx[j][half][min(lane, HT)]),
                           ((unsigned long long)(i + 1) << 32) | mine, lane <= HT);
      __syncwarp();
      ptx::mbar_arrive_if(bar_red + 8u * (2 * j + half), lane == 0);

      // ---- while the other warps of the half deliver their maxima: fold the
      // previous stage's value product. After it the value accumulator in
      // tensor memory is free for this stage's product, and this warp's P'
      // arrival for stage i (below) comes after it, so no warp can arrive
      // for stage i + 1 before every warp's stage-i arrival has completed
      // that phase (the value MMAs of stage i wait for it).
      if (i >= 1 && !fold(i - 1, aoprev)) {
        ok = false;
        break;
      }
      if (!warp_wait(bar_red + 8u * (2 * j + half), (uint32_t)((i >> 1) & 1), abort_flag)) {
        ok = false;
        break;
      }
      // Head and V-scale maxima over the four warps of this half (all tokens).
#pragma unroll
      for (int e = 0; e < HT; ++e) {
        // the inverse map: u & ~2^31 for u >= 2^31, ~u below
        const uint32_t u = (uint32_t)ms.redx[j][half][e];
        red[e] = __uint_as_float(u ^ (~(uint32_t)((int)u >> 31) | 0x80000000u));
      }
      const uint32_t vmax = (uint32_t)ms.redx[j][half][HT];

      // ---- online softmax, one rescale per stage; P' as 23-bit integers
      // ev = 23 - ceil(log2 vmax) (23 for a zero scale), within [-100, 100];
      // the scale is a positive fp16 or zero, exactly a normal float here.
      const uint32_t vu = __float_as_uint(__half2float(__ushort_as_half((unsigned short)vmax)));
      const int ev = vu == 0u ? 23 : max(min(150 - (int)(vu >> 23) - ((vu & 0x7FFFFFu) != 0u), 100), -100);
      const float fv = exp2i(ev);
      // 2^(ev - ev_run) as a product of two powers of two: exact while
      // |ev - ev_run| <= 126 (always, for scales within 2^100 of each other)
      const float fratio = fv * finv_run;
      finv_run = exp2i(-ev);
      ev_run = ev;
      // A masked row has zero scales (its metadata words were zeroed) and a
      // score of -inf, so p = 0 and every product below is 0 without a test;
      // the running maximum starts finite, so no exponent is ever inf - inf.
      float vsf[GPR];
#pragma unroll
      for (int g = 0; g < GPR; ++g) vsf[g] = vs[g] * fv;  // exact: fv is a power of two
      // P' = rint(p * vscale * 2^ev) < 2^23 (+1 at most, from the rounding of
      // p <= 1): the magic 2^23 added inside the FMA rounds the product to an
      // integer (floats in [2^23, 2^24) have a unit ulp), and the float's
      // three low bytes are that integer (2^23 itself becomes 2^24, whose low
      // bytes read 0x800000 all the same). The fourth byte (0x4B, exponent
      // bits) goes to the fourth column of the head, which the fold ignores.
      uint32_t pint[GPR][4];
#pragma unroll
      for (int g = 0; g < GPR; ++g) pint[g][2 % HT] = pint[g][3 % HT] = 0u;
#pragma unroll
      for (int e = 0; e < HT; e += 2) {
        const float2 mo = make_float2(mrun[e], mrun[e + 1]);
        const float2 mn = make_float2(fmaxf(mo.x, red[e]), fmaxf(mo.y, red[e + 1]));
        const float2 da = sub2(mo, mn), ds = sub2(make_float2(sc[e], sc[e + 1]), mn);
        const float2 alpha = make_float2(ex2_approx(da.x), ex2_approx(da.y));
        const float2 pr = make_float2(ex2_approx(ds.x), ex2_approx(ds.y));
        mrun[e] = mn.x;
        mrun[e + 1] = mn.y;
        const float2 l2 = fma2(make_float2(lrun[e], lrun[e + 1]), alpha, pr);
        lrun[e] = l2.x;
        lrun[e + 1] = l2.y;
        const float2 a2 = mul2(alpha, make_float2(fratio, fratio));
        aocur[e] = a2.x;
        aocur[e + 1] = a2.y;
#pragma unroll
        for (int g = 0; g < GPR; ++g) {
          const float2 z2 = fma2(make_float2(zrun[e][g], zrun[e + 1][g]), alpha, mul2(pr, make_float2(vz[g], vz[g])));
          zrun[e][g] = z2.x;
          zrun[e + 1][g] = z2.y;
          const float2 p2 = fma2(pr, make_float2(vsf[g], vsf[g]), make_float2(8388608.f, 8388608.f));
          pint[g][e] = __float_as_uint(p2.x);
          pint[g][e + 1] = __float_as_uint(p2.y);
        }
      }

      // ---- P' planes into the value operand tile (MN-major, 16-byte rows of
      // 16 columns per 8-token core matrix), over the stage's K tile: the
      // score MMAs that read it completed (sfull above), and the slot is
      // handed back to the producer only after the value MMAs.
      const uint32_t sp = sbase + (uint32_t)s * p.stage_bytes;
      const uint32_t rowoff = (uint32_t)(row >> 3) * 128u + (uint32_t)(row & 7) * 16u;
#pragma unroll
      for (int g = 0; g < GPR; ++g) {
        if (CH == 8) {
          asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(sp + (uint32_t)g * 2048u + rowoff + 8u * half),
                       "r"(pint[g][0]), "r"(pint[g][1])
                       : "memory");
        } else {
          asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(sp + (uint32_t)(2 * g + half) * 2048u + rowoff),
                       "r"(pint[g][0]), "r"(pint[g][1]), "r"(pint[g][2]), "r"(pint[g][3])
                       : "memory");
        }
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      ptx::mbar_arrive_if(bar_pready, lane == 0);

#pragma unroll
      for (int e = 0; e < HT; ++e) aoprev[e] = aocur[e];
    }
    if (ok && ntiles >= 1 && !fold(ntiles - 1, aoprev)) ok = false;
    if (!ok) {
      if (lane == 0) atomicOr(&g_kvfb_error, KVFB_ERR_TIMEOUT);
      *abort_flag = 1;
    }

    // ------------------------------------------------------------ epilogue
    // Token-side sums over the block, then one output column per thread.
#pragma unroll
    for (int e = 0; e < HT; ++e) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        lrun[e] += __shfl_xor_sync(0xffffffffu, lrun[e], off);
#pragma unroll
        for (int g = 0; g < GPR; ++g) zrun[e][g] += __shfl_xor_sync(0xffffffffu, zrun[e][g], off);
      }
      if (lane == 0) {
        ms.xl[warp][e] = lrun[e];
#pragma unroll
        for (int g = 0; g < GPR; ++g) ms.xz[warp][e][g] = zrun[e][g];
      }
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float finv = exp2i(max(min(-ev_run, 127), -126));
    const bool failed = *abort_flag != 0;
#pragma unroll
    for (int e = 0; e < HT; ++e) {
      const int hq = half * HT + e;
      if (hq < p.gq && !failed) {
        float L = 0.f, Z = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          L += ms.xl[half * 4 + w][e];
          Z += ms.xz[half * 4 + w][e][gd];
        }
        const float val = fmaf(ocur[e], finv, Z);
        const long long head = (long long)b * a.H + (long long)h * p.gq + hq;
        if (p.final_out) {
          a.out[head * D + row] = L > 0.f ? val / L : 0.f;
          if (row == 0 && a.lse) a.lse[head] = L > 0.f ? mrun[e] + log2f(L) : -INFINITY;
        } else {
          a.part_o[(head * p.splits + split) * D + row] = val;
          if (row == 0) {
            a.part_ml[(head * p.splits + split) * 2] = mrun[e] == kTcMinusBig ? -INFINITY : mrun[e];
            a.part_ml[(head * p.splits + split) * 2 + 1] = L;
          }
        }
      }
    }
    if (p.merge_in_kernel) {
      // Count this split in; the block that completes the count merges the
      // head's partials (log-sum-exp in log2 units, as decode_merge does) and
      // resets the counter for the next launch.
      unsigned *cnt = a.split_sem + 2 * ((long long)b * a.Hkv + h);
      __threadfence();
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (tid == 0) ms.last = atomicAdd(cnt, 1u) == (unsigned)(p.splits - 1) ? 1 : 0;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (ms.last) {
        __threadfence();
        const int S = p.splits;
        // Split weights 2^(m_s - M) and the merged denominator per query head,
        // one warp per head, into the (idle) stage ring: W[hq][s], Lsum[hq].
        float *W = reinterpret_cast<float *>(smem);
        float *Lsum = W + 8 * S;
        if (warp < p.gq) {
          const long long head = (long long)b * a.H + (long long)h * p.gq + warp;
          const float *ml = a.part_ml + head * S * 2;
          float M = -INFINITY;
          for (int sp = lane; sp < S; sp += 32) M = fmaxf(M, __ldcg(ml + 2 * sp));
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
          float L = 0.f;
          for (int sp = lane; sp < S; sp += 32) {
            const float2 v = __ldcg(reinterpret_cast<const float2 *>(ml) + sp);
            const float wgt = (M == -INFINITY || v.x == -INFINITY) ? 0.f : exp2f(v.x - M);
            W[warp * S + sp] = wgt;
            L = fmaf(v.y, wgt, L);
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
          if (lane == 0) {
            Lsum[warp] = L;
            if (a.lse) a.lse[head] = L > 0.f ? M + log2f(L) : -INFINITY;
          }
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        // out[d] = sum_s o_s[d] W[s] / L for this thread's column and heads;
        // loads issued in batches of 16 independent ones.
#pragma unroll
        for (int e = 0; e < HT; ++e) {
          const int hq = half * HT + e;
          if (hq >= p.gq) continue;
          const long long head = (long long)b * a.H + (long long)h * p.gq + hq;
          const float *po = a.part_o + head * (long long)S * D + row;
          const float *wq = W + hq * S;
          float O = 0.f;
          int sp = 0;
          for (; sp + 16 <= S; sp += 16) {
            float os[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) os[u] = __ldcg(po + (long long)(sp + u) * D);
#pragma unroll
            for (int u = 0; u < 16; ++u) O = fmaf(os[u], wq[sp + u], O);
          }
          for (; sp < S; ++sp) O = fmaf(__ldcg(po + (long long)sp * D), wq[sp], O);
          const float L = Lsum[hq];
          a.out[head * D + row] = L > 0.f ? O / L : 0.f;
        }
        if (tid == 0) *cnt = 0u;
      }
    }
    tc::fence_before();
  }

  __syncthreads();
  if (warp == kTcMmaWarp) {
    tc::fence_after();
    tc::dealloc(tbase, p.tmem_cols);
  }
}

} // namespace kvfb
