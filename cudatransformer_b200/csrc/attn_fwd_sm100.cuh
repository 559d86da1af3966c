// Flash-attention forward for sm_100a: TMA -> 128B-swizzled shared memory,
// tcgen05.mma with S and O accumulators in TMEM, online softmax in registers.
//
// Replaces the SIMT kernel `flashAttention<DType>` of the reference
// (cuda_transformer/flash_attention.cu:57-169), which streams 32-key tiles
// through shared memory with scalar dot products.  The math is the same
// online-softmax recurrence (running max, rescaled denominator, rescaled
// weighted sum: flash_attention.cu:120-153); what changes is where it runs:
//
//   CTA  = NQ query tiles of 128 rows of one (batch, head), sharing K/V tiles.
//   warps 0..4*NQ-1 : softmax, one warpgroup per query tile, one thread per
//                     query row (= TMEM lane).
//   warp  4*NQ      : TMA producer (Q once, then K tiles through KST stages and
//                     V tiles through VST stages, K one tile ahead of V: the
//                     S GEMM of tile j+1 needs K well before P V of tile j+1
//                     needs V).
//   warp  4*NQ+1    : tcgen05.mma issuer (one elected lane).
//   warps 4*NQ+2,3  : complete the producer warpgroup, which hands its
//                     registers to the softmax warpgroups via setmaxnreg.  For
//                     fp32 I/O (RND) they round every landed K/V tile to tf32
//                     (round to nearest) in shared memory before the MMAs read
//                     it and store it for the backward (each K/V tile by one
//                     designated CTA); the softmax warpgroups do the same for
//                     their Q tiles before the first S tile (Q by every CTA).
//
//   V is the MN-major B operand of P V: 128B swizzle for 16-bit types, the
//   32-byte-granule variant for tf32.
//
//   TMEM columns:  S_k = Q_k K^T  at [k*BN, (k+1)*BN)            (fp32)
//                  P_k written over S_k by the softmax warps       (tf32, or bf16/fp16 packed in pairs)
//                  O_k += P_k V   at [NQ*BN + k*HD, ... + HD)      (fp32)
//
// The MMA warp alternates the query tiles (ping-pong): while the softmax of
// tile 0 runs, the tensor core computes P_1 V and the next S_1, and vice versa.
// The running max is rescaled lazily: O is only rescaled when the max grows by
// more than 2^8 (log2 domain), which keeps the exponentials below 256.
//
// Masking: key j (local to the call) is visible to query i iff j < Tk and,
// when causal, j <= i + causal_offset.  The reference has no causal mode and
// treats keys past T as zero vectors that still enter the softmax
// (flash_attention.cu:104-109); here they are excluded.
#pragma once

#include "sm100_primitives.cuh"

namespace ctfa {

struct FwdParams {
  int BH;              // batch * heads
  int Tq, Tk;          // query rows / key rows handled by this call (per head)
  int q_row0, k_row0;  // first row of this call inside each head's allocation
  int q_rows_alloc;    // rows per head in the Q/O/LSE allocations
  int causal;          // 0: every key visible; 1: key j visible iff j <= i + causal_offset
  int causal_offset;
  int n_groups;        // CTA groups of NQ query tiles per head
  int head_chunk;      // causal: heads per chunk of the heavy-first block order (BH: one chunk)
  float scale_log2;    // softmax scale * log2(e)
  void* o;             // [BH][q_rows_alloc][HD] DT
  float* o_f32;        // when set: fp32 output rows here instead of o (block partials)
  float* lse;          // [BH][q_rows_alloc] natural-log logsumexp (nullable)
  int merge;           // with o_f32: o_f32 / lse hold a running (o, lse) of earlier key blocks,
                       // which this block is folded into (logsumexp-weighted) instead of overwriting
  int o_tma;           // O (not o_f32) covers whole heads: each tile is staged in shared memory and
                       // written by TMA stores through tm_o instead of per-row stores
  unsigned long long wait_limit_ns;
};

template <typename DT, int HD, int NQ, int BN, int KST, int VST>
struct FwdConfig {
  static constexpr int BM = 128;
  static constexpr int EB = (int)sizeof(DT);
  static constexpr int E128 = 128 / EB;           // elements per 128-byte row segment
  static constexpr int KBLK = HD * EB / 128;      // 128-byte column blocks per row
  static constexpr int Q_TILE_BYTES = BM * HD * EB;
  static constexpr int KV_TILE_BYTES = BN * HD * EB;
  static constexpr int KSTEP_S = HD * EB / 32;    // QK^T k-steps (32 bytes of head dim each)
  static constexpr int K_PER_PV = (EB == 4) ? 8 : 16;
  static constexpr int KSTEP_PV = BN / K_PER_PV;
  static constexpr int P_COLS = (EB == 4) ? BN : BN / 2;
  static constexpr uint32_t TMEM_COLS = tmem_cols_for(NQ * (BN + HD));
  static constexpr int NUM_BARS = 1 + 2 * KST + 2 * VST + 3 * NQ + 1 + (1 + KST + VST);
  static constexpr int SMEM_BYTES = 1024 + NQ * Q_TILE_BYTES + (KST + VST) * KV_TILE_BYTES + NUM_BARS * 8 + 16;
  // NQ softmax warpgroups + one producer warpgroup (TMA warp, MMA warp, two
  // spare warps) so that registers can be rebalanced per warpgroup.
  static constexpr int THREADS = NQ * 128 + 128;
  // The block launches at LAUNCH_REGS registers/thread (the launch bound's
  // share of the 64 K register file, in the allocator's steps of 8); the
  // producer warpgroup drops to 56 and the softmax warpgroups take the rest:
  // NQ = 2: 384 * 168 = 64512 >= 256 * 224 + 128 * 56;
  // NQ = 3: 512 * 128 = 65536 >= 384 * 152 + 128 * 56;
  // NQ = 4: 640 * 96 = 61440 >= 512 * 104 + 128 * 56.
  // The host checks the compiled register count against LAUNCH_REGS before
  // the first launch (a split above the launch's registers would never be
  // granted).
  static constexpr int LAUNCH_REGS = (65536 / THREADS) / 8 * 8 > 255 ? 248 : (65536 / THREADS) / 8 * 8;
  static constexpr bool REBALANCE = (NQ >= 2);
  static constexpr int PRODUCER_REGS = 56;
  static constexpr int SOFTMAX_REGS_RAW = (LAUNCH_REGS * THREADS - 128 * PRODUCER_REGS) / (NQ * 128) / 8 * 8;
  static constexpr int SOFTMAX_REGS = SOFTMAX_REGS_RAW > 248 ? 248 : SOFTMAX_REGS_RAW;
  static_assert(!REBALANCE || NQ * 128 * SOFTMAX_REGS + 128 * PRODUCER_REGS <= THREADS * LAUNCH_REGS,
                "register split");
  static_assert(HD * EB % 128 == 0, "head dim must fill whole 128-byte rows");
  static_assert(BN % 32 == 0 && BN <= 256, "key tile");
  static_assert(NQ * (BN + HD) <= 512, "TMEM budget");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

template <typename DT, int HD, int NQ, int BN, int KST, int VST, bool RND>
__global__ void __launch_bounds__(NQ * 128 + 128, 1)
    attn_fwd_sm100(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_qr,
                   const __grid_constant__ CUtensorMap tm_kr, const __grid_constant__ CUtensorMap tm_vr,
                   const __grid_constant__ CUtensorMap tm_o, const FwdParams p) {
  using C = FwdConfig<DT, HD, NQ, BN, KST, VST>;
  static_assert(!RND || C::EB == 4, "in-kernel rounding is for fp32 I/O");
  constexpr int BM = C::BM;
  constexpr int kKind = DTypeTraits<DT>::kKind;
  constexpr uint32_t kFmt = DTypeTraits<DT>::kFmt;
  constexpr int TMA_WARP = NQ * 4;
  constexpr int MMA_WARP = NQ * 4 + 1;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + NQ * C::Q_TILE_BYTES;
  uint8_t* sV = sK + KST * C::KV_TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + VST * C::KV_TILE_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + KST;
  uint64_t* v_full = k_empty + KST;
  uint64_t* v_empty = v_full + VST;
  uint64_t* s_full = v_empty + VST;
  uint64_t* p_full = s_full + NQ;
  uint64_t* o_full = p_full + NQ;
  uint64_t* done_bar = o_full + NQ;
  // RND: tiles rounded in shared memory (what the MMAs wait for instead of the TMA barriers)
  uint64_t* q_ready = done_bar + 1;
  uint64_t* k_ready = q_ready + 1;    // [KST]
  uint64_t* v_ready = k_ready + KST;  // [VST]
  uint64_t* q_go = RND ? q_ready : q_full;
  uint64_t* k_go = RND ? k_ready : k_full;
  uint64_t* v_go = RND ? v_ready : v_full;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(v_ready + VST);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work assignment: heavy query groups first under the causal mask ----
  int group, bh;
  if (p.causal) {
    int rank;
    head_chunked_item((int)blockIdx.x, p.BH, p.n_groups, p.head_chunk, rank, bh);
    group = p.n_groups - 1 - rank;
  } else {
    group = (int)(blockIdx.x % p.n_groups);
    bh = (int)(blockIdx.x / p.n_groups);
  }
  const int n_kv_all = (p.Tk + BN - 1) / BN;
  int n_kv[NQ];
  int n_max = 0;
#pragma unroll
  for (int k = 0; k < NQ; ++k) {
    const int qt = group * NQ + k;
    int n = 0;
    if (qt * BM < p.Tq) {
      n = n_kv_all;
      if (p.causal) {
        const int last_row = min(qt * BM + BM - 1, p.Tq - 1) + p.causal_offset;
        n = last_row < 0 ? 0 : min(n_kv_all, last_row / BN + 1);
      }
    }
    n_kv[k] = n;
    n_max = max(n_max, n);
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    // RND: a stage is empty once the MMAs read it and the rounding warps
    // finished with it (their store of the rounded tile included)
    for (int s = 0; s < KST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], RND ? 2 : 1);
      mbar_init(&k_ready[s], 64);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], RND ? 2 : 1);
      mbar_init(&v_ready[s], 64);
    }
    mbar_init(q_ready, NQ * 128);  // RND: the softmax warpgroups round Q
    for (int k = 0; k < NQ; ++k) {
      mbar_init(&s_full[k], 1);
      mbar_init(&p_full[k], 128);
      mbar_init(&o_full[k], 1);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const uint64_t limit = p.wait_limit_ns;
  // launched with programmatic serialization after the previous kernel on the
  // stream: nothing below may read the inputs or write the outputs before it
  // has completed
  grid_dep_wait();

  if (warp >= NQ * 4) {
    // --------------------------- producer warpgroup ---------------------------
    if constexpr (C::REBALANCE) regs_decrease<C::PRODUCER_REGS>();
  if (warp == TMA_WARP) {
    if (lane == 0 && n_max > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int q_bytes = 0;
#pragma unroll
      for (int k = 0; k < NQ; ++k) q_bytes += (n_kv[k] > 0) ? C::Q_TILE_BYTES : 0;
      mbar_arrive_expect_tx(q_full, q_bytes);
#pragma unroll
      for (int k = 0; k < NQ; ++k) {
        if (n_kv[k] == 0) continue;
        const int row = p.q_row0 + (group * NQ + k) * BM;
#pragma unroll
        for (int b = 0; b < C::KBLK; ++b)
          tma_load_3d(sQ + k * C::Q_TILE_BYTES + b * BM * 128, &tm_q, q_full, b * C::E128, row, bh);
      }
      int issued_k = 0, issued_v = 0;
      // slot t loads K_t and V_{t-1}: K runs one tile ahead of V
      for (int t = 0; t <= n_max; ++t) {
        if (t < n_max) {
          const int st = t % KST;
          if (!mbar_wait(&k_empty[st], ((t / KST) & 1) ^ 1, abort_flag, limit, 1)) break;
          mbar_arrive_expect_tx(&k_full[st], C::KV_TILE_BYTES);
#pragma unroll
          for (int b = 0; b < C::KBLK; ++b)
            tma_load_3d(sK + st * C::KV_TILE_BYTES + b * BN * 128, &tm_k, &k_full[st], b * C::E128,
                        p.k_row0 + t * BN, bh);
          issued_k = t + 1;
        }
        if (t >= 1) {
          const int j = t - 1;
          const int st = j % VST;
          if (!mbar_wait(&v_empty[st], ((j / VST) & 1) ^ 1, abort_flag, limit, 2)) break;
          mbar_arrive_expect_tx(&v_full[st], C::KV_TILE_BYTES);
#pragma unroll
          for (int b = 0; b < C::KBLK; ++b)
            tma_load_3d(sV + st * C::KV_TILE_BYTES + b * BN * 128, &tm_v, &v_full[st], b * C::E128,
                        p.k_row0 + j * BN, bh);
          issued_v = j + 1;
        }
      }
      // On an aborted run some loads may still be landing: wait (bounded,
      // ignoring the abort flag) for the last load issued into each stage.
      if (*abort_flag) {
        const uint64_t t0 = globaltimer_ns();
        for (int j = max(0, issued_k - KST); j < issued_k; ++j)
          while (!mbar_try_wait(&k_full[j % KST], (j / KST) & 1) && globaltimer_ns() - t0 < limit) {
          }
        for (int j = max(0, issued_v - VST); j < issued_v; ++j)
          while (!mbar_try_wait(&v_full[j % VST], (j / VST) & 1) && globaltimer_ns() - t0 < limit) {
          }
        while (!mbar_try_wait(q_full, 0) && globaltimer_ns() - t0 < limit) {
        }
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // The whole warp runs this loop; one elected lane issues each MMA group.
    if (n_max > 0) {
      constexpr uint32_t idesc_s = make_idesc(kFmt, 128, BN, false, false);
      constexpr uint32_t idesc_pv = make_idesc(kFmt, 128, HD, false, true);
      const uint32_t sQ_addr = smem_u32(sQ);
      const uint32_t sK_addr = smem_u32(sK);
      const uint32_t sV_addr = smem_u32(sV);

      auto issue_s = [&](int k, int st) {
        const uint32_t d = tbase + k * BN;
        const uint64_t a0 = kmajor_desc(sQ_addr + k * C::Q_TILE_BYTES, BM, 0);
        const uint64_t b0 = kmajor_desc(sK_addr + st * C::KV_TILE_BYTES, BN, 0);
#pragma unroll
        for (int ks = 0; ks < C::KSTEP_S; ++ks)
          umma_ss<kKind>(d, desc_advance(a0, kmajor_offset(BM, ks)), desc_advance(b0, kmajor_offset(BN, ks)), idesc_s,
                         ks > 0 ? 1u : 0u);
      };
      auto issue_pv = [&](int k, int st, bool acc) {
        const uint32_t d = tbase + NQ * BN + k * HD;
        const uint64_t b0 = mnmajor_desc<C::EB == 4>(sV_addr + st * C::KV_TILE_BYTES, BN, 0, C::K_PER_PV);
#pragma unroll
        for (int ks = 0; ks < C::KSTEP_PV; ++ks)
          umma_ts<kKind>(d, tbase + k * BN + ks * 8, desc_advance(b0, mnmajor_offset(ks, C::K_PER_PV)), idesc_pv,
                         (acc || ks > 0) ? 1u : 0u);
      };

      bool ok = mbar_wait_warp(q_go, 0, abort_flag, limit, 3);
      if (ok) ok = mbar_wait_warp(&k_go[0], 0, abort_flag, limit, 4);
      if (ok) {
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int k = 0; k < NQ; ++k) {
            if (n_kv[k] > 0) {
              issue_s(k, 0);
              umma_commit(&s_full[k]);
            }
          }
          umma_commit(&k_empty[0]);
        }
        __syncwarp();
      }
      for (int j = 0; ok && j < n_max; ++j) {
        const int st = j % VST;
        const int st1 = (j + 1) % KST;
        if (!(ok = mbar_wait_warp(&v_go[st], (j / VST) & 1, abort_flag, limit, 5))) break;
        bool next_k = false;
#pragma unroll
        for (int k = 0; k < NQ; ++k) {
          if (j >= n_kv[k]) continue;
          if (!(ok = mbar_wait_warp(&p_full[k], j & 1, abort_flag, limit, 6))) break;
          tc_fence_after();
          if (elect_one()) {
            issue_pv(k, st, j > 0);
            if (j == n_kv[k] - 1) umma_commit(&o_full[k]);
          }
          __syncwarp();
          if (j + 1 < n_kv[k]) {
            if (!next_k) {
              if (!(ok = mbar_wait_warp(&k_go[st1], ((j + 1) / KST) & 1, abort_flag, limit, 7))) break;
              tc_fence_after();
              next_k = true;
            }
            if (elect_one()) {
              issue_s(k, st1);
              umma_commit(&s_full[k]);
            }
            __syncwarp();
          }
        }
        if (elect_one()) {
          umma_commit(&v_empty[st]);
          if (next_k) umma_commit(&k_empty[st1]);
        }
        __syncwarp();
      }
      // Wait (bounded, regardless of abort) for every MMA issued so far, so
      // that TMEM is idle before it is released.
      if (elect_one()) umma_commit(done_bar);
      __syncwarp();
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(done_bar, 0) && globaltimer_ns() - t0 < limit) {
      }
    }
    __syncwarp();
  } else if constexpr (RND) {
    // ------------------ rounding warps (fp32 I/O, warps 4*NQ+2,3) ------------------
    const int sub = (warp - MMA_WARP - 1) * 32 + lane;  // 0..63
    const bool leader = (sub == 0);
    // Round a landed tile in place and make the writes visible to the async
    // proxy (tcgen05.mma, TMA store); the caller then arrives on the tile's
    // ready barrier (64 arrivals), which the MMA warp and the storing lane wait on.
    // Tiles are whole multiples of 256 16-byte vectors: four loads in flight
    // per thread.
    static_assert(C::Q_TILE_BYTES % (64 * 64) == 0 && C::KV_TILE_BYTES % (64 * 64) == 0, "rounding split");
    auto round_tile = [&](uint8_t* tile, int bytes) {
      float4* t4 = reinterpret_cast<float4*>(tile);
      for (int i = sub; i < bytes / 16; i += 4 * 64) {
        float4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = t4[i + u * 64];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          x[u].x = __uint_as_float(f32_to_tf32_rna(x[u].x));
          x[u].y = __uint_as_float(f32_to_tf32_rna(x[u].y));
          x[u].z = __uint_as_float(f32_to_tf32_rna(x[u].z));
          x[u].w = __uint_as_float(f32_to_tf32_rna(x[u].w));
          t4[i + u * 64] = x[u];
        }
      }
      fence_proxy_async_smem();
    };
    // K/V tile t of this head is stored by the one CTA whose query group
    // contains key row t*BN (it loads the tile under the causal mask too).
    auto designated = [&](int t) { return min((t * BN) / (NQ * BM), p.n_groups - 1) == group; };
    // (the Q tiles are rounded and stored by the softmax warpgroups, which
    // are idle until the first S tile)
    bool ok = n_max > 0;
    for (int t = 0; ok && t < n_max; ++t) {
      const bool mine = designated(t);
      const int kst = t % KST, vst = t % VST;
      if (!(ok = mbar_wait(&k_full[kst], (t / KST) & 1, abort_flag, limit, 43))) break;
      round_tile(sK + kst * C::KV_TILE_BYTES, C::KV_TILE_BYTES);
      mbar_arrive(&k_ready[kst]);
      if (leader) {
        if (mine && (ok = mbar_wait(&k_ready[kst], (t / KST) & 1, abort_flag, limit, 46))) {
#pragma unroll
          for (int b = 0; b < C::KBLK; ++b)
            tma_store_3d(&tm_kr, sK + kst * C::KV_TILE_BYTES + b * BN * 128, b * C::E128, p.k_row0 + t * BN, bh);
          tma_store_commit();
          tma_store_wait_read();
        }
        mbar_arrive(&k_empty[kst]);
      }
      if (!(ok = mbar_wait(&v_full[vst], (t / VST) & 1, abort_flag, limit, 44))) break;
      round_tile(sV + vst * C::KV_TILE_BYTES, C::KV_TILE_BYTES);
      mbar_arrive(&v_ready[vst]);
      if (leader) {
        if (mine && (ok = mbar_wait(&v_ready[vst], (t / VST) & 1, abort_flag, limit, 47))) {
#pragma unroll
          for (int b = 0; b < C::KBLK; ++b)
            tma_store_3d(&tm_vr, sV + vst * C::KV_TILE_BYTES + b * BN * 128, b * C::E128, p.k_row0 + t * BN, bh);
          tma_store_commit();
          tma_store_wait_read();
        }
        mbar_arrive(&v_empty[vst]);
      }
    }
    if (leader) tma_store_wait_all();
    __syncwarp();
  }  // without RND the two remaining warps of the producer warpgroup have no role
  } else {
    // ---------------------------- softmax warps ----------------------------
    if constexpr (C::REBALANCE) regs_increase<C::SOFTMAX_REGS>();
    const int k = threadIdx.x >> 7;          // query tile inside the CTA
    const int r = threadIdx.x & 127;         // row inside the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int qt = group * NQ + k;
    const int q_local = qt * BM + r;
    const int n = n_kv[k];
    const uint32_t s_addr = tbase + lane_off + k * BN;
    const uint32_t o_addr = tbase + lane_off + NQ * BN + k * HD;
    const float sl2 = p.scale_log2;
    bool q_stored = false;
    if constexpr (RND) {
      // Round this warpgroup's Q tile in place (four 16-byte loads in flight
      // per thread), then its thread 0 stores the rounded tile for the
      // backward.  Only tiles with keys to attend to were loaded (a CTA with
      // none loads no Q at all), so only their warpgroups wait for Q; the
      // whole warpgroup takes the named barrier whatever the wait returned,
      // so that no thread is left waiting on it.
      const bool qok = n > 0 && mbar_wait(q_full, 0, abort_flag, limit, 42);
      if (qok && n > 0) {
        float4* t4 = reinterpret_cast<float4*>(sQ + k * C::Q_TILE_BYTES);
        static_assert(C::Q_TILE_BYTES % (16 * 4 * 128) == 0, "Q rounding split");
        for (int i = r; i < C::Q_TILE_BYTES / 16; i += 4 * 128) {
          float4 x[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) x[u] = t4[i + u * 128];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            x[u].x = __uint_as_float(f32_to_tf32_rna(x[u].x));
            x[u].y = __uint_as_float(f32_to_tf32_rna(x[u].y));
            x[u].z = __uint_as_float(f32_to_tf32_rna(x[u].z));
            x[u].w = __uint_as_float(f32_to_tf32_rna(x[u].w));
            t4[i + u * 128] = x[u];
          }
        }
        fence_proxy_async_smem();
      }
      mbar_arrive(q_ready);
      if (n > 0) {
        named_bar_sync(1 + k, 128);
        if (r == 0 && qok) {
          const int row = p.q_row0 + qt * BM;
#pragma unroll
          for (int b = 0; b < C::KBLK; ++b)
            tma_store_3d(&tm_qr, sQ + k * C::Q_TILE_BYTES + b * BM * 128, b * C::E128, row, bh);
          tma_store_commit();
          q_stored = true;
        }
      }
    }
    float m = -INFINITY;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!(ok = mbar_wait(&s_full[k], j & 1, abort_flag, limit, 8))) break;
      tc_fence_after();
      const int key0 = j * BN;
      int vis = p.Tk - 1;  // last visible key for this row
      int vis_tile = p.Tk - 1;
      if (p.causal) {
        vis = min(vis, q_local + p.causal_offset);
        vis_tile = min(vis_tile, qt * BM + p.causal_offset);
      }
      const bool need_mask = key0 + BN - 1 > vis_tile;  // only diagonal / last tiles
      float sv[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32f(s_addr + c * 32, sv + c * 32);
      tmem_wait_ld();
      if (need_mask) {
        const int lim = vis - key0;  // columns > lim are masked
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c > lim) sv[c] = -INFINITY;
      }
      // row max: four independent chains
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < BN; c += 4) {
#pragma unroll
        for (int t = 0; t < 4; ++t) mx4[t] = fmaxf(mx4[t], sv[c + t]);
      }
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
      if (j == 0) {
        m = mx;
      } else {
        const bool need = mx > m + 8.f;
        if (__any_sync(0xffffffffu, need)) {
          const float m_new = fmaxf(m, mx);
          const float alpha = (m == -INFINITY) ? 0.f : ex2_approx(m - m_new);
          l *= alpha;
          m = m_new;
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            tmem_ld32f(o_addr + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32f(o_addr + c * 32, o);
          }
        }
      }
      const float m_use = (m == -INFINITY) ? 0.f : m;
      // p = exp2(s * scale*log2e - m): packed fp32x2 FMA, two row-sum chains;
      // masked columns hold -inf and give exactly 0.
      const float2 sl2x2 = make_float2(sl2, sl2);
      const float2 negm = make_float2(-m_use, -m_use);
      float2 rs2a = make_float2(0.f, 0.f), rs2b = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < BN; c += 4) {
        float2 y0 = __ffma2_rn(make_float2(sv[c], sv[c + 1]), sl2x2, negm);
        float2 y1 = __ffma2_rn(make_float2(sv[c + 2], sv[c + 3]), sl2x2, negm);
        y0.x = ex2_approx(y0.x);
        y0.y = ex2_approx(y0.y);
        y1.x = ex2_approx(y1.x);
        y1.y = ex2_approx(y1.y);
        sv[c] = y0.x;
        sv[c + 1] = y0.y;
        sv[c + 2] = y1.x;
        sv[c + 3] = y1.y;
        rs2a = __fadd2_rn(rs2a, y0);
        rs2b = __fadd2_rn(rs2b, y1);
      }
      l += (rs2a.x + rs2a.y) + (rs2b.x + rs2b.y);
      // P over the S columns: tf32 (rounded to nearest) in place, or packed pairs.
      if constexpr (C::EB == 4) {
#pragma unroll
        for (int c = 0; c < BN; ++c) sv[c] = __uint_as_float(f32_to_tf32_rna(sv[c]));
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_st32f(s_addr + c * 32, sv + c * 32);
      } else {
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t regs[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            regs[i] = (kFmt == 1) ? pack_bf16x2(sv[c * 32 + 2 * i], sv[c * 32 + 2 * i + 1])
                                  : pack_f16x2(sv[c * 32 + 2 * i], sv[c * 32 + 2 * i + 1]);
          tmem_st16(s_addr + c * 16, regs);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[k]);
    }
    // ------------------------------ epilogue ------------------------------
    // With o_tma the tile's 128 threads stage O in their Q buffer (its last
    // reader, the tile's last S MMA, completed before o_full) in the 128-byte
    // swizzled layout of tm_o, and one thread stores it with TMA: coalesced
    // lines instead of 128 rows written 16 bytes per lane.  Every thread of a
    // tile with keys takes both named barriers, whatever its waits returned.
    if (n > 0 && ok) ok = mbar_wait(&o_full[k], 0, abort_flag, limit, 9);
    bool o_stored = false;
    if (n > 0 && p.o_tma) {
      if (r == 0 && q_stored) tma_store_wait_read();  // the rounded-Q store has read the buffer
      named_bar_sync(1 + k, 128);
    }
    if (n > 0 && ok) {
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = q_local < p.Tq;
      const size_t row_index = (size_t)bh * p.q_rows_alloc + p.q_row0 + q_local;
      DT* orow = reinterpret_cast<DT*>(p.o) + row_index * HD;
      float* orow32 = p.o_f32 != nullptr ? p.o_f32 + row_index * HD : nullptr;
      // this block's logsumexp; with `merge`, the row's running (o, lse) and
      // this block's are combined as o = ca * o_run + cb * O with
      // ca = e^(lse_run - lse_new), cb = e^(lse_blk - lse_new) / l
      const float lse_blk = l > 0.f ? (((m == -INFINITY) ? 0.f : m) + __log2f(l)) * 0.69314718055994531f : -INFINITY;
      float ca = 0.f, cb = inv_l, lse_new = lse_blk;
      bool keep = false;  // no visible key in either: leave the running row as it is
      if (p.merge && row_ok && orow32 != nullptr) {
        const float lse_run = p.lse[row_index];
        const float mx = fmaxf(lse_run, lse_blk);
        if (mx == -INFINITY) {
          keep = true;
        } else {
          const float wa = __expf(lse_run - mx), wb = __expf(lse_blk - mx);
          const float inv = 1.f / (wa + wb);
          ca = wa * inv;
          cb = wb * inv * inv_l;
          lse_new = mx + __logf(wa + wb);
        }
      }
      if (p.o_tma) {
        uint8_t* tile = sQ + k * C::Q_TILE_BYTES;
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t regs[32];
          tmem_ld32(o_addr + c * 32, regs);
          tmem_wait_ld();
          // 32 columns: one 128-byte block (fp32) or half of one (16-bit),
          // 16-byte chunk j of row r at chunk position j ^ (r & 7)
          uint4 w[C::EB == 4 ? 8 : 4];
#pragma unroll
          for (int i = 0; i < (C::EB == 4 ? 8 : 4); ++i) {
            if constexpr (C::EB == 4) {
              w[i] = make_uint4(__float_as_uint(__uint_as_float(regs[4 * i]) * inv_l),
                                __float_as_uint(__uint_as_float(regs[4 * i + 1]) * inv_l),
                                __float_as_uint(__uint_as_float(regs[4 * i + 2]) * inv_l),
                                __float_as_uint(__uint_as_float(regs[4 * i + 3]) * inv_l));
            } else {
              uint32_t h4[4];
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const float a = __uint_as_float(regs[8 * i + 2 * h]) * inv_l;
                const float b = __uint_as_float(regs[8 * i + 2 * h + 1]) * inv_l;
                h4[h] = (kFmt == 1) ? pack_bf16x2(a, b) : pack_f16x2(a, b);
              }
              w[i] = make_uint4(h4[0], h4[1], h4[2], h4[3]);
            }
          }
          const int blk = C::EB == 4 ? c : c / 2;
          const int chunk0 = C::EB == 4 ? 0 : (c % 2) * 4;
          uint8_t* row = tile + blk * BM * 128 + r * 128;
#pragma unroll
          for (int i = 0; i < (C::EB == 4 ? 8 : 4); ++i)
            *reinterpret_cast<uint4*>(row + (((chunk0 + i) ^ (r & 7)) * 16)) = w[i];
        }
      } else {
  #pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t regs[32];
          tmem_ld32(o_addr + c * 32, regs);
          tmem_wait_ld();
          if (row_ok && orow32 != nullptr) {
            float4* dst = reinterpret_cast<float4*>(orow32 + c * 32);
            if (keep) continue;
            if (p.merge) {
  #pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float4 a = dst[i];
                dst[i] = make_float4(fmaf(a.x, ca, __uint_as_float(regs[4 * i]) * cb),
                                     fmaf(a.y, ca, __uint_as_float(regs[4 * i + 1]) * cb),
                                     fmaf(a.z, ca, __uint_as_float(regs[4 * i + 2]) * cb),
                                     fmaf(a.w, ca, __uint_as_float(regs[4 * i + 3]) * cb));
              }
            } else {
  #pragma unroll
              for (int i = 0; i < 8; ++i)
                dst[i] = make_float4(__uint_as_float(regs[4 * i]) * inv_l, __uint_as_float(regs[4 * i + 1]) * inv_l,
                                     __uint_as_float(regs[4 * i + 2]) * inv_l,
                                     __uint_as_float(regs[4 * i + 3]) * inv_l);
            }
          } else if (row_ok) {
            if constexpr (C::EB == 4) {
              float4* dst = reinterpret_cast<float4*>(orow + c * 32);
  #pragma unroll
              for (int i = 0; i < 8; ++i)
                dst[i] = make_float4(__uint_as_float(regs[4 * i]) * inv_l, __uint_as_float(regs[4 * i + 1]) * inv_l,
                                     __uint_as_float(regs[4 * i + 2]) * inv_l,
                                     __uint_as_float(regs[4 * i + 3]) * inv_l);
            } else {
              uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
  #pragma unroll
              for (int i = 0; i < 4; ++i) {
                uint32_t w[4];
  #pragma unroll
                for (int h = 0; h < 4; ++h) {
                  const float a = __uint_as_float(regs[8 * i + 2 * h]) * inv_l;
                  const float b = __uint_as_float(regs[8 * i + 2 * h + 1]) * inv_l;
                  w[h] = (kFmt == 1) ? pack_bf16x2(a, b) : pack_f16x2(a, b);
                }
                dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
              }
            }
          }
        }
      }
      if (row_ok && p.lse != nullptr && !keep) p.lse[row_index] = lse_new;
    }
    if (n > 0 && p.o_tma) {
      fence_proxy_async_smem();
      named_bar_sync(1 + k, 128);
      if (r == 0 && ok) {
        const int row = p.q_row0 + qt * BM;
#pragma unroll
        for (int b = 0; b < C::KBLK; ++b)
          tma_store_3d(&tm_o, sQ + k * C::Q_TILE_BYTES + b * BM * 128, b * C::E128, row, bh);
        tma_store_commit();
        o_stored = true;
      }
    }
    if (q_stored || o_stored) tma_store_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

}  // namespace ctfa
