// tcgen05 GEMMs of the attention layer's two projections, reading and writing
// the head layout [B, H, T, D] directly (no reshape / transpose passes).
//
// Reference kernels replaced (cuda_transformer/):
//   kProjQkvFwd  getQKVmatrices  attention_qkv_kernels.cu:51-122
//   kProjQkvDw   qkvBackwardWB   attention_qkv_kernels.cu:164-241
//   kProjQkvDx   qkvBackward     attention_qkv_kernels.cu:283-362
//   kProjOutFwd  attentionProj   attention_proj_kernels.cu:48-98
//   kProjOutDw   projBackwardWB  attention_proj_kernels.cu:148-199
//   kProjOutDa   projBackward    attention_proj_kernels.cu:240-288
// Weights are read as the reference's kernels index them: W{q,k,v}[h*D+d, i]
// (row = output feature, attention_qkv_kernels.cu:92) and Wo[o, h*D+d]
// (attention_proj_kernels.cu:83).  Weight and bias gradients are ADDED into
// the caller's buffers (the reference atomically accumulates them); every
// other output is overwritten.
//
// One CTA computes one 128 x 128 fp32 tile in TMEM (one 128-row M tile, one
// 128-column N tile, one range of k-steps):
//   warp 0     TMA producer: per k-step one 128-byte-wide slab of A and of B
//              (K-major: 128 rows x 128 B; MN-major: 128/CB column blocks of
//              KB rows x 128 B), STAGES-deep ring;
//   warp 1     TMEM allocation and MMA issue (4 tcgen05.mma per k-step);
//   warps 2-5  epilogue: TMEM -> registers (+ bias) -> 128-byte-swizzled
//              staging tile in the (then idle) stage buffers -> TMA store, or
//              TMA reduce-add for the split-K fp32 weight gradients (16-bit
//              weight gradients: bf16x2 / f16x2 atomic adds from registers).
// The bias gradient rides on the weight-gradient GEMM: N tile 0 appends one
// column block of ones to B, so TMEM column 128 holds sum_k A[m, k] = db[m].
// M tiles of the row-wise GEMMs are (sequence, 128 rows) pairs, and every
// tensor map has T as its own dimension, so a tile never straddles two
// sequences and rows past T read as zero / are clipped on store.
//
// Numerics: fp32 operands go to kind::tf32 as stored (the tensor core uses
// their upper 19 bits); bf16 / fp16 to kind::f16; fp32 accumulation.
#pragma once

#include "sm100_primitives.cuh"

namespace ctfa {

enum ProjKind : int {
  kProjQkvFwd = 0,  // q|k|v[b,h,t,d] = sum_i x[b,t,i] W[h*D+d, i] + bias   (M = t, N = h*D+d, K = i)
  kProjOutFwd = 1,  // y[b,t,o] = sum_{h,d} a[b,h,t,d] Wo[o, h*D+d] + bo[o] (M = t, N = o, K = (h,d))
  kProjQkvDx = 2,   // dx[b,t,i] = sum_{w,h,d} dw[b,h,t,d] W_w[h*D+d, i]    (M = t, N = i, K = (w,h,d))
  kProjOutDa = 3,   // da[b,h,t,d] = sum_o dy[b,t,o] Wo[o, h*D+d]            (M = t, N = h*D+d, K = o)
  kProjQkvDw = 4,   // dW_w[n,i] += sum_{b,t} dw[b,h,t,d] x[b,t,i]          (M = n, N = i, K = (b,t))
  kProjOutDw = 5,   // dWo[o,j] += sum_{b,t} dy[b,t,o] a[b,h,t,d]           (M = o, N = j, K = (b,t))
};

struct ProjParams {
  int B, T, H, D;
  int E;            // model-side features: inputDim (QKV) / outputDim (output projection)
  int row_tiles;    // ceil(T / 128): M tiles per sequence of the row-wise kinds
  int m_tiles, n_tiles, splits;
  int ksteps;       // k-steps of the whole reduction
  int kt;           // weight-gradient kinds: k-steps per sequence, ceil(T / KB)
  const void* bias[3];  // forward kinds (DT), may be null
  void* dbias[3];       // weight-gradient kinds (DT, accumulated), may be null
  void* dw[3];          // weight-gradient kinds with 16-bit elements: the gradients themselves
  int relu;             // kProjOutFwd: y = max(y, 0) (a Linear layer followed by ReLU)
  const void* mask;     // kProjQkvDx: dx *= (mask > 0), mask [B, T, E] (backward of a ReLU before the layer)
  unsigned long long wait_limit_ns;
};

template <typename DT, int KIND, int STAGES>
struct ProjConfig {
  static constexpr int EB = (int)sizeof(DT);
  static constexpr int CB = 128 / EB;         // elements per 128-byte column block = K per stage
  static constexpr int KB = CB;
  static constexpr int NBLK = 128 / CB;       // column blocks across a 128-wide tile
  static constexpr int K_PER_MMA = KB / 4;    // 8 (tf32) / 16 (f16)
  static constexpr bool DW = (KIND == kProjQkvDw || KIND == kProjOutDw);
  static constexpr bool A_MN = DW;
  static constexpr bool B_MN = (KIND == kProjQkvDx || KIND == kProjOutDa || DW);
  static constexpr int TILE_BYTES = 128 * 128;
  static constexpr int ONES_BYTES = DW ? KB * 128 : 0;  // one MN-major column block of ones after B
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES + ONES_BYTES;
  static constexpr int N_EXTRA = DW ? CB : 0;
  static constexpr uint32_t TMEM_COLS = tmem_cols_for(128 + N_EXTRA);
  static constexpr int NUM_BARS = 2 * STAGES + 1;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 192;
  static_assert(STAGE_BYTES % 1024 == 0, "stages keep 1024-byte alignment (128-byte swizzle atoms)");
  static_assert(STAGES * STAGE_BYTES >= 128 * 128 * EB, "the epilogue staging tile reuses the stages");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

template <typename DT>
__device__ __forceinline__ float proj_to_float(DT x) {
  if constexpr (sizeof(DT) == 4) return x;
  else if constexpr (DTypeTraits<DT>::kFmt == 1) return __bfloat162float(x);
  else return __half2float(x);
}

template <typename DT>
__device__ __forceinline__ DT proj_from_float(float x) {
  if constexpr (sizeof(DT) == 4) return x;
  else if constexpr (DTypeTraits<DT>::kFmt == 1) return __float2bfloat16_rn(x);
  else return __float2half_rn(x);
}

template <typename DT, int KIND, int STAGES>
__global__ void __launch_bounds__(192, STAGES == 2 ? 3 : 2)
    proj_gemm_sm100(const __grid_constant__ CUtensorMap ta0, const __grid_constant__ CUtensorMap ta1,
                    const __grid_constant__ CUtensorMap ta2, const __grid_constant__ CUtensorMap tb0,
                    const __grid_constant__ CUtensorMap tb1, const __grid_constant__ CUtensorMap tb2,
                    const __grid_constant__ CUtensorMap to0, const __grid_constant__ CUtensorMap to1,
                    const __grid_constant__ CUtensorMap to2, const ProjParams p) {
  using C = ProjConfig<DT, KIND, STAGES>;
  constexpr int kKind = DTypeTraits<DT>::kKind;
  constexpr uint32_t kFmt = DTypeTraits<DT>::kFmt;
  constexpr bool kTF32 = (C::EB == 4);
  constexpr int CB = C::CB, KB = C::KB;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- tile of this CTA: N fastest, so CTAs sharing an A slab run together ----
  const int item = blockIdx.x;
  const int nt = item % p.n_tiles;
  const int rest = item / p.n_tiles;
  const int split = rest % p.splits;
  const int mt = rest / p.splits;
  const int ks_begin = (int)((long long)p.ksteps * split / p.splits);
  const int nk = (int)((long long)p.ksteps * (split + 1) / p.splits) - ks_begin;
  const int HD = p.H * p.D;

  int which = 0, b = 0, t0 = 0, m0 = 0, n0 = 0;
  if constexpr (!C::DW) {
    b = mt / p.row_tiles;
    t0 = (mt % p.row_tiles) * 128;
  } else if constexpr (KIND == kProjQkvDw) {
    const int per = p.m_tiles / 3;
    which = mt / per;
    m0 = (mt % per) * 128;
  } else {
    m0 = mt * 128;
  }
  if constexpr (KIND == kProjQkvFwd) {
    const int per = p.n_tiles / 3;
    which = nt / per;
    n0 = (nt % per) * 128;
  } else {
    n0 = nt * 128;
  }
  // per-output pointers picked without indexing the parameter arrays
  // dynamically (which would copy them to local memory)
  auto pick = [which](auto const (&arr)[3]) { return which == 0 ? arr[0] : which == 1 ? arr[1] : arr[2]; };
  const void* bias_w = pick(p.bias);
  void* dbias_w = pick(p.dbias);
  void* dw_w = pick(p.dw);
  const bool bias_col = C::DW && nt == 0 && dbias_w != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if constexpr (C::DW) {
    // ones column block after each stage's B slab (never overwritten by TMA)
    const uint32_t one = (C::EB == 4) ? 0x3F800000u : (kFmt == 1 ? 0x3F803F80u : 0x3C003C00u);
    for (int s = 0; s < STAGES; ++s) {
      uint4* dst = reinterpret_cast<uint4*>(smem + s * C::STAGE_BYTES + 2 * C::TILE_BYTES);
      for (int i = threadIdx.x; i < C::ONES_BYTES / 16; i += C::THREADS) dst[i] = make_uint4(one, one, one, one);
    }
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const uint64_t limit = p.wait_limit_ns;

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------
    if (lane == 0 && nk > 0) {
      auto tmA = [&](int w) { return w == 0 ? &ta0 : w == 1 ? &ta1 : &ta2; };
      auto tmB = [&](int w) { return w == 0 ? &tb0 : w == 1 ? &tb1 : &tb2; };
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1, abort_flag, limit, 1)) break;
        uint8_t* sa = smem + s * C::STAGE_BYTES;
        uint8_t* sb = sa + C::TILE_BYTES;
        mbar_arrive_expect_tx(&full[s], 2 * C::TILE_BYTES);
        const int ks = ks_begin + i;
        if constexpr (KIND == kProjQkvFwd) {
          tma_load_4d(sa, &ta0, &full[s], ks * KB, t0, b, 0);
          tma_load_4d(sb, tmB(which), &full[s], ks * KB, n0, 0, 0);
        } else if constexpr (KIND == kProjOutFwd) {
          const int per = p.D / KB, h = ks / per, d0 = (ks % per) * KB;
          tma_load_4d(sa, &ta0, &full[s], d0, t0, h, b);
          tma_load_4d(sb, &tb0, &full[s], h * p.D + d0, n0, 0, 0);
        } else if constexpr (KIND == kProjQkvDx) {
          const int per = p.D / KB, per_w = p.H * per;
          const int w = ks / per_w, r = ks % per_w, h = r / per, d0 = (r % per) * KB;
          tma_load_4d(sa, tmA(w), &full[s], d0, t0, h, b);
#pragma unroll
          for (int c = 0; c < C::NBLK; ++c)
            tma_load_4d(sb + c * KB * 128, tmB(w), &full[s], n0 + c * CB, h * p.D + d0, 0, 0);
        } else if constexpr (KIND == kProjOutDa) {
          tma_load_4d(sa, &ta0, &full[s], ks * KB, t0, b, 0);
#pragma unroll
          for (int c = 0; c < C::NBLK; ++c)
            tma_load_4d(sb + c * KB * 128, &tb0, &full[s], n0 + c * CB, ks * KB, 0, 0);
        } else if constexpr (KIND == kProjQkvDw) {
          const int bb = ks / p.kt, tt = (ks % p.kt) * KB;
#pragma unroll
          for (int c = 0; c < C::NBLK; ++c) {
            const int m = m0 + c * CB;
            tma_load_4d(sa + c * KB * 128, tmA(which), &full[s], m % p.D, tt, m / p.D, bb);
            tma_load_4d(sb + c * KB * 128, &tb0, &full[s], n0 + c * CB, tt, bb, 0);
          }
        } else {  // kProjOutDw
          const int bb = ks / p.kt, tt = (ks % p.kt) * KB;
#pragma unroll
          for (int c = 0; c < C::NBLK; ++c) {
            const int j = n0 + c * CB;
            tma_load_4d(sa + c * KB * 128, &ta0, &full[s], m0 + c * CB, tt, bb, 0);
            tma_load_4d(sb + c * KB * 128, &tb0, &full[s], j % p.D, tt, j / p.D, bb);
          }
        }
        issued = i + 1;
      }
      // On an aborted run some loads may still be landing: wait (bounded,
      // ignoring the abort flag) for the last load issued into each stage.
      if (*abort_flag) {
        const uint64_t w0 = globaltimer_ns();
        for (int j = max(0, issued - STAGES); j < issued; ++j)
          while (!mbar_try_wait(&full[j % STAGES], (j / STAGES) & 1) && globaltimer_ns() - w0 < limit) {
          }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // -------------------------------- MMA issue --------------------------------
    const uint32_t idesc = bias_col ? make_idesc(kFmt, 128, 128 + C::N_EXTRA, C::A_MN, C::B_MN)
                                    : make_idesc(kFmt, 128, 128, C::A_MN, C::B_MN);
    const uint32_t sbase = smem_u32(smem);
    for (int i = 0; i < nk; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait_warp(&full[s], (i / STAGES) & 1, abort_flag, limit, 2)) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t sa = sbase + s * C::STAGE_BYTES;
        const uint32_t sb = sa + C::TILE_BYTES;
        const uint64_t a0 = C::A_MN ? mnmajor_desc<kTF32>(sa, KB, 0, C::K_PER_MMA) : kmajor_desc(sa, 128, 0);
        const uint64_t b0 = C::B_MN ? mnmajor_desc<kTF32>(sb, KB, 0, C::K_PER_MMA) : kmajor_desc(sb, 128, 0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = desc_advance(a0, C::A_MN ? mnmajor_offset(kk, C::K_PER_MMA) : kmajor_offset(128, kk));
          const uint64_t bd = desc_advance(b0, C::B_MN ? mnmajor_offset(kk, C::K_PER_MMA) : kmajor_offset(128, kk));
          umma_ss<kKind>(tbase, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      __syncwarp();
    }
    // acc_full: every MMA issued so far has completed (also on an aborted
    // run, so that TMEM is idle before it is released).
    if (elect_one()) umma_commit(acc_full);
    __syncwarp();
    const uint64_t w0 = globaltimer_ns();
    while (!mbar_try_wait(acc_full, 0) && globaltimer_ns() - w0 < limit) {
    }
    __syncwarp();
  } else {
    // --------------------------------- epilogue ---------------------------------
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int r = quarter * 32 + lane;
    const uint32_t trow = tbase + ((uint32_t)(quarter * 32) << 16);
    uint8_t* stg = smem;  // staging tile: NBLK column blocks of 128 rows x 128 B
    // kProjQkvDx with a ReLU mask: fetch this row's 128 mask values while the
    // MMAs run and keep one bit per column (bit j of keep[c] = column 32c + j).
    uint32_t keep[4] = {~0u, ~0u, ~0u, ~0u};
    if constexpr (KIND == kProjQkvDx) {
      if (p.mask != nullptr && t0 + r < p.T) {
        const DT* mrow = static_cast<const DT*>(p.mask) + ((size_t)b * p.T + t0 + r) * p.E + n0;
        if (n0 + 128 <= p.E) {
          // whole 128-column span; the row start is 16-byte aligned (E * size % 16 == 0)
          constexpr int PER16 = 16 / C::EB;  // elements per 16-byte load
#pragma unroll
          for (int q = 0; q < 128 / PER16; ++q) {
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(mrow) + q);
            const DT* e = reinterpret_cast<const DT*>(&u);
#pragma unroll
            for (int t = 0; t < PER16; ++t) {
              const int col = q * PER16 + t;
              if (!(proj_to_float(e[t]) > 0.f)) keep[col >> 5] &= ~(1u << (col & 31));
            }
          }
        } else {
          for (int col = 0; col < 128; ++col)
            if (n0 + col < p.E && !(proj_to_float(mrow[col]) > 0.f)) keep[col >> 5] &= ~(1u << (col & 31));
        }
      }
    }
    bool ok = nk > 0 && mbar_wait(acc_full, 0, abort_flag, limit, 3);
    tc_fence_after();
    if constexpr (C::DW && C::EB == 2) {
      // 16-bit weight gradients: add the fp32 tile row into the gradient
      // through packed atomics (two elements per address).
      const int m = m0 + r;
      const int m_lim = (KIND == kProjQkvDw) ? HD : p.E;
      const int n_lim = (KIND == kProjQkvDw) ? p.E : HD;
      DT* g = static_cast<DT*>(dw_w);
      if (ok) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32f(trow + c * 32, v);
          tmem_wait_ld();
          if (m < m_lim) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int n = n0 + c * 32 + 2 * j;
              if (n < n_lim) {
                if constexpr (kFmt == 1)
                  atomicAdd(reinterpret_cast<__nv_bfloat162*>(g + (size_t)m * n_lim + n),
                            __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]));
                else
                  atomicAdd(reinterpret_cast<__half2*>(g + (size_t)m * n_lim + n),
                            __floats2half2_rn(v[2 * j], v[2 * j + 1]));
              }
            }
          }
        }
        if (bias_col) {
          uint32_t u[16];
          tmem_ld16(trow + 128, u);
          tmem_wait_ld();
          if (m < m_lim) atomicAdd(static_cast<DT*>(dbias_w) + m, proj_from_float<DT>(__uint_as_float(u[0])));
        }
      }
    } else {
    if (ok) {
      const DT* bias = nullptr;
      if constexpr (KIND == kProjQkvFwd || KIND == kProjOutFwd) bias = static_cast<const DT*>(bias_w);
      const int n_lim = (KIND == kProjQkvFwd) ? HD : p.E;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32f(trow + c * 32, v);
        tmem_wait_ld();
        if (bias != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = n0 + c * 32 + j;
            v[j] += (n < n_lim) ? proj_to_float(bias[n]) : 0.f;
          }
        }
        if constexpr (KIND == kProjOutFwd) {
          if (p.relu) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
          }
        }
        if constexpr (KIND == kProjQkvDx) {
          const uint32_t kb = keep[c];
          if (kb != ~0u) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (!((kb >> j) & 1u)) v[j] = 0.f;
          }
        }
        if constexpr (C::EB == 4) {
          uint8_t* row = stg + c * C::TILE_BYTES + r * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(row + ((j ^ (r & 7)) << 4)) =
                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
          uint8_t* row = stg + (c >> 1) * C::TILE_BYTES + r * 128;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t w[4];
#pragma unroll
            for (int h = 0; h < 4; ++h)
              w[h] = (kFmt == 1) ? pack_bf16x2(v[8 * j + 2 * h], v[8 * j + 2 * h + 1])
                                 : pack_f16x2(v[8 * j + 2 * h], v[8 * j + 2 * h + 1]);
            const int chunk = (c & 1) * 4 + j;
            *reinterpret_cast<uint4*>(row + ((chunk ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      if (bias_col) {
        uint32_t u[16];
        tmem_ld16(trow + 128, u);
        tmem_wait_ld();
        const int m = m0 + r;
        const int m_lim = (KIND == kProjQkvDw) ? HD : p.E;
        if (m < m_lim) atomicAdd(static_cast<DT*>(dbias_w) + m, proj_from_float<DT>(__uint_as_float(u[0])));
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(1, 128);
    if (warp == 2 && lane == 0 && ok && !*abort_flag) {
      const CUtensorMap* out_map = which == 0 ? &to0 : which == 1 ? &to1 : &to2;
#pragma unroll 1
      for (int c = 0; c < C::NBLK; ++c) {
        const void* src = stg + c * C::TILE_BYTES;
        const int n = n0 + c * CB;
        if constexpr (KIND == kProjQkvFwd || KIND == kProjOutDa) {
          if (n < HD) tma_store_4d(out_map, src, n % p.D, t0, n / p.D, b);
        } else if constexpr (KIND == kProjOutFwd || KIND == kProjQkvDx) {
          if (n < p.E) tma_store_4d(&to0, src, n, t0, b, 0);
        } else if constexpr (KIND == kProjQkvDw) {
          if (n < p.E) tma_reduce_add_4d(out_map, src, n, m0, 0, 0);
        } else {
          if (n < HD) tma_reduce_add_4d(&to0, src, n, m0, 0, 0);
        }
      }
      tma_store_commit();
      tma_store_wait_read();  // smem must stay valid until read; the writes complete with the grid
    }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

}  // namespace ctfa
