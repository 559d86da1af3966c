// Flash-attention backward for sm_100a.
//
// Replaces the SIMT kernel `flashAttentionBackward<DType>` of the reference
// (cuda_transformer/flash_attention.cu:226-326).  The reference recomputes
// P from the saved max and denominator (:298), forms dS = P (dO.V - delta)/sqrt(D)
// (:299) and scatters dQ/dK/dV with atomics (:317-321); its dK/dV rows are
// wrong (it mixes the query index into key rows, :312-313).  Here the same
// recurrence is computed exactly with tensor cores, in three launches:
//
//   attn_bwd_prep     delta_i = sum_d O_i[d] dO_i[d]            (HBM-bound)
//   attn_bwd_dkdv     per key tile (128 keys, stationary K, V); streams
//                     128-query tiles (Q, dO) through ST stages:
//                       S^T  = K Q^T        (SS)   -> TMEM
//                       dP^T = V dO^T       (SS)   -> TMEM
//                       P^T  = exp2(S^T*scale*log2e - lse_q*log2e), masked
//                       dS^T = P^T (dP^T - delta_q)   (16-bit: the softmax
//                              scale is applied once, to dK in the epilogue;
//                              tf32: dS^T carries it)
//                       dV  += P^T dO       (TS, P^T from TMEM)
//                       dK  += dS^T Q       (TS, dS^T from TMEM)
//   attn_bwd_dq       per query tile (stationary Q, dO); streams K/V tiles:
//                       S  = Q K^T, dP = dO V^T (SS), dS = P (dP - delta)
//                       (row-wise lse/delta; packed fp32x2 math), dQ += dS K
//                       (TS, dS from TMEM), the softmax scale applied to dQ
//                       in the epilogue
//
// dQ is produced by its own query-stationary pass instead of atomics, so all
// three gradients are written once, deterministically, in the I/O type.
//
// Warp roles in both main kernels: compute warpgroups that split the 128
// score columns (thread = TMEM lane = row; dQ and 16-bit dK/dV: two groups
// of 64 columns, tf32 dK/dV: four of 32), then the TMA producer warp and the
// MMA-issuing warp.  The score buffer S is released as soon as the compute
// warps have it in registers, so the next S GEMM overlaps the exponentials of
// the current tile.  The tensor pipe takes a thread's next MMA only as it
// starts the previous one, so the MMA warp's issue order is chosen to keep
// it from waiting while a GEMM is ready (dK/dV: dV_g, S^T_{g+1}, dK_g,
// dP^T_{g+1}).
#pragma once

#include "sm100_primitives.cuh"

namespace ctfa {

struct BwdPrepParams {
  long long rows;    // BH * Tq_pad
  int Tq, Tq_pad;    // rows per head, and rounded up to a whole 128-row tile
  int q_rows_alloc;
  int q_row0;
  const void* o;
  const void* dO;
  const float* lse;  // [BH][q_rows_alloc] natural log
  float* ndelta;     // [BH][Tq_pad] -delta; 0 on padding rows
  float* nlse2;      // [BH][Tq_pad] -lse * log2(e); -inf on padding rows (their P is 0)
  float* dO_round;   // fp32 I/O only: round-to-nearest tf32 copy of dO (nullable)
  int* item_counters;  // [2] work-list counters of the dK/dV and dQ kernels, zeroed here
};

// slots of the work-list ring of the persistent dK/dV and dQ kernels (ItemRing)
constexpr int ITEM_SLOTS = 4;

struct BwdParams {
  int BH;
  int Tq, Tk;
  int Tq_pad;        // row stride of nlse2 / ndelta
  int q_row0, k_row0;
  int q_rows_alloc, k_rows_alloc;
  int causal, causal_offset;
  float scale;       // 1/sqrt(D)
  float scale_log2;  // log2(e)/sqrt(D)
  // Both negated, so that the compute warps form P and dS with packed adds /
  // FMAs: P = exp2(S * scale*log2e + nlse2), dS = P (dP + ndelta).
  const float* nlse2;   // [BH][Tq_pad] -lse * log2(e), -inf on padding rows
  const float* ndelta;  // [BH][Tq_pad] -delta, 0 on padding rows
  void* dq;          // [BH][q_rows_alloc][HD]
  void* dk;          // [BH][k_rows_alloc][HD]
  void* dv;
  int accumulate;    // 0: write dq/dk/dv in the I/O type; 1: add into fp32 dq/dk/dv buffers
  int dkdv_head_chunk;  // heads per chunk of the dK/dV item order (BH: one chunk)
  int dq_head_chunk;    // heads per chunk of the dQ item order
  int* item_counters;   // [2] next unclaimed dK/dV item, dQ item (zeroed by the delta pass)
  unsigned long long wait_limit_ns;
};

template <typename DT>
__device__ __forceinline__ float load_as_float(const DT* p) {
  if constexpr (sizeof(DT) == 4)
    return *reinterpret_cast<const float*>(p);
  else if constexpr (std::is_same<DT, __nv_bfloat16>::value)
    return __bfloat162float(*p);
  else
    return __half2float(*p);
}

// delta = rowsum(O * dO) in fp32, a group of 4-16 threads per query row, each
// thread loading two 16-byte vectors of O and of dO (with a full wave of
// 256-thread blocks, enough bytes in flight per SM to keep HBM busy; four
// vectors per thread measured 0.058 vs 0.048 ms at B=16 H=16 T=2048 D=128
// bf16, eight 0.088, and the same 0.017 ms at config 2).  For fp32 I/O it
// also writes the tf32-rounded dO that the MMAs read, and forms delta from
// that same rounded dO, so that
// sum_j P_ij dP_ij == delta_i holds for the values the tensor cores see (dS
// then cancels exactly where it should).
template <typename DT, int HD>
struct PrepShape {
  static constexpr int VEC = 16 / (int)sizeof(DT);  // elements per 16-byte vector
  static constexpr int NV = HD / VEC;               // vectors per row
  static constexpr int VPT = 2;                     // vectors per thread
  static constexpr int TPR = NV / VPT;              // threads per row
  static_assert(TPR >= 1 && TPR <= 32 && (32 % TPR) == 0, "row group must tile a warp");
};

template <typename DT>
__device__ __forceinline__ void vec_to_float(const uint4& u, float* f) {
  if constexpr (sizeof(DT) == 4) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<DT, __nv_bfloat16>::value) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      } else {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        const float2 x = __half22float2(h);
        f[2 * i] = x.x;
        f[2 * i + 1] = x.y;
      }
    }
  }
}

template <typename DT, int HD>
__device__ __forceinline__ void attn_bwd_prep_rowgroup(const BwdPrepParams& p, long long t) {
  using S = PrepShape<DT, HD>;
  constexpr int VEC = S::VEC, TPR = S::TPR, VPT = S::VPT;
  const long long w = t / TPR;  // padded query row
  const int sub = (int)(t % TPR);
  // whole row groups share a warp; every lane reaches the shuffles below
  const bool in = w < p.rows;
  const long long bh = in ? w / p.Tq_pad : 0, i = in ? w % p.Tq_pad : 0;
  const bool real = in && i < p.Tq;
  float s = 0.f;
  if (real) {
    const size_t row = ((size_t)bh * p.q_rows_alloc + p.q_row0 + i) * HD;
    const uint4* o4 = reinterpret_cast<const uint4*>(reinterpret_cast<const DT*>(p.o) + row);
    const uint4* g4 = reinterpret_cast<const uint4*>(reinterpret_cast<const DT*>(p.dO) + row);
    uint4 ov[VPT], gv[VPT];
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      ov[v] = __ldcs(o4 + sub + v * TPR);
      gv[v] = __ldcs(g4 + sub + v * TPR);
    }
    float* gr = p.dO_round != nullptr ? p.dO_round + row : nullptr;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      float of[VEC], gf[VEC];
      vec_to_float<DT>(ov[v], of);
      vec_to_float<DT>(gv[v], gf);
      if constexpr (sizeof(DT) == 4) {
        if (gr != nullptr) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) gf[e] = __uint_as_float(f32_to_tf32_rna(gf[e]));
          reinterpret_cast<float4*>(gr)[sub + v * TPR] = make_float4(gf[0], gf[1], gf[2], gf[3]);
        }
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) s = fmaf(of[e], gf[e], s);
    }
  }
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (in && sub == 0) {
    if (real) {
      p.ndelta[w] = -s;
      p.nlse2[w] = p.lse[bh * p.q_rows_alloc + p.q_row0 + i] * -1.4426950408889634f;
    } else {  // padding row of the last tile
      p.ndelta[w] = 0.f;
      p.nlse2[w] = -INFINITY;
    }
  }
}

// Grid-stride over row groups with one resident wave of blocks (a grid of
// rows * TPR / 256 blocks left the last wave ~30 % full at config 2); the
// loop advances whole warps, so every lane reaches the shuffles below.
template <typename DT, int HD>
__global__ void __launch_bounds__(256) attn_bwd_prep(BwdPrepParams p) {
  constexpr int TPR = PrepShape<DT, HD>::TPR;
  // launched with programmatic serialization after the forward: o and lse
  // are read only once it has completed
  grid_dep_wait();
  if (blockIdx.x == 0 && threadIdx.x == 0) {  // work-list counters of the dK/dV and dQ kernels that follow
    p.item_counters[0] = 0;
    p.item_counters[1] = 0;
  }
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long total = p.rows * TPR;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t - (threadIdx.x & 31) < total; t += stride)
    attn_bwd_prep_rowgroup<DT, HD>(p, t);
}

template <typename DT, int HD>
struct BwdConfig {
  static constexpr int EB = (int)sizeof(DT);
  static constexpr bool TF32 = (EB == 4);
  static constexpr int E128 = 128 / EB;
  static constexpr int KBLK = HD * EB / 128;          // 128-byte column blocks per row
  static constexpr int KSTEP_S = HD * EB / 32;        // k-steps over the head dim (32 bytes each)
  static constexpr int K_PER = TF32 ? 8 : 16;         // reduction rows per TS MMA
  static constexpr int ROW_BYTES = HD * EB;
  // dK/dV kernel: 128 stationary keys (MMA M); streamed query tiles of KV_QT
  // rows.  128 for every type: the S^T / dP^T MMAs are then N=128 (twice the
  // work of an N=64 MMA for ~1.35x its time; the MMA-issuing warp, which
  // bounds this kernel, issues 25 % fewer MMAs and half the waits per query).
  static constexpr int KV_KEYS = 128;
  static constexpr int KV_QT = 128;
  // dQ kernel: 128 stationary queries; streamed key tiles of Q_KT rows (128:
  // N=128 MMAs run at ~1.7x the per-MAC rate of N=64 ones, and the per-tile
  // barrier / TMEM round trips are amortised over twice the keys).
  static constexpr int Q_ROWS = 128;
  static constexpr int Q_KT = (TF32 && HD > 64) ? 64 : 128;
  // tf32 operands read both K-major and MN-major get a second copy in the
  // 32-byte-granule swizzle; 16-bit operands serve both from one buffer.
  static constexpr int BIG_TILE = 128 * ROW_BYTES;
  static constexpr int KV_QTILE = KV_QT * ROW_BYTES;
  static constexpr int Q_KTILE = Q_KT * ROW_BYTES;
  static constexpr int KV_STAGE_BYTES = (TF32 ? 4 : 2) * KV_QTILE;  // Q, dO (+ MN copies)
  // A stage's query tiles are released in KV_PARTS groups, each after its
  // last reader: tf32 (one stage fits) Q after S^T, dO after dP^T, the dO MN
  // copy after dV, the Q MN copy after dK, so every tile of the next query
  // tile loads while the current one is still in use; 16-bit (2-3 stages)
  // releases Q and dO together after dK.
  static constexpr int KV_PARTS = TF32 ? 4 : 1;
  static constexpr int Q_KSTAGE_BYTES = (TF32 ? 2 : 1) * Q_KTILE;   // K (+ K MN copy)
  static constexpr int Q_VSTAGE_BYTES = Q_KTILE;                    // V
  static constexpr int BUDGET = 216 * 1024;
  static constexpr int KV_ST = (BUDGET - 2 * BIG_TILE) / KV_STAGE_BYTES > 3 ? 3 : (BUDGET - 2 * BIG_TILE) / KV_STAGE_BYTES;
  // dQ kernel rings: K (+ its MN copy) and V separately.  tf32 at 128-key
  // tiles: two K stages (the next S needs K(j+1) while dQ(j) still reads
  // Km(j)) and one V stage (V(j+1) loads while dQ(j) runs, before dP(j+1)).
  static constexpr int Q_BUDGET = 226 * 1024;
  static constexpr int Q_PAIR = (Q_BUDGET - 2 * BIG_TILE) / (Q_KSTAGE_BYTES + Q_VSTAGE_BYTES);
  static constexpr int Q_KST = TF32 ? 2 : (Q_PAIR > 3 ? 3 : Q_PAIR);
  static constexpr int Q_VST = TF32 ? 1 : Q_KST;
  // dK/dV kernel TMEM map (columns, lanes = keys).  S^T, then the dP^T buffer
  // (dS^T after the compute pass: tf32 in place; 16-bit: dS^T|P^T packed per
  // half), then for tf32 the P^T buffer (EARLY_P: the compute warps store P^T
  // right after the exponentials and release it, so dV (+)= P^T dO runs while
  // they form dS^T; only dK waits for dS^T; P^T of tile g overwrites that of
  // tile g-1 once S^T of tile g completed, which dV of tile g-1 precedes in
  // the MMA stream), then the dK and dV accumulators.
  // A second dP^T buffer (so the next dP^T GEMM is queued before the compute
  // warps release the current one) measured 4-8% slower: thread-side TMEM
  // loads/stores take ~4x longer while the tensor pipe is busy.
  // Compute warpgroups of the dK/dV kernel (thread = key row x KV_HALF query
  // columns) plus the TMA and MMA warps.  tf32: four (576 threads, 96
  // registers each), so that each SM sub-partition interleaves four warps'
  // TMEM load -> exp / dS -> TMEM store chains (0.094 -> 0.089 ms at config
  // 2; handing the producer warps' registers over with setmaxnreg made their
  // 56-register loops spill).
  static constexpr int KV_GROUPS = TF32 ? 4 : 2;
  static constexpr int KV_HALF = KV_QT / KV_GROUPS;  // score columns per compute warpgroup
  static constexpr int KV_THREADS = KV_GROUPS * 128 + 64;
  static_assert(KV_GROUPS == 2 || HD == 64, "four compute groups split the dK|dV epilogue in 32-column quarters");
  static constexpr bool EARLY_P = TF32;
  static constexpr int KV_S = 0;
  static constexpr int KV_DP = KV_QT;
  static constexpr int KV_DK = TF32 ? 3 * KV_QT : 2 * KV_QT;
  static constexpr int KV_DV = KV_DK + HD;
  static constexpr uint32_t KV_TMEM = tmem_cols_for(KV_DV + HD);
  // P^T: tf32 its own buffer; 16-bit packed into the dP^T buffer
  __host__ __device__ static constexpr int kv_p() { return TF32 ? 2 * KV_QT : KV_DP + KV_HALF / 2; }
  // dQ kernel TMEM map (lanes = queries): S, then a dP buffer (dS after the
  // compute pass: tf32 in place, 16-bit packed per half), then the dQ
  // accumulator.
  static constexpr int Q_HALF = Q_KT / 2;
  static constexpr int Q_S = 0;
  static constexpr int Q_DQ = 2 * Q_KT;
  static constexpr uint32_t Q_TMEM = tmem_cols_for(Q_DQ + HD);
  __host__ __device__ static constexpr int q_dp(int b) { return Q_KT + b * Q_KT; }
  // dK/dV kernel, 16-bit I/O: the per-query rows (nlse2, ndelta) of each
  // streamed query tile, staged by the TMA warp in a ring of LD_SLOTS slots
  // (each 2 x KV_QT floats) and released by the compute warps after the
  // tile's dS pass, so that the compute warps read them from shared memory
  // instead of L2, and form P / dS with packed fp32x2 FMAs, adds and
  // multiplies, the softmax scale applied to dK in the epilogue (config 3:
  // dK/dV 0.712 -> 0.69 ms).  tf32 keeps its rows in registers, loaded from
  // L2 before each S^T wait, and scalar math: its four compute warpgroups
  // run at 96 registers (five warps per SM sub-partition), and the ring and
  // packed forms measured ~4 % slower there (0.089 -> 0.093 ms at config 2).
  static constexpr bool ROWS_RING = !TF32;
  static constexpr int LD_SLOTS = 4;
  static constexpr int LD_BYTES = 2 * KV_QT * 4;
  static constexpr int NUM_BARS = 40;
  // after the barriers: TMEM address, abort flag, work-list ring
  static constexpr int TAIL_BYTES = 8 + 4 * ITEM_SLOTS;
  static constexpr int KV_SMEM = 1024 + 2 * BIG_TILE + KV_ST * KV_STAGE_BYTES + (ROWS_RING ? LD_SLOTS * LD_BYTES : 0) +
                                 NUM_BARS * 8 + TAIL_BYTES;
  static constexpr int Q_SMEM =
      1024 + 2 * BIG_TILE + Q_KST * Q_KSTAGE_BYTES + Q_VST * Q_VSTAGE_BYTES + NUM_BARS * 8 + TAIL_BYTES;
  static constexpr int THREADS = 320;  // dQ kernel: 8 compute warps, TMA warp, MMA warp
  static_assert(KV_ST >= 1 && Q_KST >= 1 && Q_VST >= 1, "shared memory budget");
  static_assert(10 + 2 * KV_PARTS * KV_ST + 2 * LD_SLOTS + 2 * ITEM_SLOTS <= NUM_BARS, "dK/dV kernel barriers");
  static_assert(9 + 2 * Q_KST + 2 * Q_VST + 2 * ITEM_SLOTS <= NUM_BARS, "dQ kernel barriers");
  static_assert(KV_SMEM <= 232448, "dK/dV kernel shared memory");
  static_assert(Q_SMEM <= 232448, "dQ kernel shared memory");
  static_assert(KV_DV + HD <= 512 && Q_DQ + HD <= 512, "TMEM budget");
  static_assert(HD * EB % 128 == 0, "head dim must fill whole 128-byte rows");
  static_assert(KV_HALF % 32 == 0 && Q_HALF % 32 == 0, "compute halves are whole 32-column TMEM loads");

  // TMEM column of the A operand for k-step ks of a TS MMA whose A operand was
  // written by the two compute warpgroups.  tf32: contiguous fp32 columns.
  // 16-bit: each warpgroup packed its half (half_cols fp32 columns -> half_cols/2
  // packed columns) at the start of its own half.
  __device__ static constexpr uint32_t a_col(int ks, int half_cols) {
    return TF32 ? (uint32_t)(ks * 8)
                : (uint32_t)((ks / (half_cols / 16)) * half_cols + (ks % (half_cols / 16)) * 8);
  }
};

// Load `cols` fp32 TMEM columns starting at taddr into v[].
template <int N>
__device__ __forceinline__ void tmem_load_row(uint32_t taddr, float (&v)[N]) {
#pragma unroll
  for (int c = 0; c < N / 32; ++c) tmem_ld32f(taddr + c * 32, v + c * 32);
  tmem_wait_ld();
}

// Store v[] as an MMA A operand: tf32 (one column per value, rounded to
// nearest) or packed bf16/fp16 pairs (N/2 columns).
template <typename DT, int N>
__device__ __forceinline__ void tmem_store_operand(uint32_t taddr, const float (&v)[N]) {
  if constexpr (sizeof(DT) == 4) {
#pragma unroll
    for (int c = 0; c < N / 32; ++c) {
      uint32_t regs[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) regs[i] = f32_to_tf32_rna(v[c * 32 + i]);
      tmem_st32(taddr + c * 32, regs);
    }
  } else {
#pragma unroll
    for (int c = 0; c < N / 64; ++c) {
      uint32_t regs[32];
#pragma unroll
      for (int i = 0; i < 32; ++i)
        regs[i] = std::is_same<DT, __nv_bfloat16>::value ? pack_bf16x2(v[c * 64 + 2 * i], v[c * 64 + 2 * i + 1])
                                                         : pack_f16x2(v[c * 64 + 2 * i], v[c * 64 + 2 * i + 1]);
      tmem_st32(taddr + c * 32, regs);
    }
    if constexpr (N % 64 == 32) {
      uint32_t regs[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        regs[i] = std::is_same<DT, __nv_bfloat16>::value ? pack_bf16x2(v[N - 32 + 2 * i], v[N - 32 + 2 * i + 1])
                                                         : pack_f16x2(v[N - 32 + 2 * i], v[N - 32 + 2 * i + 1]);
      tmem_st16(taddr + (N / 64) * 32, regs);
    }
  }
}

// Add `COLS` fp32 TMEM columns of this thread's lane, times `mul`, into a row
// of an fp32 buffer (the block entry points accumulate over ring steps; each
// CTA owns its rows within one launch, so no atomics).
template <int COLS>
__device__ __forceinline__ void tmem_row_accumulate(uint32_t taddr, float* dst, bool store, float mul) {
#pragma unroll
  for (int c = 0; c < COLS / 32; ++c) {
    uint32_t regs[32];
    tmem_ld32(taddr + c * 32, regs);
    tmem_wait_ld();
    if (!store) continue;
    float4* d4 = reinterpret_cast<float4*>(dst + c * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 a = d4[i];
      a.x = fmaf(__uint_as_float(regs[4 * i]), mul, a.x);
      a.y = fmaf(__uint_as_float(regs[4 * i + 1]), mul, a.y);
      a.z = fmaf(__uint_as_float(regs[4 * i + 2]), mul, a.z);
      a.w = fmaf(__uint_as_float(regs[4 * i + 3]), mul, a.w);
      d4[i] = a;
    }
  }
}

// Write `cols` (multiple of 32) fp32 TMEM columns of this thread's lane, times
// `mul`, to a row of DT in global memory (zeros when `zero`).
template <typename DT, int COLS>
__device__ __forceinline__ void tmem_row_to_global(uint32_t taddr, DT* dst, bool store, bool zero, float mul) {
#pragma unroll
  for (int c = 0; c < COLS / 32; ++c) {
    uint32_t regs[32];
    if (!zero) {
      tmem_ld32(taddr + c * 32, regs);
      tmem_wait_ld();
      if (mul != 1.f) {
#pragma unroll
        for (int i = 0; i < 32; ++i) regs[i] = __float_as_uint(__uint_as_float(regs[i]) * mul);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) regs[i] = 0u;
    }
    if (!store) continue;
    if constexpr (sizeof(DT) == 4) {
      float4* d4 = reinterpret_cast<float4*>(dst + c * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        d4[i] = make_float4(__uint_as_float(regs[4 * i]), __uint_as_float(regs[4 * i + 1]),
                            __uint_as_float(regs[4 * i + 2]), __uint_as_float(regs[4 * i + 3]));
    } else {
      uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float a = __uint_as_float(regs[8 * i + 2 * h]);
          const float b = __uint_as_float(regs[8 * i + 2 * h + 1]);
          w[h] = std::is_same<DT, __nv_bfloat16>::value ? pack_bf16x2(a, b) : pack_f16x2(a, b);
        }
        d4[i] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

// Load `COLS` fp32 TMEM columns of this thread's lane into registers (one
// wait for all of them).
template <int COLS>
__device__ __forceinline__ void tmem_row_load(uint32_t taddr, uint32_t (&r)[COLS]) {
#pragma unroll
  for (int c = 0; c < COLS / 32; ++c) tmem_ld32(taddr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(r + c * 32));
  tmem_wait_ld();
}

// Write a row of COLS fp32 values (register bits) to global memory: as DT, or
// added into an fp32 row (`accumulate`, block entry points).
template <typename DT, int COLS>
__device__ __forceinline__ void row_store(const uint32_t (&r)[COLS], void* dst, bool accumulate) {
  if (accumulate) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int i = 0; i < COLS / 4; ++i) {
      float4 a = d4[i];
      a.x += __uint_as_float(r[4 * i]);
      a.y += __uint_as_float(r[4 * i + 1]);
      a.z += __uint_as_float(r[4 * i + 2]);
      a.w += __uint_as_float(r[4 * i + 3]);
      d4[i] = a;
    }
  } else if constexpr (sizeof(DT) == 4) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int i = 0; i < COLS / 4; ++i)
      d4[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]), __uint_as_float(r[4 * i + 2]),
                          __uint_as_float(r[4 * i + 3]));
  } else {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < COLS / 8; ++i) {
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float a = __uint_as_float(r[8 * i + 2 * h]);
        const float b = __uint_as_float(r[8 * i + 2 * h + 1]);
        w[h] = std::is_same<DT, __nv_bfloat16>::value ? pack_bf16x2(a, b) : pack_f16x2(a, b);
      }
      d4[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Dynamic work list of the persistent backward kernels.  Items are numbered
// heavy-first inside chunks of heads (head_chunked_item); block b starts with
// item b (the grid never exceeds the item count), then the TMA warp's lane 0
// claims the next unclaimed number (gridDim.x + a global counter) as it starts
// each further item and publishes it in a ring of ITEM_SLOTS shared-memory
// slots, from which the MMA and compute warps read the same sequence.  A
// block's sequence ends at the first number >= n_items it claims.  Blocks taking items as they
// free up finish within about one item of each other whatever the cost
// profile of the list; a fixed round-robin assignment balances only lists
// sorted by decreasing cost, which the head chunks break.  The delta pass
// that precedes both kernels zeroes their counters.

struct ItemRing {
  volatile int* slot;  // [ITEM_SLOTS] item numbers
  uint64_t* full;      // [ITEM_SLOTS] count 1: the producer published the slot
  uint64_t* empty;     // [ITEM_SLOTS] count = consumer threads: each read it

  // Producer (one thread): claim an item, publish it as sequence entry j.
  __device__ __forceinline__ bool publish(int j, int* counter, int& w, volatile int* abort, uint64_t limit,
                                          int site) {
    w = j == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(counter, 1);
    const int s = j % ITEM_SLOTS;
    if (!mbar_wait(&empty[s], ((j / ITEM_SLOTS) & 1) ^ 1, abort, limit, site)) return false;
    slot[s] = w;
    mbar_arrive(&full[s]);  // release: the consumers' wait orders their read after the store
    return true;
  }
  // Consumer (every thread of the MMA and compute warps): sequence entry j,
  // or -1 when the wait gave up.
  __device__ __forceinline__ int take(int j, volatile int* abort, uint64_t limit, int site) {
    const int s = j % ITEM_SLOTS;
    if (!mbar_wait(&full[s], (j / ITEM_SLOTS) & 1, abort, limit, site)) return -1;
    const int w = slot[s];
    mbar_arrive(&empty[s]);  // release: orders the read before the producer's reuse
    return w;
  }
};

// ---------------------------------------------------------------------------
// dK / dV: persistent CTAs; each takes (128-key tile, batch*head) items from
// the work list (ItemRing: heavy first inside chunks of heads).  K/V of the
// next item load once the current item's last S^T / dP^T GEMMs ran; the next
// item's GEMMs overlap the current epilogue.
// ---------------------------------------------------------------------------
template <typename DT, int HD>
__global__ void __launch_bounds__(BwdConfig<DT, HD>::KV_THREADS, 1)
    attn_bwd_dkdv_sm100(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                        const __grid_constant__ CUtensorMap tm_qm, const __grid_constant__ CUtensorMap tm_dom,
                        const BwdParams p, int n_ktiles, int n_items) {
  using C = BwdConfig<DT, HD>;
  constexpr int ST = C::KV_ST;
  constexpr int QT = C::KV_QT;
  constexpr int HALF = C::KV_HALF;
  constexpr int kKind = DTypeTraits<DT>::kKind;
  constexpr uint32_t kFmt = DTypeTraits<DT>::kFmt;
  constexpr int CW = 4 * C::KV_GROUPS;  // compute warps
  constexpr int CT = 128 * C::KV_GROUPS;  // compute threads
  constexpr int TMA_WARP = CW, MMA_WARP = CW + 1;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + C::BIG_TILE;
  uint8_t* sStage = sV + C::BIG_TILE;  // per stage: Q, dO [, Q MN copy, dO MN copy]
  auto sQ = [&](int st) { return sStage + st * C::KV_STAGE_BYTES; };
  auto sdO = [&](int st) { return sStage + st * C::KV_STAGE_BYTES + C::KV_QTILE; };
  auto sQm = [&](int st) { return C::TF32 ? sStage + st * C::KV_STAGE_BYTES + 2 * C::KV_QTILE : sQ(st); };
  auto sdOm = [&](int st) { return C::TF32 ? sStage + st * C::KV_STAGE_BYTES + 3 * C::KV_QTILE : sdO(st); };
  // per-query rows of the streamed tiles: slot l = nlse2[QT] | ndelta[QT]
  float* sRows = reinterpret_cast<float*>(sStage + ST * C::KV_STAGE_BYTES);
  constexpr int LDS = C::LD_SLOTS;
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(sStage + ST * C::KV_STAGE_BYTES + (C::ROWS_RING ? LDS * C::LD_BYTES : 0));
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = kv_full + 1;
  constexpr int NP = C::KV_PARTS;
  uint64_t* part_full = kv_empty + 1;          // [NP][ST]
  uint64_t* part_empty = part_full + NP * ST;  // [NP][ST]
  auto pfull = [&](int part, int st) { return &part_full[part * ST + st]; };
  auto pempty = [&](int part, int st) { return &part_empty[part * ST + st]; };
  uint64_t* s_full = part_empty + NP * ST;
  uint64_t* s_free = s_full + 1;
  uint64_t* dp_full = s_free + 1;
  uint64_t* p_full = dp_full + 1;   // dS^T (and 16-bit P^T) stored
  uint64_t* pt_full = p_full + 1;   // EARLY_P: P^T stored
  uint64_t* acc_full = pt_full + 1;
  uint64_t* acc_free = acc_full + 1;
  uint64_t* done_bar = acc_free + 1;
  uint64_t* rows_full = done_bar + 1;     // [LDS]
  uint64_t* rows_empty = rows_full + LDS;  // [LDS]
  ItemRing items;
  items.full = rows_empty + LDS;           // [ITEM_SLOTS]
  items.empty = items.full + ITEM_SLOTS;   // [ITEM_SLOTS]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  items.slot = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_qt_all = (p.Tq + QT - 1) / QT;
  // item -> key tile, batch*head, first query tile that sees the key tile,
  // number of query tiles (causal: heavy key tiles, i.e. low kt, first)
  auto item = [&](int w, int& kt, int& bh, int& qt_first) -> int {
    head_chunked_item(w, p.BH, n_ktiles, p.dkdv_head_chunk, kt, bh);
    qt_first = 0;
    if (p.causal) {
      const int need = kt * C::KV_KEYS - p.causal_offset;  // smallest query index that sees the tile
      qt_first = need <= 0 ? 0 : need / QT;
    }
    return max(0, n_qt_all - qt_first);
  };

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int s = 0; s < NP * ST; ++s) {
      mbar_init(&part_full[s], 1);
      mbar_init(&part_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, CT);
    mbar_init(dp_full, 1);
    mbar_init(p_full, CT);
    mbar_init(pt_full, CT);
    mbar_init(acc_full, 1);
    mbar_init(acc_free, CT);
    mbar_init(done_bar, 1);
    for (int l = 0; l < LDS; ++l) {
      mbar_init(&rows_full[l], 1);
      mbar_init(&rows_empty[l], CW);  // one arrival per compute warp
    }
    for (int l = 0; l < ITEM_SLOTS; ++l) {
      mbar_init(&items.full[l], 1);
      mbar_init(&items.empty[l], 32 + CT);  // the MMA warp's and the compute warps' threads
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_holder, C::KV_TMEM);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const uint64_t limit = p.wait_limit_ns;
  // Launched with programmatic serialization after the delta pass: the set-up
  // above overlaps its tail, everything below reads its output.
  grid_dep_wait();
  // The dQ kernel, which reads none of this kernel's outputs, is launched
  // next with programmatic serialization: let its blocks take the SMs this
  // grid's blocks leave as they finish (every block of this grid has started
  // by now, after the delta pass it reads had completed).
  grid_dep_launch_dependents();

  if (warp == TMA_WARP) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      int g = 0, ni = 0;  // query tiles and non-empty items issued so far
      int issued_kv = 0;
      int issued[NP];  // query tiles whose part q was issued
#pragma unroll
      for (int q = 0; q < NP; ++q) issued[q] = 0;
      int issued_rows = 0;
      bool ok = true;
      for (int seq = 0; ok; ++seq) {
        int w;
        if (!(ok = items.publish(seq, p.item_counters, w, abort_flag, limit, 60))) break;
        if (w >= n_items) break;
        int kt, bh, qt_first;
        const int n_it = item(w, kt, bh, qt_first);
        if (n_it == 0) continue;
        // K/V buffers are free once the previous item's last S^T/dP^T ran
        if (!(ok = mbar_wait(kv_empty, (ni & 1) ^ 1, abort_flag, limit, 10))) break;
        const int krow = p.k_row0 + kt * C::KV_KEYS;
        mbar_arrive_expect_tx(kv_full, 2 * C::BIG_TILE);
#pragma unroll
        for (int b = 0; b < C::KBLK; ++b) {
          tma_load_3d(sK + b * 128 * 128, &tm_k, kv_full, b * C::E128, krow, bh);
          tma_load_3d(sV + b * 128 * 128, &tm_v, kv_full, b * C::E128, krow, bh);
        }
        issued_kv = ni + 1;
        for (int it = 0; ok && it < n_it; ++it, ++g) {
          const int st = g % ST;
          const int row = p.q_row0 + (qt_first + it) * QT;
          if constexpr (C::ROWS_RING) {  // the tile's nlse2 / ndelta rows (QT floats each, 16-byte aligned: Tq_pad is whole tiles)
            const int l = g % LDS;
            if (!(ok = mbar_wait(&rows_empty[l], ((g / LDS) & 1) ^ 1, abort_flag, limit, 48))) break;
            const size_t off = (size_t)bh * p.Tq_pad + (size_t)(qt_first + it) * QT;
            mbar_arrive_expect_tx(&rows_full[l], C::LD_BYTES);
            bulk_load_1d(sRows + l * 2 * QT, p.nlse2 + off, QT * 4, &rows_full[l]);
            bulk_load_1d(sRows + l * 2 * QT + QT, p.ndelta + off, QT * 4, &rows_full[l]);
            issued_rows = g + 1;
          }
          // parts in the order the GEMMs read them
#pragma unroll
          for (int q = 0; q < NP; ++q) {
            if (!(ok = mbar_wait(pempty(q, st), ((g / ST) & 1) ^ 1, abort_flag, limit, 11))) break;
            uint64_t* bar = pfull(q, st);
            if constexpr (NP == 1) {
              mbar_arrive_expect_tx(bar, C::KV_STAGE_BYTES);
#pragma unroll
              for (int b = 0; b < C::KBLK; ++b) {
                tma_load_3d(sQ(st) + b * QT * 128, &tm_q, bar, b * C::E128, row, bh);
                tma_load_3d(sdO(st) + b * QT * 128, &tm_do, bar, b * C::E128, row, bh);
              }
            } else {
              mbar_arrive_expect_tx(bar, C::KV_QTILE);
              const CUtensorMap* map = q == 0 ? &tm_q : q == 1 ? &tm_do : q == 2 ? &tm_dom : &tm_qm;
              uint8_t* dst = q == 0 ? sQ(st) : q == 1 ? sdO(st) : q == 2 ? sdOm(st) : sQm(st);
#pragma unroll
              for (int b = 0; b < C::KBLK; ++b) tma_load_3d(dst + b * QT * 128, map, bar, b * C::E128, row, bh);
            }
            issued[q] = g + 1;
          }
        }
        ++ni;
      }
      // On an aborted run some loads may still be landing: wait (bounded,
      // ignoring the abort flag) for the last load issued into each buffer.
      if (*abort_flag) {
        const uint64_t t0 = globaltimer_ns();
        if (issued_kv > 0)
          while (!mbar_try_wait(kv_full, (issued_kv - 1) & 1) && globaltimer_ns() - t0 < limit) {
          }
#pragma unroll
        for (int q = 0; q < NP; ++q)
          for (int it = max(0, issued[q] - ST); it < issued[q]; ++it)
            while (!mbar_try_wait(pfull(q, it % ST), (it / ST) & 1) && globaltimer_ns() - t0 < limit) {
            }
        if constexpr (C::ROWS_RING)
          for (int it = max(0, issued_rows - LDS); it < issued_rows; ++it)
            while (!mbar_try_wait(&rows_full[it % LDS], (it / LDS) & 1) && globaltimer_ns() - t0 < limit) {
            }
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // The whole warp runs this loop; one elected lane issues each MMA group.
    constexpr uint32_t idesc_s = make_idesc(kFmt, 128, QT, false, false);
    constexpr uint32_t idesc_t = make_idesc(kFmt, 128, HD, false, true);
    const uint32_t aK = smem_u32(sK), aV = smem_u32(sV);
    // S^T = K Q^T, dP^T = V dO^T: A is the 128-key tile, B the streamed query tile.
    auto gemm_ss = [&](uint32_t d, uint32_t a_tile, uint32_t b_tile) {
      const uint64_t a0 = kmajor_desc(a_tile, 128, 0), b0 = kmajor_desc(b_tile, QT, 0);
#pragma unroll
      for (int ks = 0; ks < C::KSTEP_S; ++ks)
        umma_ss<kKind>(d, desc_advance(a0, kmajor_offset(128, ks)), desc_advance(b0, kmajor_offset(QT, ks)), idesc_s,
                       ks > 0 ? 1u : 0u);
    };
    // dV += P^T dO, dK += dS^T Q: A from TMEM, B = MN-major query tile.
    auto gemm_ts = [&](uint32_t d, uint32_t a_base, uint32_t b_tile, bool acc) {
      const uint64_t b0 = mnmajor_desc<C::TF32>(b_tile, QT, 0, C::K_PER);
#pragma unroll
      for (int ks = 0; ks < QT / C::K_PER; ++ks)
        umma_ts<kKind>(d, a_base + C::a_col(ks, HALF), desc_advance(b0, mnmajor_offset(ks, C::K_PER)), idesc_t,
                       (acc || ks > 0) ? 1u : 0u);
    };
    int g = 0, ni = 0;
    bool ok = true;
    for (int seq = 0; ok; ++seq) {
      const int w = items.take(seq, abort_flag, limit, 61);
      if (!(ok = __all_sync(0xffffffffu, w >= 0))) break;
      if (w >= n_items) break;
      int kt, bh, qt_first;
      const int n_it = item(w, kt, bh, qt_first);
      if (n_it == 0) continue;
      if (!(ok = mbar_wait_warp(kv_full, ni & 1, abort_flag, limit, 12))) break;
      // first S^T of the item: the compute warps must have read the last one
      if (g > 0 && !(ok = mbar_wait_warp(s_free, (g - 1) & 1, abort_flag, limit, 14))) break;
      if (!(ok = mbar_wait_warp(pfull(0, g % ST), (g / ST) & 1, abort_flag, limit, 13))) break;
      tc_fence_after();
      if (elect_one()) {
        gemm_ss(tbase + C::KV_S, aK, smem_u32(sQ(g % ST)));
        umma_commit(s_full);
        if constexpr (NP > 1) umma_commit(pempty(0, g % ST));
      }
      __syncwarp();
      if (NP > 1 && !(ok = mbar_wait_warp(pfull(1, g % ST), (g / ST) & 1, abort_flag, limit, 38))) break;
      tc_fence_after();
      if (elect_one()) {
        gemm_ss(tbase + C::KV_DP, aV, smem_u32(sdO(g % ST)));
        umma_commit(dp_full);
        if constexpr (NP > 1) umma_commit(pempty(1, g % ST));
        if (n_it == 1) umma_commit(kv_empty);
      }
      __syncwarp();
      for (int it = 0; it < n_it; ++it, ++g) {
        const int st = g % ST;
        const int st1 = (g + 1) % ST;
        // S^T of the next query tile.  With early P^T (tf32) it is queued after
        // dV of this tile: dV only waits for the exponentials, while the next
        // tile's Q / dO stage is refilled only once dK of the tile before this
        // one has run, so issuing S^T first would park the MMA warp on that
        // load with dV ready behind it.
        auto issue_next_s = [&](bool wait_s_free) -> bool {
          if (it + 1 < n_it) {
            if (wait_s_free && !mbar_wait_warp(s_free, g & 1, abort_flag, limit, 14)) return false;
            if (!mbar_wait_warp(pfull(0, st1), ((g + 1) / ST) & 1, abort_flag, limit, 15)) return false;
            tc_fence_after();
            if (elect_one()) {
              gemm_ss(tbase + C::KV_S, aK, smem_u32(sQ(st1)));
              umma_commit(s_full);
              if constexpr (NP > 1) umma_commit(pempty(0, st1));
            }
            __syncwarp();
          }
          return true;
        };
        if constexpr (!C::EARLY_P) {
          if (!(ok = issue_next_s(true))) break;
        }
        if constexpr (C::EARLY_P) {
          // dV (+)= P^T dO as soon as P^T is stored, while dS^T is formed
          if (!(ok = mbar_wait_warp(pt_full, g & 1, abort_flag, limit, 37))) break;
          // the accumulators are free once the previous item's epilogue read them
          if (it == 0 && ni > 0 && !(ok = mbar_wait_warp(acc_free, (ni - 1) & 1, abort_flag, limit, 34))) break;
          if (NP > 1 && !(ok = mbar_wait_warp(pfull(2, st), (g / ST) & 1, abort_flag, limit, 39))) break;
          tc_fence_after();
          if (elect_one()) {
            gemm_ts(tbase + C::KV_DV, tbase + C::kv_p(), smem_u32(sdOm(st)), it > 0);
            if constexpr (NP > 1) umma_commit(pempty(2, st));
          }
          __syncwarp();
          // every compute thread arrives on s_free (S^T read) before pt_full,
          // so the completed pt_full phase implies the s_free one
          if (!(ok = issue_next_s(false))) break;
        }
        if (!(ok = mbar_wait_warp(p_full, g & 1, abort_flag, limit, 16))) break;
        if (!C::EARLY_P && it == 0 && ni > 0 && !(ok = mbar_wait_warp(acc_free, (ni - 1) & 1, abort_flag, limit, 34)))
          break;
        if (NP > 1 && !(ok = mbar_wait_warp(pfull(NP - 1, st), (g / ST) & 1, abort_flag, limit, 40))) break;
        tc_fence_after();
        if (elect_one()) {
          if constexpr (!C::EARLY_P) gemm_ts(tbase + C::KV_DV, tbase + C::kv_p(), smem_u32(sdOm(st)), it > 0);
          gemm_ts(tbase + C::KV_DK, tbase + C::KV_DP, smem_u32(sQm(st)), it > 0);
          umma_commit(pempty(NP - 1, st));
          if (it + 1 == n_it) umma_commit(acc_full);
        }
        __syncwarp();
        if (it + 1 < n_it) {
          if (NP > 1 && !(ok = mbar_wait_warp(pfull(1, st1), ((g + 1) / ST) & 1, abort_flag, limit, 41))) break;
          tc_fence_after();
          if (elect_one()) {
            gemm_ss(tbase + C::KV_DP, aV, smem_u32(sdO(st1)));
            umma_commit(dp_full);
            if constexpr (NP > 1) umma_commit(pempty(1, st1));
            if (it + 2 == n_it) umma_commit(kv_empty);  // last GEMMs reading K / V of this item
          }
          __syncwarp();
        }
      }
      ++ni;
    }
    // Wait (bounded, regardless of abort) for every MMA issued so far, so
    // that TMEM is idle before it is released.
    if (elect_one()) umma_commit(done_bar);
    __syncwarp();
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(done_bar, 0) && globaltimer_ns() - t0 < limit) {
    }
    __syncwarp();
  } else if (warp < CW) {
    // --------------------------- compute warps ---------------------------
    const int h = threadIdx.x >> 7;   // column group
    const int rr = threadIdx.x & 127;  // key row inside the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const float sl2 = p.scale_log2;
    const float scale = p.scale;
    const int col = h * (HD / 2);
    int g = 0, ni = 0;
    bool ok = true;
    for (int seq = 0; ok; ++seq) {
      const int w = items.take(seq, abort_flag, limit, 62);
      ok = w >= 0;
      if (!ok) break;
      if (w >= n_items) break;
      int kt, bh, qt_first;
      const int n_it = item(w, kt, bh, qt_first);
      const int key0 = kt * C::KV_KEYS;
      const int key = key0 + rr;
      const bool key_ok = key < p.Tk;
      const size_t row_index = (size_t)bh * p.k_rows_alloc + p.k_row0 + key;
      if (n_it == 0) {  // no query sees this key tile: dK = dV = 0
        if (!p.accumulate && key_ok) {
          if constexpr (C::KV_GROUPS == 4) {
            uint32_t zero[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) zero[i] = 0u;
            row_store<DT, 32>(zero, reinterpret_cast<DT*>(h < 2 ? p.dk : p.dv) + row_index * HD + (h & 1) * 32,
                              false);
          } else {
            uint32_t zero[HD / 2];
#pragma unroll
            for (int i = 0; i < HD / 2; ++i) zero[i] = 0u;
            row_store<DT, HD / 2>(zero, reinterpret_cast<DT*>(p.dk) + row_index * HD + col, false);
            row_store<DT, HD / 2>(zero, reinterpret_cast<DT*>(p.dv) + row_index * HD + col, false);
          }
        }
        continue;
      }
      for (int it = 0; it < n_it; ++it, ++g) {
        const int qtile0 = (qt_first + it) * QT;
        const int q0 = qtile0 + h * HALF;
        // this tile's -lse*log2(e) and -delta rows (padded to whole tiles: -inf
        // / 0 on padding rows): 16-bit from the shared-memory ring the TMA warp
        // fills; tf32 from L2, -lse*log2(e) into registers before the S^T wait
        const int l = g % LDS;
        const float4* nL4;
        const float4* nD4;
        float nLr[C::ROWS_RING ? 4 : HALF];
        if constexpr (C::ROWS_RING) {
          if (!(ok = mbar_wait(&rows_full[l], (g / LDS) & 1, abort_flag, limit, 49))) break;
          nL4 = reinterpret_cast<const float4*>(sRows + l * 2 * QT + h * HALF);
          nD4 = reinterpret_cast<const float4*>(sRows + l * 2 * QT + QT + h * HALF);
        } else {
          nL4 = reinterpret_cast<const float4*>(p.nlse2 + (size_t)bh * p.Tq_pad + q0);
          nD4 = reinterpret_cast<const float4*>(p.ndelta + (size_t)bh * p.Tq_pad + q0);
#pragma unroll
          for (int c = 0; c < HALF / 4; ++c) {
            const float4 v4 = __ldg(nL4 + c);
            nLr[4 * c] = v4.x;
            nLr[4 * c + 1] = v4.y;
            nLr[4 * c + 2] = v4.z;
            nLr[4 * c + 3] = v4.w;
          }
        }
        if (!(ok = mbar_wait(s_full, g & 1, abort_flag, limit, 17))) break;
        tc_fence_after();
        float sv[HALF];
        tmem_load_row(tbase + lane_off + C::KV_S + h * HALF, sv);
        tc_fence_before();
        mbar_arrive(s_free);
        // P^T = exp2(S^T * scale*log2e - lse*log2e); padding queries have
        // -lse*log2e = -inf, so P = 0
        if constexpr (!C::ROWS_RING) {
#pragma unroll
          for (int c = 0; c < HALF; ++c) sv[c] = ex2_approx(fmaf(sv[c], sl2, nLr[c]));
        } else {  // two columns per packed FMA
          const float2 sl2x2 = make_float2(sl2, sl2);
#pragma unroll
          for (int c = 0; c < HALF; c += 4) {
            const float4 n4 = nL4[c / 4];  // shared-memory broadcast: every lane reads the same row
            const float2 y0 = __ffma2_rn(make_float2(sv[c], sv[c + 1]), sl2x2, make_float2(n4.x, n4.y));
            const float2 y1 = __ffma2_rn(make_float2(sv[c + 2], sv[c + 3]), sl2x2, make_float2(n4.z, n4.w));
            sv[c] = ex2_approx(y0.x);
            sv[c + 1] = ex2_approx(y0.y);
            sv[c + 2] = ex2_approx(y1.x);
            sv[c + 3] = ex2_approx(y1.y);
          }
        }
        // causal diagonal tile / keys past Tk: zero the invisible entries
        if (!key_ok) {
#pragma unroll
          for (int c = 0; c < HALF; ++c) sv[c] = 0.f;
        } else if (p.causal && key0 + C::KV_KEYS - 1 > qtile0 + p.causal_offset) {
          const int cmin = key - p.causal_offset - q0;  // first visible column
#pragma unroll
          for (int c = 0; c < HALF; ++c)
            if (c < cmin) sv[c] = 0.f;
        }
        if constexpr (C::EARLY_P) {
          // P^T over the previous tile's (its reader, dV of tile g-1, was
          // queued before S^T of this tile, which the s_full wait above covered)
          tmem_store_operand<DT>(tbase + lane_off + C::kv_p() + h * HALF, sv);
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(pt_full);
        }
        if (!(ok = mbar_wait(dp_full, g & 1, abort_flag, limit, 18))) break;
        tc_fence_after();
        // dS^T = P^T (dP^T - delta) (tf32: times the softmax scale; 16-bit:
        // packed adds / multiplies, the scale goes on dK in the epilogue), 32
        // columns at a time, written in place (tf32) or packed into the
        // already-read front of the dP buffer.  16-bit: every dP^T column of
        // this thread is loaded first, with one wait for all of them (the
        // packed stores below then overwrite only columns already read).
        uint32_t dpall[C::ROWS_RING ? HALF : 32];
        if constexpr (C::ROWS_RING) {
#pragma unroll
          for (int ch = 0; ch < HALF / 32; ++ch)
            tmem_ld32(tbase + lane_off + C::KV_DP + h * HALF + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(dpall + ch * 32));
          tmem_wait_ld();
        }
#pragma unroll
        for (int ch = 0; ch < HALF / 32; ++ch) {
          float dsv[32];
          {
            uint32_t regs[32];
            if constexpr (C::ROWS_RING) {
#pragma unroll
              for (int i = 0; i < 32; ++i) regs[i] = dpall[ch * 32 + i];
            } else {
              tmem_ld32(tbase + lane_off + C::KV_DP + h * HALF + ch * 32, regs);
              tmem_wait_ld();
            }
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const int i = 4 * c4;
              if constexpr (!C::ROWS_RING) {
                const float4 d4 = __ldg(nD4 + ch * 8 + c4);
                dsv[i] = sv[ch * 32 + i] * (__uint_as_float(regs[i]) + d4.x) * scale;
                dsv[i + 1] = sv[ch * 32 + i + 1] * (__uint_as_float(regs[i + 1]) + d4.y) * scale;
                dsv[i + 2] = sv[ch * 32 + i + 2] * (__uint_as_float(regs[i + 2]) + d4.z) * scale;
                dsv[i + 3] = sv[ch * 32 + i + 3] * (__uint_as_float(regs[i + 3]) + d4.w) * scale;
                continue;
              }
              const float4 d4 = nD4[ch * 8 + c4];
              const float2 t0 = __fadd2_rn(make_float2(__uint_as_float(regs[i]), __uint_as_float(regs[i + 1])),
                                           make_float2(d4.x, d4.y));
              const float2 t1 = __fadd2_rn(make_float2(__uint_as_float(regs[i + 2]), __uint_as_float(regs[i + 3])),
                                           make_float2(d4.z, d4.w));
              const float2 r0 = __fmul2_rn(make_float2(sv[ch * 32 + i], sv[ch * 32 + i + 1]), t0);
              const float2 r1 = __fmul2_rn(make_float2(sv[ch * 32 + i + 2], sv[ch * 32 + i + 3]), t1);
              dsv[i] = r0.x;
              dsv[i + 1] = r0.y;
              dsv[i + 2] = r1.x;
              dsv[i + 3] = r1.y;
            }
          }
          if constexpr (C::TF32)
            tmem_store_operand<DT>(tbase + lane_off + C::KV_DP + h * HALF + ch * 32, dsv);
          else
            tmem_store_operand<DT>(tbase + lane_off + C::KV_DP + h * HALF + ch * 16, dsv);
        }
        // the tile's rows in shared memory are no longer read by this warp
        if constexpr (C::ROWS_RING) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&rows_empty[l]);
        }
        if constexpr (!C::EARLY_P) tmem_store_operand<DT>(tbase + lane_off + C::kv_p() + h * HALF, sv);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_full);
      }
      if (!ok) break;
      // ------------------------------ epilogue ------------------------------
      if (!(ok = mbar_wait(acc_full, ni & 1, abort_flag, limit, 19))) break;
      tc_fence_after();
      if constexpr (C::KV_GROUPS == 4) {
        // groups 0, 1: the two 32-column halves of dK; 2, 3: of dV
        const uint32_t src = tbase + lane_off + (h < 2 ? C::KV_DK : C::KV_DV) + (h & 1) * 32;
        void* dst_row = reinterpret_cast<char*>(h < 2 ? p.dk : p.dv) +
                        (row_index * HD + (h & 1) * 32) * (p.accumulate ? sizeof(float) : sizeof(DT));
        const float mul = 1.f;  // (tf32: dS^T carries the softmax scale)
        if (p.accumulate)
          tmem_row_accumulate<32>(src, reinterpret_cast<float*>(dst_row), key_ok, mul);
        else
          tmem_row_to_global<DT, 32>(src, reinterpret_cast<DT*>(dst_row), key_ok, false, mul);
      } else if (p.accumulate) {
        tmem_row_accumulate<HD / 2>(tbase + lane_off + C::KV_DK + col,
                                    reinterpret_cast<float*>(p.dk) + row_index * HD + col, key_ok, scale);
        tmem_row_accumulate<HD / 2>(tbase + lane_off + C::KV_DV + col,
                                    reinterpret_cast<float*>(p.dv) + row_index * HD + col, key_ok, 1.f);
      } else {
        tmem_row_to_global<DT, HD / 2>(tbase + lane_off + C::KV_DK + col,
                                       reinterpret_cast<DT*>(p.dk) + row_index * HD + col, key_ok, false, scale);
        tmem_row_to_global<DT, HD / 2>(tbase + lane_off + C::KV_DV + col,
                                       reinterpret_cast<DT*>(p.dv) + row_index * HD + col, key_ok, false, 1.f);
      }
      tc_fence_before();
      mbar_arrive(acc_free);
      ++ni;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tbase, C::KV_TMEM);
  }
}

// ---------------------------------------------------------------------------
// dQ: persistent CTAs; each takes (128-query tile, batch*head) items from the
// work list (ItemRing: heavy first inside chunks of heads).  Q/dO of the next
// item load while the current item's last tiles run;
// the dQ accumulator is read into registers and released before it is written
// out, so the next item's GEMMs start under the current item's epilogue.
// ---------------------------------------------------------------------------
template <typename DT, int HD>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_dq_sm100(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                      const __grid_constant__ CUtensorMap tm_km, const BwdParams p, int n_qtiles, int n_items) {
  using C = BwdConfig<DT, HD>;
  constexpr int KST = C::Q_KST;
  constexpr int VST = C::Q_VST;
  constexpr int KT = C::Q_KT;
  constexpr int HALF = C::Q_HALF;
  constexpr int kKind = DTypeTraits<DT>::kKind;
  constexpr uint32_t kFmt = DTypeTraits<DT>::kFmt;
  constexpr int TMA_WARP = 8, MMA_WARP = 9;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sdO = sQ + C::BIG_TILE;
  uint8_t* sKring = sdO + C::BIG_TILE;  // per stage: K [, K MN copy]
  uint8_t* sVring = sKring + KST * C::Q_KSTAGE_BYTES;
  auto sK = [&](int st) { return sKring + st * C::Q_KSTAGE_BYTES; };
  auto sKm = [&](int st) { return C::TF32 ? sKring + st * C::Q_KSTAGE_BYTES + C::Q_KTILE : sK(st); };
  auto sV = [&](int st) { return sVring + st * C::Q_VSTAGE_BYTES; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(sVring + VST * C::Q_VSTAGE_BYTES);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 1;
  uint64_t* k_full = q_empty + 1;    // [KST]
  uint64_t* k_empty = k_full + KST;  // [KST]
  uint64_t* v_full = k_empty + KST;  // [VST]
  uint64_t* v_empty = v_full + VST;  // [VST]
  uint64_t* s_full = v_empty + VST;
  uint64_t* s_free = s_full + 1;
  uint64_t* dp_full = s_free + 1;
  uint64_t* ds_full = dp_full + 1;
  uint64_t* acc_full = ds_full + 1;
  uint64_t* acc_free = acc_full + 1;
  uint64_t* done_bar = acc_free + 1;
  ItemRing items;
  items.full = done_bar + 1;              // [ITEM_SLOTS]
  items.empty = items.full + ITEM_SLOTS;  // [ITEM_SLOTS]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  items.slot = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_kv_all = (p.Tk + KT - 1) / KT;
  // item -> query tile, batch*head, number of key tiles it sees
  auto item = [&](int w, int& qt, int& bh) -> int {
    if (p.causal) {  // heavy query tiles first
      int rank;
      head_chunked_item(w, p.BH, n_qtiles, p.dq_head_chunk, rank, bh);
      qt = n_qtiles - 1 - rank;
      const int last_row = min(qt * C::Q_ROWS + C::Q_ROWS - 1, p.Tq - 1) + p.causal_offset;
      return last_row < 0 ? 0 : min(n_kv_all, last_row / KT + 1);
    }
    qt = w % n_qtiles;
    bh = w / n_qtiles;
    return n_kv_all;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(dp_full, 1);
    mbar_init(ds_full, 256);
    mbar_init(acc_full, 1);
    mbar_init(acc_free, 256);
    mbar_init(done_bar, 1);
    for (int l = 0; l < ITEM_SLOTS; ++l) {
      mbar_init(&items.full[l], 1);
      mbar_init(&items.empty[l], 32 + 256);  // the MMA warp's and the compute warps' threads
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_holder, C::Q_TMEM);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const uint64_t limit = p.wait_limit_ns;

  if (warp == TMA_WARP) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      int g = 0, ni = 0;  // key tiles and non-empty items issued so far
      int issued_q = 0, issued_k = 0, issued_v = 0;
      bool ok = true;
      for (int seq = 0; ok; ++seq) {
        int w;
        if (!(ok = items.publish(seq, p.item_counters + 1, w, abort_flag, limit, 63))) break;
        if (w >= n_items) break;
        int qt, bh;
        const int n_kv = item(w, qt, bh);
        if (n_kv == 0) continue;
        // Q/dO buffers are free once the previous item's last S/dP GEMMs ran
        if (!(ok = mbar_wait(q_empty, (ni & 1) ^ 1, abort_flag, limit, 20))) break;
        const int qrow = p.q_row0 + qt * C::Q_ROWS;
        mbar_arrive_expect_tx(q_full, 2 * C::BIG_TILE);
#pragma unroll
        for (int b = 0; b < C::KBLK; ++b) {
          tma_load_3d(sQ + b * 128 * 128, &tm_q, q_full, b * C::E128, qrow, bh);
          tma_load_3d(sdO + b * 128 * 128, &tm_do, q_full, b * C::E128, qrow, bh);
        }
        issued_q = ni + 1;
        for (int j = 0; j < n_kv; ++j, ++g) {
          const int kst = g % KST, vst = g % VST;
          const int row = p.k_row0 + j * KT;
          if (!(ok = mbar_wait(&k_empty[kst], ((g / KST) & 1) ^ 1, abort_flag, limit, 21))) break;
          mbar_arrive_expect_tx(&k_full[kst], C::Q_KSTAGE_BYTES);
#pragma unroll
          for (int b = 0; b < C::KBLK; ++b) {
            tma_load_3d(sK(kst) + b * KT * 128, &tm_k, &k_full[kst], b * C::E128, row, bh);
            if constexpr (C::TF32) tma_load_3d(sKm(kst) + b * KT * 128, &tm_km, &k_full[kst], b * C::E128, row, bh);
          }
          issued_k = g + 1;
          if (!(ok = mbar_wait(&v_empty[vst], ((g / VST) & 1) ^ 1, abort_flag, limit, 22))) break;
          mbar_arrive_expect_tx(&v_full[vst], C::Q_VSTAGE_BYTES);
#pragma unroll
          for (int b = 0; b < C::KBLK; ++b)
            tma_load_3d(sV(vst) + b * KT * 128, &tm_v, &v_full[vst], b * C::E128, row, bh);
          issued_v = g + 1;
        }
        ++ni;
      }
      // On an aborted run some loads may still be landing: wait (bounded,
      // ignoring the abort flag) for the last load issued into each buffer.
      if (*abort_flag) {
        const uint64_t t0 = globaltimer_ns();
        if (issued_q > 0)
          while (!mbar_try_wait(q_full, (issued_q - 1) & 1) && globaltimer_ns() - t0 < limit) {
          }
        for (int j = max(0, issued_k - KST); j < issued_k; ++j)
          while (!mbar_try_wait(&k_full[j % KST], (j / KST) & 1) && globaltimer_ns() - t0 < limit) {
          }
        for (int j = max(0, issued_v - VST); j < issued_v; ++j)
          while (!mbar_try_wait(&v_full[j % VST], (j / VST) & 1) && globaltimer_ns() - t0 < limit) {
          }
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // The whole warp runs this loop; one elected lane issues each MMA group.
    constexpr uint32_t idesc_s = make_idesc(kFmt, 128, KT, false, false);
    constexpr uint32_t idesc_t = make_idesc(kFmt, 128, HD, false, true);
    const uint32_t aQ = smem_u32(sQ), adO = smem_u32(sdO);
    // S = Q K^T, dP = dO V^T: A is the 128-query tile, B the streamed key tile.
    auto gemm_ss = [&](uint32_t d, uint32_t a_tile, uint32_t b_tile) {
      const uint64_t a0 = kmajor_desc(a_tile, 128, 0), b0 = kmajor_desc(b_tile, KT, 0);
#pragma unroll
      for (int ks = 0; ks < C::KSTEP_S; ++ks)
        umma_ss<kKind>(d, desc_advance(a0, kmajor_offset(128, ks)), desc_advance(b0, kmajor_offset(KT, ks)), idesc_s,
                       ks > 0 ? 1u : 0u);
    };
    // dQ (+)= dS K: A = dS from TMEM, B = the key tile read MN-major.
    auto gemm_dq = [&](int st, bool acc) {
      const uint64_t b0 = mnmajor_desc<C::TF32>(smem_u32(sKm(st)), KT, 0, C::K_PER);
#pragma unroll
      for (int ks = 0; ks < KT / C::K_PER; ++ks)
        umma_ts<kKind>(tbase + C::Q_DQ, tbase + C::q_dp(0) + C::a_col(ks, HALF),
                       desc_advance(b0, mnmajor_offset(ks, C::K_PER)), idesc_t, (acc || ks > 0) ? 1u : 0u);
    };
    int g = 0, ni = 0;
    bool ok = true;
    for (int seq = 0; ok; ++seq) {
      const int w = items.take(seq, abort_flag, limit, 64);
      if (!(ok = __all_sync(0xffffffffu, w >= 0))) break;
      if (w >= n_items) break;
      int qt, bh;
      const int n_kv = item(w, qt, bh);
      if (n_kv == 0) continue;
      if (!(ok = mbar_wait_warp(q_full, ni & 1, abort_flag, limit, 23))) break;
      // first S of the item: the compute warps must have read the last one
      if (g > 0 && !(ok = mbar_wait_warp(s_free, (g - 1) & 1, abort_flag, limit, 26))) break;
      if (!(ok = mbar_wait_warp(&k_full[g % KST], (g / KST) & 1, abort_flag, limit, 24))) break;
      tc_fence_after();
      if (elect_one()) {
        gemm_ss(tbase + C::Q_S, aQ, smem_u32(sK(g % KST)));
        umma_commit(s_full);
      }
      __syncwarp();
      if (!(ok = mbar_wait_warp(&v_full[g % VST], (g / VST) & 1, abort_flag, limit, 25))) break;
      tc_fence_after();
      if (elect_one()) {
        gemm_ss(tbase + C::q_dp(0), adO, smem_u32(sV(g % VST)));
        umma_commit(dp_full);
        umma_commit(&v_empty[g % VST]);
        if (n_kv == 1) umma_commit(q_empty);
      }
      __syncwarp();
      for (int j = 0; j < n_kv; ++j, ++g) {
        const int st = g % KST;
        if (j + 1 < n_kv) {
          const int st1 = (g + 1) % KST;
          if (!(ok = mbar_wait_warp(s_free, g & 1, abort_flag, limit, 26))) break;
          if (!(ok = mbar_wait_warp(&k_full[st1], ((g + 1) / KST) & 1, abort_flag, limit, 27))) break;
          tc_fence_after();
          if (elect_one()) {
            gemm_ss(tbase + C::Q_S, aQ, smem_u32(sK(st1)));
            umma_commit(s_full);
          }
          __syncwarp();
        }
        if (!(ok = mbar_wait_warp(ds_full, g & 1, abort_flag, limit, 28))) break;
        // the accumulator is free once the previous item's epilogue read it
        if (j == 0 && ni > 0 && !(ok = mbar_wait_warp(acc_free, (ni - 1) & 1, abort_flag, limit, 33))) break;
        tc_fence_after();
        if (elect_one()) {
          gemm_dq(st, j > 0);
          umma_commit(&k_empty[st]);
        }
        __syncwarp();
        if (j + 1 < n_kv) {
          const int vst1 = (g + 1) % VST;
          if (!(ok = mbar_wait_warp(&v_full[vst1], ((g + 1) / VST) & 1, abort_flag, limit, 29))) break;
          tc_fence_after();
          if (elect_one()) {
            gemm_ss(tbase + C::q_dp(0), adO, smem_u32(sV(vst1)));
            umma_commit(dp_full);
            umma_commit(&v_empty[vst1]);
            if (j + 2 == n_kv) umma_commit(q_empty);  // last GEMM reading Q / dO of this item
          }
          __syncwarp();
        } else {
          if (elect_one()) umma_commit(acc_full);
          __syncwarp();
        }
      }
      ++ni;
    }
    // Wait (bounded, regardless of abort) for every MMA issued so far, so
    // that TMEM is idle before it is released.
    if (elect_one()) umma_commit(done_bar);
    __syncwarp();
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(done_bar, 0) && globaltimer_ns() - t0 < limit) {
    }
    __syncwarp();
  } else if (warp < 8) {
    // --------------------------- compute warps ---------------------------
    const int h = threadIdx.x >> 7;   // key-column half
    const int rr = threadIdx.x & 127;  // query row (TMEM lane)
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const float sl2 = p.scale_log2;
    const float scale = p.scale;
    const int col = h * (HD / 2);
    int g = 0, ni = 0;
    bool ok = true;
    for (int seq = 0; ok; ++seq) {
      const int w = items.take(seq, abort_flag, limit, 65);
      ok = w >= 0;
      if (!ok) break;
      if (w >= n_items) break;
      int qt, bh;
      const int n_kv = item(w, qt, bh);
      const int q = qt * C::Q_ROWS + rr;
      const bool q_ok = q < p.Tq;
      const size_t lrow = (size_t)bh * p.q_rows_alloc + p.q_row0 + q;
      if (n_kv == 0) {  // no key visible to this query tile: dQ = 0
        if (!p.accumulate && q_ok) {
          uint32_t zero[HD / 2];
#pragma unroll
          for (int i = 0; i < HD / 2; ++i) zero[i] = 0u;
          row_store<DT, HD / 2>(zero, reinterpret_cast<DT*>(p.dq) + lrow * HD + col, false);
        }
        continue;
      }
      const float nL = q_ok ? p.nlse2[(size_t)bh * p.Tq_pad + q] : 0.f;  // -lse * log2(e)
      const float nd = q_ok ? p.ndelta[(size_t)bh * p.Tq_pad + q] : 0.f;  // -delta
      const float2 sl2x2 = make_float2(sl2, sl2), nL2 = make_float2(nL, nL), nd2 = make_float2(nd, nd);
      int vis = p.Tk - 1;
      if (p.causal) vis = min(vis, q + p.causal_offset);
      if (!q_ok) vis = -1;
      for (int j = 0; j < n_kv; ++j, ++g) {
        const int kc0 = j * KT + h * HALF;  // first key of this thread's half
        if (!(ok = mbar_wait(s_full, g & 1, abort_flag, limit, 30))) break;
        tc_fence_after();
        float sv[HALF];
        tmem_load_row(tbase + lane_off + C::Q_S + h * HALF, sv);
        tc_fence_before();
        mbar_arrive(s_free);
        const int lim = vis - kc0;  // columns > lim are masked (diagonal / tail tiles only)
#pragma unroll
        for (int c = 0; c < HALF; c += 2) {
          const float2 y = __ffma2_rn(make_float2(sv[c], sv[c + 1]), sl2x2, nL2);
          sv[c] = ex2_approx(y.x);
          sv[c + 1] = ex2_approx(y.y);
        }
        if (lim < HALF - 1) {
#pragma unroll
          for (int c = 0; c < HALF; ++c)
            if (c > lim) sv[c] = 0.f;
        }
        if (!(ok = mbar_wait(dp_full, g & 1, abort_flag, limit, 31))) break;
        tc_fence_after();
        float dsv[HALF];
        tmem_load_row(tbase + lane_off + C::q_dp(0) + h * HALF, dsv);
#pragma unroll
        for (int c = 0; c < HALF; c += 2) {  // dS = P (dP - delta); the scale goes on dQ in the epilogue
          const float2 r = __fmul2_rn(make_float2(sv[c], sv[c + 1]),
                                      __fadd2_rn(make_float2(dsv[c], dsv[c + 1]), nd2));
          dsv[c] = r.x;
          dsv[c + 1] = r.y;
        }
        tmem_store_operand<DT>(tbase + lane_off + C::q_dp(0) + h * HALF, dsv);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(ds_full);
      }
      if (!ok) break;
      // epilogue: accumulator -> registers, release it, then write the row
      if (!(ok = mbar_wait(acc_full, ni & 1, abort_flag, limit, 32))) break;
      tc_fence_after();
      uint32_t acc[HD / 2];
      tmem_row_load<HD / 2>(tbase + lane_off + C::Q_DQ + col, acc);
      tc_fence_before();
      mbar_arrive(acc_free);
#pragma unroll
      for (int i = 0; i < HD / 2; ++i) acc[i] = __float_as_uint(__uint_as_float(acc[i]) * scale);
      if (q_ok) {
        if (p.accumulate)
          row_store<DT, HD / 2>(acc, reinterpret_cast<float*>(p.dq) + lrow * HD + col, true);
        else
          row_store<DT, HD / 2>(acc, reinterpret_cast<DT*>(p.dq) + lrow * HD + col, false);
      }
      ++ni;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tbase, C::Q_TMEM);
  }
  // Launched with programmatic serialization after the dK/dV kernel: finish
  // only after it has, so that work queued after this kernel on the stream
  // (which may overwrite the inputs both read) also runs after the dK/dV kernel.
  grid_dep_wait();
}

}  // namespace ctfa
