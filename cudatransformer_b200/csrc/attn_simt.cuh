// SIMT attention kernels for the element types and head dims that the
// tcgen05 kernels do not cover: double (no fp64 tensor-core kind on sm_100a),
// and any head dim up to 256 that is not 64 or 128.  The reference
// instantiates its layer for float, double, half and bfloat16
// (cuda_transformer/cuda_transformer.cu:839-842) and accepts any head dim up to
// 256 (flash_attention.cu:52,95), so these keep that surface on the GPU.
//
// One warp per query row (forward, dQ) or per key row (dK/dV); each lane holds
// up to 8 elements of the head dim.  Exact exponentials, accumulation in fp32
// (fp64 for double).  Masking matches the tcgen05 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

namespace ctfa {

template <typename DT>
using AccT = typename std::conditional<std::is_same<DT, double>::value, double, float>::type;

template <typename DT>
__device__ __forceinline__ AccT<DT> to_acc(DT x) {
  return static_cast<AccT<DT>>(x);
}
template <>
__device__ __forceinline__ float to_acc<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_acc<__half>(__half x) {
  return __half2float(x);
}

template <typename DT>
__device__ __forceinline__ DT from_acc(AccT<DT> x) {
  return static_cast<DT>(x);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half from_acc<__half>(float x) {
  return __float2half_rn(x);
}

__device__ __forceinline__ float acc_exp(float x) { return expf(x); }
__device__ __forceinline__ double acc_exp(double x) { return exp(x); }
__device__ __forceinline__ float acc_log(float x) { return logf(x); }
__device__ __forceinline__ double acc_log(double x) { return log(x); }

template <typename A>
__device__ __forceinline__ A warp_sum(A v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct SimtParams {
  int BH, Tq, Tk, D;
  int q_row0, k_row0;
  int q_rows_alloc, k_rows_alloc;
  int causal, causal_offset;
  double scale;
};

__device__ __forceinline__ int simt_last_key(const SimtParams& p, int i) {
  int last = p.Tk - 1;
  if (p.causal) last = min(last, i + p.causal_offset);
  return last;
}

template <typename DT>
__global__ void attn_fwd_simt(const DT* __restrict__ q, const DT* __restrict__ k, const DT* __restrict__ v,
                              DT* __restrict__ o, float* __restrict__ lse, SimtParams p) {
  using A = AccT<DT>;
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)p.BH * p.Tq) return;
  const int bh = (int)(w / p.Tq), i = (int)(w % p.Tq);
  const size_t qrow = ((size_t)bh * p.q_rows_alloc + p.q_row0 + i) * p.D;
  const size_t kbase = ((size_t)bh * p.k_rows_alloc + p.k_row0) * p.D;
  A qv[8], acc[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int d = lane + 32 * t;
    qv[t] = d < p.D ? to_acc(q[qrow + d]) : A(0);
    acc[t] = A(0);
  }
  const A scale = (A)p.scale;
  A m = -INFINITY, l = 0;
  const int last = simt_last_key(p, i);
  for (int j = 0; j <= last; ++j) {
    const size_t kr = kbase + (size_t)j * p.D;
    A s = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int d = lane + 32 * t;
      if (d < p.D) s += qv[t] * to_acc(k[kr + d]);
    }
    s = warp_sum(s) * scale;
    const A mn = s > m ? s : m;
    const A a = acc_exp(m - mn);
    const A pj = acc_exp(s - mn);
    l = l * a + pj;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int d = lane + 32 * t;
      if (d < p.D) acc[t] = acc[t] * a + pj * to_acc(v[kr + d]);
    }
    m = mn;
  }
  const A inv = l > A(0) ? A(1) / l : A(0);
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int d = lane + 32 * t;
    if (d < p.D) o[qrow + d] = from_acc<DT>(acc[t] * inv);
  }
  if (lane == 0 && lse != nullptr)
    lse[(size_t)bh * p.q_rows_alloc + p.q_row0 + i] = l > A(0) ? (float)(m + acc_log(l)) : -INFINITY;
}

// delta_i = sum_d O_i[d] * dO_i[d].  For double I/O the row logsumexp is
// also recomputed in double (lse_acc), because the float lse of the C ABI
// would cap the backward at float accuracy.
template <typename DT>
__global__ void attn_bwd_delta_simt(const DT* __restrict__ q, const DT* __restrict__ k, const DT* __restrict__ o,
                                    const DT* __restrict__ dO, AccT<DT>* __restrict__ delta,
                                    AccT<DT>* __restrict__ lse_acc, SimtParams p) {
  using A = AccT<DT>;
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)p.BH * p.Tq) return;
  const int bh = (int)(w / p.Tq), i = (int)(w % p.Tq);
  const size_t row = ((size_t)bh * p.q_rows_alloc + p.q_row0 + i) * p.D;
  A s = 0;
  for (int d = lane; d < p.D; d += 32) s += to_acc(o[row + d]) * to_acc(dO[row + d]);
  s = warp_sum(s);
  if (lane == 0) delta[(size_t)bh * p.Tq + i] = s;
  if (lse_acc != nullptr) {
    const size_t kbase = ((size_t)bh * p.k_rows_alloc + p.k_row0) * p.D;
    A qv[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int d = lane + 32 * t;
      qv[t] = d < p.D ? to_acc(q[row + d]) : A(0);
    }
    A m = -INFINITY, l = 0;
    const int last = simt_last_key(p, i);
    for (int j = 0; j <= last; ++j) {
      A x = 0;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int d = lane + 32 * t;
        if (d < p.D) x += qv[t] * to_acc(k[kbase + (size_t)j * p.D + d]);
      }
      x = warp_sum(x) * (A)p.scale;
      const A mn = x > m ? x : m;
      l = l * acc_exp(m - mn) + acc_exp(x - mn);
      m = mn;
    }
    if (lane == 0) lse_acc[(size_t)bh * p.Tq + i] = m + acc_log(l);
  }
}

// Row logsumexp for the backward: the recomputed one when present, else the forward's.
template <typename A>
__device__ __forceinline__ A row_lse(const float* lse, const A* lse_acc, const SimtParams& p, int bh, int i) {
  return lse_acc != nullptr ? lse_acc[(size_t)bh * p.Tq + i] : (A)lse[(size_t)bh * p.q_rows_alloc + p.q_row0 + i];
}

// dQ_i = scale * sum_j P_ij (dP_ij - delta_i) K_j, with P_ij = exp(scale*q_i.k_j - lse_i), dP_ij = dO_i.v_j
template <typename DT>
__global__ void attn_bwd_dq_simt(const DT* __restrict__ q, const DT* __restrict__ k, const DT* __restrict__ v,
                                 const DT* __restrict__ dO, const float* __restrict__ lse,
                                 const AccT<DT>* __restrict__ lse_acc, const AccT<DT>* __restrict__ delta,
                                 DT* __restrict__ dq, SimtParams p) {
  using A = AccT<DT>;
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)p.BH * p.Tq) return;
  const int bh = (int)(w / p.Tq), i = (int)(w % p.Tq);
  const size_t qrow = ((size_t)bh * p.q_rows_alloc + p.q_row0 + i) * p.D;
  const size_t kbase = ((size_t)bh * p.k_rows_alloc + p.k_row0) * p.D;
  A qv[8], gv[8], acc[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int d = lane + 32 * t;
    qv[t] = d < p.D ? to_acc(q[qrow + d]) : A(0);
    gv[t] = d < p.D ? to_acc(dO[qrow + d]) : A(0);
    acc[t] = A(0);
  }
  const A scale = (A)p.scale;
  const A L = row_lse(lse, lse_acc, p, bh, i);
  const A dl = delta[(size_t)bh * p.Tq + i];
  const int last = simt_last_key(p, i);
  for (int j = 0; j <= last; ++j) {
    const size_t kr = kbase + (size_t)j * p.D;
    A s = 0, dp = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int d = lane + 32 * t;
      if (d < p.D) {
        s += qv[t] * to_acc(k[kr + d]);
        dp += gv[t] * to_acc(v[kr + d]);
      }
    }
    s = warp_sum(s);
    dp = warp_sum(dp);
    const A pij = acc_exp(s * scale - L);
    const A ds = pij * (dp - dl) * scale;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int d = lane + 32 * t;
      if (d < p.D) acc[t] += ds * to_acc(k[kr + d]);
    }
  }
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int d = lane + 32 * t;
    if (d < p.D) dq[qrow + d] = from_acc<DT>(acc[t]);
  }
}

// dV_j = sum_i P_ij dO_i ; dK_j = scale * sum_i P_ij (dP_ij - delta_i) Q_i  (one warp per key row)
template <typename DT>
__global__ void attn_bwd_dkdv_simt(const DT* __restrict__ q, const DT* __restrict__ k, const DT* __restrict__ v,
                                   const DT* __restrict__ dO, const float* __restrict__ lse,
                                   const AccT<DT>* __restrict__ lse_acc, const AccT<DT>* __restrict__ delta,
                                   DT* __restrict__ dk, DT* __restrict__ dv, SimtParams p) {
  using A = AccT<DT>;
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)p.BH * p.Tk) return;
  const int bh = (int)(w / p.Tk), j = (int)(w % p.Tk);
  const size_t krow = ((size_t)bh * p.k_rows_alloc + p.k_row0 + j) * p.D;
  const size_t qbase = ((size_t)bh * p.q_rows_alloc + p.q_row0) * p.D;
  A kv[8], vv[8], adk[8], adv[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int d = lane + 32 * t;
    kv[t] = d < p.D ? to_acc(k[krow + d]) : A(0);
    vv[t] = d < p.D ? to_acc(v[krow + d]) : A(0);
    adk[t] = A(0);
    adv[t] = A(0);
  }
  const A scale = (A)p.scale;
  int first = 0;
  if (p.causal) first = max(0, j - p.causal_offset);
  for (int i = first; i < p.Tq; ++i) {
    const size_t qr = qbase + (size_t)i * p.D;
    A s = 0, dp = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int d = lane + 32 * t;
      if (d < p.D) {
        s += to_acc(q[qr + d]) * kv[t];
        dp += to_acc(dO[qr + d]) * vv[t];
      }
    }
    s = warp_sum(s);
    dp = warp_sum(dp);
    const A L = row_lse(lse, lse_acc, p, bh, i);
    const A pij = acc_exp(s * scale - L);
    const A ds = pij * (dp - delta[(size_t)bh * p.Tq + i]) * scale;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int d = lane + 32 * t;
      if (d < p.D) {
        adv[t] += pij * to_acc(dO[qr + d]);
        adk[t] += ds * to_acc(q[qr + d]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int d = lane + 32 * t;
    if (d < p.D) {
      dk[krow + d] = from_acc<DT>(adk[t]);
      dv[krow + d] = from_acc<DT>(adv[t]);
    }
  }
}

}  // namespace ctfa
