// The block's other layers for the config-4 training step (survey §8 "next",
// item 4): the MLP's Linear layers (with the ReLU between them fused into the
// GEMM epilogues) and LayerNorm.  Included by ctfa_api.cu after
// proj_api.cuh, inside the library's single translation unit.
//
// Linear (cuda_transformer/LinearLayer.cu, kernels linear_kernels.cu):
// y = x W^T + b with W [N, K] (row = output feature, linear_kernels.cu:64).
// The GEMMs are the projection kernels with one head spanning the whole
// feature dimension: forward = kProjOutFwd with H = 1, D = K; input gradient =
// kProjQkvDx with one weight (H = 1, D = N); weight + bias gradient =
// kProjOutDw (H = 1, D = K).  A ReLU after the layer (relu_kernels.cu:26-38)
// is fused into the forward epilogue; the ReLU before a layer is fused into
// that layer's input-gradient epilogue (dx_mask: the ReLU's output, dx is
// zeroed where it is not positive, relu_kernels.cu:62-75).
//
// LayerNorm (cuda_transformer/LayerNorm.cu, kernels layer_norm_kernels.cu):
// biased variance, eps given (1e-5 in the reference), y = x_hat * w + b;
// backward dx = rstd * (g - mean(g) - x_hat * mean(g * x_hat)) with
// g = dy * w, dw += sum dy * x_hat, db += sum dy (accumulated like the
// reference's atomicAdd, layer_norm_kernels.cu:131-133).  One warp per row;
// the parameter gradients are reduced per block before one atomic add per
// column.  HBM-bound.
#pragma once

namespace {

// ---------------------------------------------------------------------------
// LayerNorm kernels
// ---------------------------------------------------------------------------
template <typename AT>
__device__ __forceinline__ AT warp_sum(AT v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename AT>
__device__ __forceinline__ AT inv_sqrt(AT v) {
  if constexpr (sizeof(AT) == 8) return 1.0 / sqrt(v);
  else return rsqrtf(v);
}

template <typename DT>
__global__ void __launch_bounds__(256) layernorm_fwd_kernel(const DT* __restrict__ x, const DT* __restrict__ w,
                                                            const DT* __restrict__ b, DT* __restrict__ y,
                                                            float* __restrict__ mean, float* __restrict__ rstd,
                                                            int M, int E, float eps) {
  using AT = typename ProjAcc<DT>::type;
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M; row += warps) {
    const DT* xr = x + row * E;
    AT s = 0;
    for (int i = lane; i < E; i += 32) s += pacc(xr[i]);
    const AT mu = warp_sum(s) / (AT)E;
    AT v = 0;
    for (int i = lane; i < E; i += 32) {
      const AT d = pacc(xr[i]) - mu;
      v += d * d;
    }
    const AT rs = inv_sqrt(warp_sum(v) / (AT)E + (AT)eps);
    DT* yr = y + row * E;
    for (int i = lane; i < E; i += 32) yr[i] = pout<DT>((pacc(xr[i]) - mu) * rs * pacc(w[i]) + pacc(b[i]));
    if (lane == 0) {
      if (mean) mean[row] = (float)mu;
      if (rstd) rstd[row] = (float)rs;
    }
  }
}

// Rows are spread over the warps of the grid; each lane keeps partial
// dw / db for its columns (i = lane + 32 k, k < kMaxCols) in registers, the
// block reduces them in shared memory and adds one value per column.
constexpr int kLnMaxCols = 32;  // E <= 1024; wider rows: layernorm_bwd_wide_kernel

template <typename DT>
__global__ void __launch_bounds__(256) layernorm_bwd_kernel(const DT* __restrict__ x, const DT* __restrict__ dy,
                                                            const DT* __restrict__ w, const float* __restrict__ mean,
                                                            const float* __restrict__ rstd, DT* __restrict__ dx,
                                                            DT* __restrict__ dw, DT* __restrict__ db, int M, int E,
                                                            float eps) {
  using AT = typename ProjAcc<DT>::type;
  extern __shared__ unsigned char ln_smem[];
  AT* red = reinterpret_cast<AT*>(ln_smem);  // [2][E]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int i = threadIdx.x; i < 2 * E; i += blockDim.x) red[i] = 0;
  __syncthreads();
  AT pw[kLnMaxCols], pb[kLnMaxCols];
#pragma unroll
  for (int k = 0; k < kLnMaxCols; ++k) pw[k] = pb[k] = 0;
  const long long warps = (long long)gridDim.x * nw;
  for (long long row = (long long)blockIdx.x * nw + wid; row < M; row += warps) {
    const DT* xr = x + row * E;
    const DT* gr = dy + row * E;
    AT mu, rs;
    if (sizeof(AT) == 8 || mean == nullptr || rstd == nullptr) {
      // recompute the statistics (double: the fp32 caches would cost precision)
      AT s = 0;
      for (int i = lane; i < E; i += 32) s += pacc(xr[i]);
      mu = warp_sum(s) / (AT)E;
      AT v = 0;
      for (int i = lane; i < E; i += 32) {
        const AT d = pacc(xr[i]) - mu;
        v += d * d;
      }
      rs = inv_sqrt(warp_sum(v) / (AT)E + (AT)eps);
    } else {
      mu = mean[row];
      rs = rstd[row];
    }
    AT s1 = 0, s2 = 0;
#pragma unroll
    for (int k = 0; k < kLnMaxCols; ++k) {
      const int i = lane + 32 * k;
      if (i < E) {
        const AT xh = (pacc(xr[i]) - mu) * rs;
        const AT g = pacc(gr[i]);
        const AT gw = g * pacc(w[i]);
        s1 += gw;
        s2 += gw * xh;
        pw[k] += g * xh;
        pb[k] += g;
      }
    }
    s1 = warp_sum(s1) / (AT)E;
    s2 = warp_sum(s2) / (AT)E;
    DT* dr = dx + row * E;
#pragma unroll
    for (int k = 0; k < kLnMaxCols; ++k) {
      const int i = lane + 32 * k;
      if (i < E) {
        const AT xh = (pacc(xr[i]) - mu) * rs;
        dr[i] = pout<DT>(rs * (pacc(gr[i]) * pacc(w[i]) - s1 - xh * s2));
      }
    }
  }
  if (dw != nullptr || db != nullptr) {
#pragma unroll
    for (int k = 0; k < kLnMaxCols; ++k) {
      const int i = lane + 32 * k;
      if (i < E) {
        atomicAdd(&red[i], pw[k]);
        atomicAdd(&red[E + i], pb[k]);
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
      if (dw) atomicAdd(&dw[i], pout<DT>(red[i]));
      if (db) atomicAdd(&db[i], pout<DT>(red[E + i]));
    }
  }
}

// Rows wider than 32 * kLnMaxCols: the same row math with strided loops;
// the per-column dw / db partials go straight into the block's shared-memory
// sums (`smem_red`, 2 E accumulators) or, when those do not fit, into the
// global gradients.
template <typename DT>
__global__ void __launch_bounds__(256) layernorm_bwd_wide_kernel(const DT* __restrict__ x, const DT* __restrict__ dy,
                                                                 const DT* __restrict__ w,
                                                                 const float* __restrict__ mean,
                                                                 const float* __restrict__ rstd, DT* __restrict__ dx,
                                                                 DT* __restrict__ dw, DT* __restrict__ db, int M, int E,
                                                                 float eps, int smem_red) {
  using AT = typename ProjAcc<DT>::type;
  extern __shared__ unsigned char ln_smem[];
  AT* red = reinterpret_cast<AT*>(ln_smem);  // [2][E] when smem_red
  const bool want_p = dw != nullptr || db != nullptr;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (smem_red) {
    for (int i = threadIdx.x; i < 2 * E; i += blockDim.x) red[i] = 0;
    __syncthreads();
  }
  const long long warps = (long long)gridDim.x * nw;
  for (long long row = (long long)blockIdx.x * nw + wid; row < M; row += warps) {
    const DT* xr = x + row * E;
    const DT* gr = dy + row * E;
    AT mu, rs;
    if (sizeof(AT) == 8 || mean == nullptr || rstd == nullptr) {
      AT s = 0;
      for (int i = lane; i < E; i += 32) s += pacc(xr[i]);
      mu = warp_sum(s) / (AT)E;
      AT v = 0;
      for (int i = lane; i < E; i += 32) {
        const AT d = pacc(xr[i]) - mu;
        v += d * d;
      }
      rs = inv_sqrt(warp_sum(v) / (AT)E + (AT)eps);
    } else {
      mu = mean[row];
      rs = rstd[row];
    }
    AT s1 = 0, s2 = 0;
    for (int i = lane; i < E; i += 32) {
      const AT xh = (pacc(xr[i]) - mu) * rs;
      const AT g = pacc(gr[i]);
      const AT gw = g * pacc(w[i]);
      s1 += gw;
      s2 += gw * xh;
      if (want_p) {
        if (smem_red) {
          atomicAdd(&red[i], g * xh);
          atomicAdd(&red[E + i], g);
        } else {
          if (dw) atomicAdd(&dw[i], pout<DT>(g * xh));
          if (db) atomicAdd(&db[i], pout<DT>(g));
        }
      }
    }
    s1 = warp_sum(s1) / (AT)E;
    s2 = warp_sum(s2) / (AT)E;
    DT* dr = dx + row * E;
    for (int i = lane; i < E; i += 32) {
      const AT xh = (pacc(xr[i]) - mu) * rs;
      dr[i] = pout<DT>(rs * (pacc(gr[i]) * pacc(w[i]) - s1 - xh * s2));
    }
  }
  if (want_p && smem_red) {
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
      if (dw) atomicAdd(&dw[i], pout<DT>(red[i]));
      if (db) atomicAdd(&db[i], pout<DT>(red[E + i]));
    }
  }
}

template <typename DT>
int launch_layernorm_fwd(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd, int M, int E,
                         float eps, cudaStream_t st) {
  const long long blocks = std::max<long long>(1, std::min<long long>((M + 7) / 8, sm_count() * 8));
  layernorm_fwd_kernel<DT><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const DT*>(x), static_cast<const DT*>(w),
                                                              static_cast<const DT*>(b), static_cast<DT*>(y), mean,
                                                              rstd, M, E, eps);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CTFA_OK : cuda_fail(e, "launch layernorm_fwd_kernel");
}

template <typename DT>
int launch_layernorm_bwd(const void* x, const void* dy, const void* w, const float* mean, const float* rstd, void* dx,
                         void* dw, void* db, int M, int E, float eps, cudaStream_t st) {
  using AT = typename ProjAcc<DT>::type;
  const long long blocks = std::max<long long>(1, std::min<long long>((M + 7) / 8, sm_count() * 2));
  const size_t smem = 2 * (size_t)E * sizeof(AT);
  if (E <= 32 * kLnMaxCols) {
    layernorm_bwd_kernel<DT><<<(unsigned)blocks, 256, smem, st>>>(
        static_cast<const DT*>(x), static_cast<const DT*>(dy), static_cast<const DT*>(w), mean, rstd,
        static_cast<DT*>(dx), static_cast<DT*>(dw), static_cast<DT*>(db), M, E, eps);
  } else {
    // shared-memory column sums while they fit in the opt-in limit
    const bool smem_red = smem <= (size_t)max_dynamic_smem();
    if (smem_red && smem > 48 * 1024) {
      cudaError_t a = cudaFuncSetAttribute(layernorm_bwd_wide_kernel<DT>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (a != cudaSuccess) return cuda_fail(a, "cudaFuncSetAttribute(layernorm_bwd_wide_kernel)");
    }
    layernorm_bwd_wide_kernel<DT><<<(unsigned)blocks, 256, smem_red ? smem : 0, st>>>(
        static_cast<const DT*>(x), static_cast<const DT*>(dy), static_cast<const DT*>(w), mean, rstd,
        static_cast<DT*>(dx), static_cast<DT*>(dw), static_cast<DT*>(db), M, E, eps, smem_red ? 1 : 0);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CTFA_OK : cuda_fail(e, "launch layernorm_bwd_kernel");
}

int check_dtype_any(int dtype) {
  return dtype_bytes(dtype) == 0 ? fail(CTFA_ERR_INVALID_ARGUMENT, "unknown dtype") : CTFA_OK;
}

// Linear shapes on the projection GEMM: x as one head of dim K, y as rows of N.
bool linear_tensor_core(int dtype, int K, int N, std::initializer_list<const void*> ptrs) {
  if (!(dtype == CTFA_DTYPE_F32 || dtype == CTFA_DTYPE_TF32 || dtype == CTFA_DTYPE_BF16 || dtype == CTFA_DTYPE_F16))
    return false;
  const int CB = 128 / (int)dtype_bytes(dtype);
  if (K % CB != 0 || N % CB != 0) return false;
  for (const void* p : ptrs)
    if (p != nullptr && !aligned16(p)) return false;
  return true;
}

}  // namespace

// ---------------------------------------------------------------------------
// Entry points
// ---------------------------------------------------------------------------
extern "C" int ctfa_linear_forward(const void* x, const void* w, const void* b, void* y, int M, int K, int N, int relu,
                                   int dtype, void* stream) {
  int s = check_dtype_any(dtype);
  if (s != CTFA_OK) return s;
  if (M <= 0 || K <= 0 || N <= 0) return fail(CTFA_ERR_INVALID_ARGUMENT, "M, K and N must be positive");
  if (!x || !w || !y) return fail(CTFA_ERR_INVALID_ARGUMENT, "x, w and y must be non-null");
  cudaStream_t st = (cudaStream_t)stream;
  const ProjShape sh{1, M, N, 1, K, dtype};  // rows = M, E = N, one head of dim K
  if (!linear_tensor_core(dtype, K, N, {x, w, b, y})) {
    ProjSimtArgs g{1, M, 1, K, N, {x, nullptr, nullptr}, {w, nullptr, nullptr}, {b, nullptr, nullptr},
                   {y, nullptr, nullptr}, {}, relu, nullptr};
    return proj_simt_dispatch(dtype, kProjOutFwd, g, st);
  }
  CUtensorMap ta[3], tb[3], to[3];
  if ((s = map_heads(&ta[0], x, sh, 128, false)) != CTFA_OK) return s;
  if ((s = map_weight(&tb[0], w, sh, N, K, 128, false)) != CTFA_OK) return s;
  if ((s = map_rows(&to[0], y, sh, 128, false)) != CTFA_OK) return s;
  ta[1] = ta[2] = ta[0];
  tb[1] = tb[2] = tb[0];
  to[1] = to[2] = to[0];
  ProjParams p = proj_params(sh);
  p.m_tiles = p.row_tiles;
  p.n_tiles = ceil_div(N, 128);
  p.ksteps = K / (128 / (int)dtype_bytes(dtype));
  p.bias[0] = b;
  p.relu = relu ? 1 : 0;
  return proj_tc_dispatch<kProjOutFwd>(dtype, p, ta, tb, to, st);
}

extern "C" int ctfa_linear_backward(const void* x, const void* dy, const void* w, const void* dx_mask, void* dw,
                                    void* db, void* dx, int M, int K, int N, int dtype, void* stream) {
  int s = check_dtype_any(dtype);
  if (s != CTFA_OK) return s;
  if (M <= 0 || K <= 0 || N <= 0) return fail(CTFA_ERR_INVALID_ARGUMENT, "M, K and N must be positive");
  if (!dy) return fail(CTFA_ERR_INVALID_ARGUMENT, "dy must be non-null");
  const bool want_dw = dw || db;
  if (want_dw && (!dw || !x)) return fail(CTFA_ERR_INVALID_ARGUMENT, "dw and x are needed for the weight gradient");
  if (dx && !w) return fail(CTFA_ERR_INVALID_ARGUMENT, "w is needed for dx");
  cudaStream_t st = (cudaStream_t)stream;
  const bool tc = linear_tensor_core(dtype, K, N, {x, dy, w, dx_mask, dw, db, dx});
  const int CB = 128 / (int)dtype_bytes(dtype);
  if (want_dw) {
    const ProjShape sh{1, M, N, 1, K, dtype};  // dy rows of N (E), x one head of dim K
    if (!tc) {
      ProjSimtArgs g{1, M, 1, K, N, {dy, nullptr, nullptr}, {x, nullptr, nullptr}, {}, {dw, nullptr, nullptr},
                     {db, nullptr, nullptr}};
      if ((s = proj_simt_dispatch(dtype, kProjOutDw, g, st)) != CTFA_OK) return s;
    } else {
      CUtensorMap ta[3], tb[3], to[3];
      if ((s = map_rows(&ta[0], dy, sh, CB, true)) != CTFA_OK) return s;
      if ((s = map_heads(&tb[0], x, sh, CB, true)) != CTFA_OK) return s;
      if ((s = map_weight(&to[0], dw, sh, N, K, 128, false)) != CTFA_OK) return s;
      ta[1] = ta[2] = ta[0];
      tb[1] = tb[2] = tb[0];
      to[1] = to[2] = to[0];
      ProjParams p = proj_params(sh);
      p.m_tiles = ceil_div(N, 128);
      p.n_tiles = ceil_div(K, 128);
      p.kt = ceil_div(M, CB);
      p.ksteps = p.kt;
      p.splits = dw_splits(p.m_tiles * p.n_tiles, p.ksteps);
      p.dbias[0] = db;
      p.dw[0] = dw;
      if ((s = proj_tc_dispatch<kProjOutDw>(dtype, p, ta, tb, to, st)) != CTFA_OK) return s;
    }
  }
  if (dx) {
    const ProjShape sh{1, M, K, 1, N, dtype};  // dy as one head of dim N, dx rows of K (E)
    if (!tc) {
      ProjSimtArgs g{1, M, 1, N, K, {dy, nullptr, nullptr}, {w, nullptr, nullptr}, {}, {dx, nullptr, nullptr}, {},
                     0, dx_mask};
      return proj_simt_dispatch(dtype, kProjQkvDx, g, st);
    }
    CUtensorMap ta[3], tb[3], to[3];
    if ((s = map_heads(&ta[0], dy, sh, 128, false)) != CTFA_OK) return s;
    if ((s = map_weight(&tb[0], w, sh, N, K, CB, true)) != CTFA_OK) return s;
    if ((s = map_rows(&to[0], dx, sh, 128, false)) != CTFA_OK) return s;
    ta[1] = ta[2] = ta[0];
    tb[1] = tb[2] = tb[0];
    to[1] = to[2] = to[0];
    ProjParams p = proj_params(sh);
    p.m_tiles = p.row_tiles;
    p.n_tiles = ceil_div(K, 128);
    p.ksteps = N / CB;  // one weight
    p.mask = dx_mask;
    if ((s = proj_tc_dispatch<kProjQkvDx>(dtype, p, ta, tb, to, st)) != CTFA_OK) return s;
  }
  return CTFA_OK;
}

extern "C" int ctfa_layernorm_forward(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd,
                                      int M, int E, float eps, int dtype, void* stream) {
  int s = check_dtype_any(dtype);
  if (s != CTFA_OK) return s;
  if (M <= 0 || E <= 0) return fail(CTFA_ERR_INVALID_ARGUMENT, "M and E must be positive");
  if (!(eps > 0.f)) return fail(CTFA_ERR_INVALID_ARGUMENT, "eps must be positive");
  if (!x || !w || !b || !y) return fail(CTFA_ERR_INVALID_ARGUMENT, "x, w, b and y must be non-null");
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case CTFA_DTYPE_F32:
    case CTFA_DTYPE_TF32: return launch_layernorm_fwd<float>(x, w, b, y, mean, rstd, M, E, eps, st);
    case CTFA_DTYPE_BF16: return launch_layernorm_fwd<__nv_bfloat16>(x, w, b, y, mean, rstd, M, E, eps, st);
    case CTFA_DTYPE_F16: return launch_layernorm_fwd<__half>(x, w, b, y, mean, rstd, M, E, eps, st);
    default: return launch_layernorm_fwd<double>(x, w, b, y, mean, rstd, M, E, eps, st);
  }
}

extern "C" int ctfa_layernorm_backward(const void* x, const void* dy, const void* w, const float* mean,
                                       const float* rstd, void* dx, void* dw, void* db, int M, int E, float eps,
                                       int dtype, void* stream) {
  int s = check_dtype_any(dtype);
  if (s != CTFA_OK) return s;
  if (M <= 0 || E <= 0) return fail(CTFA_ERR_INVALID_ARGUMENT, "M and E must be positive");
  if (!(eps > 0.f)) return fail(CTFA_ERR_INVALID_ARGUMENT, "eps must be positive");
  if (!x || !dy || !w || !dx) return fail(CTFA_ERR_INVALID_ARGUMENT, "x, dy, w and dx must be non-null");
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case CTFA_DTYPE_F32:
    case CTFA_DTYPE_TF32: return launch_layernorm_bwd<float>(x, dy, w, mean, rstd, dx, dw, db, M, E, eps, st);
    case CTFA_DTYPE_BF16:
      return launch_layernorm_bwd<__nv_bfloat16>(x, dy, w, mean, rstd, dx, dw, db, M, E, eps, st);
    case CTFA_DTYPE_F16: return launch_layernorm_bwd<__half>(x, dy, w, mean, rstd, dx, dw, db, M, E, eps, st);
    default: return launch_layernorm_bwd<double>(x, dy, w, mean, rstd, dx, dw, db, M, E, eps, st);
  }
}
