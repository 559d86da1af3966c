// Host side of the projection GEMMs (ctfa_qkv_* / ctfa_out_proj_* in
// include/ctfa.h).  Included by ctfa_api.cu after its helpers (status
// handling, tensor-map entry point, wait limit), inside the library's single
// translation unit.
//
// Path selection is by element type and shape only: f32 / bf16 / f16 with
// D = 64 or 128, 16-byte-aligned tensors and rows (E * element size a multiple
// of 16 bytes) run proj_gemm_sm100; everything else (double, other D, odd E)
// runs the SIMT kernels below.  Both are GPU kernels; there is no host path.
#pragma once

#include <algorithm>
#include <initializer_list>
#include <type_traits>

#include "proj_gemm_sm100.cuh"

namespace {

using namespace ctfa;

// Pipeline depth per kind.  Row-wise kinds: 2 stages (64 KB, also the fp32
// staging tile) so that three CTAs share an SM (3 x 128 TMEM columns): the
// output-projection and dx/da grids (B*T/128 x E/128 CTAs, 384 at config 4)
// then run in one wave.  Weight-gradient kinds: 3 stages, two CTAs per SM
// (their accumulator is 256 TMEM columns wide for the bias-gradient block).
template <int KIND>
constexpr int proj_stages() {
  return (KIND == kProjQkvDw || KIND == kProjOutDw) ? 3 : 2;
}

// ---------------------------------------------------------------------------
// SIMT kernels: one thread per output element, accumulation in double for
// double tensors and in float otherwise.
// ---------------------------------------------------------------------------
template <typename DT>
struct ProjAcc {
  using type = float;
};
template <>
struct ProjAcc<double> {
  using type = double;
};

template <typename DT>
__device__ __forceinline__ typename ProjAcc<DT>::type pacc(DT x) {
  if constexpr (std::is_same<DT, __nv_bfloat16>::value) return __bfloat162float(x);
  else if constexpr (std::is_same<DT, __half>::value) return __half2float(x);
  else return x;
}
template <typename DT>
__device__ __forceinline__ DT pout(typename ProjAcc<DT>::type x) {
  if constexpr (std::is_same<DT, __nv_bfloat16>::value) return __float2bfloat16_rn(x);
  else if constexpr (std::is_same<DT, __half>::value) return __float2half_rn(x);
  else return (DT)x;
}

struct ProjSimtArgs {
  int B, T, H, D, E;
  const void* a[3];  // x | a | dq,dk,dv | dy
  const void* w[3];  // weights
  const void* bias[3];
  void* out[3];
  void* dbias[3];
  int relu;          // kProjOutFwd: max(y, 0)
  const void* mask;  // kProjQkvDx: dx *= (mask > 0)
};

// kind: a ProjKind.  Element counts per kind are computed by the launcher.
template <typename DT>
__global__ void __launch_bounds__(256) proj_simt_kernel(int kind, ProjSimtArgs g, long long total) {
  using AT = typename ProjAcc<DT>::type;
  const int B = g.B, T = g.T, H = g.H, D = g.D, E = g.E, HD = H * D;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    AT acc = 0;
    if (kind == kProjQkvFwd) {  // idx over [3][B][H][T][D]
      const long long per = (long long)B * H * T * D;
      const int w = (int)(idx / per);
      const long long r = idx % per;
      const int d = (int)(r % D), t = (int)((r / D) % T), h = (int)((r / ((long long)D * T)) % H),
                b = (int)(r / ((long long)D * T * H));
      const DT* x = static_cast<const DT*>(g.a[0]) + ((size_t)b * T + t) * E;
      const DT* wr = static_cast<const DT*>(g.w[w]) + (size_t)(h * D + d) * E;
      for (int i = 0; i < E; ++i) acc += pacc(x[i]) * pacc(wr[i]);
      if (g.bias[w]) acc += pacc(static_cast<const DT*>(g.bias[w])[h * D + d]);
      static_cast<DT*>(g.out[w])[r] = pout<DT>(acc);
    } else if (kind == kProjOutFwd || kind == kProjQkvDx) {  // idx over [B][T][E]
      const int o = (int)(idx % E);
      const long long bt = idx / E;
      const int t = (int)(bt % T), b = (int)(bt / T);
      const int nw = (kind == kProjQkvDx && g.w[1] != nullptr) ? 3 : 1;  // one weight: a Linear layer's dx
      for (int w = 0; w < nw; ++w) {
        const DT* a = static_cast<const DT*>(g.a[w]);
        const DT* wt = static_cast<const DT*>(g.w[w]);
        for (int h = 0; h < H; ++h) {
          const DT* arow = a + (((size_t)b * H + h) * T + t) * D;
          for (int d = 0; d < D; ++d) {
            const AT wv = (kind == kProjOutFwd) ? pacc(wt[(size_t)o * HD + h * D + d])
                                                : pacc(wt[(size_t)(h * D + d) * E + o]);
            acc += pacc(arow[d]) * wv;
          }
        }
      }
      if (kind == kProjOutFwd && g.bias[0]) acc += pacc(static_cast<const DT*>(g.bias[0])[o]);
      if (kind == kProjOutFwd && g.relu && !(acc > 0)) acc = 0;
      if (kind == kProjQkvDx && g.mask && !(pacc(static_cast<const DT*>(g.mask)[idx]) > 0)) acc = 0;
      static_cast<DT*>(g.out[0])[idx] = pout<DT>(acc);
    } else if (kind == kProjOutDa) {  // idx over [B][H][T][D]
      const int d = (int)(idx % D), t = (int)((idx / D) % T), h = (int)((idx / ((long long)D * T)) % H),
                b = (int)(idx / ((long long)D * T * H));
      const DT* dy = static_cast<const DT*>(g.a[0]) + ((size_t)b * T + t) * E;
      const DT* wo = static_cast<const DT*>(g.w[0]);
      for (int o = 0; o < E; ++o) acc += pacc(dy[o]) * pacc(wo[(size_t)o * HD + h * D + d]);
      static_cast<DT*>(g.out[0])[idx] = pout<DT>(acc);
    } else if (kind == kProjQkvDw) {  // idx over [3][HD][E + 1]: column E is the bias gradient
      const long long per = (long long)HD * (E + 1);
      const int w = (int)(idx / per);
      const long long r = idx % per;
      const int n = (int)(r / (E + 1)), i = (int)(r % (E + 1));
      if (i == E && !g.dbias[w]) continue;
      if (i < E && !g.out[w]) continue;
      const int h = n / D, d = n % D;
      const DT* dw = static_cast<const DT*>(g.a[w]);
      const DT* x = static_cast<const DT*>(g.w[0]);
      for (int b = 0; b < B; ++b)
        for (int t = 0; t < T; ++t) {
          const AT gv = pacc(dw[(((size_t)b * H + h) * T + t) * D + d]);
          acc += (i == E) ? gv : gv * pacc(x[((size_t)b * T + t) * E + i]);
        }
      DT* dst = (i == E) ? static_cast<DT*>(g.dbias[w]) + n : static_cast<DT*>(g.out[w]) + (size_t)n * E + i;
      *dst = pout<DT>(pacc(*dst) + acc);
    } else {  // kProjOutDw, idx over [E][HD + 1]: column HD is the bias gradient
      const int o = (int)(idx / (HD + 1)), j = (int)(idx % (HD + 1));
      if (j == HD && !g.dbias[0]) continue;
      if (j < HD && !g.out[0]) continue;
      const int h = j / D, d = j % D;
      const DT* dy = static_cast<const DT*>(g.a[0]);
      const DT* a = static_cast<const DT*>(g.w[0]);
      for (int b = 0; b < B; ++b)
        for (int t = 0; t < T; ++t) {
          const AT gv = pacc(dy[((size_t)b * T + t) * E + o]);
          acc += (j == HD) ? gv : gv * pacc(a[(((size_t)b * H + h) * T + t) * D + d]);
        }
      DT* dst = (j == HD) ? static_cast<DT*>(g.dbias[0]) + o : static_cast<DT*>(g.out[0]) + (size_t)o * HD + j;
      *dst = pout<DT>(pacc(*dst) + acc);
    }
  }
}

template <typename DT>
int launch_proj_simt(int kind, const ProjSimtArgs& g, cudaStream_t stream) {
  const long long HD = (long long)g.H * g.D;
  long long total = 0;
  switch (kind) {
    case kProjQkvFwd: total = 3LL * g.B * HD * g.T; break;
    case kProjOutFwd:
    case kProjQkvDx: total = (long long)g.B * g.T * g.E; break;
    case kProjOutDa: total = (long long)g.B * HD * g.T; break;
    case kProjQkvDw: total = 3LL * HD * (g.E + 1); break;
    default: total = (long long)g.E * (HD + 1); break;
  }
  const long long blocks = std::min<long long>((total + 255) / 256, sm_count() * 16);
  proj_simt_kernel<DT><<<(unsigned)std::max<long long>(1, blocks), 256, 0, stream>>>(kind, g, total);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CTFA_OK : cuda_fail(e, "launch proj_simt_kernel");
}

int proj_simt_dispatch(int dtype, int kind, const ProjSimtArgs& g, cudaStream_t stream) {
  switch (dtype) {
    case CTFA_DTYPE_F32:
    case CTFA_DTYPE_TF32: return launch_proj_simt<float>(kind, g, stream);
    case CTFA_DTYPE_BF16: return launch_proj_simt<__nv_bfloat16>(kind, g, stream);
    case CTFA_DTYPE_F16: return launch_proj_simt<__half>(kind, g, stream);
    default: return launch_proj_simt<double>(kind, g, stream);
  }
}

// ---------------------------------------------------------------------------
// Tensor-core path
// ---------------------------------------------------------------------------
// 4-D map over a contiguous tensor with dims[0] innermost; box = one 128-byte
// column block x box_rows x 1 x 1.  mn32: the 32-byte-granule 128-byte swizzle
// that tf32 operands read MN-major need; otherwise the plain 128-byte swizzle.
int make_map4(CUtensorMap* map, const void* base, int dtype, const uint64_t (&dims)[4], int box_rows, bool mn32) {
  auto fn = encode_fn();
  if (!fn) return fail(CTFA_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const size_t eb = dtype_bytes(dtype);
  CUtensorMapDataType dt = (eb == 4) ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : dtype == CTFA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t strides[3] = {dims[0] * eb, dims[0] * dims[1] * eb, dims[0] * dims[1] * dims[2] * eb};
  cuuint32_t box[4] = {(cuuint32_t)(128 / eb), (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), d, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  mn32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CTFA_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return CTFA_OK;
}

struct ProjShape {
  int B, T, E, H, D, dtype;
  int HD() const { return H * D; }
  bool tensor_core(std::initializer_list<const void*> ptrs) const {
    if (!(dtype == CTFA_DTYPE_F32 || dtype == CTFA_DTYPE_TF32 || dtype == CTFA_DTYPE_BF16 ||
          dtype == CTFA_DTYPE_F16))
      return false;
    if (!(D == 64 || D == 128)) return false;
    if ((size_t)E * dtype_bytes(dtype) % 16 != 0) return false;
    for (const void* p : ptrs)
      if (p != nullptr && !aligned16(p)) return false;
    return true;
  }
};

// Maps of the tensors the projections touch.
//   rows: [B, T, E]        dims (E, T, B, 1)
//   heads: [B, H, T, D]    dims (D, T, H, B)
//   weight [rows, cols]    dims (cols, rows, 1, 1)
int map_rows(CUtensorMap* m, const void* p, const ProjShape& s, int box_rows, bool mn) {
  const uint64_t dims[4] = {(uint64_t)s.E, (uint64_t)s.T, (uint64_t)s.B, 1};
  return make_map4(m, p, s.dtype, dims, box_rows, mn && dtype_bytes(s.dtype) == 4);
}
int map_heads(CUtensorMap* m, const void* p, const ProjShape& s, int box_rows, bool mn) {
  const uint64_t dims[4] = {(uint64_t)s.D, (uint64_t)s.T, (uint64_t)s.H, (uint64_t)s.B};
  return make_map4(m, p, s.dtype, dims, box_rows, mn && dtype_bytes(s.dtype) == 4);
}
int map_weight(CUtensorMap* m, const void* p, const ProjShape& s, int rows, int cols, int box_rows, bool mn) {
  const uint64_t dims[4] = {(uint64_t)cols, (uint64_t)rows, 1, 1};
  return make_map4(m, p, s.dtype, dims, box_rows, mn && dtype_bytes(s.dtype) == 4);
}

template <typename DT, int KIND>
int launch_proj_tc(ProjParams p, const CUtensorMap (&ta)[3], const CUtensorMap (&tb)[3], const CUtensorMap (&to)[3],
                   cudaStream_t stream) {
  constexpr int kStages = proj_stages<KIND>();
  using C = ProjConfig<DT, KIND, kStages>;
  auto kern = proj_gemm_sm100<DT, KIND, kStages>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(proj_gemm_sm100)");
  p.wait_limit_ns = g_wait_limit_ns;
  const long long grid = (long long)p.m_tiles * p.splits * p.n_tiles;
  if (grid <= 0 || grid > 0x7fffffffLL) return fail(CTFA_ERR_UNSUPPORTED, "projection grid out of range");
  kern<<<(unsigned)grid, C::THREADS, C::SMEM_BYTES, stream>>>(ta[0], ta[1], ta[2], tb[0], tb[1], tb[2], to[0],
                                                               to[1], to[2], p);
  e = cudaGetLastError();
  return e == cudaSuccess ? CTFA_OK : cuda_fail(e, "launch proj_gemm_sm100");
}

template <int KIND>
int proj_tc_dispatch(int dtype, const ProjParams& p, const CUtensorMap (&ta)[3], const CUtensorMap (&tb)[3],
                     const CUtensorMap (&to)[3], cudaStream_t stream) {
  switch (dtype) {
    case CTFA_DTYPE_F32:
    case CTFA_DTYPE_TF32: return launch_proj_tc<float, KIND>(p, ta, tb, to, stream);
    case CTFA_DTYPE_BF16: return launch_proj_tc<__nv_bfloat16, KIND>(p, ta, tb, to, stream);
    default: return launch_proj_tc<__half, KIND>(p, ta, tb, to, stream);
  }
}

ProjParams proj_params(const ProjShape& s) {
  ProjParams p;
  std::memset(&p, 0, sizeof(p));
  p.B = s.B;
  p.T = s.T;
  p.H = s.H;
  p.D = s.D;
  p.E = s.E;
  p.row_tiles = (s.T + 127) / 128;
  p.splits = 1;
  return p;
}

int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

// Split count for the weight-gradient GEMMs: as many CTAs as fit in ONE wave
// (two per SM, see proj_stages), at least two k-steps per CTA.  Rounding up instead would put
// a few CTAs into a second wave and double the kernel's duration.
int dw_splits(int tiles, int ksteps) {
  const long long want = (2 * sm_count()) / tiles;
  return (int)std::max<long long>(1, std::min<long long>(want, ksteps / 2));
}

int check_proj(int B, int T, int E, int H, int D, int dtype) {
  if (B <= 0 || T <= 0 || E <= 0 || H <= 0 || D <= 0)
    return fail(CTFA_ERR_INVALID_ARGUMENT, "B, T, E, H and D must be positive");
  if (dtype_bytes(dtype) == 0) return fail(CTFA_ERR_INVALID_ARGUMENT, "unknown dtype");
  if ((long long)B * T * std::max<long long>(E, (long long)H * D) > (1LL << 40))
    return fail(CTFA_ERR_UNSUPPORTED, "problem too large");
  return CTFA_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// Entry points
// ---------------------------------------------------------------------------
extern "C" int ctfa_qkv_forward(const void* x, const void* wq, const void* bq, const void* wk, const void* bk,
                                const void* wv, const void* bv, void* q, void* k, void* v, int B, int T, int E,
                                int H, int D, int dtype, void* stream) {
  int s = check_proj(B, T, E, H, D, dtype);
  if (s != CTFA_OK) return s;
  if (!x || !wq || !wk || !wv || !q || !k || !v)
    return fail(CTFA_ERR_INVALID_ARGUMENT, "x, wq, wk, wv, q, k and v must be non-null");
  const ProjShape sh{B, T, E, H, D, dtype};
  cudaStream_t st = (cudaStream_t)stream;
  if (!sh.tensor_core({x, wq, bq, wk, bk, wv, bv, q, k, v})) {
    ProjSimtArgs g{B, T, H, D, E, {x, nullptr, nullptr}, {wq, wk, wv}, {bq, bk, bv}, {q, k, v}, {}};
    return proj_simt_dispatch(dtype, kProjQkvFwd, g, st);
  }
  CUtensorMap ta[3], tb[3], to[3];
  const void* w[3] = {wq, wk, wv};
  void* o[3] = {q, k, v};
  if ((s = map_rows(&ta[0], x, sh, 128, false)) != CTFA_OK) return s;
  ta[1] = ta[2] = ta[0];
  for (int i = 0; i < 3; ++i) {
    if ((s = map_weight(&tb[i], w[i], sh, sh.HD(), E, 128, false)) != CTFA_OK) return s;
    if ((s = map_heads(&to[i], o[i], sh, 128, false)) != CTFA_OK) return s;
  }
  ProjParams p = proj_params(sh);
  p.m_tiles = B * p.row_tiles;
  p.n_tiles = 3 * ceil_div(sh.HD(), 128);
  p.ksteps = ceil_div(E, 128 / (int)dtype_bytes(dtype));
  p.bias[0] = bq;
  p.bias[1] = bk;
  p.bias[2] = bv;
  return proj_tc_dispatch<kProjQkvFwd>(dtype, p, ta, tb, to, st);
}

extern "C" int ctfa_qkv_backward(const void* x, const void* dq, const void* dk, const void* dv, const void* wq,
                                 const void* wk, const void* wv, void* dwq, void* dbq, void* dwk, void* dbk,
                                 void* dwv, void* dbv, void* dx, int B, int T, int E, int H, int D, int dtype,
                                 void* stream) {
  int s = check_proj(B, T, E, H, D, dtype);
  if (s != CTFA_OK) return s;
  if (!dq || !dk || !dv) return fail(CTFA_ERR_INVALID_ARGUMENT, "dq, dk and dv must be non-null");
  const bool want_dw = dwq || dwk || dwv || dbq || dbk || dbv;
  if (want_dw && !(dwq && dwk && dwv)) return fail(CTFA_ERR_INVALID_ARGUMENT, "dwq, dwk and dwv go together");
  if (want_dw && !x) return fail(CTFA_ERR_INVALID_ARGUMENT, "x is needed for the weight gradients");
  if (dx && !(wq && wk && wv)) return fail(CTFA_ERR_INVALID_ARGUMENT, "wq, wk and wv are needed for dx");
  const ProjShape sh{B, T, E, H, D, dtype};
  cudaStream_t st = (cudaStream_t)stream;
  if (!sh.tensor_core({x, dq, dk, dv, wq, wk, wv, dwq, dbq, dwk, dbk, dwv, dbv, dx})) {
    if (want_dw) {
      ProjSimtArgs g{B, T, H, D, E, {dq, dk, dv}, {x, nullptr, nullptr}, {}, {dwq, dwk, dwv}, {dbq, dbk, dbv}};
      if ((s = proj_simt_dispatch(dtype, kProjQkvDw, g, st)) != CTFA_OK) return s;
    }
    if (dx) {
      ProjSimtArgs g{B, T, H, D, E, {dq, dk, dv}, {wq, wk, wv}, {}, {dx, nullptr, nullptr}, {}};
      if ((s = proj_simt_dispatch(dtype, kProjQkvDx, g, st)) != CTFA_OK) return s;
    }
    return CTFA_OK;
  }
  const int CB = 128 / (int)dtype_bytes(dtype);
  const void* g3[3] = {dq, dk, dv};
  const void* w3[3] = {wq, wk, wv};
  if (want_dw) {
    CUtensorMap ta[3], tb[3], to[3];
    void* dw3[3] = {dwq, dwk, dwv};
    for (int i = 0; i < 3; ++i) {
      if ((s = map_heads(&ta[i], g3[i], sh, CB, true)) != CTFA_OK) return s;
      if ((s = map_weight(&to[i], dw3[i], sh, sh.HD(), E, 128, false)) != CTFA_OK) return s;
    }
    if ((s = map_rows(&tb[0], x, sh, CB, true)) != CTFA_OK) return s;
    tb[1] = tb[2] = tb[0];
    ProjParams p = proj_params(sh);
    p.m_tiles = 3 * ceil_div(sh.HD(), 128);
    p.n_tiles = ceil_div(E, 128);
    p.kt = ceil_div(T, CB);
    p.ksteps = B * p.kt;
    p.splits = dw_splits(p.m_tiles * p.n_tiles, p.ksteps);
    p.dbias[0] = dbq;
    p.dbias[1] = dbk;
    p.dbias[2] = dbv;
    for (int i = 0; i < 3; ++i) p.dw[i] = dw3[i];
    if ((s = proj_tc_dispatch<kProjQkvDw>(dtype, p, ta, tb, to, st)) != CTFA_OK) return s;
  }
  if (dx) {
    CUtensorMap ta[3], tb[3], to[3];
    for (int i = 0; i < 3; ++i) {
      if ((s = map_heads(&ta[i], g3[i], sh, 128, false)) != CTFA_OK) return s;
      if ((s = map_weight(&tb[i], w3[i], sh, sh.HD(), E, CB, true)) != CTFA_OK) return s;
    }
    if ((s = map_rows(&to[0], dx, sh, 128, false)) != CTFA_OK) return s;
    to[1] = to[2] = to[0];
    ProjParams p = proj_params(sh);
    p.m_tiles = B * p.row_tiles;
    p.n_tiles = ceil_div(E, 128);
    p.ksteps = 3 * H * (D / CB);
    if ((s = proj_tc_dispatch<kProjQkvDx>(dtype, p, ta, tb, to, st)) != CTFA_OK) return s;
  }
  return CTFA_OK;
}

extern "C" int ctfa_out_proj_forward(const void* a, const void* wo, const void* bo, void* y, int B, int T, int E,
                                     int H, int D, int dtype, void* stream) {
  int s = check_proj(B, T, E, H, D, dtype);
  if (s != CTFA_OK) return s;
  if (!a || !wo || !y) return fail(CTFA_ERR_INVALID_ARGUMENT, "a, wo and y must be non-null");
  const ProjShape sh{B, T, E, H, D, dtype};
  cudaStream_t st = (cudaStream_t)stream;
  if (!sh.tensor_core({a, wo, bo, y})) {
    ProjSimtArgs g{B, T, H, D, E, {a, nullptr, nullptr}, {wo, nullptr, nullptr}, {bo, nullptr, nullptr},
                   {y, nullptr, nullptr}, {}};
    return proj_simt_dispatch(dtype, kProjOutFwd, g, st);
  }
  const int CB = 128 / (int)dtype_bytes(dtype);
  CUtensorMap ta[3], tb[3], to[3];
  if ((s = map_heads(&ta[0], a, sh, 128, false)) != CTFA_OK) return s;
  if ((s = map_weight(&tb[0], wo, sh, E, sh.HD(), 128, false)) != CTFA_OK) return s;
  if ((s = map_rows(&to[0], y, sh, 128, false)) != CTFA_OK) return s;
  ta[1] = ta[2] = ta[0];
  tb[1] = tb[2] = tb[0];
  to[1] = to[2] = to[0];
  ProjParams p = proj_params(sh);
  p.m_tiles = B * p.row_tiles;
  p.n_tiles = ceil_div(E, 128);
  p.ksteps = H * (D / CB);
  p.bias[0] = bo;
  return proj_tc_dispatch<kProjOutFwd>(dtype, p, ta, tb, to, st);
}

extern "C" int ctfa_out_proj_backward(const void* a, const void* dy, const void* wo, void* dwo, void* dbo, void* da,
                                      int B, int T, int E, int H, int D, int dtype, void* stream) {
  int s = check_proj(B, T, E, H, D, dtype);
  if (s != CTFA_OK) return s;
  if (!dy) return fail(CTFA_ERR_INVALID_ARGUMENT, "dy must be non-null");
  const bool want_dw = dwo || dbo;
  if (want_dw && (!dwo || !a)) return fail(CTFA_ERR_INVALID_ARGUMENT, "dwo and a are needed for the weight gradients");
  if (da && !wo) return fail(CTFA_ERR_INVALID_ARGUMENT, "wo is needed for da");
  const ProjShape sh{B, T, E, H, D, dtype};
  cudaStream_t st = (cudaStream_t)stream;
  if (!sh.tensor_core({a, dy, wo, dwo, dbo, da})) {
    if (want_dw) {
      ProjSimtArgs g{B, T, H, D, E, {dy, nullptr, nullptr}, {a, nullptr, nullptr}, {}, {dwo, nullptr, nullptr},
                     {dbo, nullptr, nullptr}};
      if ((s = proj_simt_dispatch(dtype, kProjOutDw, g, st)) != CTFA_OK) return s;
    }
    if (da) {
      ProjSimtArgs g{B, T, H, D, E, {dy, nullptr, nullptr}, {wo, nullptr, nullptr}, {}, {da, nullptr, nullptr}, {}};
      if ((s = proj_simt_dispatch(dtype, kProjOutDa, g, st)) != CTFA_OK) return s;
    }
    return CTFA_OK;
  }
  const int CB = 128 / (int)dtype_bytes(dtype);
  if (want_dw) {
    CUtensorMap ta[3], tb[3], to[3];
    if ((s = map_rows(&ta[0], dy, sh, CB, true)) != CTFA_OK) return s;
    if ((s = map_heads(&tb[0], a, sh, CB, true)) != CTFA_OK) return s;
    if ((s = map_weight(&to[0], dwo, sh, E, sh.HD(), 128, false)) != CTFA_OK) return s;
    ta[1] = ta[2] = ta[0];
    tb[1] = tb[2] = tb[0];
    to[1] = to[2] = to[0];
    ProjParams p = proj_params(sh);
    p.m_tiles = ceil_div(E, 128);
    p.n_tiles = ceil_div(sh.HD(), 128);
    p.kt = ceil_div(T, CB);
    p.ksteps = B * p.kt;
    p.splits = dw_splits(p.m_tiles * p.n_tiles, p.ksteps);
    p.dbias[0] = dbo;
    p.dw[0] = dwo;
    if ((s = proj_tc_dispatch<kProjOutDw>(dtype, p, ta, tb, to, st)) != CTFA_OK) return s;
  }
  if (da) {
    CUtensorMap ta[3], tb[3], to[3];
    if ((s = map_rows(&ta[0], dy, sh, 128, false)) != CTFA_OK) return s;
    if ((s = map_weight(&tb[0], wo, sh, E, sh.HD(), CB, true)) != CTFA_OK) return s;
    if ((s = map_heads(&to[0], da, sh, 128, false)) != CTFA_OK) return s;
    ta[1] = ta[2] = ta[0];
    tb[1] = tb[2] = tb[0];
    to[1] = to[2] = to[0];
    ProjParams p = proj_params(sh);
    p.m_tiles = B * p.row_tiles;
    p.n_tiles = ceil_div(sh.HD(), 128);
    p.ksteps = ceil_div(E, CB);
    if ((s = proj_tc_dispatch<kProjOutDa>(dtype, p, ta, tb, to, st)) != CTFA_OK) return s;
  }
  return CTFA_OK;
}
