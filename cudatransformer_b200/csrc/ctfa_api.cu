// extern "C" entry points of libctfa_b200.so (declared in include/ctfa.h).
//
// Host side of the attention path: argument checks, TMA tensor-map encoding,
// kernel selection (compile-time element type x head dim), launches.  All
// launches go to the caller's stream; nothing here allocates device memory or
// synchronises, except ctfa_check_device_error / ctfa_selftest_wait_timeout.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/ctfa.h"
#include "attn_bwd_sm100.cuh"
#include "attn_fwd_sm100.cuh"
#include "attn_simt.cuh"

using namespace ctfa;

namespace {

constexpr int kVersion = 10000;  // 1.0.0
unsigned long long g_wait_limit_ns = 2000000000ull;
thread_local std::string g_last_error;

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(CTFA_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

size_t dtype_bytes(int dtype) {
  switch (dtype) {
    case CTFA_DTYPE_F32: return 4;
    case CTFA_DTYPE_BF16: return 2;
    case CTFA_DTYPE_F16: return 2;
    case CTFA_DTYPE_F64: return 8;
    case CTFA_DTYPE_TF32: return 4;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Tensor maps (driver entry point fetched through the runtime, no -lcuda)
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 3-D map over an allocation [BH][rows][D] with a (128-byte x box_rows x 1)
// box and 128-byte swizzle.  Rows past `rows` read as zero.  mn32: 128-byte
// swizzle with 32-byte granules, the layout of tf32 operands that the MMA
// reads N-major (V in the forward, the MN-major copies in the backward).
int make_map(CUtensorMap* map, const void* base, int dtype, int D, int rows, int BH, int box_rows,
             bool mn32 = false) {
  auto fn = encode_fn();
  if (!fn) return fail(CTFA_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const size_t eb = dtype_bytes(dtype);
  CUtensorMapDataType dt = (dtype == CTFA_DTYPE_F32 || dtype == CTFA_DTYPE_TF32) ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : dtype == CTFA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)D * eb, (cuuint64_t)rows * D * eb};
  cuuint32_t box[3] = {(cuuint32_t)(128 / eb), (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  mn32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CTFA_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return CTFA_OK;
}

int device_is_sm100(bool* yes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  *yes = (major == 10 && minor == 0);
  return CTFA_OK;
}

// Streaming multiprocessors of the current device (persistent grids).
long long sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0)
    return 148;
  return sms;
}

// Opt-in dynamic shared memory per block of the current device (bytes).
long long max_dynamic_smem() {
  int dev = 0, bytes = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&bytes, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || bytes <= 0)
    return 48 * 1024;
  return bytes;
}

// ---------------------------------------------------------------------------
// Problem description shared by the full-sequence and block entry points.
// ---------------------------------------------------------------------------
struct Problem {
  int B, H, D, dtype;
  int Tq, Tk;
  int q_rows, k_rows;  // rows per head in the allocations
  int q_row0, k_row0;
  int causal, causal_offset;
  float* o_f32 = nullptr;  // forward: fp32 output rows instead of o (block partials)
  int merge = 0;           // forward with o_f32: fold into the running (o_f32, lse) instead of overwriting
  int accumulate = 0;      // backward: add into fp32 dq/dk/dv instead of writing the I/O type
};

bool tensor_core_shape(const Problem& pr) {
  return (pr.dtype == CTFA_DTYPE_F32 || pr.dtype == CTFA_DTYPE_TF32 || pr.dtype == CTFA_DTYPE_BF16 ||
          pr.dtype == CTFA_DTYPE_F16) &&
         (pr.D == 64 || pr.D == 128);
}

// Launch `kern` on `stream`; with `pdl`, with programmatic stream
// serialization, so that its blocks may start while the previous kernel on the
// stream finishes (each kernel launched this way runs griddepcontrol.wait
// before it touches what the previous kernel writes).  Without it (per-kernel
// timing events between the launches) an ordinary launch.
template <typename... KArgs, typename... Args>
cudaError_t launch_after_previous(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t stream, Args... args) {
  if (!pdl) {
    kern<<<grid, block, smem, stream>>>(args...);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Heads per chunk of a heavy-first work order whose blocks stream
// `per_head_bytes` of one head's operands (K/V for the forward and dQ, Q/dO for
// dK/dV).  While every head's operands fit in half of the 126 MB L2 the plain
// order is kept (one chunk); beyond that the list is walked in chunks of about
// 16 MiB of heads, so that the blocks in flight re-read their operands from L2
// instead of HBM.  Measured on one B200 (forward + backward step, ms, plain
// order -> 8 / 16 / 32 / 48 MiB chunks): B=16 H=16 T=2048 D=128 bf16 1.79 ->
// 1.53 / 1.50 / 1.53 / 1.55; B=4 H=16 T=4096 D=128 bf16 1.37 -> 1.31 / 1.28 /
// 1.31 / 1.29; B=16 H=16 T=2048 D=64 bf16 1.067 -> 1.028 / 1.031 / 1.047 /
// 1.026; B=8 H=12 T=2048 D=64 fp32 0.662 -> 0.643 / 0.638 / 0.652 / 0.631.
constexpr long long kL2AllHeadsBytes = 64ll << 20;
constexpr long long kL2ChunkBytes = 16ll << 20;
int head_chunk(int BH, long long per_head_bytes) {
  if (per_head_bytes <= 0 || (long long)BH * per_head_bytes <= kL2AllHeadsBytes) return BH;
  return (int)std::max<long long>(1, std::min<long long>(BH, kL2ChunkBytes / per_head_bytes));
}

// RND (fp32 I/O): q, k, v are the caller's fp32 tensors; the kernel rounds
// every tile to tf32 in shared memory and writes the rounded copies to
// rounded[0..2] (same layout) for the backward.
template <typename DT, int HD, int NQ, int BN, int KST, int VST, bool RND = false>
int launch_fwd_tc(const Problem& pr, const void* q, const void* k, const void* v, void* o, float* lse,
                  cudaStream_t stream, void* const* rounded = nullptr) {
  using C = FwdConfig<DT, HD, NQ, BN, KST, VST>;
  CUtensorMap mq, mk, mv, mqr, mkr, mvr;
  int s;
  if ((s = make_map(&mq, q, pr.dtype, HD, pr.q_rows, pr.B * pr.H, 128)) != CTFA_OK) return s;
  if ((s = make_map(&mk, k, pr.dtype, HD, pr.k_rows, pr.B * pr.H, BN)) != CTFA_OK) return s;
  if ((s = make_map(&mv, v, pr.dtype, HD, pr.k_rows, pr.B * pr.H, BN, sizeof(DT) == 4)) != CTFA_OK) return s;
  if constexpr (RND) {
    if ((s = make_map(&mqr, rounded[0], pr.dtype, HD, pr.q_rows, pr.B * pr.H, 128)) != CTFA_OK) return s;
    if ((s = make_map(&mkr, rounded[1], pr.dtype, HD, pr.k_rows, pr.B * pr.H, BN)) != CTFA_OK) return s;
    if ((s = make_map(&mvr, rounded[2], pr.dtype, HD, pr.k_rows, pr.B * pr.H, BN, true)) != CTFA_OK) return s;
  } else {
    mqr = mq;
    mkr = mk;
    mvr = mv;
  }
  FwdParams p;
  p.BH = pr.B * pr.H;
  p.Tq = pr.Tq;
  p.Tk = pr.Tk;
  p.q_row0 = pr.q_row0;
  p.k_row0 = pr.k_row0;
  p.q_rows_alloc = pr.q_rows;
  p.causal = pr.causal;
  p.causal_offset = pr.causal_offset;
  const int q_tiles = (pr.Tq + 127) / 128;
  p.n_groups = (q_tiles + NQ - 1) / NQ;
  p.head_chunk = head_chunk(p.BH, 2ll * pr.Tk * HD * (long long)sizeof(DT));
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)HD));
  p.o = o;
  p.o_f32 = pr.o_f32;
  p.merge = pr.merge;
  // whole-head O in the I/O type: staged tiles stored by TMA (rows past T are
  // clipped by the map, which ends at the last row)
  CUtensorMap mo = mq;
  p.o_tma = (o != nullptr && pr.o_f32 == nullptr && pr.q_row0 == 0 && pr.Tq == pr.q_rows) ? 1 : 0;
  if (p.o_tma && (s = make_map(&mo, o, pr.dtype, HD, pr.q_rows, pr.B * pr.H, 128)) != CTFA_OK) return s;
  p.lse = lse;
  p.wait_limit_ns = g_wait_limit_ns;
  auto kern = attn_fwd_sm100<DT, HD, NQ, BN, KST, VST, RND>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attn_fwd_sm100)");
  if constexpr (C::REBALANCE) {
    // setmaxnreg can only redistribute the registers the block launched with
    static int checked_regs = 0;
    if (checked_regs == 0) {
      cudaFuncAttributes fa;
      if ((e = cudaFuncGetAttributes(&fa, kern)) != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
      checked_regs = fa.numRegs;
    }
    if (checked_regs < C::LAUNCH_REGS)
      return fail(CTFA_ERR_UNSUPPORTED, "attn_fwd_sm100 compiled below its register split");
  }
  const long long grid = (long long)p.n_groups * p.BH;
  if (grid > 0x7fffffffLL) return fail(CTFA_ERR_UNSUPPORTED, "grid too large");
  // programmatic serialization after whatever kernel precedes on the stream:
  // the forward's set-up overlaps its tail, and the forward waits for it
  // (griddepcontrol.wait) before reading q / k / v or writing anything
  e = launch_after_previous(true, kern, dim3((unsigned)grid), dim3(C::THREADS), C::SMEM_BYTES, stream, mq, mk, mv, mqr,
                            mkr, mvr, mo, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch attn_fwd_sm100");
  return CTFA_OK;
}

SimtParams simt_params(const Problem& pr) {
  SimtParams p;
  p.BH = pr.B * pr.H;
  p.Tq = pr.Tq;
  p.Tk = pr.Tk;
  p.D = pr.D;
  p.q_row0 = pr.q_row0;
  p.k_row0 = pr.k_row0;
  p.q_rows_alloc = pr.q_rows;
  p.k_rows_alloc = pr.k_rows;
  p.causal = pr.causal;
  p.causal_offset = pr.causal_offset;
  p.scale = 1.0 / std::sqrt((double)pr.D);
  return p;
}

unsigned warps_grid(long long warps) { return (unsigned)((warps * 32 + 255) / 256); }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Round-to-nearest tf32 copies of up to four fp32 tensors (one launch).  The
// tensor core truncates fp32 operands to tf32 (drops 13 mantissa bits toward
// zero); feeding it rounded values removes that bias.
struct RoundJob {
  const float4* in[4];
  float4* out[4];
  long long n4;  // float4 per tensor
  int count;
};

__global__ void __launch_bounds__(256) round_tf32_kernel(RoundJob job) {
  const int t = blockIdx.y;
  const float4* in = job.in[t];
  float4* out = job.out[t];
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  // four independent 16-byte loads in flight per thread; the inputs are read
  // once (evict-first), the rounded copies stay in L2 for the kernel after
  for (; i + 3 * stride < job.n4; i += 4 * stride) {
    float4 x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) x[u] = __ldcs(in + i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      x[u].x = __uint_as_float(f32_to_tf32_rna(x[u].x));
      x[u].y = __uint_as_float(f32_to_tf32_rna(x[u].y));
      x[u].z = __uint_as_float(f32_to_tf32_rna(x[u].z));
      x[u].w = __uint_as_float(f32_to_tf32_rna(x[u].w));
      out[i + u * stride] = x[u];
    }
  }
  for (; i < job.n4; i += stride) {
    float4 x = __ldcs(in + i);
    x.x = __uint_as_float(f32_to_tf32_rna(x.x));
    x.y = __uint_as_float(f32_to_tf32_rna(x.y));
    x.z = __uint_as_float(f32_to_tf32_rna(x.z));
    x.w = __uint_as_float(f32_to_tf32_rna(x.w));
    out[i] = x;
  }
}

int launch_round(const void* const* in, void* const* out, int count, size_t elems, cudaStream_t stream) {
  RoundJob job;
  for (int i = 0; i < 4; ++i) {
    job.in[i] = i < count ? reinterpret_cast<const float4*>(in[i]) : nullptr;
    job.out[i] = i < count ? reinterpret_cast<float4*>(out[i]) : nullptr;
  }
  job.n4 = (long long)(elems / 4);
  job.count = count;
  const long long sms = sm_count();
  // one resident wave (8 blocks of 256 threads per SM) over all tensors
  const long long want = (job.n4 + 255) / 256;
  dim3 grid((unsigned)std::max<long long>(1, std::min<long long>(want, (sms * 8 + count - 1) / count)), count);
  round_tf32_kernel<<<grid, 256, 0, stream>>>(job);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CTFA_OK : cuda_fail(e, "launch round_tf32_kernel");
}

// fp32 I/O on the tensor cores works on rounded operand copies in the workspace.
bool needs_rounding(int dtype, int D) { return dtype == CTFA_DTYPE_F32 && (D == 64 || D == 128); }

template <typename DT>
int launch_fwd_simt(const Problem& pr, const void* q, const void* k, const void* v, void* o, float* lse,
                    cudaStream_t stream) {
  SimtParams p = simt_params(pr);
  attn_fwd_simt<DT><<<warps_grid((long long)p.BH * p.Tq), 256, 0, stream>>>(
      (const DT*)q, (const DT*)k, (const DT*)v, (DT*)o, lse, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CTFA_OK : cuda_fail(e, "launch attn_fwd_simt");
}

size_t fwd_workspace(const Problem& pr) {
  if (!needs_rounding(pr.dtype, pr.D)) return 0;
  return 3 * align256((size_t)pr.B * pr.H * pr.q_rows * pr.D * sizeof(float));
}

int forward_impl(const Problem& pr, const void* q, const void* k, const void* v, void* o, float* lse,
                 void* ws, cudaStream_t stream) {
  int s;
  if (tensor_core_shape(pr)) {
    bool sm100 = false;
    s = device_is_sm100(&sm100);
    if (s != CTFA_OK) return s;
    if (!sm100) return fail(CTFA_ERR_UNSUPPORTED, "tensor-core attention kernels need an sm_100 (B200) device");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
      return fail(CTFA_ERR_MISALIGNED, "q/k/v/o must be 16-byte aligned");
    switch (pr.dtype) {
      case CTFA_DTYPE_F32: {
        const size_t n = (size_t)pr.B * pr.H * pr.q_rows * pr.D;
        char* w = reinterpret_cast<char*>(ws);
        void* r[3] = {w, w + align256(n * 4), w + 2 * align256(n * 4)};
        // rounding to tf32 happens inside the kernel, which also writes the
        // rounded copies the backward reads (CTFA_DTYPE_TF32)
        return pr.D == 64 ? launch_fwd_tc<float, 64, 2, 128, 2, 2, true>(pr, q, k, v, o, lse, stream, r)
                          : launch_fwd_tc<float, 128, 1, 64, 3, 2, true>(pr, q, k, v, o, lse, stream, r);
      }
      case CTFA_DTYPE_TF32:
        return pr.D == 64 ? launch_fwd_tc<float, 64, 2, 128, 3, 2>(pr, q, k, v, o, lse, stream)
                          : launch_fwd_tc<float, 128, 1, 64, 3, 2>(pr, q, k, v, o, lse, stream);
      case CTFA_DTYPE_BF16:
        return pr.D == 64 ? launch_fwd_tc<__nv_bfloat16, 64, 2, 128, 4, 3>(pr, q, k, v, o, lse, stream)
                          : launch_fwd_tc<__nv_bfloat16, 128, 2, 128, 2, 2>(pr, q, k, v, o, lse, stream);
      default:
        return pr.D == 64 ? launch_fwd_tc<__half, 64, 2, 128, 4, 3>(pr, q, k, v, o, lse, stream)
                          : launch_fwd_tc<__half, 128, 2, 128, 2, 2>(pr, q, k, v, o, lse, stream);
    }
  }
  switch (pr.dtype) {
    case CTFA_DTYPE_F32:
    case CTFA_DTYPE_TF32: return launch_fwd_simt<float>(pr, q, k, v, o, lse, stream);
    case CTFA_DTYPE_BF16: return launch_fwd_simt<__nv_bfloat16>(pr, q, k, v, o, lse, stream);
    case CTFA_DTYPE_F16: return launch_fwd_simt<__half>(pr, q, k, v, o, lse, stream);
    default: return launch_fwd_simt<double>(pr, q, k, v, o, lse, stream);
  }
}

int check_common(int B, int H, int T, int D, int dtype) {
  if (B <= 0 || H <= 0 || T <= 0 || D <= 0) return fail(CTFA_ERR_INVALID_ARGUMENT, "B, H, T and D must be positive");
  if (dtype_bytes(dtype) == 0) return fail(CTFA_ERR_INVALID_ARGUMENT, "unknown dtype");
  if (D > 256) return fail(CTFA_ERR_UNSUPPORTED, "head dim above 256 is not supported");
  if ((long long)B * H > 0x7fffffffLL) return fail(CTFA_ERR_UNSUPPORTED, "B*H too large");
  return CTFA_OK;
}

Problem full_problem(int B, int H, int T, int D, int dtype, int causal) {
  Problem pr;
  pr.B = B;
  pr.H = H;
  pr.D = D;
  pr.dtype = dtype;
  pr.Tq = pr.Tk = T;
  pr.q_rows = pr.k_rows = T;
  pr.q_row0 = pr.k_row0 = 0;
  pr.causal = causal ? 1 : 0;
  pr.causal_offset = 0;
  return pr;
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
// Rows of the padded per-row arrays of the tensor-core backward: each head's
// rows rounded up to a whole 128-row tile, so tiles read them with aligned
// vector loads and without bounds checks.
size_t padded_tq(const Problem& pr) { return (size_t)((pr.Tq + 127) / 128) * 128; }
size_t padded_rows(const Problem& pr) { return (size_t)pr.B * pr.H * padded_tq(pr); }
// Head of the tensor-core backward's workspace: -delta and -lse*log2(e) over
// the padded rows, then 256 bytes holding the dK/dV and dQ work-list counters.
size_t bwd_rows_bytes(const Problem& pr) { return 2 * align256(padded_rows(pr) * sizeof(float)) + 256; }

size_t bwd_workspace(const Problem& pr) {
  const size_t rows = (size_t)pr.B * pr.H * pr.Tq;
  if (tensor_core_shape(pr) && !(pr.D == 128 && (pr.dtype == CTFA_DTYPE_F32 || pr.dtype == CTFA_DTYPE_TF32))) {
    size_t ws = bwd_rows_bytes(pr);  // -delta, -lse*log2(e) (padded rows), work-list counters
    const size_t n = align256(rows * pr.D * sizeof(float));
    if (pr.dtype == CTFA_DTYPE_F32) ws += 4 * n;   // rounded q, k, v, dO
    if (pr.dtype == CTFA_DTYPE_TF32) ws += n;      // rounded dO
    return ws;
  }
  if (pr.dtype == CTFA_DTYPE_F64) return 2 * align256(rows * sizeof(double));  // delta + lse in double
  return align256(rows * sizeof(float));
}

// Optional profiling events: ev[0] before the first launch, ev[1] after the
// delta pass, ev[2] after the dK/dV pass, ev[3] after the dQ pass.
void record(cudaEvent_t* ev, int i, cudaStream_t stream) {
  if (ev) cudaEventRecord(ev[i], stream);
}

template <typename DT>
int launch_bwd_simt(const Problem& pr, const void* q, const void* k, const void* v, const void* o, const void* dO,
                    const float* lse, void* dq, void* dk, void* dv, void* ws, cudaStream_t stream,
                    cudaEvent_t* ev) {
  using A = AccT<DT>;
  SimtParams p = simt_params(pr);
  A* delta = reinterpret_cast<A*>(ws);
  // double I/O: the row logsumexp is recomputed in double (second workspace array)
  A* lse_acc = std::is_same<DT, double>::value
                   ? reinterpret_cast<A*>(reinterpret_cast<char*>(ws) + align256((size_t)p.BH * p.Tq * sizeof(A)))
                   : nullptr;
  record(ev, 0, stream);
  attn_bwd_delta_simt<DT><<<warps_grid((long long)p.BH * p.Tq), 256, 0, stream>>>(
      (const DT*)q, (const DT*)k, (const DT*)o, (const DT*)dO, delta, lse_acc, p);
  record(ev, 1, stream);
  attn_bwd_dkdv_simt<DT><<<warps_grid((long long)p.BH * p.Tk), 256, 0, stream>>>(
      (const DT*)q, (const DT*)k, (const DT*)v, (const DT*)dO, lse, lse_acc, delta, (DT*)dk, (DT*)dv, p);
  record(ev, 2, stream);
  attn_bwd_dq_simt<DT><<<warps_grid((long long)p.BH * p.Tq), 256, 0, stream>>>(
      (const DT*)q, (const DT*)k, (const DT*)v, (const DT*)dO, lse, lse_acc, delta, (DT*)dq, p);
  record(ev, 3, stream);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CTFA_OK : cuda_fail(e, "launch attn_bwd_simt");
}

template <typename DT, int HD>
int launch_bwd_tc(const Problem& pr, const void* q, const void* k, const void* v, const void* o, const void* dO,
                  const void* dO_mma, const float* lse, void* dq, void* dk, void* dv, void* ws, cudaStream_t stream,
                  cudaEvent_t* ev) {
  using C = BwdConfig<DT, HD>;
  const int BH = pr.B * pr.H;
  float* ndelta = reinterpret_cast<float*>(ws);
  // 1. -delta = -rowsum(O * dO), and -lse * log2(e)
  const int Tq_pad = (int)padded_tq(pr);
  float* nlse2 = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + align256(padded_rows(pr) * sizeof(float)));
  BwdPrepParams pp;
  pp.rows = (long long)BH * Tq_pad;
  pp.Tq = pr.Tq;
  pp.Tq_pad = Tq_pad;
  pp.lse = lse;
  pp.nlse2 = nlse2;
  pp.q_rows_alloc = pr.q_rows;
  pp.q_row0 = pr.q_row0;
  pp.o = o;
  pp.dO = dO;
  pp.ndelta = ndelta;
  pp.dO_round = (dO_mma != dO) ? reinterpret_cast<float*>(const_cast<void*>(dO_mma)) : nullptr;
  int* item_counters =
      reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + 2 * align256(padded_rows(pr) * sizeof(float)));
  pp.item_counters = item_counters;
  if (!std::is_same<DT, float>::value) record(ev, 0, stream);
  const long long prep_blocks =
      std::max<long long>(1, std::min<long long>((pp.rows * PrepShape<DT, HD>::TPR + 255) / 256, sm_count() * 8));
  // programmatic serialization after whatever kernel precedes on the stream
  // (normally the forward): the prep kernel waits for it before reading o / lse
  cudaError_t e = launch_after_previous(ev == nullptr, attn_bwd_prep<DT, HD>, dim3((unsigned)prep_blocks), dim3(256), 0,
                                        stream, pp);
  record(ev, 1, stream);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch attn_bwd_prep");
  // 2. dK/dV (key-stationary) and dQ (query-stationary).  Each kernel has its
  // own box heights; tf32 operands read N-major get a 32-byte-granule map.
  constexpr bool kMN32 = C::TF32;
  CUtensorMap kv_q, kv_do, kv_k, kv_v, kv_qm, kv_dom, q_q, q_do, q_k, q_v, q_km;
  int s;
  if ((s = make_map(&kv_q, q, pr.dtype, HD, pr.q_rows, BH, C::KV_QT)) != CTFA_OK) return s;
  if ((s = make_map(&kv_do, dO_mma, pr.dtype, HD, pr.q_rows, BH, C::KV_QT)) != CTFA_OK) return s;
  if ((s = make_map(&kv_k, k, pr.dtype, HD, pr.k_rows, BH, C::KV_KEYS)) != CTFA_OK) return s;
  if ((s = make_map(&kv_v, v, pr.dtype, HD, pr.k_rows, BH, C::KV_KEYS)) != CTFA_OK) return s;
  if ((s = make_map(&q_q, q, pr.dtype, HD, pr.q_rows, BH, C::Q_ROWS)) != CTFA_OK) return s;
  if ((s = make_map(&q_do, dO_mma, pr.dtype, HD, pr.q_rows, BH, C::Q_ROWS)) != CTFA_OK) return s;
  if ((s = make_map(&q_k, k, pr.dtype, HD, pr.k_rows, BH, C::Q_KT)) != CTFA_OK) return s;
  if ((s = make_map(&q_v, v, pr.dtype, HD, pr.k_rows, BH, C::Q_KT)) != CTFA_OK) return s;
  if (kMN32) {
    if ((s = make_map(&kv_qm, q, pr.dtype, HD, pr.q_rows, BH, C::KV_QT, true)) != CTFA_OK) return s;
    if ((s = make_map(&kv_dom, dO_mma, pr.dtype, HD, pr.q_rows, BH, C::KV_QT, true)) != CTFA_OK) return s;
    if ((s = make_map(&q_km, k, pr.dtype, HD, pr.k_rows, BH, C::Q_KT, true)) != CTFA_OK) return s;
  } else {
    kv_qm = kv_q;
    kv_dom = kv_do;
    q_km = q_k;
  }
  BwdParams p;
  p.BH = BH;
  p.Tq = pr.Tq;
  p.Tk = pr.Tk;
  p.q_row0 = pr.q_row0;
  p.k_row0 = pr.k_row0;
  p.q_rows_alloc = pr.q_rows;
  p.k_rows_alloc = pr.k_rows;
  p.causal = pr.causal;
  p.causal_offset = pr.causal_offset;
  p.scale = (float)(1.0 / std::sqrt((double)HD));
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)HD));
  p.Tq_pad = Tq_pad;
  p.nlse2 = nlse2;
  p.ndelta = ndelta;
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.accumulate = pr.accumulate;
  p.dkdv_head_chunk = head_chunk(BH, 2ll * pr.Tq * HD * (long long)sizeof(DT));
  p.dq_head_chunk = head_chunk(BH, 2ll * pr.Tk * HD * (long long)sizeof(DT));
  p.item_counters = item_counters;
  p.wait_limit_ns = g_wait_limit_ns;
  const int n_kt = (pr.Tk + C::KV_KEYS - 1) / C::KV_KEYS;
  const int n_qt = (pr.Tq + C::Q_ROWS - 1) / C::Q_ROWS;
  auto kdkdv = attn_bwd_dkdv_sm100<DT, HD>;
  e = cudaFuncSetAttribute(kdkdv, cudaFuncAttributeMaxDynamicSharedMemorySize, C::KV_SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attn_bwd_dkdv_sm100)");
  // persistent: one CTA per SM (or per item when there are fewer items)
  const long long kv_items = (long long)n_kt * BH;
  const unsigned kv_grid = (unsigned)std::min<long long>(kv_items, sm_count());
  e = launch_after_previous(ev == nullptr, kdkdv, dim3(kv_grid), dim3(C::KV_THREADS), C::KV_SMEM, stream, kv_q, kv_k,
                            kv_v, kv_do, kv_qm, kv_dom, p, n_kt, (int)kv_items);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch attn_bwd_dkdv_sm100");
  record(ev, 2, stream);
  auto kdq = attn_bwd_dq_sm100<DT, HD>;
  e = cudaFuncSetAttribute(kdq, cudaFuncAttributeMaxDynamicSharedMemorySize, C::Q_SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attn_bwd_dq_sm100)");
  // persistent: one CTA per SM (or per item when there are fewer items)
  const long long dq_items = (long long)n_qt * BH;
  const unsigned dq_grid = (unsigned)std::min<long long>(dq_items, sm_count());
  // programmatic serialization: dQ blocks start on the SMs the dK/dV blocks
  // free as they finish (the dQ kernel reads nothing the dK/dV kernel writes
  // and waits for it before exiting)
  e = launch_after_previous(ev == nullptr, kdq, dim3(dq_grid), dim3(C::THREADS), C::Q_SMEM, stream, q_q, q_k, q_v,
                            q_do, q_km, p, n_qt, (int)dq_items);
  if (e != cudaSuccess) return cuda_fail(e, "launch attn_bwd_dq_sm100");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch attn_bwd_dq_sm100");
  record(ev, 3, stream);
  return CTFA_OK;
}

int backward_impl(const Problem& pr, const void* q, const void* k, const void* v, const void* o, const void* dO,
                  const float* lse, void* dq, void* dk, void* dv, void* ws, cudaStream_t stream,
                  cudaEvent_t* ev = nullptr) {
  int s;
  if (tensor_core_shape(pr)) {
    bool sm100 = false;
    s = device_is_sm100(&sm100);
    if (s != CTFA_OK) return s;
    if (!sm100) return fail(CTFA_ERR_UNSUPPORTED, "tensor-core attention kernels need an sm_100 (B200) device");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(dO) || !aligned16(dq) ||
        !aligned16(dk) || !aligned16(dv))
      return fail(CTFA_ERR_MISALIGNED, "q/k/v/o/dO/dq/dk/dv must be 16-byte aligned");
    switch (pr.dtype) {
      case CTFA_DTYPE_F32:
      case CTFA_DTYPE_TF32:
        if (pr.D == 64) {
          const size_t n = (size_t)pr.B * pr.H * pr.Tq * pr.D;
          char* w = reinterpret_cast<char*>(ws) + bwd_rows_bytes(pr);
          record(ev, 0, stream);
          if (pr.dtype == CTFA_DTYPE_TF32)  // q, k, v already rounded; the delta pass rounds dO into w
            return launch_bwd_tc<float, 64>(pr, q, k, v, o, dO, w, lse, dq, dk, dv, ws, stream, ev);
          void* r[4] = {w, w + align256(n * 4), w + 2 * align256(n * 4), w + 3 * align256(n * 4)};
          const void* in[3] = {q, k, v};
          if ((s = launch_round(in, r, 3, n, stream)) != CTFA_OK) return s;
          // the delta pass writes the rounded dO (r[3]) the GEMMs read
          return launch_bwd_tc<float, 64>(pr, r[0], r[1], r[2], o, dO, r[3], lse, dq, dk, dv, ws, stream, ev);
        }
        break;  // fp32 D=128 does not fit the tensor-core backward's shared memory: SIMT below
      case CTFA_DTYPE_BF16:
        return pr.D == 64 ? launch_bwd_tc<__nv_bfloat16, 64>(pr, q, k, v, o, dO, dO, lse, dq, dk, dv, ws, stream, ev)
                          : launch_bwd_tc<__nv_bfloat16, 128>(pr, q, k, v, o, dO, dO, lse, dq, dk, dv, ws, stream, ev);
      default:
        return pr.D == 64 ? launch_bwd_tc<__half, 64>(pr, q, k, v, o, dO, dO, lse, dq, dk, dv, ws, stream, ev)
                          : launch_bwd_tc<__half, 128>(pr, q, k, v, o, dO, dO, lse, dq, dk, dv, ws, stream, ev);
    }
  }
  switch (pr.dtype) {
    case CTFA_DTYPE_F32:
    case CTFA_DTYPE_TF32: return launch_bwd_simt<float>(pr, q, k, v, o, dO, lse, dq, dk, dv, ws, stream, ev);
    case CTFA_DTYPE_BF16: return launch_bwd_simt<__nv_bfloat16>(pr, q, k, v, o, dO, lse, dq, dk, dv, ws, stream, ev);
    case CTFA_DTYPE_F16: return launch_bwd_simt<__half>(pr, q, k, v, o, dO, lse, dq, dk, dv, ws, stream, ev);
    default: return launch_bwd_simt<double>(pr, q, k, v, o, dO, lse, dq, dk, dv, ws, stream, ev);
  }
}

// One CTA waits on an mbarrier that nothing arrives on.
__global__ void selftest_wait_kernel(unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, limit_ns, 100);
}

}  // namespace

// ---------------------------------------------------------------------------
// extern "C"
// ---------------------------------------------------------------------------
extern "C" int ctfa_version(void) { return kVersion; }

extern "C" const char* ctfa_status_string(int status) {
  switch (status) {
    case CTFA_OK: return "CTFA_OK";
    case CTFA_ERR_INVALID_ARGUMENT: return "CTFA_ERR_INVALID_ARGUMENT";
    case CTFA_ERR_UNSUPPORTED: return "CTFA_ERR_UNSUPPORTED";
    case CTFA_ERR_MISALIGNED: return "CTFA_ERR_MISALIGNED";
    case CTFA_ERR_CUDA: return "CTFA_ERR_CUDA";
    case CTFA_ERR_DEVICE_TIMEOUT: return "CTFA_ERR_DEVICE_TIMEOUT";
    case CTFA_ERR_WORKSPACE: return "CTFA_ERR_WORKSPACE";
    default: return "CTFA_ERR_UNKNOWN";
  }
}

extern "C" const char* ctfa_last_error_message(void) { return g_last_error.c_str(); }

extern "C" int ctfa_set_wait_limit_ns(unsigned long long ns) {
  if (ns == 0) return fail(CTFA_ERR_INVALID_ARGUMENT, "wait limit must be positive");
  g_wait_limit_ns = ns;
  return CTFA_OK;
}

extern "C" size_t ctfa_forward_workspace_bytes(int B, int H, int T, int D, int dtype) {
  if (check_common(B, H, T, D, dtype) != CTFA_OK) return 0;
  return fwd_workspace(full_problem(B, H, T, D, dtype, 0));
}

extern "C" int ctfa_forward(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H, int T,
                            int D, int dtype, int causal, void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_common(B, H, T, D, dtype);
  if (s != CTFA_OK) return s;
  if (!q || !k || !v || !o) return fail(CTFA_ERR_INVALID_ARGUMENT, "q, k, v and o must be non-null");
  Problem pr = full_problem(B, H, T, D, dtype, causal);
  const size_t need = fwd_workspace(pr);
  if (need > 0) {
    if (!workspace || workspace_bytes < need)
      return fail(CTFA_ERR_WORKSPACE, "workspace needs " + std::to_string(need) + " bytes");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
      return fail(CTFA_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  }
  return forward_impl(pr, q, k, v, o, lse, workspace, (cudaStream_t)stream);
}

extern "C" size_t ctfa_backward_workspace_bytes(int B, int H, int T, int D, int dtype) {
  if (check_common(B, H, T, D, dtype) != CTFA_OK) return 0;
  return bwd_workspace(full_problem(B, H, T, D, dtype, 0));
}

extern "C" int ctfa_backward(const void* q, const void* k, const void* v, const void* o, const void* dO,
                             const float* lse, void* dq, void* dk, void* dv, void* workspace,
                             size_t workspace_bytes, int B, int H, int T, int D, int dtype, int causal,
                             void* stream) {
  int s = check_common(B, H, T, D, dtype);
  if (s != CTFA_OK) return s;
  if (!q || !k || !v || !o || !dO || !lse || !dq || !dk || !dv)
    return fail(CTFA_ERR_INVALID_ARGUMENT, "q, k, v, o, dO, lse, dq, dk and dv must be non-null");
  Problem pr = full_problem(B, H, T, D, dtype, causal);
  const size_t need = bwd_workspace(pr);
  if (!workspace || workspace_bytes < need)
    return fail(CTFA_ERR_WORKSPACE, "workspace needs " + std::to_string(need) + " bytes");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(CTFA_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  return backward_impl(pr, q, k, v, o, dO, lse, dq, dk, dv, workspace, (cudaStream_t)stream);
}

extern "C" int ctfa_backward_with_events(const void* q, const void* k, const void* v, const void* o, const void* dO,
                                         const float* lse, void* dq, void* dk, void* dv, void* workspace,
                                         size_t workspace_bytes, int B, int H, int T, int D, int dtype, int causal,
                                         void* stream, void** events) {
  int s = check_common(B, H, T, D, dtype);
  if (s != CTFA_OK) return s;
  if (!q || !k || !v || !o || !dO || !lse || !dq || !dk || !dv || !events)
    return fail(CTFA_ERR_INVALID_ARGUMENT, "tensors and events must be non-null");
  Problem pr = full_problem(B, H, T, D, dtype, causal);
  const size_t need = bwd_workspace(pr);
  if (!workspace || workspace_bytes < need)
    return fail(CTFA_ERR_WORKSPACE, "workspace needs " + std::to_string(need) + " bytes");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(CTFA_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  return backward_impl(pr, q, k, v, o, dO, lse, dq, dk, dv, workspace, (cudaStream_t)stream,
                       reinterpret_cast<cudaEvent_t*>(events));
}

// ---------------------------------------------------------------------------
// Backward without allocation: scratch in a static device array.
// ---------------------------------------------------------------------------
namespace {

// Scratch of ctfa_backward_noalloc.  Static device memory: every GPU that
// loads this library holds these CTFA_NOALLOC_SCRATCH_BYTES until exit.
static __device__ __align__(256) unsigned char g_noalloc_scratch[CTFA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 128;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};
CUcontext g_noalloc_ctx[kMaxDevices] = {};

// The driver's cuCtxGetCurrent, fetched through the runtime (no -lcuda).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  return fn;
}

// Device address of g_noalloc_scratch on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is looked up
// (with that device current) once per device and context and cached.  The
// cache is keyed on the current context as well as the device: after a
// cudaDeviceReset the primary context is a new one, the module is loaded
// again and the array has a new address, which the next call looks up.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(CTFA_ERR_UNSUPPORTED, "device index out of range");
  auto get_ctx = ctx_get_current_fn();
  if (get_ctx == nullptr) return fail(CTFA_ERR_CUDA, "cuCtxGetCurrent entry point unavailable");
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;  // none current yet: look the address up below
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (ctx == nullptr || g_noalloc_addr[dev] == nullptr || g_noalloc_ctx[dev] != ctx) {
    // (the lookup makes the device's primary context current if none is)
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) return fail(CTFA_ERR_CUDA, "no current CUDA context");
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_addr[dev];
  return CTFA_OK;
}

}  // namespace

extern "C" int ctfa_backward_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dO,
                                     const float* lse, void* dq, void* dk, void* dv, int B, int H, int T, int D,
                                     int dtype, int causal, void* stream) {
  int s = check_common(B, H, T, D, dtype);
  if (s != CTFA_OK) return s;
  if (!q || !k || !v || !o || !dO || !lse || !dq || !dk || !dv)
    return fail(CTFA_ERR_INVALID_ARGUMENT, "q, k, v, o, dO, lse, dq, dk and dv must be non-null");
  Problem pr = full_problem(B, H, T, D, dtype, causal);
  const size_t need = bwd_workspace(pr);
  if (need > CTFA_NOALLOC_SCRATCH_BYTES)
    return fail(CTFA_ERR_WORKSPACE, "ctfa_backward_noalloc: this problem needs " + std::to_string(need) +
                                        " bytes of scratch, the static scratch holds " +
                                        std::to_string(CTFA_NOALLOC_SCRATCH_BYTES) +
                                        "; call ctfa_backward with a caller-provided workspace");
  void* ws = nullptr;
  if ((s = noalloc_scratch(&ws)) != CTFA_OK) return s;
  return backward_impl(pr, q, k, v, o, dO, lse, dq, dk, dv, ws, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Block entry points for sequence-parallel (ring) attention.
// ---------------------------------------------------------------------------
namespace {

__global__ void __launch_bounds__(256)
    merge_blocks_kernel(float* o_acc, float* lse_acc, const float* o_blk, const float* lse_blk, int BH, int rows,
                        int row0, int T, int D, int init) {
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)BH * T) return;
  const long long bh = w / T, i = w % T;
  const size_t r = (size_t)bh * rows + row0 + i;
  float* oa = o_acc + r * D;
  const float* ob = o_blk + r * D;
  if (init) {
    for (int d = lane; d < D; d += 32) oa[d] = ob[d];
    if (lane == 0) lse_acc[r] = lse_blk[r];
    return;
  }
  const float l1 = lse_acc[r], l2 = lse_blk[r];
  const float mx = fmaxf(l1, l2);
  if (mx == -INFINITY) return;
  const float w1 = __expf(l1 - mx), w2 = __expf(l2 - mx);
  const float inv = 1.f / (w1 + w2);
  for (int d = lane; d < D; d += 32) oa[d] = (oa[d] * w1 + ob[d] * w2) * inv;
  __syncwarp();
  if (lane == 0) lse_acc[r] = mx + __logf(w1 + w2);
}

template <typename DT>
__global__ void __launch_bounds__(256) convert_f32_kernel(const float* src, DT* dst, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = from_acc<DT>(src[i]);
}

int check_block(const void* q, const void* k, const void* v, int B, int H, int D, int dtype, int q_rows,
                int q_row0, int Tq, int k_rows, int k_row0, int Tk) {
  int s = check_common(B, H, Tq > 0 ? Tq : 1, D, dtype);
  if (s != CTFA_OK) return s;
  if (!q || !k || !v) return fail(CTFA_ERR_INVALID_ARGUMENT, "q, k and v must be non-null");
  if (dtype != CTFA_DTYPE_BF16 && dtype != CTFA_DTYPE_F16)
    return fail(CTFA_ERR_UNSUPPORTED, "block entry points take bf16 or fp16 I/O");
  if (D != 64 && D != 128) return fail(CTFA_ERR_UNSUPPORTED, "block entry points take head dim 64 or 128");
  if (Tq <= 0 || Tk <= 0 || q_row0 < 0 || k_row0 < 0 || q_row0 + Tq > q_rows || k_row0 + Tk > k_rows)
    return fail(CTFA_ERR_INVALID_ARGUMENT, "row range outside the allocation");
  return CTFA_OK;
}

Problem block_problem(int B, int H, int D, int dtype, int q_rows, int q_row0, int Tq, int k_rows, int k_row0,
                      int Tk, int causal, int causal_offset) {
  Problem pr;
  pr.B = B;
  pr.H = H;
  pr.D = D;
  pr.dtype = dtype;
  pr.Tq = Tq;
  pr.Tk = Tk;
  pr.q_rows = q_rows;
  pr.k_rows = k_rows;
  pr.q_row0 = q_row0;
  pr.k_row0 = k_row0;
  pr.causal = causal ? 1 : 0;
  pr.causal_offset = causal_offset;
  return pr;
}

}  // namespace

extern "C" int ctfa_forward_block(const void* q, const void* k, const void* v, float* o_blk, float* lse_blk, int B,
                                  int H, int D, int dtype, int q_rows, int q_row0, int Tq, int k_rows, int k_row0,
                                  int Tk, int causal, int causal_offset, void* stream) {
  int s = check_block(q, k, v, B, H, D, dtype, q_rows, q_row0, Tq, k_rows, k_row0, Tk);
  if (s != CTFA_OK) return s;
  if (!o_blk || !lse_blk) return fail(CTFA_ERR_INVALID_ARGUMENT, "o_blk and lse_blk must be non-null");
  Problem pr = block_problem(B, H, D, dtype, q_rows, q_row0, Tq, k_rows, k_row0, Tk, causal, causal_offset);
  pr.o_f32 = o_blk;
  return forward_impl(pr, q, k, v, o_blk, lse_blk, nullptr, (cudaStream_t)stream);
}

extern "C" int ctfa_forward_block_merge(const void* q, const void* k, const void* v, float* o_acc, float* lse_acc,
                                        int B, int H, int D, int dtype, int q_rows, int q_row0, int Tq, int k_rows,
                                        int k_row0, int Tk, int causal, int causal_offset, int init, void* stream) {
  int s = check_block(q, k, v, B, H, D, dtype, q_rows, q_row0, Tq, k_rows, k_row0, Tk);
  if (s != CTFA_OK) return s;
  if (!o_acc || !lse_acc) return fail(CTFA_ERR_INVALID_ARGUMENT, "o_acc and lse_acc must be non-null");
  Problem pr = block_problem(B, H, D, dtype, q_rows, q_row0, Tq, k_rows, k_row0, Tk, causal, causal_offset);
  pr.o_f32 = o_acc;
  pr.merge = init ? 0 : 1;
  return forward_impl(pr, q, k, v, o_acc, lse_acc, nullptr, (cudaStream_t)stream);
}

extern "C" int ctfa_merge_blocks(float* o_acc, float* lse_acc, const float* o_blk, const float* lse_blk, int B,
                                 int H, int D, int rows, int row0, int T, int init, void* stream) {
  if (!o_acc || !lse_acc || !o_blk || !lse_blk) return fail(CTFA_ERR_INVALID_ARGUMENT, "null pointer");
  if (B <= 0 || H <= 0 || D <= 0 || T <= 0 || row0 < 0 || row0 + T > rows)
    return fail(CTFA_ERR_INVALID_ARGUMENT, "bad sizes");
  const long long warps = (long long)B * H * T;
  merge_blocks_kernel<<<warps_grid(warps), 256, 0, (cudaStream_t)stream>>>(o_acc, lse_acc, o_blk, lse_blk, B * H,
                                                                           rows, row0, T, D, init);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CTFA_OK : cuda_fail(e, "launch merge_blocks_kernel");
}

extern "C" int ctfa_convert_f32(const float* src, void* dst, int dtype, size_t n, void* stream) {
  if (!src || !dst) return fail(CTFA_ERR_INVALID_ARGUMENT, "null pointer");
  const unsigned grid = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 16);
  if (n == 0) return CTFA_OK;
  if (dtype == CTFA_DTYPE_BF16)
    convert_f32_kernel<__nv_bfloat16><<<grid, 256, 0, (cudaStream_t)stream>>>(src, (__nv_bfloat16*)dst, n);
  else if (dtype == CTFA_DTYPE_F16)
    convert_f32_kernel<__half><<<grid, 256, 0, (cudaStream_t)stream>>>(src, (__half*)dst, n);
  else if (dtype == CTFA_DTYPE_F32)
    convert_f32_kernel<float><<<grid, 256, 0, (cudaStream_t)stream>>>(src, (float*)dst, n);
  else
    return fail(CTFA_ERR_UNSUPPORTED, "convert to fp32, bf16 or fp16 only");
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CTFA_OK : cuda_fail(e, "launch convert_f32_kernel");
}

extern "C" size_t ctfa_backward_block_workspace_bytes(int B, int H, int Tq, int D, int dtype) {
  if (check_common(B, H, Tq, D, dtype) != CTFA_OK) return 0;
  Problem pr = block_problem(B, H, D, dtype, Tq, 0, Tq, Tq, 0, Tq, 0, 0);
  return bwd_rows_bytes(pr);
}

extern "C" int ctfa_backward_block(const void* q, const void* k, const void* v, const void* o, const void* dO,
                                   const float* lse, float* dq_acc, float* dk_acc, float* dv_acc, void* workspace,
                                   size_t workspace_bytes, int B, int H, int D, int dtype, int q_rows, int q_row0,
                                   int Tq, int k_rows, int k_row0, int Tk, int causal, int causal_offset,
                                   void* stream) {
  int s = check_block(q, k, v, B, H, D, dtype, q_rows, q_row0, Tq, k_rows, k_row0, Tk);
  if (s != CTFA_OK) return s;
  if (!o || !dO || !lse || !dq_acc || !dk_acc || !dv_acc)
    return fail(CTFA_ERR_INVALID_ARGUMENT, "o, dO, lse, dq_acc, dk_acc and dv_acc must be non-null");
  Problem pr = block_problem(B, H, D, dtype, q_rows, q_row0, Tq, k_rows, k_row0, Tk, causal, causal_offset);
  pr.accumulate = 1;
  const size_t need = ctfa_backward_block_workspace_bytes(B, H, Tq, D, dtype);
  if (!workspace || workspace_bytes < need)
    return fail(CTFA_ERR_WORKSPACE, "workspace needs " + std::to_string(need) + " bytes");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(CTFA_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  return backward_impl(pr, q, k, v, o, dO, lse, dq_acc, dk_acc, dv_acc, workspace, (cudaStream_t)stream);
}

extern "C" int ctfa_check_device_error(void* stream) {
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  DeviceError err;
  e = cudaMemcpyFromSymbol(&err, g_device_error, sizeof(err));
  if (e != cudaSuccess) return cuda_fail(e, "read device error word");
  if (err.code != 0) {
    DeviceError zero = {0, 0, 0, 0};
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    char buf[160];
    snprintf(buf, sizeof(buf), "kernel wait gave up (site %d, block %d, thread %d)", err.site, err.block,
             err.thread);
    return fail(CTFA_ERR_DEVICE_TIMEOUT, buf);
  }
  return CTFA_OK;
}

extern "C" int ctfa_selftest_wait_timeout(unsigned long long limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 10000000000ull)
    return fail(CTFA_ERR_INVALID_ARGUMENT, "limit must be in (0, 10 s]");
  selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(limit_ns);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch selftest_wait_kernel");
  return ctfa_check_device_error(stream);
}

#include "proj_api.cuh"
#include "mlp_api.cuh"
