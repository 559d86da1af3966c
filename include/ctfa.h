/*
 * ctfa.h -- C ABI of the B200 (sm_100a) flash-attention library
 * (libctfa_b200.so).
 *
 * These entry points are the seam under CudaTransformer's
 * FlashAttentionLayer<DType> (cuda_transformer/FlashAttentionLayer.cu).  The
 * layer keeps its C++ API; its two kernel launches become calls into this
 * library.  Every function takes plain device pointers, sizes and a CUDA
 * stream (cudaStream_t passed as void*; NULL = legacy default stream, which
 * is what the reference launches on), returns a status code, and never
 * allocates or synchronises unless stated.
 *
 * Tensor layout (unchanged from the reference, Tensor<DType> contiguous
 * row-major, cuda_transformer/Tensor.cu:10-170):
 *   q, k, v, o, dO, dq, dk, dv : [B, H, T, D], D fastest
 *   lse                        : [B, H, T] float32, natural-log logsumexp
 *                                of the scaled scores of each query row
 * Softmax scale: 1/sqrt(D) (flash_attention.cu:116).
 */
#ifndef CTFA_H_
#define CTFA_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define CTFA_OK 0
#define CTFA_ERR_INVALID_ARGUMENT 1 /* null pointer, non-positive size, bad dtype */
#define CTFA_ERR_UNSUPPORTED 2      /* shape / dtype / device the library cannot run */
#define CTFA_ERR_MISALIGNED 3       /* tensor-core path needs 16-byte aligned tensors */
#define CTFA_ERR_CUDA 4             /* a CUDA runtime call or launch failed */
#define CTFA_ERR_DEVICE_TIMEOUT 5   /* a kernel gave up on a bounded wait */
#define CTFA_ERR_WORKSPACE 6        /* workspace missing or too small */

/* Element types of q/k/v/o/dO/dq/dk/dv (the DType template argument of the
 * reference layer: float, __nv_bfloat16, __half, double). */
#define CTFA_DTYPE_F32 0  /* fp32 I/O, tcgen05 kind::tf32, fp32 softmax/accumulation */
#define CTFA_DTYPE_BF16 1 /* bf16 I/O, tcgen05 kind::f16, fp32 softmax/accumulation */
#define CTFA_DTYPE_F16 2  /* fp16 I/O, tcgen05 kind::f16, fp32 softmax/accumulation */
#define CTFA_DTYPE_F64 3  /* fp64 I/O, SIMT fp64 kernels */
#define CTFA_DTYPE_TF32 4 /* fp32 storage whose values are already rounded to tf32 (for example the
                           * copies ctfa_forward leaves in its workspace): the fp32 tensor-core path
                           * without the rounding pass over q, k, v */

/* Library version: major*10000 + minor*100 + patch. */
int ctfa_version(void);

/* Human-readable name of a status code. */
const char* ctfa_status_string(int status);

/* Detail message of the last failing call made by this host thread. */
const char* ctfa_last_error_message(void);

/*
 * Forward: o = softmax(q k^T / sqrt(D) [+ causal mask]) v, lse per row.
 * Replaces the launch of flashAttention<DType> in
 * FlashAttentionLayer::computeAttention (FlashAttentionLayer.cu:45-87, kernel
 * at flash_attention.cu:57-169).  causal = 0 reproduces the reference's
 * semantics (every query attends every key); causal = 1 masks key j > query i.
 * lse may be NULL when the caller does not keep it for the backward pass.
 * workspace: ctfa_forward_workspace_bytes(...) bytes of device memory,
 * 256-byte aligned (NULL when that is 0).
 * D: any value in [1, 256]; D = 64 and D = 128 with f32/bf16/f16 run on the
 * tcgen05 tensor-core kernels, everything else on SIMT kernels.
 */
int ctfa_forward(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H, int T, int D,
                 int dtype, int causal, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of device workspace ctfa_forward needs (0 except for fp32 I/O on the
 * tensor cores, where it holds the round-to-nearest tf32 copies of q, k, v:
 * the MMA itself truncates fp32 operands to tf32, which costs a factor ~4 in
 * accuracy).  workspace may be NULL when this is 0.  After an fp32 forward
 * the workspace holds the rounded q, k, v at byte offsets 0, a and 2a, with
 * a = B*H*T*D*4 rounded up to a multiple of 256; a caller that keeps it may
 * pass those copies to ctfa_backward as q, k, v with CTFA_DTYPE_TF32, which
 * skips rounding them again. */
size_t ctfa_forward_workspace_bytes(int B, int H, int T, int D, int dtype);

/* Bytes of device workspace ctfa_backward needs for this problem. */
size_t ctfa_backward_workspace_bytes(int B, int H, int T, int D, int dtype);

/*
 * Backward: dq, dk, dv from q, k, v, the forward output o, its gradient dO and
 * the forward's lse.  Replaces the launch of flashAttentionBackward<DType> in
 * FlashAttentionLayer::computeBackward (FlashAttentionLayer.cu:97-142, kernel
 * at flash_attention.cu:226-326).  Unlike the reference, dk and dv are the
 * exact gradients (the reference kernel mixes the query index into the key
 * rows it updates, flash_attention.cu:310-321).  dq/dk/dv are fully written
 * (no zero-filled inputs required).  workspace: device memory of at least
 * ctfa_backward_workspace_bytes(...) bytes, 256-byte aligned; it holds the
 * per-row delta / logsumexp arrays and the work-list counters of the
 * backward kernels, so calls that may run at the same time (other streams)
 * need separate workspaces.
 */
int ctfa_backward(const void* q, const void* k, const void* v, const void* o, const void* dO, const float* lse,
                  void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes, int B, int H, int T,
                  int D, int dtype, int causal, void* stream);

/*
 * Profiling variant of ctfa_backward (no reference counterpart): identical
 * work, and it records events[0..3] (cudaEvent_t) on `stream` before the
 * first launch and after the delta, dK/dV and dQ passes, so a caller can time
 * each kernel on its own launch stream.
 */
int ctfa_backward_with_events(const void* q, const void* k, const void* v, const void* o, const void* dO,
                              const float* lse, void* dq, void* dk, void* dv, void* workspace,
                              size_t workspace_bytes, int B, int H, int T, int D, int dtype, int causal,
                              void* stream, void** events);

/*
 * Backward that allocates nothing.  No counterpart in the reference (its
 * FlashAttentionLayer::computeBackward always allocates).  It exists for
 * callers that cannot call cudaMalloc while they run attention: a serving or
 * plugin host that has already handed all device memory to its own pool (so
 * a new allocation fails or breaks its accounting), or a caller that cannot
 * afford the device-wide synchronisation cudaMalloc may imply.  Same inputs,
 * outputs and results as ctfa_backward, but the scratch (delta rows and, for
 * fp32 I/O, the tf32-rounded operand copies) lives in a static device array
 * of CTFA_NOALLOC_SCRATCH_BYTES inside this library, which every GPU that
 * loads the library holds until the process exits.  Problems whose
 * ctfa_backward_workspace_bytes(...) exceed that size are rejected with
 * CTFA_ERR_WORKSPACE before anything is launched.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current); make that first call
 *     before any stream capture on the device.  The address is cached per
 *     device and CUDA context: after a cudaDeviceReset the device's next
 *     context gets a new copy of the array, and the first call made in it
 *     looks the address up again (so, again, before any capture).
 *   - All calls share the one array and leave their contents in it; calls
 *     that overlap on the GPU (two streams, two host threads) race and must
 *     be serialised by the caller.  Nothing in the array needs to start at zero.
 */
#define CTFA_NOALLOC_SCRATCH_BYTES (32ull << 20)
int ctfa_backward_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dO,
                          const float* lse, void* dq, void* dk, void* dv, int B, int H, int T, int D, int dtype,
                          int causal, void* stream);

/*
 * Block entry points for sequence-parallel (ring) attention.  No counterpart
 * in the reference, which runs one device and one sequence (its kernel loops
 * over all keys, flash_attention.cu:97).  They run the same tensor-core
 * kernels on row ranges of each head (bf16 / fp16 I/O, head dim 64 or 128):
 * query rows [q_row0, q_row0+Tq) of an allocation [B, H, q_rows, D] against
 * key/value rows [k_row0, k_row0+Tk) of an allocation [B, H, k_rows, D].
 * causal = 1: key j (local to the block) is visible to query i (local) iff
 * j <= i + causal_offset; causal = 0: every key is visible.
 */

/* Partial attention of one block: normalised output rows (fp32) into o_blk
 * ([B, H, q_rows, D], same rows as q) and their logsumexp into lse_blk
 * ([B, H, q_rows]). */
int ctfa_forward_block(const void* q, const void* k, const void* v, float* o_blk, float* lse_blk, int B, int H,
                       int D, int dtype, int q_rows, int q_row0, int Tq, int k_rows, int k_row0, int Tk,
                       int causal, int causal_offset, void* stream);

/* ctfa_forward_block with the merge done in the kernel's epilogue: the block's
 * output is folded straight into the running fp32 (o_acc, lse_acc) of rows
 * [q_row0, q_row0+Tq) (logsumexp-weighted, as ctfa_merge_blocks does), so no
 * per-block partial is written and read back.  init = 1: the first block of
 * those rows (o_acc / lse_acc are overwritten).  Rows with no visible key in
 * this block or before keep their running values. */
int ctfa_forward_block_merge(const void* q, const void* k, const void* v, float* o_acc, float* lse_acc, int B,
                             int H, int D, int dtype, int q_rows, int q_row0, int Tq, int k_rows, int k_row0,
                             int Tk, int causal, int causal_offset, int init, void* stream);

/* Fold one block's partial (o_blk, lse_blk) into the running (o_acc, lse_acc)
 * on rows [row0, row0+T) of [B, H, rows, *] fp32 buffers: logsumexp-weighted
 * average.  init = 1 copies instead (first block of those rows). */
int ctfa_merge_blocks(float* o_acc, float* lse_acc, const float* o_blk, const float* lse_blk, int B, int H, int D,
                      int rows, int row0, int T, int init, void* stream);

/* n fp32 values to CTFA_DTYPE_BF16 / F16 / F32 (round to nearest). */
int ctfa_convert_f32(const float* src, void* dst, int dtype, size_t n, void* stream);

/* Workspace of ctfa_backward_block for Tq query rows. */
size_t ctfa_backward_block_workspace_bytes(int B, int H, int Tq, int D, int dtype);

/* Gradient contributions of one block, added into fp32 buffers: dq_acc rows
 * like q, dk_acc / dv_acc rows like k.  o, dO: the final forward output and
 * its gradient (rows like q); lse: the final logsumexp ([B, H, q_rows]). */
int ctfa_backward_block(const void* q, const void* k, const void* v, const void* o, const void* dO,
                        const float* lse, float* dq_acc, float* dk_acc, float* dv_acc, void* workspace,
                        size_t workspace_bytes, int B, int H, int D, int dtype, int q_rows, int q_row0, int Tq,
                        int k_rows, int k_row0, int Tk, int causal, int causal_offset, void* stream);

/*
 * Bound, in nanoseconds, on every wait inside the kernels (default 2e9).  A
 * kernel that waits longer records CTFA_ERR_DEVICE_TIMEOUT in a device error
 * word and exits without touching its outputs further.
 */
int ctfa_set_wait_limit_ns(unsigned long long ns);

/*
 * Synchronise `stream`, then read and clear the device error word.  Returns
 * CTFA_OK, CTFA_ERR_DEVICE_TIMEOUT (a kernel gave up on a wait) or
 * CTFA_ERR_CUDA (an asynchronous CUDA error).
 */
int ctfa_check_device_error(void* stream);

/*
 * Self-test of the bounded-wait path: launches one CTA that waits on an
 * mbarrier nothing arrives on, with the given limit, then checks the device
 * error word.  Returns CTFA_ERR_DEVICE_TIMEOUT when the wait gave up as
 * designed (the expected result), CTFA_OK if it did not.
 */
int ctfa_selftest_wait_timeout(unsigned long long limit_ns, void* stream);

/*
 * Projections either side of the attention (the QKV projection and the output
 * projection of cuda_transformer/AttentionLayer.cu), as tcgen05 GEMMs that read
 * and write the head layout [B, H, T, D] directly.
 *   x, y, dx, dy : [B, T, E]   (E = the layer's inputDim; rows of the model)
 *   q, k, v, a, dq, dk, dv, da : [B, H, T, D]
 *   wq, wk, wv   : H*D rows of E  (row n = output feature n; the buffer the
 *                  reference's kernels index as W[n * inputDim + i],
 *                  attention_qkv_kernels.cu:92)
 *   wo           : E rows of H*D  (row o = output feature o,
 *                  attention_proj_kernels.cu:83)
 *   bq, bk, bv   : [H*D];  bo : [E]
 * Element types as for the attention (CTFA_DTYPE_*).  f32 / bf16 / f16 with
 * D = 64 or 128, 16-byte-aligned tensors and E * element size a multiple of 16
 * bytes run on the tensor cores (fp32 operands as tf32: the tensor core reads
 * their upper 19 bits; fp32 accumulation); other shapes and double run SIMT
 * kernels.  Nothing is allocated or synchronised.
 */
/* q|k|v = x W^T + b, written as [B, H, T, D].  Replaces getQKVmatrices
 * (QKVProjectionLayer::computeQKV, QKVProjectionLayer.cu:73-96).  Biases may
 * be NULL (zero). */
int ctfa_qkv_forward(const void* x, const void* wq, const void* bq, const void* wk, const void* bk, const void* wv,
                     const void* bv, void* q, void* k, void* v, int B, int T, int E, int H, int D, int dtype,
                     void* stream);
/* Backward of the QKV projection.  Replaces qkvBackwardWB + qkvBackward
 * (QKVProjectionLayer::computeBackward, QKVProjectionLayer.cu:100-141):
 *   dw{q,k,v} += dq|dk|dv^T x, db{q,k,v} += column sums of dq|dk|dv (ADDED into
 *   the buffers, like the reference's atomic accumulation);
 *   dx = sum over q, k, v of d{q,k,v} W{q,k,v} (overwritten).
 * dx == NULL skips the input gradient; dwq == dwk == dwv == NULL and the
 * bias-gradient pointers NULL skip the parameter gradients (a bias-gradient
 * pointer alone may be NULL). */
int ctfa_qkv_backward(const void* x, const void* dq, const void* dk, const void* dv, const void* wq, const void* wk,
                      const void* wv, void* dwq, void* dbq, void* dwk, void* dbk, void* dwv, void* dbv, void* dx,
                      int B, int T, int E, int H, int D, int dtype, void* stream);
/* y = a Wo^T + bo, a read as [B, H, T, D] with the heads concatenated per row.
 * Replaces attentionProj (OutputProjectionLayer::forward,
 * OutputProjectionLayer.cu:52-66).  bo may be NULL. */
int ctfa_out_proj_forward(const void* a, const void* wo, const void* bo, void* y, int B, int T, int E, int H, int D,
                          int dtype, void* stream);
/* Backward of the output projection.  Replaces projBackwardWB + projBackward
 * (OutputProjectionLayer::backward, OutputProjectionLayer.cu:69-97):
 *   dwo += dy^T a, dbo += column sums of dy (added); da = dy Wo as
 *   [B, H, T, D] (overwritten).  da == NULL or dwo == dbo == NULL skip the
 *   respective part. */
int ctfa_out_proj_backward(const void* a, const void* dy, const void* wo, void* dwo, void* dbo, void* da, int B,
                           int T, int E, int H, int D, int dtype, void* stream);

/*
 * The block's other layers (the config-4 training step): the MLP's Linear
 * layers and LayerNorm.  Same element types.  Row-major tensors; M rows.
 */
/* y [M, N] = x [M, K] W^T + b, W [N, K] (row = output feature, as
 * cuda_transformer/linear_kernels.cu:64 reads it); relu != 0 applies
 * max(y, 0) (a ReLU layer after the Linear, relu_kernels.cu:26-38).  Replaces
 * linearForward (LinearLayer::forward, LinearLayer.cu:55).  b may be NULL.
 * f32 / bf16 / f16 with K and N multiples of 128 bytes of elements run on the
 * tensor cores (the projection GEMM with one head), other shapes on SIMT. */
int ctfa_linear_forward(const void* x, const void* w, const void* b, void* y, int M, int K, int N, int relu, int dtype,
                        void* stream);
/* Backward of y = x W^T + b.  Replaces linearBackwardWB + linearBackward
 * (LinearLayer::backward, LinearLayer.cu:83, :95): dw += dy^T x, db += column
 * sums of dy (added into the buffers), dx = dy W (overwritten).  dx_mask
 * (optional, [M, K]): dx is zeroed where dx_mask <= 0 -- the backward of a
 * ReLU whose output is this layer's input (pass that output, x itself).  dx ==
 * NULL or dw == db == NULL skip the respective part. */
int ctfa_linear_backward(const void* x, const void* dy, const void* w, const void* dx_mask, void* dw, void* db,
                         void* dx, int M, int K, int N, int dtype, void* stream);
/* y = (x - mean) * rstd * w + b per row of E, biased variance; mean and rstd
 * (fp32 [M], may be NULL) are kept for the backward.  Replaces
 * layerNormForwardKernel (LayerNorm.cu:119). */
int ctfa_layernorm_forward(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd, int M,
                           int E, float eps, int dtype, void* stream);
/* dx (overwritten), dw += sum dy * x_hat, db += sum dy (added; either may be
 * NULL).  Replaces layerNormBackwardKernel (LayerNorm.cu:143).  Any E (rows
 * wider than 1024 take a strided-loop kernel).
 * mean / rstd: the forward's (NULL: recomputed from x with eps; double data
 * always recomputes, the fp32 statistics would cost it precision). */
int ctfa_layernorm_backward(const void* x, const void* dy, const void* w, const float* mean, const float* rstd,
                            void* dx, void* dw, void* db, int M, int E, float eps, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CTFA_H_ */
