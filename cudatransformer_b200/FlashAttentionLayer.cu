// Drop-in replacement for CudaTransformer's cuda_transformer/FlashAttentionLayer.cu.
//
// Same template, same public members and signatures as the reference
// (FlashAttentionLayer.cu:13-150), same Tensor<DType> layout ([B, H, T, D],
// contiguous row-major) and the same include guard, so AttentionLayer.cu,
// TransformerBlockLayer.cu, NanoGPT.cu and the pybind module compile against
// it unchanged.  The two kernel launches of the reference
// (flashAttention<<<>>> at FlashAttentionLayer.cu:76-79/123-126 and
// flashAttentionBackward<<<>>> at :133-140) become calls into the C ABI of
// libctfa_b200.so (include/ctfa.h): tcgen05 tensor-core kernels for float,
// __nv_bfloat16 and __half with head dim 64/128, SIMT kernels otherwise
// (double, other head dims up to 256).
//
// Build: put this directory before the reference's cuda_transformer/ on the
// include path and include this header before the reference's headers (or
// replace the reference file with it), add include/ to the path and link
// libctfa_b200.so.  Outputs and caches are Tensor<DType> / shared_ptr buffers
// on the default stream like the reference's, but stream-ordered
// (cudaMallocAsync / cudaFreeAsync, ctfa_dropin.h): no device-wide
// synchronisation per allocation (the reference's cudaMakeShared has one,
// headers.cu:206-207).
//
// Additions (all defaulted, existing call sites unchanged):
//   * bool causal (constructor's optional third argument, default false = the
//     reference's behaviour): masks key j > query i.
//   * cachedLSE: fp32 logsumexp per row, what the kernels keep for the
//     backward.  cachedMaxScores holds the same logsumexp in DType and
//     cachedDenominators holds ones, so exp(s - max) / denom is still the
//     softmax for code that reads the old fields.
//   * float: the forward writes round-to-nearest tf32 copies of q, k, v into
//     its workspace (include/ctfa.h).  With saveStates that workspace is kept
//     with the other cached state, and computeBackward on the same q, k, v
//     buffers passes the copies to the backward (CTFA_DTYPE_TF32), which then
//     rounds only dO.  Like the reference's cached output and max/denominator
//     (FlashAttentionLayer.cu:81-84, :114-127), the cache assumes q, k, v were
//     not modified in place between the two calls.
//   * cachedOutput shares the buffer of the tensor computeAttention returns
//     (the reference keeps a device-to-device copy, FlashAttentionLayer.cu:81-84):
//     one 4·B·H·T·D-byte copy less per step; a caller that writes into the
//     returned output before computeBackward must copy it first.  The
//     reference's callers (AttentionLayer, TransformerBlockLayer) only read it.
// Errors: every non-zero status from the library throws std::runtime_error
// (the reference throws from cudaMakeShared and ignores launch errors).
#include "ModuleLayer.cu"
#include "ctfa_dropin.h"

#ifndef FLASH_ATTENTION_LAYER
#define FLASH_ATTENTION_LAYER

template <typename DType = float>
struct FlashAttentionLayer {
  int headDim = 1;   /// Dimension of each attention head.
  int numHeads = 1;  /// Number of attention heads.

  // Cached values from the forward pass for the backward pass.
  std::shared_ptr<DType[]> cachedMaxScores = nullptr;
  std::shared_ptr<DType[]> cachedDenominators = nullptr;
  std::shared_ptr<DType[]> cachedOutput = nullptr;
  int cachedBatchSize = 0;
  int cachedSequenceLength = 0;

  bool causal = false;                        /// key j visible to query i iff j <= i
  std::shared_ptr<float[]> cachedLSE = nullptr;  /// fp32 logsumexp per row
  /// float only: the forward workspace holding tf32-rounded q, k, v, and the
  /// buffers they were rounded from
  std::shared_ptr<unsigned char[]> cachedRounded = nullptr;
  const void* cachedRoundedFrom[3] = {nullptr, nullptr, nullptr};

  FlashAttentionLayer(int headDim, int numHeads, bool causal = false)
      : headDim(headDim), numHeads(numHeads), causal(causal) {}

  std::shared_ptr<FlashAttentionLayer<DType>> clone() const {
    return std::make_shared<FlashAttentionLayer<DType>>(headDim, numHeads, causal);
  }

  /**
   * Forward: o = softmax(q k^T / sqrt(headDim)) v on [batch, numHeads, seq, headDim].
   * saveStates keeps o and the row logsumexp for computeBackward.
   */
  Tensor<DType> computeAttention(const Tensor<DType>& queries, const Tensor<DType>& keys,
                                 const Tensor<DType>& values, bool saveStates = false) {
    const int batchSize = queries.shape()[0];
    const int sequenceLength = queries.shape()[2];
    const size_t rows = (size_t)batchSize * numHeads * sequenceLength;
    Tensor<DType> output = ctfa_dropin::stream_tensor<DType>(queries.shape().toVector());
    std::shared_ptr<float[]> lse = ctfa_dropin::stream_buffer<float>(rows);
    std::shared_ptr<unsigned char[]> ws =
        runForward(queries, keys, values, output.data(), lse.get(), batchSize, sequenceLength);
    if (saveStates) {
      cachedRounded = ws;
      cachedRoundedFrom[0] = queries.get();
      cachedRoundedFrom[1] = keys.get();
      cachedRoundedFrom[2] = values.get();
      cachedLSE = lse;
      cachedMaxScores = ctfa_dropin::stream_buffer<DType>(rows);
      cachedDenominators = ctfa_dropin::stream_buffer<DType>(rows);
      const unsigned blocks = (unsigned)std::min<size_t>((rows + 255) / 256, 1184);
      ctfa_dropin::legacy_row_caches<DType><<<blocks, 256>>>(lse.get(), cachedMaxScores.get(),
                                                            cachedDenominators.get(), rows);
      // the cached output shares the returned tensor's buffer (the reference
      // copies it, FlashAttentionLayer.cu:81-84)
      cachedOutput = output.dataPtr();
      cachedBatchSize = batchSize;
      cachedSequenceLength = sequenceLength;
    }
    return output;
  }

  /**
   * Backward: [dq, dk, dv] for the upstream gradient outputGrad.  Recomputes
   * the forward when computeAttention did not save states.
   */
  std::array<Tensor<DType>, 3> computeBackward(const Tensor<DType>& queries, const Tensor<DType>& keys,
                                               const Tensor<DType>& values, const Tensor<DType>& outputGrad) {
    std::array<Tensor<DType>, 3> grads;
    grads[0] = ctfa_dropin::stream_tensor<DType>(queries.shape().toVector());
    grads[1] = ctfa_dropin::stream_tensor<DType>(keys.shape().toVector());
    grads[2] = ctfa_dropin::stream_tensor<DType>(values.shape().toVector());
    const int batchSize = queries.shape()[0];
    const int sequenceLength = queries.shape()[2];
    const size_t rows = (size_t)batchSize * numHeads * sequenceLength;

    std::shared_ptr<DType[]> output = cachedOutput;
    std::shared_ptr<float[]> lse = cachedLSE;
    if (output == nullptr || lse == nullptr || cachedBatchSize != batchSize ||
        cachedSequenceLength != sequenceLength) {
      output = ctfa_dropin::stream_buffer<DType>(rows * headDim);
      lse = ctfa_dropin::stream_buffer<float>(rows);
      runForward(queries, keys, values, output.get(), lse.get(), batchSize, sequenceLength);
    }
    int code = ctfa_dropin::DtypeCode<DType>::value;
    const void* in[3] = {queries.get(), keys.get(), values.get()};
    if (cachedRounded != nullptr && output == cachedOutput && in[0] == cachedRoundedFrom[0] &&
        in[1] == cachedRoundedFrom[1] && in[2] == cachedRoundedFrom[2]) {
      // the forward's tf32-rounded copies of these very buffers, at byte
      // offsets 0, a, 2a of its workspace (a = B*H*T*D*4 rounded up to 256)
      const size_t a = (rows * headDim * sizeof(float) + 255) / 256 * 256;
      for (int i = 0; i < 3; ++i) in[i] = cachedRounded.get() + i * a;
      code = CTFA_DTYPE_TF32;
    }
    const size_t wsBytes = ctfa_backward_workspace_bytes(batchSize, numHeads, sequenceLength, headDim, code);
    std::shared_ptr<unsigned char[]> ws = ctfa_dropin::stream_buffer<unsigned char>(wsBytes > 0 ? wsBytes : 256);
    ctfa_dropin::check(ctfa_backward(in[0], in[1], in[2], output.get(), outputGrad.get(), lse.get(),
                                     grads[0].data(), grads[1].data(), grads[2].data(), ws.get(), wsBytes,
                                     batchSize, numHeads, sequenceLength, headDim, code, causal ? 1 : 0, nullptr),
                       "ctfa_backward");
    return grads;
  }

  /** Clear cached values to free memory. */
  void clearCache() {
    cachedMaxScores = nullptr;
    cachedDenominators = nullptr;
    cachedOutput = nullptr;
    cachedLSE = nullptr;
    cachedRounded = nullptr;
    cachedRoundedFrom[0] = cachedRoundedFrom[1] = cachedRoundedFrom[2] = nullptr;
  }

 private:
  // Runs the forward; returns its workspace (float: the rounded q, k, v;
  // null when the dtype needs none).
  std::shared_ptr<unsigned char[]> runForward(const Tensor<DType>& queries, const Tensor<DType>& keys,
                                              const Tensor<DType>& values, DType* output, float* lse,
                                              int batchSize, int sequenceLength) {
    const int code = ctfa_dropin::DtypeCode<DType>::value;
    const size_t wsBytes = ctfa_forward_workspace_bytes(batchSize, numHeads, sequenceLength, headDim, code);
    std::shared_ptr<unsigned char[]> ws = ctfa_dropin::stream_buffer<unsigned char>(wsBytes);
    ctfa_dropin::check(ctfa_forward(queries.get(), keys.get(), values.get(), output, lse, batchSize, numHeads,
                                    sequenceLength, headDim, code, causal ? 1 : 0, ws.get(), wsBytes, nullptr),
                       "ctfa_forward");
    return ws;
  }
};

#endif  // FLASH_ATTENTION_LAYER
