// ref_harness.cu -- TEST INFRASTRUCTURE ONLY.  Builds the reference's own
// FlashAttentionLayer<DType> (cuda_transformer/FlashAttentionLayer.cu, kernels
// in cuda_transformer/flash_attention.cu) unmodified, from the reference tree,
// into oracle/_ref/libctref.so, and exposes it through a small C ABI so that
// tests can compare the reference's CUDA output with libctfa_b200.so and
// bench.py --impl reference can time the reference's stock code path.
//
// Every entry point drives the reference through its public API:
//   FlashAttentionLayer<DType>(headDim, numHeads)            (:29)
//   computeAttention(q, k, v, saveStates)                    (:45-87)
//   computeBackward(q, k, v, outputGrad)                     (:97-142)
//   clearCache()                                             (:145)
// with caller-owned device buffers wrapped as Tensor<DType> through the
// reference's shallow-wrap constructor (Tensor.cu:63).  Nothing of the
// reference is copied here; the sources are compiled where they lie.
#include "FlashAttentionLayer.cu"

namespace {

template <typename DT>
Tensor<DT> wrap(const void* p, int B, int H, int T, int D) {
  std::shared_ptr<DT[]> sp(const_cast<DT*>(static_cast<const DT*>(p)), [](DT*) {});
  return Tensor<DT>(sp, {(size_t)B, (size_t)H, (size_t)T, (size_t)D});
}

template <typename DT>
int fwd(const void* q, const void* k, const void* v, void* o, void* m, void* l, int B, int H, int T, int D) {
  FlashAttentionLayer<DT> layer(D, H);
  Tensor<DT> out = layer.computeAttention(wrap<DT>(q, B, H, T, D), wrap<DT>(k, B, H, T, D),
                                          wrap<DT>(v, B, H, T, D), true);
  const size_t n = (size_t)B * H * T * D, r = (size_t)B * H * T;
  if (o) cudaMemcpy(o, out.data(), n * sizeof(DT), cudaMemcpyDeviceToDevice);
  if (m) cudaMemcpy(m, layer.cachedMaxScores.get(), r * sizeof(DT), cudaMemcpyDeviceToDevice);
  if (l) cudaMemcpy(l, layer.cachedDenominators.get(), r * sizeof(DT), cudaMemcpyDeviceToDevice);
  return (int)cudaDeviceSynchronize();
}

template <typename DT>
int fwd_bwd(const void* q, const void* k, const void* v, const void* dO, void* o, void* dq, void* dk, void* dv,
            int B, int H, int T, int D) {
  FlashAttentionLayer<DT> layer(D, H);
  Tensor<DT> tq = wrap<DT>(q, B, H, T, D), tk = wrap<DT>(k, B, H, T, D), tv = wrap<DT>(v, B, H, T, D);
  Tensor<DT> out = layer.computeAttention(tq, tk, tv, true);
  std::array<Tensor<DT>, 3> g = layer.computeBackward(tq, tk, tv, wrap<DT>(dO, B, H, T, D));
  const size_t n = (size_t)B * H * T * D;
  if (o) cudaMemcpy(o, out.data(), n * sizeof(DT), cudaMemcpyDeviceToDevice);
  if (dq) cudaMemcpy(dq, g[0].data(), n * sizeof(DT), cudaMemcpyDeviceToDevice);
  if (dk) cudaMemcpy(dk, g[1].data(), n * sizeof(DT), cudaMemcpyDeviceToDevice);
  if (dv) cudaMemcpy(dv, g[2].data(), n * sizeof(DT), cudaMemcpyDeviceToDevice);
  layer.clearCache();
  return (int)cudaDeviceSynchronize();
}

}  // namespace

// dtype: 0 = float, 1 = __nv_bfloat16
extern "C" int ctref_forward(int dtype, const void* q, const void* k, const void* v, void* o, void* maxScores,
                             void* denominators, int B, int H, int T, int D) {
  if (dtype == 0) return fwd<float>(q, k, v, o, maxScores, denominators, B, H, T, D);
  if (dtype == 1) return fwd<__nv_bfloat16>(q, k, v, o, maxScores, denominators, B, H, T, D);
  return -1;
}

extern "C" int ctref_forward_backward(int dtype, const void* q, const void* k, const void* v, const void* dO,
                                      void* o, void* dq, void* dk, void* dv, int B, int H, int T, int D) {
  if (dtype == 0) return fwd_bwd<float>(q, k, v, dO, o, dq, dk, dv, B, H, T, D);
  if (dtype == 1) return fwd_bwd<__nv_bfloat16>(q, k, v, dO, o, dq, dk, dv, B, H, T, D);
  return -1;
}
