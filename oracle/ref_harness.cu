// ref_harness.cu -- TEST INFRASTRUCTURE ONLY.  Builds the reference's own
// FlashAttentionLayer<DType> (cuda_transformer/FlashAttentionLayer.cu, kernels
// in cuda_transformer/flash_attention.cu), QKVProjectionLayer and
// OutputProjectionLayer (kernels in attention_qkv_kernels.cu and
// attention_proj_kernels.cu), LinearLayer and LayerNormLayer (linear_kernels.cu,
// layer_norm_kernels.cu) unmodified, from the reference tree,
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
#include "LayerNorm.cu"
#include "LinearLayer.cu"
#include "OutputProjectionLayer.cu"
#include "QKVProjectionLayer.cu"

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

// Non-owning shared_ptr over a caller buffer (the layers' parameter fields).
template <typename DT>
std::shared_ptr<DT[]> borrow(const void* p) {
  return std::shared_ptr<DT[]>(const_cast<DT*>(static_cast<const DT*>(p)), [](DT*) {});
}

template <typename DT>
void copy_out(void* dst, const std::shared_ptr<DT[]>& src, size_t n) {
  if (dst && src) cudaMemcpy(dst, src.get(), n * sizeof(DT), cudaMemcpyDeviceToDevice);
}

// QKVProjectionLayer<DT>(E, H, D) (QKVProjectionLayer.cu:38) with the
// caller's weights, computeQKV (:73) and, when gq is given,
// computeBackward (:100); the gradient buffers start at zero (:107-116).
template <typename DT>
int qkv(const void* x, const void* const* w, const void* const* bias, void* const* out, const void* const* grad,
        void* dx, void* const* dw, void* const* db, int B, int T, int E, int H, int D) {
  QKVProjectionLayer<DT> layer(E, H, D);
  layer.weightsQuery = borrow<DT>(w[0]);
  layer.weightsKey = borrow<DT>(w[1]);
  layer.weightsValue = borrow<DT>(w[2]);
  layer.biasesQuery = borrow<DT>(bias[0]);
  layer.biasesKey = borrow<DT>(bias[1]);
  layer.biasesValue = borrow<DT>(bias[2]);
  Tensor<DT> tx(borrow<DT>(x), {(size_t)B, (size_t)T, (size_t)E});
  std::array<Tensor<DT>, 3> qkv_out = layer.computeQKV(tx);
  const size_t n = (size_t)B * H * T * D, hd = (size_t)H * D;
  for (int i = 0; i < 3; ++i) copy_out<DT>(out[i], qkv_out[i].dataPtr(), n);
  if (grad[0]) {
    auto g = [&](int i) { return Tensor<DT>(borrow<DT>(grad[i]), {(size_t)B, (size_t)H, (size_t)T, (size_t)D}); };
    Tensor<DT> gx = layer.computeBackward(tx, g(0), g(1), g(2));
    copy_out<DT>(dx, gx.dataPtr(), (size_t)B * T * E);
    copy_out<DT>(dw[0], layer.weightsQueryGrad, hd * E);
    copy_out<DT>(dw[1], layer.weightsKeyGrad, hd * E);
    copy_out<DT>(dw[2], layer.weightsValueGrad, hd * E);
    copy_out<DT>(db[0], layer.biasesQueryGrad, hd);
    copy_out<DT>(db[1], layer.biasesKeyGrad, hd);
    copy_out<DT>(db[2], layer.biasesValueGrad, hd);
  }
  return (int)cudaDeviceSynchronize();
}

// OutputProjectionLayer<DT>(E, D, H) (OutputProjectionLayer.cu:28) with the
// caller's weights, forward (:52) and, when dy is given, backward (:69).
template <typename DT>
int out_proj(const void* a, const void* wo, const void* bo, void* y, const void* dy, void* da, void* dwo, void* dbo,
             int B, int T, int E, int H, int D) {
  OutputProjectionLayer<DT> layer(E, D, H);
  layer.weightsProj = borrow<DT>(wo);
  layer.biasesProj = borrow<DT>(bo);
  Tensor<DT> ta(borrow<DT>(a), {(size_t)B, (size_t)H, (size_t)T, (size_t)D});
  Tensor<DT> ty = layer.forward(ta);
  copy_out<DT>(y, ty.dataPtr(), (size_t)B * T * E);
  if (dy) {
    Tensor<DT> ga = layer.backward(ta, Tensor<DT>(borrow<DT>(dy), {(size_t)B, (size_t)T, (size_t)E}));
    copy_out<DT>(da, ga.dataPtr(), (size_t)B * H * T * D);
    copy_out<DT>(dwo, layer.weightsProjGrad, (size_t)E * H * D);
    copy_out<DT>(dbo, layer.biasesProjGrad, (size_t)E);
  }
  return (int)cudaDeviceSynchronize();
}

// LinearLayer<float>(K, N) (LinearLayer.cu:25) with the caller's weights:
// forward (:45) and, when dy is given, backward (:73); gradients start at 0.
int linear(const void* x, const void* w, const void* b, void* y, const void* dy, void* dx, void* dw, void* db, int M,
           int K, int N) {
  LinearLayer<float> layer(K, N);
  layer.weights = borrow<float>(w);
  layer.biases = borrow<float>(b);
  Tensor<float> tx(borrow<float>(x), {(size_t)M, (size_t)K});
  Tensor<float> ty = layer.forward(tx);
  copy_out<float>(y, ty.dataPtr(), (size_t)M * N);
  if (dy) {
    Tensor<float> gx = layer.backward(tx, Tensor<float>(borrow<float>(dy), {(size_t)M, (size_t)N}));
    copy_out<float>(dx, gx.dataPtr(), (size_t)M * K);
    copy_out<float>(dw, layer.weightGrad, (size_t)N * K);
    copy_out<float>(db, layer.biasGrad, (size_t)N);
  }
  return (int)cudaDeviceSynchronize();
}

// LayerNormLayer<float>(E) (LayerNorm.cu:31, eps 1e-5) with the caller's
// scale / shift: forward (:104) and, when dy is given, backward (:135).
int layernorm(const void* x, const void* w, const void* b, void* y, const void* dy, void* dx, void* dw, void* db,
              int M, int E) {
  LayerNormLayer<float> layer(E);
  layer.weights = borrow<float>(w);
  layer.biases = borrow<float>(b);
  Tensor<float> tx(borrow<float>(x), {(size_t)M, (size_t)E});
  Tensor<float> ty = layer.forward(tx);
  copy_out<float>(y, ty.dataPtr(), (size_t)M * E);
  if (dy) {
    Tensor<float> gx = layer.backward(tx, Tensor<float>(borrow<float>(dy), {(size_t)M, (size_t)E}));
    copy_out<float>(dx, gx.dataPtr(), (size_t)M * E);
    copy_out<float>(dw, layer.weightsGrad, (size_t)E);
    copy_out<float>(db, layer.biasesGrad, (size_t)E);
  }
  return (int)cudaDeviceSynchronize();
}

}  // namespace

extern "C" int ctref_linear(const void* x, const void* w, const void* b, void* y, const void* dy, void* dx, void* dw,
                            void* db, int M, int K, int N) {
  return linear(x, w, b, y, dy, dx, dw, db, M, K, N);
}

extern "C" int ctref_layernorm(const void* x, const void* w, const void* b, void* y, const void* dy, void* dx,
                               void* dw, void* db, int M, int E) {
  return layernorm(x, w, b, y, dy, dx, dw, db, M, E);
}

// fp32 only.  w/bias/out/grad/dw/db: arrays of 3 device pointers (q, k, v).
extern "C" int ctref_qkv_projection(const void* x, const void* const* w, const void* const* bias, void* const* out,
                                    const void* const* grad, void* dx, void* const* dw, void* const* db, int B,
                                    int T, int E, int H, int D) {
  return qkv<float>(x, w, bias, out, grad, dx, dw, db, B, T, E, H, D);
}

extern "C" int ctref_out_projection(const void* a, const void* wo, const void* bo, void* y, const void* dy,
                                    void* da, void* dwo, void* dbo, int B, int T, int E, int H, int D) {
  return out_proj<float>(a, wo, bo, y, dy, da, dwo, dbo, B, T, E, H, D);
}

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
