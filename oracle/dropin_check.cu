// dropin_check.cu -- TEST INFRASTRUCTURE ONLY.  Compiles the reference's own
// AttentionLayer / TransformerBlockLayer (cuda_transformer/*.cu, unmodified,
// from the reference tree) against cudatransformer_b200/FlashAttentionLayer.cu,
// QKVProjectionLayer.cu, OutputProjectionLayer.cu, LinearLayer.cu and
// LayerNorm.cu (the drop-ins),
// for every element type the reference instantiates (float, double, half,
// bfloat16; cuda_transformer.cu:839-842), and exposes one C entry point that
// runs the reference's AttentionLayer<float>::forward through it, another
// its TransformerBlockLayer<float> forward + backward (whose backward stops
// at the reference AttentionLayer's released attention output, which the
// output-projection drop-in rejects), and one that times the
// FlashAttentionLayer<float> drop-in's forward + backward step.  It proves the
// drop-ins compile where the reference's layers did, and lets a GPU test
// compare the composed layer with an fp64 restatement.
#include "FlashAttentionLayer.cu"  // ours: same include guard as the reference file
#include "OutputProjectionLayer.cu"  // ours, likewise
#include "QKVProjectionLayer.cu"  // ours, likewise
#include "LinearLayer.cu"  // ours, likewise
#include "LayerNorm.cu"  // ours, likewise
#include "TransformerBlockLayer.cu"  // reference: pulls AttentionLayer.cu -> our layers
#include "block_step.cuh"  // g_last_error, dropin_last_error, dropin_block_step

template struct FlashAttentionLayer<float>;
template struct FlashAttentionLayer<double>;
template struct FlashAttentionLayer<__half>;
template struct FlashAttentionLayer<__nv_bfloat16>;
template struct QKVProjectionLayer<float>;
template struct QKVProjectionLayer<double>;
template struct QKVProjectionLayer<__half>;
template struct QKVProjectionLayer<__nv_bfloat16>;
template struct OutputProjectionLayer<float>;
template struct OutputProjectionLayer<double>;
template struct OutputProjectionLayer<__half>;
template struct OutputProjectionLayer<__nv_bfloat16>;
template struct LinearLayer<float>;
template struct LinearLayer<double>;
template struct LinearLayer<__half>;
template struct LinearLayer<__nv_bfloat16>;
template struct LayerNormLayer<float>;
template struct LayerNormLayer<double>;
template struct LayerNormLayer<__half>;
template struct LayerNormLayer<__nv_bfloat16>;
template struct AttentionLayer<float>;
template struct AttentionLayer<__nv_bfloat16>;
template struct TransformerBlockLayer<float>;

// x: [B, N, E] host array; w*: [E, E] host arrays (row-major, y = x W^T);
// out: [B, N, E] host array.  Biases are zero.  causal selects the mask.
extern "C" int dropin_attention_forward(const float* x, const float* wq, const float* wk, const float* wv,
                                        const float* wo, float* out, int B, int N, int E, int H, int causal) {
  try {
    const int D = E / H;
    AttentionLayer<float> layer(E, H, D);
    layer.flashAttn.causal = causal != 0;
    auto load = [](const float* host, std::vector<size_t> shape) {
      Tensor<float> t(shape);
      cudaMemcpy(t.data(), host, t.size() * sizeof(float), cudaMemcpyHostToDevice);
      return t;
    };
    layer.setQueryWeights(load(wq, {(size_t)E, (size_t)E}));
    layer.setKeyWeights(load(wk, {(size_t)E, (size_t)E}));
    layer.setValueWeights(load(wv, {(size_t)E, (size_t)E}));
    layer.setOutputWeights(load(wo, {(size_t)E, (size_t)E}));
    Tensor<float> y = layer.forward(load(x, {(size_t)B, (size_t)N, (size_t)E}));
    cudaMemcpy(out, y.data(), y.size() * sizeof(float), cudaMemcpyDeviceToHost);
    return (int)cudaDeviceSynchronize();
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return -1;
  }
}

// Device-resident variant (x, w*, y device pointers; biases zero): builds the
// reference's AttentionLayer<float> over the drop-ins, runs forward, copies y
// with a stream-ordered copy and returns WITHOUT synchronising, so that a test
// can check that nothing in construction, forward or teardown waited for the
// device (the drop-ins' buffers are stream-ordered).
extern "C" int dropin_attention_forward_device(const float* x, const float* wq, const float* wk, const float* wv,
                                               const float* wo, float* y, int B, int N, int E, int H, int causal) {
  try {
    const int D = E / H;
    AttentionLayer<float> layer(E, H, D);
    layer.flashAttn.causal = causal != 0;
    auto view = [](const float* p, std::vector<size_t> shape) {
      return Tensor<float>(std::shared_ptr<float[]>(const_cast<float*>(p), [](float*) {}), shape);
    };
    layer.setQueryWeights(view(wq, {(size_t)E, (size_t)E}));
    layer.setKeyWeights(view(wk, {(size_t)E, (size_t)E}));
    layer.setValueWeights(view(wv, {(size_t)E, (size_t)E}));
    layer.setOutputWeights(view(wo, {(size_t)E, (size_t)E}));
    Tensor<float> out = layer.forward(view(x, {(size_t)B, (size_t)N, (size_t)E}));
    cudaMemcpyAsync(y, out.data(), out.size() * sizeof(float), cudaMemcpyDeviceToDevice, 0);
    return (int)cudaGetLastError();
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return -1;
  }
}

// FlashAttentionLayer<float> (the drop-in) on device-resident [B, H, T, D]
// buffers: `iters` steps of computeAttention(saveStates=true) +
// computeBackward + clearCache on the default stream, the way the reference's
// AttentionLayer drives it (AttentionLayer.cu:87, :141).  Writes the last
// step's o, dq, dk, dv and the mean step time (CUDA events on the default
// stream, after one untimed step).
extern "C" int dropin_flash_step_f32(const float* q, const float* k, const float* v, const float* dO, float* o,
                                     float* dq, float* dk, float* dv, int B, int H, int T, int D, int causal,
                                     int iters, float* ms_per_step) {
  try {
    FlashAttentionLayer<float> layer(D, H, causal != 0);
    const std::vector<size_t> shape = {(size_t)B, (size_t)H, (size_t)T, (size_t)D};
    auto view = [&](const float* p) {
      return Tensor<float>(std::shared_ptr<float[]>(const_cast<float*>(p), [](float*) {}), shape);
    };
    Tensor<float> tq = view(q), tk = view(k), tv = view(v), tdo = view(dO);
    const size_t n = (size_t)B * H * T * D;
    auto step = [&](bool keep) {
      Tensor<float> out = layer.computeAttention(tq, tk, tv, true);
      std::array<Tensor<float>, 3> g = layer.computeBackward(tq, tk, tv, tdo);
      layer.clearCache();
      if (keep) {
        cudaMemcpyAsync(o, out.data(), n * sizeof(float), cudaMemcpyDeviceToDevice, 0);
        float* dst[3] = {dq, dk, dv};
        for (int i = 0; i < 3; ++i) cudaMemcpyAsync(dst[i], g[i].data(), n * sizeof(float), cudaMemcpyDeviceToDevice, 0);
      }
    };
    step(true);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, 0);
    for (int i = 0; i < iters; ++i) step(false);
    cudaEventRecord(e1, 0);
    cudaEventSynchronize(e1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *ms_per_step = iters > 0 ? ms / iters : 0.f;
    return (int)cudaDeviceSynchronize();
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return -1;
  }
}
