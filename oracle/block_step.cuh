// block_step.cuh -- TEST INFRASTRUCTURE ONLY.  C entry points around the
// reference's TransformerBlockLayer<float>, included by dropin_check.cu (the
// reference's AttentionLayer over the sub-layer drop-ins) and by
// dropin_block.cu (every layer a drop-in, AttentionLayer included).  Include
// after TransformerBlockLayer.cu.
#pragma once

#include <map>
#include <string>
#include <vector>

static std::string g_last_error;  // what() of the last exception an entry point caught

extern "C" const char* dropin_last_error() { return g_last_error.c_str(); }

// The reference's TransformerBlockLayer<float> (LayerNorm -> attention ->
// LayerNorm -> Linear, ReLU, Linear; TransformerBlockLayer.cu:60-66).  Every
// parameter named in names[0..n) is handed to the block's own
// setParameters() from the host array params[i] (sizes[i] floats, the shapes
// getParameters() reports), and params[i] is then overwritten with what
// getParameters() holds afterwards (the parameters the step really used:
// the block's setParameters drops the secondNorm.* entries,
// TransformerBlockLayer.cu:159 strips a 12-character prefix from the
// 11-character "secondNorm.").  Then y = forward(x), dx = backward(x, dy),
// and the gradient getGradients() reports under names[i] is copied to
// grads[i].  hidden ([B, N, mlp_dim], may be NULL) receives the first MLP
// Linear's output (the ReLU's input) of the same forward, so that a checker
// can apply the ReLU pattern this precision produced.  Returns 0, -2 when
// getGradients() lacks one of the names (the reference's LayerNorm has none),
// -3 for an unknown parameter name, -1 on an exception (message:
// dropin_last_error()), or a CUDA error code.
extern "C" int dropin_block_step(const float* x, const float* dy, float* y, float* dx, int B, int N, int E, int H,
                                 int mlp_dim, int causal, int n, const char** names, float** params,
                                 float** grads, const long long* sizes, float* hidden) {
  try {
    TransformerBlockLayer<float> block(E, H, E / H, mlp_dim);
    std::static_pointer_cast<AttentionLayer<float>>(block.attention)->flashAttn.causal = causal != 0;
    auto load = [](const float* host, std::vector<size_t> shape) {
      Tensor<float> t(shape);
      cudaMemcpy(t.data(), host, t.size() * sizeof(float), cudaMemcpyHostToDevice);
      return t;
    };
    auto current = block.getParameters();
    std::map<std::string, Tensor<float>> set;
    for (int i = 0; i < n; ++i) {
      auto it = current.find(names[i]);
      if (it == current.end() || (long long)it->second.size() != sizes[i]) return -3;
      set[names[i]] = load(params[i], it->second.shape().toVector());
    }
    block.setParameters(set);
    auto held = block.getParameters();
    for (int i = 0; i < n; ++i)
      cudaMemcpy(params[i], held.at(names[i]).data(), sizes[i] * sizeof(float), cudaMemcpyDeviceToHost);
    const std::vector<size_t> xs{(size_t)B, (size_t)N, (size_t)E};
    Tensor<float> tx = load(x, xs);
    Tensor<float> ty = block.forward(tx);
    cudaMemcpy(y, ty.data(), ty.size() * sizeof(float), cudaMemcpyDeviceToHost);
    if (hidden != nullptr) {
      Tensor<float> a = block.attention->forward(block.firstNorm->forward(tx));
      auto& layers = std::static_pointer_cast<MLPLayer<float>>(block.mlp)->modelLayers;
      Tensor<float> h = layers[0]->forward(block.secondNorm->forward(a));
      cudaMemcpy(hidden, h.data(), h.size() * sizeof(float), cudaMemcpyDeviceToHost);
    }
    Tensor<float> tdx = block.backward(tx, load(dy, xs));
    cudaMemcpy(dx, tdx.data(), tdx.size() * sizeof(float), cudaMemcpyDeviceToHost);
    auto g = block.getGradients();
    for (int i = 0; i < n; ++i) {
      auto it = g.find(names[i]);
      if (it == g.end()) return -2;
      cudaMemcpy(grads[i], it->second.data(), sizes[i] * sizeof(float), cudaMemcpyDeviceToHost);
    }
    return (int)cudaDeviceSynchronize();
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return -1;
  }
}
