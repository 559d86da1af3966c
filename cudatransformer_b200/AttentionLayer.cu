// Drop-in replacement for cuda_transformer/AttentionLayer.cu: the same
// template, members, methods and include guard, so TransformerBlockLayer.cu,
// TransformerLayer.cu, NanoGPT.cu and the pybind module compile against it
// unchanged (include it, and cudatransformer_b200/FlashAttentionLayer.cu,
// before the reference's cuda_transformer.cu).
//
// One behaviour differs, on purpose: the reference's forward with state
// caching stores the attention output in outStates[3] and then releases it
// (AttentionLayer.cu:88-100), so backward passes an empty tensor to the
// output projection's backward (AttentionLayer.cu:136), which divides by a
// zero sequence length (OutputProjectionLayer.cu:76-77) on every backward
// through the layer.  Here outStates[3] keeps the attention output until the
// backward has used it.
//
// QKV projection -> FlashAttentionLayer -> output projection, as in the
// reference; the parameter / gradient plumbing is table driven.
#include <array>
#include <map>
#include <string>
#include <vector>

#include "QKVProjectionLayer.cu"
#include "FlashAttentionLayer.cu"
#include "OutputProjectionLayer.cu"

#ifndef ATTENTION_LAYER_REFACTORED
#define ATTENTION_LAYER_REFACTORED

template <typename DType = float> struct AttentionLayer : public Layer<DType> {
    QKVProjectionLayer<DType> qkvProj;
    FlashAttentionLayer<DType> flashAttn;
    OutputProjectionLayer<DType> outProj;

    int inputDim = 1;
    int numHeads = 1;
    int headDim = 1;

    AttentionLayer(int inputDim, int numHeads, int headDim)
        : Layer<DType>(),
          qkvProj(inputDim, numHeads, headDim),
          flashAttn(headDim, numHeads),
          outProj(inputDim, headDim, numHeads),
          inputDim(inputDim), numHeads(numHeads), headDim(headDim) {}

    // ---- trainable tensors: name, parameter buffer, gradient buffer, shape ----
    struct Slot {
        const char* name;
        std::shared_ptr<DType[]>* param;
        std::shared_ptr<DType[]>* grad;
        std::vector<size_t> shape;
        size_t count() const {
            size_t n = 1;
            for (size_t d : shape) n *= d;
            return n;
        }
    };

    std::array<Slot, 8> slots() {
        const size_t in = (size_t)inputDim, hd = (size_t)(headDim * numHeads);
        return {{
            {"query.weights", &qkvProj.weightsQuery, &qkvProj.weightsQueryGrad, {in, hd}},
            {"query.biases", &qkvProj.biasesQuery, &qkvProj.biasesQueryGrad, {hd}},
            {"key.weights", &qkvProj.weightsKey, &qkvProj.weightsKeyGrad, {in, hd}},
            {"key.biases", &qkvProj.biasesKey, &qkvProj.biasesKeyGrad, {hd}},
            {"value.weights", &qkvProj.weightsValue, &qkvProj.weightsValueGrad, {in, hd}},
            {"value.biases", &qkvProj.biasesValue, &qkvProj.biasesValueGrad, {hd}},
            {"output.weights", &outProj.weightsProj, &outProj.weightsProjGrad, {hd, in}},
            {"output.biases", &outProj.biasesProj, &outProj.biasesProjGrad, {in}},
        }};
    }

    Tensor<DType> slotTensor(const Slot& s, bool grad) {
        std::shared_ptr<DType[]>& buf = grad ? *s.grad : *s.param;
        if (grad && buf == nullptr) buf = ctfa_dropin::stream_buffer<DType>(s.count(), true);  // lazily, zero-filled
        return Tensor<DType>(buf, s.shape);
    }

    std::shared_ptr<Layer<DType>> clone() override {
        auto copy = std::make_shared<AttentionLayer<DType>>(inputDim, numHeads, headDim);
        std::array<Slot, 8> mine = slots(), theirs = copy->slots();
        for (size_t i = 0; i < mine.size(); ++i)
            cudaMemcpyAsync(theirs[i].param->get(), mine[i].param->get(), mine[i].count() * sizeof(DType),
                            cudaMemcpyDeviceToDevice, 0);
        return copy;
    }

    Tensor<DType> forward(Tensor<DType> input) override { return forward(input, nullptr); }

    // outStates (optional, 4 entries): queries, keys, values and the attention
    // output, all kept for backward(input, gradOutput, outStates).
    Tensor<DType> forward(Tensor<DType> input, Tensor<DType>* outStates) {
        std::array<Tensor<DType>, 3> qkv = qkvProj.computeQKV(input);
        Tensor<DType> attention = flashAttn.computeAttention(qkv[0], qkv[1], qkv[2], outStates != nullptr);
        if (outStates != nullptr) {
            outStates[0] = qkv[0];
            outStates[1] = qkv[1];
            outStates[2] = qkv[2];
            outStates[3] = attention;
        }
        return outProj.forward(attention);
    }

    Tensor<DType> backward(Tensor<DType> input, Tensor<DType> gradOutput) override {
        std::array<Tensor<DType>, 4> states;
        forward(input, states.data());
        return backward(input, gradOutput, states.data());
    }

    // Uses and releases the tensors cached by forward(input, states).
    Tensor<DType> backward(Tensor<DType> input, Tensor<DType> gradOutput, Tensor<DType>* states) {
        Tensor<DType> attentionGrad = outProj.backward(states[3], gradOutput);
        states[3] = Tensor<DType>();
        std::array<Tensor<DType>, 3> qkvGrads = flashAttn.computeBackward(states[0], states[1], states[2], attentionGrad);
        for (int i = 0; i < 3; ++i) states[i] = Tensor<DType>();
        attentionGrad = Tensor<DType>();
        Tensor<DType> inputGrad = qkvProj.computeBackward(input, qkvGrads[0], qkvGrads[1], qkvGrads[2]);
        flashAttn.clearCache();
        return inputGrad;
    }

    // ---- weight / bias views (shallow: they share the layer's buffers) ----
    Tensor<DType> getQueryWeights() { return slotTensor(slots()[0], false); }
    Tensor<DType> getQueryBiases() { return slotTensor(slots()[1], false); }
    Tensor<DType> getKeyWeights() { return slotTensor(slots()[2], false); }
    Tensor<DType> getKeyBiases() { return slotTensor(slots()[3], false); }
    Tensor<DType> getValueWeights() { return slotTensor(slots()[4], false); }
    Tensor<DType> getValueBiases() { return slotTensor(slots()[5], false); }
    Tensor<DType> getOutputWeights() { return slotTensor(slots()[6], false); }
    Tensor<DType> getOutputBiases() { return slotTensor(slots()[7], false); }
    void setQueryWeights(Tensor<DType> t) { qkvProj.weightsQuery = t.dataPtr(); }
    void setQueryBiases(Tensor<DType> t) { qkvProj.biasesQuery = t.dataPtr(); }
    void setKeyWeights(Tensor<DType> t) { qkvProj.weightsKey = t.dataPtr(); }
    void setKeyBiases(Tensor<DType> t) { qkvProj.biasesKey = t.dataPtr(); }
    void setValueWeights(Tensor<DType> t) { qkvProj.weightsValue = t.dataPtr(); }
    void setValueBiases(Tensor<DType> t) { qkvProj.biasesValue = t.dataPtr(); }
    void setOutputWeights(Tensor<DType> t) { outProj.weightsProj = t.dataPtr(); }
    void setOutputBiases(Tensor<DType> t) { outProj.biasesProj = t.dataPtr(); }

    void zeroGrad() override {
        for (const Slot& s : slots())
            if (*s.grad != nullptr) cudaMemset(s.grad->get(), 0, s.count() * sizeof(DType));
    }

    void sgdUpdate(DType lr) override {
        for (const Slot& s : slots()) {
            if (*s.grad == nullptr) *s.grad = ctfa_dropin::stream_buffer<DType>(s.count(), true);
            runSgdUpdate<DType>(*s.param, *s.grad, lr, (int)s.count());
        }
    }

    std::map<std::string, Tensor<DType>> getParameters() override {
        std::map<std::string, Tensor<DType>> out;
        for (const Slot& s : slots()) out[s.name] = slotTensor(s, false);
        return out;
    }

    void setParameters(const std::map<std::string, Tensor<DType>>& params) override {
        for (const Slot& s : slots()) {
            auto it = params.find(s.name);
            if (it != params.end()) *s.param = it->second.dataPtr();
        }
    }

    std::map<std::string, Tensor<DType>> getGradients() override {
        std::map<std::string, Tensor<DType>> out;
        for (const Slot& s : slots()) out[s.name] = slotTensor(s, true);
        return out;
    }
};

template <typename DType = float> Module<DType> Attention(int inputDim, int numHeads, int headDim) {
    return std::make_shared<AttentionLayer<DType>>(inputDim, numHeads, headDim);
}

#endif  // ATTENTION_LAYER_REFACTORED
