// The reference's pybind module (cuda_transformer/cuda_transformer.cu:
// tensors, layers, NanoGPT, optimizers, every binding unchanged), compiled
// with this repository's AttentionLayer.cu drop-in (the F3 fix: the attention
// output is kept for the output projection's backward) and with the
// FlashAttentionLayer named by FLASH_LAYER_HEADER
// (cudatransformer_b200/FlashAttentionLayer.cu: the tcgen05 kernels).  Built
// by oracle/Makefile (target pybind) for tests/test_gpu_pybind.py; TEST /
// MEASUREMENT INFRASTRUCTURE ONLY.
#include FLASH_LAYER_HEADER
#include "../cudatransformer_b200/AttentionLayer.cu"
#include "cuda_transformer.cu"
