// The reference's pybind module (cuda_transformer/cuda_transformer.cu:
// NanoGPT, layers, optimizers), compiled with this repository's
// AttentionLayer.cu drop-in (the F3 fix: the attention output is kept for the
// output projection's backward) and with the FlashAttentionLayer chosen by
// FLASH_LAYER_HEADER: cudatransformer_b200/FlashAttentionLayer.cu (the
// tcgen05 kernels) or the reference's own.  Built by oracle/Makefile (target
// nanogpt) for the config-4 NanoGPT comparison; TEST / MEASUREMENT
// INFRASTRUCTURE ONLY.
#include FLASH_LAYER_HEADER
#include "../cudatransformer_b200/AttentionLayer.cu"
#include "cuda_transformer.cu"
