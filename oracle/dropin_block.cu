// dropin_block.cu -- TEST INFRASTRUCTURE ONLY.  The reference's
// TransformerBlockLayer / MLPLayer / ActivationLayer (cuda_transformer/*.cu,
// unmodified, from the reference tree) compiled against every drop-in of
// cudatransformer_b200/: AttentionLayer.cu (the F3 fix: the attention output
// is kept for the output projection's backward), QKVProjectionLayer.cu,
// FlashAttentionLayer.cu, OutputProjectionLayer.cu, LinearLayer.cu and
// LayerNorm.cu.  dropin_block_step (block_step.cuh) runs the block's forward
// and backward for a GPU parity test against an fp64 restatement.
#include "../cudatransformer_b200/AttentionLayer.cu"  // ours: same include guard as the reference file
#include "../cudatransformer_b200/LinearLayer.cu"     // ours, likewise
#include "../cudatransformer_b200/LayerNorm.cu"       // ours, likewise
#include "TransformerBlockLayer.cu"                   // reference

template struct TransformerBlockLayer<float>;
template struct TransformerBlockLayer<__nv_bfloat16>;

#include "block_step.cuh"
