/*
 * liblaya_cuda — fused ModernBERT encoder over unpadded variable-length
 * batches (the throughput path behind the contract).
 *
 * The reference runs the encoder as ~18 contract ops per layer on padded
 * [B, L] batches with host-built boolean masks
 * (packages/modernbert/src/index.ts:342-357 ModernBert.layer, :407-429
 * encode, :240-259 attentionMasks). These entry points compute the same
 * function on packed sequences (cu_seqlens), with the permutes, RoPE, GeGLU
 * and residual adds fused into the GEMM epilogues and the masks replaced by
 * the window rule inside the attention kernel. Valid-token outputs equal the
 * padded forward's (every mask only admits keys of the query's own sequence).
 *
 * Weights are tensors already uploaded with lc_from_host (or
 * lc_from_host_quantized), in the order of buildEncoderWeights
 * (packages/modernbert/src/index.ts:532-559):
 *   tok_embeddings [V, H], embeddings.norm [H],
 *   per layer i: attn_norm [H] (0 for layer 0), Wqkv [3H, H], Wo [H, H],
 *                mlp_norm [H], Wi [2I, H], mlp.Wo [H, I],
 *   final_norm [H].
 * Norm biases and linear biases are not part of ModernBERT-base/large
 * (norm_bias = attention_bias = mlp_bias = false) and are not accepted here.
 */
#ifndef LAYA_CUDA_ENCODER_H
#define LAYA_CUDA_ENCODER_H
#include "laya_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int32_t vocab_size, hidden_size, intermediate_size, num_layers, num_heads;
  int32_t local_attention; /* sliding window width; keys with |i - j| <= local_attention / 2 */
  int32_t dtype;           /* 1 = f16, 2 = bf16 (compute/storage dtype) */
  int32_t quant_bits;      /* 0 = dense weights; 4 or 8 = affine/symmetric packed Linear weights */
  int32_t quant_group;     /* group size of the packed weights */
  int32_t quant_mode;      /* 0 symmetric, 1 affine */
  double norm_eps, rope_theta_global, rope_theta_local;
} lc_encoder_config;

/*
 * Builds an encoder (parseModernBertConfig + loadModernBert,
 * packages/modernbert/src/index.ts:58-110, 498-529). `layer_kinds[i]` is 0 for
 * full_attention and 1 for sliding_attention. `weights` holds the handles in
 * the order above; for quant_bits != 0 each Linear weight (Wqkv, Wo, Wi,
 * mlp.Wo) is replaced by three consecutive handles (packed, scales, biases|0)
 * from lc_from_host_quantized. The encoder keeps its own references.
 * Shapes: head dim 64 (hidden_size = 64 * num_heads), hidden_size a multiple
 * of 64 up to 2048, intermediate_size a multiple of 32 (any size relative to
 * hidden_size), f16 or bf16; the forwards take sequences of 1 to 8192 tokens.
 * Other shapes return an error; the contract ops (ModernBert.forward) serve
 * them.
 */
int lc_encoder_create(uint64_t* enc, const lc_encoder_config* cfg, const int32_t* layer_kinds, const lc_tensor* weights, int nweights);
int lc_encoder_free(uint64_t enc);

/*
 * One forward over packed sequences: ids i32 [T] on the device,
 * cu_seqlens (host, nseq + 1 entries, 0 .. T). Outputs (each optional):
 * hidden = final-norm hidden states [T, H] (ModernBert.encode on the valid
 * tokens), probs = softmax(CLS row · head_wᵀ + head_b) f32 [nseq, C]
 * (the classifier pattern of packages/laya/src/model.ts:228).
 */
int lc_encoder_forward(lc_tensor* hidden, lc_tensor* probs, uint64_t enc, lc_tensor ids, const int32_t* cu_seqlens, int nseq,
                       lc_tensor head_w, lc_tensor head_b);

/*
 * End-to-end form with host buffers: copies ids (host, T values) to the
 * device, runs lc_encoder_forward, copies probs back to `probs_host`
 * (nseq x C floats) and synchronises.
 */
int lc_encoder_forward_host(uint64_t enc, const int32_t* ids_host, const int32_t* cu_seqlens, int nseq, lc_tensor head_w, lc_tensor head_b,
                            float* probs_host);

/*
 * Replay of lc_encoder_forward_host for one fixed batch shape as a CUDA
 * graph (no counterpart in the reference, whose TypeScript host issues every
 * op itself). create captures, for the given cu_seqlens and head, the copy of
 * the ids into the device, the whole forward and the copy of the
 * probabilities out, with workspace, metadata and I/O buffers owned by the
 * graph. run takes ids (host, T = cu_seqlens[nseq] values), replays the graph
 * and writes probs (host, nseq x C floats); it returns after the result is on
 * the host. Freeing the encoder frees its graphs. Per-kernel tracing does not
 * apply to replays.
 */
int lc_encoder_graph_create(uint64_t* graph, uint64_t enc, const int32_t* cu_seqlens, int nseq, lc_tensor head_w, lc_tensor head_b);
int lc_encoder_graph_run(uint64_t graph, const int32_t* ids_host, float* probs_host);
int lc_encoder_graph_free(uint64_t graph);

/*
 * Per-kernel-class device timing of the forwards that follow (tracing):
 * when enabled, every forward records CUDA events around its kernels on the
 * library stream. lc_encoder_profile_read returns, per class, the summed
 * milliseconds and launch counts since the last read, then resets them.
 * Classes: 0 Wqkv GEMM (+RoPE), 1 attention, 2 LayerNorm/embedding,
 * 3 head/dequant/other, 4 Wo GEMM (+residual), 5 Wi GEMM (+GeGLU),
 * 6 mlp.Wo GEMM (+residual), 7 unused.
 */
int lc_encoder_set_profiling(uint64_t enc, int on);
int lc_encoder_profile_read(uint64_t enc, double* ms /* [8] */, int64_t* launches /* [8] */);

/*
 * Attention of one encoder layer on its own: qkv [T, 3H] (RoPE applied),
 * heads of 64; half_window < 0 = global attention. Returns att [T, H].
 * kernel 0 = tcgen05/TMEM kernel (the one the encoder runs), 1 = the
 * mma.sync kernel (kept as an independent cross-check).
 */
int lc_attention_varlen(lc_tensor* out, lc_tensor qkv, const int32_t* cu_seqlens, int nseq, int half_window, double scale, int kernel);

#ifdef __cplusplus
}
#endif
#endif /* LAYA_CUDA_ENCODER_H */
