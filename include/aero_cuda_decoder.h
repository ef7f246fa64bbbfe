/*
 * aero_cuda_decoder — the qwen-style decoder around the MoE layer on one B200,
 * plain C ABI (same library as aero_cuda_moe.h).
 *
 * One step runs the reference's block loop (src/model.cpp:234-330) for T tokens,
 * each of its own sequence at its own position:
 *   x = embedding rows (token_embd, a row gather)
 *   per layer: h = RMSNorm(x, attn_norm); q, k, v = h W_q, h W_k, h W_v;
 *              per-head RMSNorm of q and k (attn_q_norm / attn_k_norm), neox RoPE
 *              (src/attention_layer.cpp:95-156); k, v appended to the sequence's
 *              f16 cache; causal GQA attention over the sequence's positions
 *              0..pos (src/transformer.cpp:120-205); x += att W_o;
 *              h = RMSNorm(x, post_attention_norm); x += MoE(h) (this library's layer);
 *   logits = RMSNorm(x, output_norm) W_head (output.weight, or token_embd tied).
 * The cache is f16 (the reference's native slots hold fp32, int8 or int4,
 * src/kv.cpp); the projections are quantised (Q8_0 / Q4_K) GEMVs with f32
 * accumulation. There is no CPU fallback.
 */
#ifndef AERO_CUDA_DECODER_H
#define AERO_CUDA_DECODER_H

#include <stdint.h>

#include "aero_cuda_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct aero_cuda_decoder_layer {
    /* (n_head * head_dim, n_embd), (n_head_kv * head_dim, n_embd) x 2, (n_embd, n_head * head_dim):
     * Q8_0 or Q4_K GGUF bytes, host or device */
    aero_cuda_tensor attn_q, attn_k, attn_v, attn_output;
    const float* attn_norm;  /* (n_embd) f32 */
    const float* ffn_norm;   /* (n_embd) f32: the reference's post_attention_norm */
    const float* q_norm;     /* (head_dim) f32, or NULL */
    const float* k_norm;     /* (head_dim) f32, or NULL */
    void* moe;               /* this layer's aero_cuda_moe handle (borrowed: the caller closes it after
                                the decoder; the decoder moves it to its own stream) */
} aero_cuda_decoder_layer;

typedef struct aero_cuda_decoder_desc {
    int32_t n_layer, n_embd, n_head, n_head_kv, head_dim, vocab;
    int32_t n_seq, n_ctx; /* sequences and positions per sequence the f16 cache holds */
    int32_t device, reserved;
    float eps, rope_base;
    aero_cuda_tensor token_embd; /* (vocab, n_embd) Q8_0 */
    aero_cuda_tensor output;     /* (vocab, n_embd) Q8_0 / Q4_K; data NULL: the head is token_embd */
    const float* output_norm;    /* (n_embd) f32 */
    const aero_cuda_decoder_layer* layers; /* n_layer entries */
} aero_cuda_decoder_desc;

/* Upload the weights and allocate the caches (every allocation charged to the
 * library's memory guard). head_dim must be a multiple of 64 and at most 256,
 * n_head a multiple of n_head_kv with at most 16 query heads per kv head, RoPE
 * over the whole head. NULL with the reason in err. */
void* aero_cuda_decoder_open(const aero_cuda_decoder_desc* desc, char* err, int errlen);

/* Device bytes the decoder itself allocates for this description (its weights
 * and caches; the MoE handles are planned by aero_cuda_moe_open), as the memory
 * guard charges them: the total, and by_class[0] weights / by_class[1] KV cache
 * when by_class is not NULL. Open checks this plan with admit_plan before it
 * allocates. With the MoE handles' own plans (aero_b200.decoder.plan_footprint
 * adds them) it replaces the reference's plan_footprint (engine/model.py:776-840),
 * whose expert term (:828-832) counts fp32 bytes of the active experts, with
 * quantised device bytes. -1 for an invalid description. */
int64_t aero_cuda_decoder_plan_bytes(const aero_cuda_decoder_desc* desc, int64_t* by_class);

/* The same from a GGUF file: metadata "<arch>.block_count", embedding_length,
 * attention.head_count, attention.head_count_kv, attention.key_length,
 * rope.freq_base, attention.layer_norm_rms_epsilon (engine/model.py:193-224);
 * tensors token_embd, output (optional: tied), output_norm and per layer
 * attn_norm, post_attention_norm (or ffn_norm), attn_q/k/v/output,
 * attn_q_norm/attn_k_norm (optional) and the MoE tensors (opened with
 * aero_cuda_moe_open_gguf; owned by the decoder). */
void* aero_cuda_decoder_open_gguf(const char* path, int device, int n_seq, int n_ctx, char* err, int errlen);

/* aero_model_forward's contract (src/model.cpp:389-392) on sequence 0: n_tokens
 * tokens at `positions` (host arrays), logits of the last one (vocab floats,
 * host or device). Returns 1 on success, 0 on refusal. */
int aero_cuda_decoder_forward(void* dec, const int32_t* tokens, int n_tokens, const int64_t* positions,
                              float* logits);

/* One step over T tokens: token i of sequence seqs[i] at positions[i] (host
 * arrays; every (sequence, position) pair at most once, positions < n_ctx). The
 * cache rows of the step are written before any token attends, so a prompt's
 * tokens in one step attend causally to each other. logits: (T, vocab), host or
 * device, or NULL (no head: a prefill that only fills the cache). 0 / -1. */
int aero_cuda_decoder_step(void* dec, const int32_t* tokens, const int32_t* seqs, const int64_t* positions, int T,
                           float* logits);

/* Run on a cudaStream_t (the layers' MoE handles follow); NULL restores the
 * decoder's own. Calls with host logits synchronise it; others only enqueue. 0 / -1. */
int aero_cuda_decoder_set_stream(void* dec, void* stream);

/* Device pointers of layer's caches: (n_seq, n_head_kv, n_ctx, head_dim) f16 each. 0 / -1. */
int aero_cuda_decoder_kv(void* dec, int layer, void** k, void** v);

/* Profiling: with on != 0 each step records the device time of its phases
 * (ms[0..4]: embed + norms, q/k/v + o projections, rope + attention, MoE layers,
 * head), accumulated until read; a NULL ms only switches. 0 / -1. */
int aero_cuda_decoder_profile(void* dec, int on, double* ms);

/* out8 = n_layer, n_embd, n_head, n_head_kv, head_dim, vocab, n_seq, n_ctx. 0 / -1. */
int aero_cuda_decoder_info(void* dec, int64_t* out8);

const char* aero_cuda_decoder_last_error(void* dec);
void aero_cuda_decoder_close(void* dec);

#ifdef __cplusplus
}
#endif

#endif /* AERO_CUDA_DECODER_H */
