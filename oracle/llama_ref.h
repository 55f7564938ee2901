/*
 * CPU oracle for the decoder token loop -- TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the Llama-style decoder that the B200 library
 * implements.  It exists to check the CUDA path: only tests/, the smoke() entry in
 * __graft_entry__.py and the cpu_baseline / reference legs of bench.py may load it.
 * The product library never links or calls it.
 *
 * Parity anchors in the reference (gosutek/inference-project):
 *   - token-embedding gather     src/cuda/kernels/input_embeddings.cu:23-34 (out[t,:] = E[id_t,:])
 *   - RMSNorm, fp32 accumulation src/cuda/kernels/rmsnorm.cu:11-59, with the eps the
 *     Llama configs state (the reference omits eps; its defects D1-D6 are not restated)
 *   - weight layout [out x in] row-major, y = W.x   src/model.cuh:44-50, src/cuda/cuda_helpers.cuh:37-55
 *   - bf16 storage with fp32 accumulation            src/cuda/kernels/rmsnorm.cu:17-22
 * RoPE, GQA attention, SwiGLU, the LM head and greedy argmax have no code in the
 * reference; they are defined here from the Llama architecture the configs name.
 */
#ifndef INF_ORACLE_LLAMA_REF_H
#define INF_ORACLE_LLAMA_REF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct OrcConfig {
	uint32_t vocab;
	uint32_t dim;
	uint32_t n_layers;
	uint32_t n_heads;
	uint32_t n_kv_heads;
	uint32_t head_dim;
	uint32_t ffn;
	uint32_t max_seq;
	uint32_t n_slots;   /* independent sequences (KV caches) */
	uint32_t bf16;      /* 1: bf16 storage points emulated, 0: fp32 everywhere */
	float    eps;
	float    rope_theta;
	float    init_std;
	/* Gemma-style decoder (arch 1), the features the reference lists as TODO for Gemma-4
	 * (src/model.cuh:11 global_head_dim, :32-41 per-layer embeddings and the q/k, post-attention,
	 * pre- and post-FFN norms, :51-55 the MLP and the PLE block); none has reference code, so
	 * they are defined here from the published Gemma architecture:
	 *   r = E[id] * bf16(sqrt(dim)); every RMSNorm scales by (1 + w); per head, q and k are
	 *   RMS-normalised (gains [head_dim]) before RoPE; the attention and MLP outputs are
	 *   RMS-normalised before their residual adds; the MLP is gelu_tanh(gate) * up; with
	 *   ple_dim > 0 each layer ends with the per-layer-embedding block; the LM head is the
	 *   embedding; final logits c * tanh(l / c) when final_softcap c > 0. */
	uint32_t arch;          /* 0: Llama, 1: Gemma-style */
	uint32_t ple_dim;       /* per-layer embedding width (Gemma; 0: none) */
	float    final_softcap; /* Gemma; 0: none */
} OrcConfig;

typedef struct OrcModel OrcModel;

/* ---- synthetic data (shared definition with the device generator) ---- */
uint64_t orc_splitmix64(uint64_t x);
void     orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
void     orc_stream_key(uint64_t seed, uint64_t stream, uint32_t key[2]);
float    orc_init_scale(float std);
float    orc_normal_value(uint64_t seed, uint64_t stream, uint64_t idx, float scale);
uint16_t orc_f32_to_bf16(float x);
float    orc_bf16_to_f32(uint16_t h);
/* out is uint16 bf16 (bf16=1) or float (bf16=0) */
void     orc_fill_tensor(uint64_t seed, uint64_t stream, uint64_t n, float std, int bf16, void* out);
uint32_t orc_uniform_u32(uint64_t seed, uint64_t stream, uint64_t idx, uint32_t lo, uint32_t hi_inclusive);
void     orc_gen_ids(uint64_t seed, uint64_t stream, uint64_t n, uint32_t vocab, uint32_t* out);
uint64_t orc_tensor_stream(int32_t layer, uint32_t kind);
/* RoPE table: cos/sin [max_seq][head_dim/2], computed in double, stored as float */
void     orc_rope_table(uint32_t max_seq, uint32_t head_dim, float theta, float* cos_out, float* sin_out);

/* ---- stage oracles used by the kernel-level parity tests ---- */
void orc_embed_gather(const uint32_t* ids, uint64_t n, uint32_t dim, const void* table, int bf16, float* out);
/* y = round(x * (1/sqrt(mean(x^2)+eps)) * g); x fp32 [rows x dim]; g [dim] (bf16 or f32) */
void orc_rmsnorm(const float* x, uint64_t rows, uint32_t dim, const void* g, int bf16, float eps, float* y);
/* y[r] = sum_c W[r,c] x[c]  (W bf16 or f32, x fp32) */
void orc_matvec(const void* W, int bf16, uint64_t rows, uint64_t cols, const float* x, float* y);

/* ---- model ---- */
OrcModel* orc_model_create(const OrcConfig* cfg, uint64_t seed, int n_threads);
void      orc_model_destroy(OrcModel* m);
/* raw weight pointers for tests (uint16 bf16 or float); kind as in orc_tensor_stream */
const void* orc_model_weight(const OrcModel* m, int32_t layer, uint32_t kind);
/* Run n tokens of one slot starting at start_pos (KV written for each).  logits_all
 * [n x vocab] and/or logits_last [vocab] may be NULL.  Returns 0 or a negative error. */
int orc_forward(OrcModel* m, uint32_t slot, const uint32_t* ids, uint32_t n, uint32_t start_pos,
                float* logits_all, float* logits_last, uint32_t* argmax_last);
/* prefill + n_new greedy steps; logits_steps [n_new x vocab] may be NULL.  out_ids[0] is the
 * argmax after the prompt, out_ids[i] the argmax after feeding out_ids[i-1]. */
int orc_generate(OrcModel* m, uint32_t slot, const uint32_t* prompt, uint32_t n_prompt, uint32_t n_new,
                 uint32_t* out_ids, float* logits_steps);
/* Fill KV positions [0, ctx) of a slot with synthetic values (timing samples only). */
int orc_fill_kv_synthetic(OrcModel* m, uint32_t slot, uint32_t ctx, uint64_t seed);
/* per-stage debug output of the last forward (layer 0 only): q,k,v after RoPE, attention out */
int orc_last_layer0(const OrcModel* m, float* q, float* k, float* v, float* attn);
/* layer 0 MLP product h (SwiGLU, or GELU-tanh for Gemma) and the residual after layer 0, of the
 * last token */
int orc_last_layer0_mlp(const OrcModel* m, float* h, float* resid);
/* K and V the cache holds for (slot, layer, pos): [n_kv_heads * head_dim] each */
int orc_kv_read(const OrcModel* m, uint32_t slot, uint32_t layer, uint32_t pos, float* k, float* v);

uint32_t orc_argmax(const float* x, uint64_t n);
/* 1: accumulate projections in float (to measure the drift between two fp32 orders) */
void     orc_set_accum_f32(int on);

/* Sampling as the library defines it (inf_set_sampling, include/inf.h): the fixed-point
 * weights q_i = min(floor(expf((logit_i - max) * inv_temp) * 2^32), 2^32 - 1), and the integer
 * selection from q (top-k, top-p, Philox draw at `counter`).  Sorting, not a radix select. */
void     orc_sample_weights(const float* logits, uint64_t n, float inv_temp, uint32_t* q);
uint32_t orc_sample_select(const uint32_t* q, uint64_t n, float top_p, uint32_t top_k, uint64_t seed, uint64_t counter);

#ifdef __cplusplus
}
#endif
#endif
