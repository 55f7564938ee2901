/*
 * inf.h -- C ABI of the B200 decoder token loop (libinf.so).
 *
 * Drop-in for the entry points of gosutek/inference-project's src/main.cu: the model-load
 * (model_build, src/main.cu:200), the forward (the embed -> RMSNorm prefix in main(),
 * src/main.cu:396-412, completed into a full decoder) and a generate loop (absent in the
 * reference).  Types, arenas and the error enum keep the reference's names and meaning
 * (src/helpers.h:17-41, src/allocator.h:13-38, src/cuda/api/cuda_allocator.cuh:11-26,
 * src/cuda/api/cuda_mem_wrapper.cuh:10-16).  Unlike the reference, no function aborts:
 * every failure is returned as an Error_t and described by inf_last_error_detail().
 *
 * Plain pointers and sizes only; no torch or CUDA types appear in the signatures
 * (streams are passed as void*).  One context per GPU; calls on one model are not
 * re-entrant.
 */
#ifndef INF_H
#define INF_H

#include <stddef.h>
#include <stdint.h>

#if defined(__cplusplus)
extern "C" {
#endif

/* src/helpers.h:17-28 */
typedef uint8_t  u8;
typedef uint16_t u16;
typedef uint32_t u32;
typedef uint64_t u64;
typedef int8_t   i8;
typedef int16_t  i16;
typedef int32_t  i32;
typedef int64_t  i64;
typedef float    f32;
typedef double   f64;
typedef i32      b32;

/* src/helpers.h:30-41; values 0-7 keep the reference's numbering. */
typedef enum Error_t {
	Success                 = 0,
	ErrorMemoryAllocation   = 1,
	ErrorArenaOutOfMemory   = 2,
	ErrorAlreadyInitialized = 3,
	ErrorInvalidValue       = 4,
	ErrorInvalidHostPtr     = 5,
	ErrorInvalidDevPtr      = 6,
	ErrorGeneric            = 7,
	ErrorCuda               = 8,  /* a CUDA runtime call failed; see inf_last_error_detail() */
	ErrorBadConfig          = 9,  /* InfConfig violates a shape rule */
	ErrorTokenOutOfRange    = 10, /* an id >= vocab_size reached a kernel */
	ErrorKvOutOfRange       = 11, /* a position or KV page outside the cache */
	ErrorNccl               = 12,
	ErrorTimeout            = 13, /* a bounded device wait expired */
	ErrorIo                 = 14,
	ErrorUnsupported        = 15,
} Error_t;

typedef enum InfDtype {
	InfF32  = 0,
	InfBF16 = 1,
} InfDtype;

/* src/model.cuh:7-15 (Config), extended with the fields a Llama decoder needs. */
typedef struct InfConfig {
	u32 vocab_size;
	u32 dim;
	u32 n_layers;
	u32 n_heads;
	u32 n_kv_heads;
	u32 head_dim;
	u32 ffn_dim;
	u32 max_seq;        /* positions per sequence */
	u32 max_batch;      /* sequences decoded together (KV slots) */
	u32 kv_block;       /* tokens per KV page; 16 */
	u32 kv_pages;       /* 0: max_batch * ceil(max_seq / kv_block) */
	u32 prefill_chunk;  /* tokens per prefill pass; 0: min(max_seq, 4096) */
	u32 dtype;          /* InfDtype of weights, KV cache and activations between kernels */
	f32 norm_eps;
	f32 rope_theta;
	f32 init_std;       /* std of the synthetic weights */
	u32 tp_rank;
	u32 tp_size;
	u32 prefill_attention; /* InfPrefillAttention */
	u32 arch;           /* InfArch */
	u32 ple_dim;        /* Gemma: per-layer embedding width (0: none) */
	f32 final_softcap;  /* Gemma: logits = c * tanh(logit / c) when c > 0 */
} InfConfig;

/* The decoder family.  Gemma-style models are the features the reference lists as TODO for its
 * Gemma-4 target (src/model.cuh:11 global_head_dim, :32-41 per-layer embeddings and the q/k,
 * post-attention, pre- and post-FFN norms, :51-55 the MLP and the PLE block); the reference has
 * no code for them, so they follow the published Gemma architecture:
 *   r = E[id] * bf16(sqrt(dim)); every RMSNorm scales by (1 + w) (gains of Gemma models are
 *   drawn like the weights, not 1.0); per head, q and k are RMS-normalised over head_dim
 *   (gains [head_dim]) before RoPE; the attention output and the MLP output are RMS-normalised
 *   before their residual adds; the MLP is gelu_tanh(gate) * up; with ple_dim > 0 a per-layer
 *   input ple_l = bf16((E_ple[id, l] * bf16(sqrt(ple_dim)) + rmsnorm(W_pmp . bf16(E[id] * s) *
 *   bf16(dim^-1/2))) * bf16(2^-1/2)) is formed per token and each layer ends with
 *   r += rmsnorm(W_pp . bf16(gelu_tanh(W_pg . bf16(r)) * ple_l)); the LM head is the embedding;
 *   logits are soft-capped when final_softcap > 0.  Head dims up to 512 (GQA groups up to 4),
 *   bf16, one GPU, greedy or sampled batch-1 decode (inf_forward, inf_generate, inf_decode;
 *   prompts are fed through the decode step token by token); inf_forward_batch and the server
 *   answer ErrorUnsupported.  Sliding-window layers and Gemma-3n's AltUp/Laurel blocks are not
 *   implemented. */
typedef enum InfArch {
	InfArchLlama = 0,
	InfArchGemma = 1,
} InfArch;

/* Which kernel computes causal attention in prefill passes. */
typedef enum InfPrefillAttention {
	InfPrefillAttnAuto = 0, /* tensor cores (tcgen05/TMEM) for bf16 with head_dim 64 or 128, else SIMT */
	InfPrefillAttnSimt = 1, /* the fp32 SIMT kernel (P kept in fp32) */
} InfPrefillAttention;

/* src/allocator.h:13-25 */
typedef struct HostArena {
	u64 reserve_size;
	u64 commit_size;
	u64 commit_pos;
	u64 pos;
} HostArena;

/* src/cuda/api/cuda_allocator.cuh:11-17.  Pushes are 256-byte aligned (the reference
 * aligns to 8, which is too little for 16-byte vector loads and TMA). */
typedef struct DevArena {
	u8* _d_ptr;
	u64 size;
	u64 pos;
} DevArena;

typedef struct ExecCtx {
	HostArena host_arena;
	DevArena  dev_arena;
} ExecCtx;

typedef struct InfEngine InfEngine;

/* src/model.cuh:62-74 (Model): config, the device weight slab and the engine state. */
typedef struct Model {
	InfConfig  config;
	void*      data;        /* device weight slab */
	u64        model_bsize; /* bytes of weights */
	InfEngine* engine;
} Model;

typedef struct InfStats {
	f64 prefill_ms;
	f64 decode_ms;
	u32 n_prompt;
	u32 n_new;
	u64 kernel_launches;
} InfStats;

/* ---- execution context and arenas ------------------------------------------------ */
/* src/allocator.h:34-35 */
Error_t exec_ctx_create(ExecCtx** ctx);
Error_t exec_ctx_destroy(ExecCtx** ctx);
/* src/allocator.h:36-41 */
Error_t arena_host_create(HostArena** const arena, const u64 reserve_size, const u64 commit_size);
Error_t arena_host_destroy(HostArena* arena);
Error_t arena_host_push(HostArena* const arena, const u64 req_size, void** ptr_out);
void    arena_host_pop(HostArena* const arena, u64 size);
void    arena_host_pop_at(HostArena* const arena, u64 pos);
u64     mem_arena_host_pos_get(const HostArena* const arena);
/* src/cuda/api/cuda_allocator.cuh:19-26 */
Error_t arena_dev_create(DevArena* const arena, const u64 bsize);
Error_t arena_dev_destroy(DevArena* arena);
Error_t arena_dev_push(DevArena* const arena, const u64 bsize, void** ptr_out);
void    arena_dev_pop(DevArena* const arena, u64 bsize);
void    arena_dev_pop_at(DevArena* const arena, u64 pos);
u64     arena_dev_pos_get(const DevArena* const arena);

/* ---- CUDA memory wrappers: src/cuda/api/cuda_mem_wrapper.cuh:10-16 -------------------
 * Same names and return types as the reference: the b32 functions return 1 on success and 0
 * on failure, the Error_t ones Success or a code; none aborts (the reference's CHECK_CUDA does),
 * and inf_last_error_detail() describes every failure.  `stream` is a cudaStream_t passed as
 * void* (the same pointer at the C ABI). */
/* cuda_mem_wrapper.cuh:10.  Takes the address of the caller's pointer, which receives the
 * allocation (the reference takes the pointer by value, so its allocation is lost: defect D10;
 * a reference caller passing &ptr gets the fixed behaviour). */
b32     cu_malloc(void** dev_ptr, const u64 bsize);
/* cuda_mem_wrapper.cuh:11.  0 if dev_ptr is not device memory. */
b32     cu_free(void* dev_ptr);
/* cuda_mem_wrapper.cuh:12.  ErrorInvalidDevPtr if dst is not device memory. */
Error_t cu_memcpy_htd(void* dst, const void* src, const u64 bsize);
/* cuda_mem_wrapper.cuh:13.  0 if dst is not device memory. */
b32     cu_memcpy_htd_async(void* dst, const void* src, const u64 bsize, void* stream);
/* cuda_mem_wrapper.cuh:14.  ErrorInvalidHostPtr if src is not device memory (the reference's code). */
Error_t cu_memcpy_dth(void* dst, const void* src, const u64 bsize);
/* cuda_mem_wrapper.cuh:15.  Page-locks host memory for reading by the device (cudaHostRegister
 * with cudaHostRegisterReadOnly); 0 for a device pointer. */
b32     cu_host_register_read_only(void* ptr, const u64 bsize);
/* cuda_mem_wrapper.cuh:16.  0 if s is not device memory. */
b32     cu_memset(void* s, i32 c, u64 n);

/* ---- stand-alone kernels ----------------------------------------------------------- */
/* Replaces k_fetch_input_embeddings (src/cuda/kernels/input_embeddings.cuh:20-24) and its
 * launch (src/main.cu:396-404): out[t,:] = table[ids[t],:] for any dim, bit-exact.  Ids
 * >= vocab_size produce ErrorTokenOutOfRange (and zero rows) instead of reading out of
 * bounds.  dtype: InfDtype of table and out.  Device pointers; synchronous. */
Error_t inf_fetch_input_embeddings(const u32* d_ids, u64 n_tokens, u32 dim, u32 vocab_size, const void* d_table,
                                   void* d_out, u32 dtype, void* stream);
/* Replaces k_rmsnorm (src/cuda/kernels/rmsnorm.cuh:15-18, launch src/main.cu:409):
 * y[t,i] = x[t,i] * g[i] / sqrt(mean_i(x[t,i]^2) + eps), fp32 accumulation, one gain
 * vector for every row, any dim, y may equal x.  Device pointers; synchronous. */
Error_t inf_rmsnorm(const void* d_x, void* d_y, u32 rows, u32 dim, const void* d_gain, f32 eps, u32 dtype,
                    void* stream);

/* The prefill projection on the tensor cores (tcgen05, TMA): Y[T x N] = X[T x K] . W[N x K]^T,
 * bf16 inputs (row-major, 16-byte aligned, K % 8 == 0), fp32 accumulation, Y bf16 (RNE) or
 * f32 (out_f32 != 0).  Device pointers; synchronous.  The reference has no projection
 * (src/model.cuh:44-50 declares wq/wk/wv/wo only). */
Error_t inf_gemm_bf16(const void* d_x, const void* d_w, void* d_y, u32 T, u32 N, u32 K, u32 out_f32, void* stream);

/* Decode attention over a paged KV cache for n_tokens query tokens (one per sequence), with
 * the kernel the model's decode step runs for that shape (no reference counterpart:
 * src/model.cuh:44-50 stops at the projection weights).  q, out: [n_tokens][n_heads*head_dim];
 * kpool, vpool: [n_pages][n_kv_heads][kv_block][head_dim]; block_table: [slots][pages_per_seq]
 * i32; tok_slot, tok_pos: [n_tokens] i32 -- token i attends positions 0..tok_pos[i] of its
 * slot.  dtype: InfDtype of q, K/V and out.  d_scratch: device memory of at least
 * inf_attn_decode_scratch_bytes(...) bytes (split partials, tickets, error word; enough for
 * every kernel of InfAttnKernel), 16-byte aligned; its contents on entry do not matter.
 * Synchronous. */
u64     inf_attn_decode_scratch_bytes(u32 n_tokens, u32 n_heads, u32 n_kv_heads, u32 head_dim, u32 kv_block,
                                      u32 pages_per_seq, u32 dtype);
Error_t inf_attn_decode(const void* d_q, const void* d_kpool, const void* d_vpool, const i32* d_block_table,
                        u32 pages_per_seq, u32 n_pages, const i32* d_tok_slot, const i32* d_tok_pos, u32 n_tokens,
                        u32 n_heads, u32 n_kv_heads, u32 head_dim, u32 kv_block, u32 dtype, void* d_out,
                        void* d_scratch, u64 scratch_bytes, void* stream);

/* The decode attention kernels.  A kernel's split plan depends on pages_per_seq (the longest
 * context a sequence may reach) exactly as in the model, whose pages_per_seq is
 * ceil(max_seq / kv_block). */
typedef enum InfAttnKernel {
	InfAttnAuto    = 0, /* what the decode step picks for one token: InfAttnClusterTc when it applies
	                       and fits, else InfAttnCluster when it fits; for several tokens InfAttnMma
	                       where it applies; else InfAttnSplitK */
	InfAttnSplitK  = 1, /* CTAs per (token, KV head, split), partials combined through the scratch by
	                       the last CTA of each (token, KV head) */
	InfAttnCluster = 2, /* one thread-block cluster of 8 or 16 CTAs per (token, KV head), the split
	                       combine in distributed shared memory; pages_per_seq up to 16 per CTA */
	InfAttnMma     = 3, /* the batched step's tensor-core kernel (mma.m16n8k16, TMA page loads): bf16,
	                       kv_block 16, head_dim 64 or 128 */
	InfAttnClusterTc = 4, /* the cluster split of InfAttnCluster on the tensor cores (mma.m16n8k16, TMA
	                       page loads, the combine pushed into each output's owner CTA): bf16,
	                       kv_block 16, head_dim 64 or 128, GQA group <= 8, up to 16 pages per CTA */
} InfAttnKernel;
/* inf_attn_decode with the kernel chosen by the caller (InfAttnKernel); ErrorUnsupported when
 * that kernel cannot serve the shape.  For tests and measurements of one kernel. */
Error_t inf_attn_decode_with(u32 kernel, const void* d_q, const void* d_kpool, const void* d_vpool,
                             const i32* d_block_table, u32 pages_per_seq, u32 n_pages, const i32* d_tok_slot,
                             const i32* d_tok_pos, u32 n_tokens, u32 n_heads, u32 n_kv_heads, u32 head_dim, u32 kv_block,
                             u32 dtype, void* d_out, void* d_scratch, u64 scratch_bytes, void* stream);
/* Causal attention of one prefill pass, the kernel the model's prefill runs (no reference
 * counterpart): n_tokens consecutive tokens of one sequence, token t at position tok_pos[t]
 * attending positions 0..tok_pos[t] of slot tok_slot[t], whose K/V (this pass's tokens
 * included) are already in the cache.  bf16 only; q, out: [n_tokens][n_heads*head_dim], the
 * other arguments as for inf_attn_decode.  kernel: InfPrefillAttention (Auto: the tcgen05/TMEM
 * kernel for head_dim 64 or 128, GQA groups dividing 128 and kv_block a multiple of 8 dividing
 * 128; else the SIMT kernel).  Synchronous. */
Error_t inf_attn_prefill(u32 kernel, const void* d_q, const void* d_kpool, const void* d_vpool,
                         const i32* d_block_table, u32 pages_per_seq, u32 n_pages, const i32* d_tok_slot,
                         const i32* d_tok_pos, u32 n_tokens, u32 n_heads, u32 n_kv_heads, u32 head_dim, u32 kv_block,
                         void* d_out, void* stream);
/* inf_attn_decode for callers that cannot allocate device memory -- a serving loop that must
 * not call cudaMalloc/cudaFree mid-step (they synchronize the device), or a runtime whose device
 * memory is all committed to a pre-sized arena.  No counterpart in the reference.  The scratch is
 * a 4 MiB array built into the library (held on every GPU that loads it until the process
 * exits); shapes needing more return ErrorInvalidValue, shapes the attention cannot serve the
 * error inf_attn_decode gives for them.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress) and keeps it; make that first call before any stream
 * capture, and do not use the library on a device after cudaDeviceReset.  The call waits for its
 * stream before returning (it reads the kernel's error word).  All calls share the array, so calls
 * issued from other host threads, or on other streams, must not run at the same time as this
 * one: the caller orders them.  Allocates nothing. */
Error_t inf_attn_decode_noalloc(const void* d_q, const void* d_kpool, const void* d_vpool, const i32* d_block_table,
                                u32 pages_per_seq, u32 n_pages, const i32* d_tok_slot, const i32* d_tok_pos,
                                u32 n_tokens, u32 n_heads, u32 n_kv_heads, u32 head_dim, u32 kv_block, u32 dtype,
                                void* d_out, void* stream);

/* ---- model ------------------------------------------------------------------------- */
/* Built-in shapes: 1 tiny fp32 (d288), 2 TinyLlama-1.1B, 3 Llama-3-8B, 4 Llama-3-8B batch 64,
 * 5 Llama-3-8B 32k prefill, 6 the Gemma-4-E2B shape the reference's comments give
 * (src/model.cuh:9-14: dim 1536, ffn 6144, global_head_dim 512, 8 heads, vocab 262144, 35
 * layers) with 2 KV heads, per-layer embeddings of 256, RoPE theta 1e6, eps 1e-6, soft-cap 30. */
Error_t inf_config_preset(u32 preset, InfConfig* out);
/* model_build (src/main.cu:200-352).  weights_path NULL: synthetic weights N(0, init_std)
 * from `seed` (Philox4x32-10), gains 1.0.  Otherwise a safetensors checkpoint (one file, a
 * *.safetensors.index.json of shards, or a directory holding model.safetensors.index.json or
 * model.safetensors), checked as inf_safetensors_check does before any device memory is
 * taken, then copied to the device through pinned staging buffers; seed is unused.
 * Creates *ctx if it is NULL. */
Error_t inf_model_build(ExecCtx** ctx, Model* model, const InfConfig* config, const char* weights_path, u64 seed);
/* model_destroy (src/main.cu:354-358) */
Error_t inf_model_destroy(ExecCtx** ctx, Model* model);

/* Forward n_tokens of one sequence starting at start_pos (KV written for each).  ids,
 * logits_out (vocab_size f32 of the last token, may be NULL) and argmax_out (may be NULL)
 * may be host or device pointers. */
Error_t inf_forward(Model* model, const u32* ids, u32 n_tokens, u32 start_pos, u32 seq_slot, f32* logits_out,
                    u32* argmax_out);
/* One decode token for each of n_seqs sequences: token ids[i] at position positions[i]
 * of slot seq_slots[i].  logits_out [n_seqs x vocab_size] may be NULL. */
Error_t inf_forward_batch(Model* model, u32 n_seqs, const u32* seq_slots, const u32* ids, const u32* positions,
                          f32* logits_out, u32* argmax_out);
/* Prefill the prompt into slot 0, then n_new greedy steps; out_ids[i] is the i-th
 * generated id.  Host pointers. */
Error_t inf_generate(Model* model, const u32* prompt, u32 n_prompt, u32 n_new, u32* out_ids, InfStats* stats);
/* Continue a sequence: feed first_id at start_pos, then n_steps - 1 more greedy steps, all
 * chained on the device (one CUDA graph replay per token, no host round trip).  out_ids
 * (host or device, may be NULL) receives the n_steps generated ids. */
Error_t inf_decode(Model* model, u32 seq_slot, u32 start_pos, u32 first_id, u32 n_steps, u32* out_ids,
                   InfStats* stats);
/* ---- tensor parallelism (one process and one model per GPU, tp_rank/tp_size in the config)
 * Column-parallel QKV (KV heads per rank) and gate/up, row-parallel O and down, vocabulary-
 * parallel LM head.  The two all-reduces of each layer and the cross-shard argmax run inside
 * the projection kernels over NVLink peer memory.  Setup: every rank calls inf_tp_export,
 * the caller gathers the tp_size handles (any host transport, e.g. torch.distributed), and
 * every rank calls inf_tp_connect with all handles in rank order.  All ranks must then run
 * the same sequence of calls.  With tp_size > 1, logits_out receives this rank's vocabulary
 * shard (vocab_size / tp_size floats) and argmax_out the global greedy id. */
Error_t inf_tp_export(Model* model, void* handle_out, u64 handle_bytes); /* 64-byte CUDA IPC handle */
Error_t inf_tp_connect(Model* model, const void* handles, u32 n_ranks);
/* Release the KV pages of a sequence slot. */
Error_t inf_seq_reset(Model* model, u32 seq_slot);

/* ---- sampling ----------------------------------------------------------------------- */
typedef struct InfSampling {
	f32 temperature; /* 0: greedy argmax (the default) */
	f32 top_p;       /* (0, 1]; 1 keeps every token */
	u32 top_k;       /* 0 keeps every token */
	u32 reserved;
	u64 seed;
} InfSampling;
/* Temperature / top-k / top-p sampling for every token the model chooses from then on
 * (inf_generate, inf_decode, and the id inf_forward reports; per-slot settings for the batched
 * step are inf_set_slot_sampling's).  With m the largest logit, each
 * token weighs q = min(floor(expf((logit - m) / temperature) * 2^32), 2^32 - 1); top-k keeps the
 * tokens at or above the k-th largest q, top-p then the fewest of those (ties kept) whose q sum to
 * at least ceil(top_p * their total); the token is the first, in id order, whose running sum of
 * kept q exceeds floor(r * total / 2^64), r the 64-bit Philox4x32-10 draw keyed by
 * SplitMix64(SplitMix64(seed) ^ 0x3000000) at counter (position, slot << 32).  Deterministic
 * for a seed.  Batch-1 decode on one GPU only (ErrorUnsupported under tensor parallelism). */
Error_t inf_set_sampling(Model* model, const InfSampling* sampling);
/* Sampling settings of one sequence slot for the tokens inf_forward_batch (and the server)
 * chooses for it: the rule above with the counter (position of the new token, 0), so a sequence
 * draws exactly what the batch-1 decode of slot 0 with the same seed would from the same logits,
 * whichever slot it runs in.  One sampler CTA per
 * sampled row follows the batched LM head; rows of greedy slots keep their argmax.  Temperature
 * 0 (the default of every slot) is greedy.  The settings stay with the slot until changed.
 * One GPU only; vocab_size a multiple of 4.  No counterpart in the reference (it has no
 * decoder); a serving loop sets it per request. */
Error_t inf_set_slot_sampling(Model* model, u32 seq_slot, const InfSampling* sampling);

/* ---- continuous batching ------------------------------------------------------------ */
typedef struct InfServer InfServer;
/* A request queue in front of the model's max_batch sequence slots (at most max_active of them
 * in use, 0: all).  Each inf_server_step admits waiting requests first come first served into
 * free slots (pages released, prompt prefilled with inf_forward, its greedy next token the
 * first output), advances every sequence admitted in an earlier step by one token with one
 * batched decode step (the tensor-core batch path even for a lone sequence, so a request's ids
 * do not depend on the load), and retires sequences that produced eos_id, reached max_new tokens or
 * ran out of positions, releasing their pages.  A request is admitted only when the KV pool can
 * hold every position it may write (prompt + max_new - 1, at most max_seq) on top of what the
 * running requests reserved; until then it waits at the head of the queue.  Greedy unless a
 * request asks for sampling (inf_server_submit_sampled): its slot then carries its settings
 * (inf_set_slot_sampling) for its first token and every batched step, so its ids are what it would
 * draw alone; the model-wide inf_set_sampling must be off (ErrorUnsupported at admission).  A
 * request whose prefill fails is retired
 * with that error and the others go on; a failing batched step retires the requests of its batch
 * with its error and returns it.  Not thread-safe. */
Error_t inf_server_create(Model* model, u32 max_active, InfServer** out);
/* The same scheduler over a host-only stand-in model (next id = a hash of the sequence's
 * previous id and position) that checks every sequence is fed its own positions in order and
 * holds kv_pages pages of 16 positions (0: enough for every slot's max_seq), failing with
 * ErrorArenaOutOfMemory like the device cache when they run out: for testing the scheduling
 * without a GPU.  A prompt that starts with id vocab - 1 makes the first batched step its
 * sequence joins fail with ErrorGeneric. */
Error_t inf_server_create_synthetic(u32 n_slots, u32 max_seq, u32 vocab, u32 kv_pages, u32 max_active,
                                    InfServer** out);
Error_t inf_server_destroy(InfServer** server);
/* Queue a request; n_prompt < max_seq.  eos_id 0xFFFFFFFF: none.  ErrorArenaOutOfMemory if its
 * positions need more KV pages than the whole pool holds. */
Error_t inf_server_submit(InfServer* server, const u32* prompt, u32 n_prompt, u32 max_new, u32 eos_id,
                          u64* request_id);
/* inf_server_submit with the request's own sampling settings (NULL or temperature 0: greedy). */
Error_t inf_server_submit_sampled(InfServer* server, const u32* prompt, u32 n_prompt, u32 max_new, u32 eos_id,
                                  const InfSampling* sampling, u64* request_id);
/* One scheduling step; *n_finished (may be NULL) = requests retired in it. */
Error_t inf_server_step(InfServer* server, u32* n_finished);
/* The ids a request has produced so far (out_ids NULL: count only), *done = 1 once retired,
 * *status = the error that retired it (Success if none).  done and status may be NULL. */
Error_t inf_server_result(InfServer* server, u64 request_id, u32* out_ids, u32 cap, u32* n_out, u32* done,
                          Error_t* status);
/* Forget a retired request. */
Error_t inf_server_release(InfServer* server, u64 request_id);
Error_t inf_server_stats(const InfServer* server, u32* n_waiting, u32* n_active, u64* batched_steps,
                         u64* batched_tokens);

/* ---- checkpoints ------------------------------------------------------------------ */
/* model_parse_config (src/main.cu:120-157): reads a Hugging Face config.json -- its
 * "text_config" object when there is one (as the reference does), else the top level -- into
 * *inout: hidden_size, intermediate_size, num_hidden_layers, num_attention_heads,
 * num_key_value_heads (default num_attention_heads), head_dim (default hidden_size /
 * num_attention_heads), vocab_size, rms_norm_eps, rope_theta and torch_dtype ("bfloat16" or
 * "float32").  A field the file lacks keeps its value; max_seq, max_batch, the KV paging and the
 * tensor-parallel fields are never taken from the file.  ErrorIo if the file cannot be read,
 * ErrorInvalidValue for malformed JSON or a field of the wrong type or range, ErrorUnsupported
 * for what this decoder does not compute (a model_type other than "llama", an activation other
 * than SiLU, attention or MLP biases, RoPE scaling). */
Error_t inf_config_from_json(const char* config_path, InfConfig* inout);

/* The checkpoint checks of model_build without a GPU.  Every tensor the decoder of `config`
 * needs must be present under its Hugging Face Llama name, "model." or
 * "model.language_model." + embed_tokens.weight, norm.weight and
 * layers.<i>.{input_layernorm, post_attention_layernorm}.weight,
 * layers.<i>.self_attn.{q,k,v,o}_proj.weight, layers.<i>.mlp.{gate,up,down}_proj.weight, plus
 * lm_head.weight (absent: the embedding is the LM head), in dtype BF16 or F32 (converted to
 * config->dtype, bf16 by round-to-nearest-even) and with the shape config implies.  The file
 * itself must follow the safetensors format: an 8-byte little-endian header length, a JSON
 * header of at most 100,000,000 bytes, offsets relative to the byte buffer after the header
 * (the reference adds them to the file start, defect D7), sizes equal to shape x dtype size,
 * and a buffer indexed without holes or overlaps.
 * ErrorIo: a file cannot be opened or mapped.  ErrorInvalidValue: malformed header, offsets or
 * index, or a missing tensor.  ErrorBadConfig: a shape that does not match config.
 * ErrorUnsupported: a needed tensor in another dtype, or a tensor under the decoder's prefix
 * that this decoder does not use (q/k norms, extra norms, biases, per-layer embeddings: the
 * checkpoint is another model family).  Gemma-style configs (arch InfArchGemma) need, beside the
 * projections and input_layernorm: layers.<i>.self_attn.{q_norm, k_norm}, post_attention_layernorm
 * (the norm of the attention output), pre_feedforward_layernorm, post_feedforward_layernorm and,
 * with ple_dim > 0, per_layer_input_gate, per_layer_projection, post_per_layer_input_norm, plus
 * embed_tokens_per_layer, per_layer_model_projection and per_layer_projection_norm; their LM head
 * is the embedding (a separate lm_head.weight is refused). */
Error_t inf_safetensors_check(const char* weights_path, const InfConfig* config);

/* Weights of the decoder, by their place in the device layout. */
typedef enum InfWeightKind {
	InfWEmbed     = 0,  /* [vocab_size x dim] */
	InfWLmHead    = 1,  /* [vocab_size / tp x dim], rank's vocabulary rows */
	InfWFinalNorm = 2,  /* [1 x dim] */
	InfWQkv       = 8,  /* [(H + 2 KV) / tp * head_dim x dim]: q, k, v heads, rows (i, i + head_dim/2) paired */
	InfWO         = 11, /* [dim x H / tp * head_dim], rank's columns */
	InfWGateUp    = 12, /* [2 ffn_dim / tp x dim], rows gate_0, up_0, gate_1, ... */
	InfWDown      = 14, /* [dim x ffn_dim / tp], rank's columns */
	InfWAttnNorm  = 15, /* [1 x dim] */
	InfWFfnNorm   = 16, /* [1 x dim]; Gemma: pre_feedforward_layernorm */
	/* Gemma-style models (InfArchGemma) */
	InfWEmbedPle     = 3,  /* [vocab_size x n_layers * ple_dim]  embed_tokens_per_layer */
	InfWPleModelProj = 4,  /* [n_layers * ple_dim x dim]         per_layer_model_projection */
	InfWPleProjNorm  = 5,  /* [1 x ple_dim]                      per_layer_projection_norm */
	InfWQNorm        = 17, /* [1 x head_dim]                     self_attn.q_norm */
	InfWKNorm        = 18, /* [1 x head_dim]                     self_attn.k_norm */
	InfWPostAttnNorm = 19, /* [1 x dim]                          post_attention_layernorm */
	InfWPostFfnNorm  = 20, /* [1 x dim]                          post_feedforward_layernorm */
	InfWPleGate      = 21, /* [ple_dim x dim]                    per_layer_input_gate */
	InfWPleProj      = 22, /* [dim x ple_dim]                    per_layer_projection */
	InfWPlePostNorm  = 23, /* [1 x dim]                          post_per_layer_input_norm */
} InfWeightKind;
/* One weight of `layer` (ignored for embed, LM head and final norm) as inf_model_build writes
 * it to rank config->tp_rank's device memory, read from the checkpoint into host memory `out`
 * (out_bytes at least rows x cols x the dtype's size).  Host only, no device work. */
Error_t inf_safetensors_read(const char* weights_path, const InfConfig* config, u32 layer, u32 kind, void* out,
                             u64 out_bytes);

/* ---- tokenizer (src/tokenizer.h:13-38) ------------------------------------------- */
typedef struct InfTokenizer InfTokenizer;
/* tokenizer_build (src/tokenizer.c:186-262): the BPE model of a Hugging Face tokenizer.json,
 * "model": {"vocab": {piece: id}, "merges": [[left, right], ...] or ["left right", ...],
 * "byte_fallback", "unk_token"}; a merge's rank is its position in the list.  "added_tokens"
 * are decoded too.  ErrorIo if the file cannot be read; ErrorInvalidValue if it is malformed;
 * ErrorUnsupported for another model type or a byte-level BPE (GPT-2 / Llama-3 style, whose
 * regex pre-tokenizer this segmentation does not implement). */
Error_t inf_tokenizer_build(const char* tokenizer_json_path, InfTokenizer** out);
/* tokenizer_destroy (src/tokenizer.c:264-278) */
Error_t inf_tokenizer_destroy(InfTokenizer** tok);
/* One past the largest id that has a piece. */
u32     inf_tokenizer_vocab_size(const InfTokenizer* tok);
/* tokenizer_encode (src/tokenizer.c:39-183), the reference's segmentation: words split at
 * ' ' (two spaces make an empty word, a trailing space ends the text), every word after the
 * first prefixed with U+2581, characters by the reference's UTF-8 lead-byte rule (clamped to
 * the word), then per round the pair of lowest merge rank merged at all its non-overlapping
 * occurrences, left to right, until no adjacent pair has a rank.  A final piece outside the
 * vocabulary becomes its bytes as <0xXX> tokens (byte_fallback), else the unk token, else
 * ErrorInvalidValue (the reference drops it and still counts it, defect D13).  A text that
 * starts with a space starts with an empty word that yields nothing (the reference reads out
 * of bounds there).  *n_ids is the number of ids; ids NULL counts only; more than max_ids:
 * ErrorInvalidValue. */
Error_t inf_tokenizer_encode(const InfTokenizer* tok, const char* text, u32* ids, u64 max_ids, u64* n_ids);
/* inf_tokenizer_encode after cutting out the added tokens marked "special" (longest match at
 * the earliest position, e.g. "<start_of_turn>"): each special becomes its id and every piece of
 * text between them is encoded as a whole text (its first word without U+2581).  The
 * reference has no special tokens; this is for chat templates. */
Error_t inf_tokenizer_encode_special(const InfTokenizer* tok, const char* text, u32* ids, u64 max_ids, u64* n_ids);
/* tokenizer_decode (declared at src/tokenizer.h:38, never defined by the reference): the
 * pieces of ids concatenated, U+2581 -> ' ', <0xXX> -> that byte (byte_fallback models).
 * Writes a NUL-terminated string of *out_len bytes; out NULL gives the length only; out_bytes
 * below *out_len + 1: ErrorInvalidValue; an id without a piece: ErrorTokenOutOfRange. */
Error_t inf_tokenizer_decode(const InfTokenizer* tok, const u32* ids, u64 n_ids, char* out, u64 out_bytes,
                             u64* out_len);

/* Synthetic inputs: n integers uniform in [lo, hi_inclusive] from Philox4x32-10 keyed by
 * SplitMix64(SplitMix64(seed) ^ stream), counter i, Lemire multiply-shift.  Prompt ids use
 * stream 0x1000000 + sequence, context lengths 0x2000000.  Host memory, no device work. */
Error_t inf_synth_ids(u64 seed, u64 stream, u64 n, u32 lo, u32 hi_inclusive, u32* out);

/* ---- introspection ------------------------------------------------------------------ */
typedef enum InfBuffer {
	InfBufResid  = 0, /* residual stream of the last decode token, f32 [dim] */
	InfBufQ      = 1, /* query of the last decode token, last layer [n_heads * head_dim] */
	InfBufAttn   = 2, /* attention output, last layer [n_heads * head_dim] */
	InfBufH      = 3, /* SwiGLU product, last layer [ffn_dim] */
	InfBufLogits = 4, /* logits of the last token [vocab_size] */
	InfBufK      = 5, /* K the cache holds for (layer, slot, pos) [n_kv_heads * head_dim] */
	InfBufV      = 6, /* V the cache holds for (layer, slot, pos) */
	InfBufSampleQ = 7, /* the sampler's fixed-point weights of the last step [vocab_size], raw u32 bits */
	InfBufSampleQRow = 8, /* the per-slot sampler's weights of row `pos` of the last sampled rows
	                        (the batched step's row order; 0 after a single forward) [vocab_size], raw u32 bits */
} InfBuffer;
/* Copy one engine buffer to host floats (bf16 widened).  For test and debugging; the
 * reference's equivalent is print_dev_buf_bf16 (src/main.cu:44-61). */
Error_t     inf_debug_read(Model* model, u32 buffer, u32 layer, u32 seq_slot, u32 pos, f32* out, u64 n_out);
const char* inf_error_string(Error_t err);
const char* inf_last_error_detail(void);
void*       inf_model_stream(Model* model);
u64         inf_kernel_launches(Model* model);
/* Bytes inf_forward_batch has copied host -> device so far (ids, positions, slots and the
 * attention work list of each step); the ids it returns are the device -> host side. */
u64         inf_batch_h2d_bytes(Model* model);
/* Bytes the decode step of one token streams from HBM: weights + KV read for ctx. */
u64         inf_decode_bytes(const InfConfig* config, u32 ctx);
/* Time each kernel kind of one eager (non-graph) decode step of token `id` at `pos` of
 * the slot, with CUDA events around every launch on the model's stream: ms_out[k] for k in
 * InfKernelKind.  Returns the number of kinds (0 on error). */
u32         inf_profile_decode_step(Model* model, u32 seq_slot, u32 pos, u32 id, f32* ms_out, u32 max_kinds);

typedef enum InfKernelKind {
	InfKEmbed = 0,
	InfKQkv   = 1,
	InfKAttn  = 2,
	InfKO     = 3,
	InfKGateUp = 4,
	InfKDown  = 5,
	InfKLmHead = 6,
	InfKNumKinds = 7,
} InfKernelKind;

#if defined(__cplusplus)
}
#endif

#endif /* INF_H */
