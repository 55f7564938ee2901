// The kernels only the Gemma-style decoder runs (InfConfig.arch = InfArchGemma): the features
// the reference lists as TODO for Gemma-4 (src/model.cuh:32-41 per-layer embeddings and the q/k
// norms, :51-55 the MLP and PLE block).  The projections themselves are the k_gemv kernels with
// the Gemma prologue and epilogues (k_gemv.cuh).
//
//   k_gemma_embed   r = E[id] * bf16(sqrt(dim)) (fp32 residual) and, for the per-layer-input
//                   projection, its bf16 rounding
//   k_ple_combine   per layer l: ple_l = bf16((E_ple[id, l] * s_ple + rms1p(pm_l * s_proj)) * s_sum),
//                   pm = W_pmp . bf16(r) from the projection GEMV; one CTA per layer
//   k_qk_norm_rope  per head: RMSNorm of the raw q or k row over head_dim with (1 + w) gains,
//                   RoPE on (i, i + head_dim/2) pairs, bf16 q out or K into the paged cache; v
//                   heads go to the cache unchanged.  One CTA per head, a thread per pair.
// rms1p(x) = (x * rsqrt(mean(x^2) + eps)) * (1 + w), fp32 products in that order.
#pragma once

#include "common.cuh"

namespace inf {

struct GemmaEmbedArgs {
	const uint32_t* id;
	uint32_t vocab;
	int dim;
	const bf16* table; // [vocab][dim]
	float scale;       // bf16(sqrt(dim))
	float* resid;      // fp32 [dim]
	bf16* xb;          // bf16 copy [dim] (may be null)
	int* err;
};

__global__ void k_gemma_embed(const GemmaEmbedArgs a)
{
	pdl_wait();
	pdl_trigger();
	const uint32_t id = *a.id;
	const bool bad = id >= a.vocab;
	if (bad && threadIdx.x == 0 && blockIdx.x == 0) report_err(a.err, kDevTokenRange);
	for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.dim; i += gridDim.x * blockDim.x) {
		const float v = bad ? 0.0f : __fmul_rn(Store<bf16>::get(a.table + (size_t)id * a.dim + i), a.scale);
		a.resid[i] = v;
		if (a.xb) Store<bf16>::put(a.xb + i, v);
	}
}

// sum over the CTA (blockDim.x a multiple of 32, at most 1024)
__device__ __forceinline__ float block_sum(float v, float* red)
{
	v = warp_sum(v);
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
	if (lane == 0) red[warp] = v;
	__syncthreads();
	float t = 0.0f;
	for (int w = 0; w < nw; ++w) t += red[w];
	__syncthreads(); // red may be reused
	return t;
}

struct PleCombineArgs {
	const uint32_t* id;
	uint32_t vocab;
	int L, P;
	const float* pm;         // [L * P] fp32, W_pmp . bf16(r)
	const bf16* embed_ple;   // [vocab][L * P]
	const bf16* norm_gain;   // [P]
	float s_ple, s_proj, s_sum, eps;
	bf16* ple;               // [L][P]
};

__global__ void k_ple_combine(const PleCombineArgs a)
{
	__shared__ float red[32];
	pdl_wait();
	pdl_trigger();
	const int l = blockIdx.x, j = threadIdx.x;
	const uint32_t id = *a.id < a.vocab ? *a.id : 0u; // an out-of-range id is reported by the embedding
	const float v = j < a.P ? __fmul_rn(a.pm[(size_t)l * a.P + j], a.s_proj) : 0.0f;
	const float ss = block_sum(v * v, red);
	if (j >= a.P) return;
	const float inv = 1.0f / sqrtf(__fdiv_rn(ss, (float)a.P) + a.eps);
	const float b = __fmul_rn(__fmul_rn(v, inv), __fadd_rn(1.0f, Store<bf16>::get(a.norm_gain + j)));
	const float e = __fmul_rn(Store<bf16>::get(a.embed_ple + (size_t)id * a.L * a.P + (size_t)l * a.P + j), a.s_ple);
	Store<bf16>::put(a.ple + (size_t)l * a.P + j, __fmul_rn(__fadd_rn(e, b), a.s_sum));
}

struct QkNormArgs {
	const float* raw;       // [(H + 2 KV) * hd] raw projection rows, each head's rows in (i, i+hd/2) pairs
	int H, KV, hd;
	const bf16* q_gain;     // [hd]
	const bf16* k_gain;     // [hd]
	float eps;
	const float* rope_cos;  // [max_seq][hd/2]
	const float* rope_sin;
	const int* pos;
	const int* slot;
	bf16* q_out;            // [H * hd]
	bf16* kpool;            // this layer's pages [pages][KV][blk][hd]
	bf16* vpool;
	const int* block_table;
	int pages_per_seq, max_pages, kv_block, max_seq;
	int* err;
};

__global__ void k_qk_norm_rope(const QkNormArgs a)
{
	__shared__ float red[32];
	pdl_wait();
	pdl_trigger();
	const int head = blockIdx.x, i = threadIdx.x, hd = a.hd, half = hd >> 1;
	const bool in = i < half;
	const float* row = a.raw + (size_t)head * hd;
	float x0 = in ? row[2 * i] : 0.0f, x1 = in ? row[2 * i + 1] : 0.0f; // canonical i and i + half
	const int pos = *a.pos, slot = *a.slot;
	if (head < a.H + a.KV) {
		const float ss = block_sum(fmaf(x0, x0, x1 * x1), red);
		if (!in) return;
		const float inv = 1.0f / sqrtf(__fdiv_rn(ss, (float)hd) + a.eps);
		const bf16* g = head < a.H ? a.q_gain : a.k_gain;
		const float n0 = __fmul_rn(__fmul_rn(x0, inv), __fadd_rn(1.0f, Store<bf16>::get(g + i)));
		const float n1 = __fmul_rn(__fmul_rn(x1, inv), __fadd_rn(1.0f, Store<bf16>::get(g + i + half)));
		const float c = a.rope_cos[(size_t)pos * half + i], s = a.rope_sin[(size_t)pos * half + i];
		x0 = __fsub_rn(__fmul_rn(n0, c), __fmul_rn(n1, s));
		x1 = __fadd_rn(__fmul_rn(n1, c), __fmul_rn(n0, s));
	}
	if (!in) return;
	if (head < a.H) {
		Store<bf16>::put(a.q_out + (size_t)head * hd + i, x0);
		Store<bf16>::put(a.q_out + (size_t)head * hd + i + half, x1);
		return;
	}
	const bool is_k = head < a.H + a.KV;
	const int kvh = head - a.H - (is_k ? 0 : a.KV);
	const int page = pos < a.max_seq ? a.block_table[(size_t)slot * a.pages_per_seq + pos / a.kv_block] : -1;
	if (page < 0 || page >= a.max_pages) {
		if (i == 0) report_err(a.err, kDevKvRange);
		return;
	}
	bf16* base = (is_k ? a.kpool : a.vpool) + (((size_t)page * a.KV + kvh) * a.kv_block + (pos % a.kv_block)) * hd;
	Store<bf16>::put(base + i, x0);
	Store<bf16>::put(base + i + half, x1);
}

} // namespace inf
