// Decode attention over the paged KV cache (flash-decoding with a split-K combine).
//
// One query token per sequence (batch of B tokens, each with its own slot and position).
// Grid (kv_heads, splits, B); a CTA owns one KV head of one token -- i.e. the G = H/KV
// query heads that share it (GQA), so every K/V page is read once for the whole group --
// and a contiguous range of the token's pages.  Per page: K tile -> shared memory (fp32),
// scores for G x kv_block, online softmax, V tile -> shared memory, accumulate.  Partial
// (max, sum, acc) go to scratch; the last CTA of each (token, KV head) -- found with an
// atomic ticket, no spinning -- combines the splits and writes the rounded output.
// Pages past the context hold stale data and are masked by position.
#pragma once

#include "common.cuh"

namespace inf {

constexpr int kAttnThreads = 128;
constexpr int kAttnMaxAcc = 8; // (G * head_dim) / kAttnThreads outputs per thread

struct AttnDecodeArgs {
	const void* q;           // [B][H*hd]
	const void* kpool;       // layer base [pages][KV][blk][hd]
	const void* vpool;
	const int* block_table;  // [slots][pages_per_seq]
	int pages_per_seq, max_pages;
	const int* tok_slot;     // [B]
	const int* tok_pos;      // [B]
	int H, KV, hd, blk, n_splits;
	float scale;
	float* part;             // [B][H][n_splits][hd + 2]
	unsigned* counters;      // [B][KV]
	void* out;               // [B][H*hd]
	int* err;
};

template <typename T>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const AttnDecodeArgs a)
{
	extern __shared__ __align__(16) float sm[];
	const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
	const int G = a.H / a.KV, hd = a.hd, blk = a.blk;
	float* q_s = sm;                 // [G][hd]
	float* kv_s = q_s + G * hd;      // [blk][hd]
	float* p_s = kv_s + blk * hd;    // [G][blk]
	float* m_s = p_s + G * blk;      // [G]
	float* l_s = m_s + G;            // [G]
	float* al_s = l_s + G;           // [G]
	__shared__ int last_flag;

	const int tid = threadIdx.x;
	pdl_wait();
	pdl_trigger();

	const int slot = a.tok_slot[b];
	const int pos = a.tok_pos[b];
	const int ctx = pos + 1;
	const int n_pages = (ctx + blk - 1) / blk;
	const int pps = (n_pages + a.n_splits - 1) / a.n_splits;
	const int p_begin = split * pps;
	const int p_end = min(n_pages, p_begin + pps);

	const T* qb = reinterpret_cast<const T*>(a.q) + (size_t)b * a.H * hd + (size_t)kvh * G * hd;
	for (int i = tid; i < G * hd; i += kAttnThreads) q_s[i] = Store<T>::get(qb + i);
	if (tid < G) {
		m_s[tid] = -INFINITY;
		l_s[tid] = 0.0f;
	}
	float acc[kAttnMaxAcc];
#pragma unroll
	for (int j = 0; j < kAttnMaxAcc; ++j) acc[j] = 0.0f;
	__syncthreads();

	const size_t page_elems = (size_t)a.KV * blk * hd;
	for (int p = p_begin; p < p_end; ++p) {
		const int page = a.block_table[(size_t)slot * a.pages_per_seq + p];
		const bool bad = page < 0 || page >= a.max_pages;
		if (bad && tid == 0) report_err(a.err, kDevKvRange);
		const T* kt = reinterpret_cast<const T*>(a.kpool) + (bad ? 0 : (size_t)page * page_elems) + (size_t)kvh * blk * hd;
		const T* vt = reinterpret_cast<const T*>(a.vpool) + (bad ? 0 : (size_t)page * page_elems) + (size_t)kvh * blk * hd;
		for (int i = tid; i < blk * hd; i += kAttnThreads) kv_s[i] = bad ? 0.0f : Store<T>::get(kt + i);
		__syncthreads();
		for (int e = tid; e < G * blk; e += kAttnThreads) {
			const int g = e / blk, t = e % blk;
			const int tok = p * blk + t;
			float s = -INFINITY;
			if (tok < ctx && !bad) {
				const float* qr = q_s + g * hd;
				const float* kr = kv_s + t * hd;
				float d = 0.0f;
				for (int i = 0; i < hd; ++i) d = fmaf(qr[i], kr[i], d);
				s = d * a.scale;
			}
			p_s[e] = s;
		}
		__syncthreads();
		if (tid < G) {
			float mx = m_s[tid];
			for (int t = 0; t < blk; ++t) mx = fmaxf(mx, p_s[tid * blk + t]);
			float alpha = 1.0f, sum = 0.0f;
			if (mx != -INFINITY) {
				alpha = expf(m_s[tid] - mx);
				for (int t = 0; t < blk; ++t) {
					const float e = expf(p_s[tid * blk + t] - mx);
					p_s[tid * blk + t] = e;
					sum += e;
				}
			} else {
				for (int t = 0; t < blk; ++t) p_s[tid * blk + t] = 0.0f;
			}
			l_s[tid] = l_s[tid] * alpha + sum;
			m_s[tid] = mx;
			al_s[tid] = alpha;
		}
		__syncthreads();
		for (int i = tid; i < blk * hd; i += kAttnThreads) kv_s[i] = bad ? 0.0f : Store<T>::get(vt + i);
		__syncthreads();
#pragma unroll
		for (int j = 0; j < kAttnMaxAcc; ++j) {
			const int o = tid + j * kAttnThreads;
			if (o < G * hd) {
				const int g = o / hd, i = o % hd;
				float v = acc[j] * al_s[g];
				for (int t = 0; t < blk; ++t) v = fmaf(p_s[g * blk + t], kv_s[t * hd + i], v);
				acc[j] = v;
			}
		}
		__syncthreads();
	}

	// partials: [b][h][split][hd + 2] = (acc..., m, l)
	const int hd2 = hd + 2;
#pragma unroll
	for (int j = 0; j < kAttnMaxAcc; ++j) {
		const int o = tid + j * kAttnThreads;
		if (o < G * hd) {
			const int g = o / hd, i = o % hd;
			const int h = kvh * G + g;
			a.part[(((size_t)b * a.H + h) * a.n_splits + split) * hd2 + i] = acc[j];
		}
	}
	if (tid < G) {
		const int h = kvh * G + tid;
		float* pr = a.part + (((size_t)b * a.H + h) * a.n_splits + split) * hd2;
		pr[hd] = m_s[tid];
		pr[hd + 1] = l_s[tid];
	}
	__threadfence();
	__syncthreads();
	if (tid == 0) {
		const unsigned t = atomicAdd(&a.counters[b * a.KV + kvh], 1u);
		last_flag = (t == (unsigned)a.n_splits - 1);
	}
	__syncthreads();
	if (!last_flag) return;
	__threadfence();

	T* ob = reinterpret_cast<T*>(a.out) + (size_t)b * a.H * hd;
	for (int o = tid; o < G * hd; o += kAttnThreads) {
		const int g = o / hd, i = o % hd;
		const int h = kvh * G + g;
		const float* pr = a.part + (((size_t)b * a.H + h) * a.n_splits) * hd2;
		float M = -INFINITY;
		for (int s = 0; s < a.n_splits; ++s) M = fmaxf(M, __ldcg(pr + (size_t)s * hd2 + hd));
		float L = 0.0f, v = 0.0f;
		if (M != -INFINITY) {
			for (int s = 0; s < a.n_splits; ++s) {
				const float ms = __ldcg(pr + (size_t)s * hd2 + hd);
				if (ms == -INFINITY) continue;
				const float w = expf(ms - M);
				L += w * __ldcg(pr + (size_t)s * hd2 + hd + 1);
				v += w * __ldcg(pr + (size_t)s * hd2 + i);
			}
		}
		Store<T>::put(ob + h * hd + i, L > 0.0f ? v / L : 0.0f);
	}
	if (tid == 0) a.counters[b * a.KV + kvh] = 0u;
}

inline size_t attn_decode_smem_bytes(int G, int hd, int blk)
{
	return sizeof(float) * ((size_t)G * hd + (size_t)blk * hd + (size_t)G * blk + 3 * G);
}

} // namespace inf
