// Causal prefill attention over the paged KV cache (online softmax, fp32).
//
// Grid (kv_heads, ceil(T / 16)); a CTA takes 16 consecutive query tokens of one sequence
// and the G = H/KV query heads that share one KV head, so each K/V page is staged into
// shared memory once for 16 x G query rows.  Keys are masked by position (key_pos <= the
// query's position), which also covers chunked prefill: earlier chunks' keys are already
// in the cache.  Queries come from the fused QKV epilogue ([T][H][hd], RoPE applied).
#pragma once

#include "common.cuh"

namespace inf {

constexpr int kPfThreads = 256;
constexpr int kPfTq = 16;        // query tokens per CTA
constexpr int kPfMaxAcc = 32;    // (16 * G * head_dim) / 256 outputs per thread

struct AttnPrefillArgs {
	const void* q;          // [T][H][hd]
	const void* kpool;      // layer base [pages][KV][blk][hd]
	const void* vpool;
	const int* block_table;
	int pages_per_seq, max_pages;
	const int* tok_pos;     // [T], consecutive within a sequence
	const int* tok_slot;    // [T]
	int T, H, KV, hd, blk;
	float scale;
	void* out;              // [T][H*hd]
	int* err;
};

template <typename T>
__global__ void __launch_bounds__(kPfThreads) k_attn_prefill(const AttnPrefillArgs a)
{
	extern __shared__ __align__(16) float sm[];
	const int G = a.H / a.KV, hd = a.hd, blk = a.blk, R = kPfTq * G, ld = hd + 1;
	float* q_s = sm;                    // [R][hd+1], row r = tq * G + g
	float* k_s = q_s + R * ld;          // [blk][hd+1]
	float* v_s = k_s + blk * ld;        // [blk][hd]
	float* s_s = v_s + blk * hd;        // [R][blk]
	float* m_s = s_s + R * blk;         // [R]
	float* l_s = m_s + R;
	float* al_s = l_s + R;

	const int kvh = blockIdx.x, t0 = blockIdx.y * kPfTq, tid = threadIdx.x;
	pdl_wait();
	pdl_trigger();
	const int n_tok = min(kPfTq, a.T - t0);
	const int slot = a.tok_slot[t0];
	const int last_pos = a.tok_pos[t0 + n_tok - 1];

	for (int e = tid; e < R * hd; e += kPfThreads) {
		const int r = e / hd, i = e % hd;
		const int tq = r / G, g = r % G;
		float v = 0.0f;
		if (tq < n_tok) v = Store<T>::get(reinterpret_cast<const T*>(a.q) + ((size_t)(t0 + tq) * a.H + kvh * G + g) * hd + i);
		q_s[r * ld + i] = v;
	}
	for (int r = tid; r < R; r += kPfThreads) {
		m_s[r] = -INFINITY;
		l_s[r] = 0.0f;
	}
	float acc[kPfMaxAcc];
#pragma unroll
	for (int j = 0; j < kPfMaxAcc; ++j) acc[j] = 0.0f;
	__syncthreads();

	const int n_pages = last_pos / blk + 1;
	const size_t page_elems = (size_t)a.KV * blk * hd;
	for (int p = 0; p < n_pages; ++p) {
		const int page = a.block_table[(size_t)slot * a.pages_per_seq + p];
		const bool bad = page < 0 || page >= a.max_pages;
		if (bad && tid == 0) report_err(a.err, kDevKvRange);
		const size_t off = (bad ? 0 : (size_t)page * page_elems) + (size_t)kvh * blk * hd;
		const T* kt = reinterpret_cast<const T*>(a.kpool) + off;
		const T* vt = reinterpret_cast<const T*>(a.vpool) + off;
		for (int e = tid; e < blk * hd; e += kPfThreads) {
			const int j = e / hd, i = e % hd;
			k_s[j * ld + i] = bad ? 0.0f : Store<T>::get(kt + e);
			v_s[e] = bad ? 0.0f : Store<T>::get(vt + e);
		}
		__syncthreads();
		for (int e = tid; e < R * blk; e += kPfThreads) {
			const int r = e / blk, j = e % blk;
			const int tq = r / G;
			const int kpos = p * blk + j;
			float s = -INFINITY;
			if (tq < n_tok && !bad && kpos <= a.tok_pos[t0 + tq]) {
				const float* qr = q_s + r * ld;
				const float* kr = k_s + j * ld;
				float d0 = 0.0f, d1 = 0.0f;
				int i = 0;
				for (; i + 1 < hd; i += 2) {
					d0 = fmaf(qr[i], kr[i], d0);
					d1 = fmaf(qr[i + 1], kr[i + 1], d1);
				}
				if (i < hd) d0 = fmaf(qr[i], kr[i], d0);
				s = (d0 + d1) * a.scale;
			}
			s_s[e] = s;
		}
		__syncthreads();
		for (int r = tid; r < R; r += kPfThreads) {
			float mx = m_s[r];
			for (int j = 0; j < blk; ++j) mx = fmaxf(mx, s_s[r * blk + j]);
			float alpha = 1.0f, sum = 0.0f;
			if (mx != -INFINITY) {
				alpha = expf(m_s[r] - mx);
				for (int j = 0; j < blk; ++j) {
					const float e = expf(s_s[r * blk + j] - mx);
					s_s[r * blk + j] = e;
					sum += e;
				}
			} else {
				for (int j = 0; j < blk; ++j) s_s[r * blk + j] = 0.0f;
			}
			l_s[r] = l_s[r] * alpha + sum;
			m_s[r] = mx;
			al_s[r] = alpha;
		}
		__syncthreads();
#pragma unroll
		for (int jj = 0; jj < kPfMaxAcc; ++jj) {
			const int o = tid + jj * kPfThreads;
			if (o < R * hd) {
				const int r = o / hd, i = o % hd;
				float v = acc[jj] * al_s[r];
				const float* pr = s_s + r * blk;
				for (int j = 0; j < blk; ++j) v = fmaf(pr[j], v_s[j * hd + i], v);
				acc[jj] = v;
			}
		}
		__syncthreads();
	}

#pragma unroll
	for (int jj = 0; jj < kPfMaxAcc; ++jj) {
		const int o = tid + jj * kPfThreads;
		if (o < R * hd) {
			const int r = o / hd, i = o % hd;
			const int tq = r / G, g = r % G;
			if (tq < n_tok) {
				const float l = l_s[r];
				T* dst = reinterpret_cast<T*>(a.out) + (size_t)(t0 + tq) * a.H * hd + (size_t)(kvh * G + g) * hd + i;
				Store<T>::put(dst, l > 0.0f ? acc[jj] / l : 0.0f);
			}
		}
	}
}

inline size_t attn_prefill_smem_bytes(int G, int hd, int blk)
{
	const int R = kPfTq * G;
	return sizeof(float) * ((size_t)R * (hd + 1) + (size_t)blk * (hd + 1) + (size_t)blk * hd + (size_t)R * blk + 3 * R);
}

} // namespace inf
