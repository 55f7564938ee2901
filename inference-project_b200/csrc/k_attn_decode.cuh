// Decode attention over the paged KV cache (flash-decoding with a split-K combine).
//
// One query token per sequence (a batch of B tokens, each with its own slot and position).
// Grid (kv_heads, splits, B): a CTA owns one KV head of one token -- the G = H/KV query heads
// that share it (GQA), so every K/V page is read once for the whole group -- and a
// contiguous range of at most max_pages_split pages of the token's context.
//
// Latency is what matters at batch 1 (a layer's KV is a few MB), so:
//   * every page of the split is fetched at once with a 1-D bulk copy per K and V block,
//     each page on its own mbarrier; pages older than the current token's page are issued
//     before griddepcontrol.wait (they were written by earlier steps), overlapping the QKV
//     kernel that is still writing this token's K/V;
//   * the CTA works on slabs of 128/G tokens so each thread owns one (head, token) score;
//   * partial (max, sum, acc) go to scratch and the last CTA of each (token, KV head) --
//     found with an atomic ticket, no spinning -- combines the splits, computing the split
//     weights once.
// Positions past the context (stale slots in the last page) are masked.
#pragma once

#include "common.cuh"

namespace inf {

constexpr int kAttnThreads = 128;
constexpr int kAttnMaxAcc = 8;        // (G * head_dim) / 128 outputs per thread
constexpr int kAttnMaxPagesSplit = 16; // mbarriers per CTA
constexpr int kAttnSmemBudget = 96 * 1024;

struct AttnDecodeArgs {
	const void* q;           // [B][H*hd]
	const void* kpool;       // layer base [pages][KV][blk][hd]
	const void* vpool;
	const int* block_table;  // [slots][pages_per_seq]
	int pages_per_seq, max_pages;
	const int* tok_slot;     // [B]
	const int* tok_pos;      // [B]
	int H, KV, hd, blk, n_splits, max_pages_split;
	float scale;
	float* part;             // [B][H][n_splits][hd + 2]
	unsigned* counters;      // [B][KV]
	void* out;               // [B][H*hd]
	int* err;
};

template <typename T>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const AttnDecodeArgs a)
{
	extern __shared__ __align__(128) uint8_t sm_raw[];
	const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
	const int G = a.H / a.KV, hd = a.hd, blk = a.blk;
	const int TS = kAttnThreads / G;               // tokens per slab
	const size_t blk_bytes = (size_t)blk * hd * sizeof(T);
	uint8_t* kbuf = sm_raw;                                        // [max_pages_split][blk][hd]
	uint8_t* vbuf = kbuf + (size_t)a.max_pages_split * blk_bytes;
	float* q_s = reinterpret_cast<float*>(vbuf + (size_t)a.max_pages_split * blk_bytes); // [G][hd]
	float* s_s = q_s + G * hd;                                     // [G][TS]
	float* m_s = s_s + G * TS;                                     // [G]
	float* l_s = m_s + G;
	float* al_s = l_s + G;
	float* w_s = al_s + G;                                         // combine weights [G][n_splits]
	uint64_t* bars = reinterpret_cast<uint64_t*>(w_s + G * a.n_splits + 2);
	bars = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(bars) + 7) & ~(uintptr_t)7);
	__shared__ int last_flag;
	__shared__ int abort_flag;

	const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
	// slot, position and block table are not written by the kernels of this step
	const int slot = a.tok_slot[b];
	const int pos = a.tok_pos[b];
	const int ctx = pos + 1;
	const int n_pages = (ctx + blk - 1) / blk;
	const int pps = (n_pages + a.n_splits - 1) / a.n_splits;
	const int p_begin = split * pps;
	const int p_end = min(n_pages, p_begin + pps);
	const int np = max(0, p_end - p_begin);
	const int cur_page = pos / blk; // holds this step's K/V: fetched after the wait

	if (tid == 0) {
		abort_flag = 0;
		for (int j = 0; j < np; ++j) mbar_init(&bars[j], 1);
		mbar_fence_init();
	}
	__syncthreads();
	// thread j issues page j's two copies (page ids are read in parallel, not one by one)
	auto issue = [&](int j) {
		const int p = p_begin + j;
		const int page = a.block_table[(size_t)slot * a.pages_per_seq + p];
		if (page < 0 || page >= a.max_pages) {
			report_err(a.err, kDevKvRange);
			mbar_arrive(&bars[j]); // completes the phase with nothing in flight; data masked below
			return;
		}
		const size_t off = (((size_t)page * a.KV + kvh) * blk) * hd;
		mbar_arrive_expect_tx(&bars[j], (uint32_t)(2 * blk_bytes));
		const uint64_t pol = policy_evict_first();
		bulk_g2s(kbuf + j * blk_bytes, reinterpret_cast<const T*>(a.kpool) + off, (uint32_t)blk_bytes, &bars[j], pol);
		bulk_g2s(vbuf + j * blk_bytes, reinterpret_cast<const T*>(a.vpool) + off, (uint32_t)blk_bytes, &bars[j], pol);
	};
	if (tid < np && p_begin + tid < cur_page) issue(tid);
	pdl_wait();
	pdl_trigger();
	if (tid < np && p_begin + tid >= cur_page) issue(tid);

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

	const int n_tok = np * blk;
	const int my_g = tid / TS, my_t = tid % TS;
	int waited = 0; // pages known to have landed
	for (int t0 = 0; t0 < n_tok; t0 += TS) {
		// make sure every page this slab touches has landed
		const int need = min(np, (t0 + TS + blk - 1) / blk);
		for (; waited < need; ++waited)
			if (!abort_flag && !mbar_wait(&bars[waited], 0, (volatile int*)&abort_flag, a.err)) abort_flag = 1;
		// scores: one (head, token) per thread; rotated reads avoid bank conflicts
		{
			const int tl = t0 + my_t;
			const int tok = p_begin * blk + tl;
			float s = -INFINITY;
			if (tl < n_tok && tok < ctx && !abort_flag) {
				const T* kr = reinterpret_cast<const T*>(kbuf) + (size_t)tl * hd;
				const float* qr = q_s + my_g * hd;
				const int rot = (2 * my_t) % hd;
				float d0 = 0.0f, d1 = 0.0f;
				for (int i = 0; i < hd; i += 2) {
					int k0 = i + rot;
					if (k0 >= hd) k0 -= hd;
					d0 = fmaf(qr[k0], Store<T>::get(kr + k0), d0);
					d1 = fmaf(qr[k0 + 1], Store<T>::get(kr + k0 + 1), d1);
				}
				s = (d0 + d1) * a.scale;
			}
			s_s[my_g * TS + my_t] = s;
		}
		__syncthreads();
		// online softmax, one warp per head
		for (int g = warp; g < G; g += kAttnThreads / 32) {
			float mx = -INFINITY;
			for (int j = lane; j < TS; j += 32) mx = fmaxf(mx, s_s[g * TS + j]);
			mx = warp_max(mx);
			const float m_old = m_s[g];
			const float m_new = fmaxf(m_old, mx);
			float sum = 0.0f;
			for (int j = lane; j < TS; j += 32) {
				const float sv = s_s[g * TS + j];
				const float e = (m_new == -INFINITY) ? 0.0f : expf(sv - m_new);
				s_s[g * TS + j] = e;
				sum += e;
			}
			sum = warp_sum(sum);
			if (lane == 0) {
				const float alpha = (m_new == -INFINITY) ? 1.0f : expf(m_old - m_new);
				l_s[g] = l_s[g] * alpha + sum;
				m_s[g] = m_new;
				al_s[g] = alpha;
			}
		}
		__syncthreads();
		const int t_hi = min(TS, n_tok - t0);
#pragma unroll
		for (int jj = 0; jj < kAttnMaxAcc; ++jj) {
			const int o = tid + jj * kAttnThreads;
			if (o < G * hd) {
				const int g = o / hd, i = o % hd;
				float v = acc[jj] * al_s[g];
				const float* pr = s_s + g * TS;
				const T* vc = reinterpret_cast<const T*>(vbuf) + (size_t)t0 * hd + i;
				for (int j = 0; j < t_hi; ++j) v = fmaf(pr[j], Store<T>::get(vc + (size_t)j * hd), v);
				acc[jj] = v;
			}
		}
		__syncthreads();
	}
	// pages issued but never waited for (abort) must land before the CTA exits or the page
	// buffers are reused for the combine
	if (tid == 0)
		for (int j = waited; j < np; ++j) {
			const uint64_t t0 = global_timer_ns();
			while (!mbar_try_wait(&bars[j], 0))
				if (global_timer_ns() - t0 > kWaitLimitNs) break;
		}

	// partials: [b][h][split][hd + 2] = (acc..., m, l)
	const int hd2 = hd + 2;
#pragma unroll
	for (int jj = 0; jj < kAttnMaxAcc; ++jj) {
		const int o = tid + jj * kAttnThreads;
		if (o < G * hd) {
			const int g = o / hd, i = o % hd;
			a.part[(((size_t)b * a.H + kvh * G + g) * a.n_splits + split) * hd2 + i] = acc[jj];
		}
	}
	if (tid < G) {
		float* pr = a.part + (((size_t)b * a.H + kvh * G + tid) * a.n_splits + split) * hd2;
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

	// combine.  The G heads' partials of this (token, KV head) are one contiguous block of
	// G * n_splits * (hd + 2) floats; copy it into the (now idle) page buffers with
	// independent 16-byte loads, eight in flight per thread, then reduce from shared memory.
	float* pc = reinterpret_cast<float*>(sm_raw);
	const size_t n_part = (size_t)G * a.n_splits * hd2;
	if (n_part * sizeof(float) <= 2 * (size_t)a.max_pages_split * blk_bytes && (n_part & 3) == 0) {
		const float4* src = reinterpret_cast<const float4*>(a.part + (((size_t)b * a.H + kvh * G) * a.n_splits) * hd2);
		float4* dst = reinterpret_cast<float4*>(pc);
		const int n4 = (int)(n_part >> 2);
		for (int base = 0; base < n4; base += 8 * kAttnThreads) {
			float4 r[8];
#pragma unroll
			for (int u = 0; u < 8; ++u) {
				const int idx = base + u * kAttnThreads + tid;
				if (idx < n4) r[u] = __ldcg(src + idx);
			}
#pragma unroll
			for (int u = 0; u < 8; ++u) {
				const int idx = base + u * kAttnThreads + tid;
				if (idx < n4) dst[idx] = r[u];
			}
		}
	} else {
		const float* src = a.part + (((size_t)b * a.H + kvh * G) * a.n_splits) * hd2;
		for (size_t idx = tid; idx < n_part; idx += kAttnThreads) pc[idx] = __ldcg(src + idx);
	}
	__syncthreads();
	// weights exp(m_s - M) / L once per (head, split)
	for (int g = warp; g < G; g += kAttnThreads / 32) {
		const float* pr = pc + (size_t)g * a.n_splits * hd2;
		float M = -INFINITY;
		for (int s = lane; s < a.n_splits; s += 32) M = fmaxf(M, pr[(size_t)s * hd2 + hd]);
		M = warp_max(M);
		float L = 0.0f;
		for (int s = lane; s < a.n_splits; s += 32) {
			const float ms = pr[(size_t)s * hd2 + hd];
			const float w = (ms == -INFINITY) ? 0.0f : expf(ms - M);
			w_s[g * a.n_splits + s] = w;
			L += w * pr[(size_t)s * hd2 + hd + 1];
		}
		L = warp_sum(L);
		__syncwarp();
		const float invL = L > 0.0f ? 1.0f / L : 0.0f;
		for (int s = lane; s < a.n_splits; s += 32) w_s[g * a.n_splits + s] *= invL;
	}
	__syncthreads();
	T* ob = reinterpret_cast<T*>(a.out) + (size_t)b * a.H * hd;
	for (int o = tid; o < G * hd; o += kAttnThreads) {
		const int g = o / hd, i = o % hd;
		const float* pr = pc + (size_t)g * a.n_splits * hd2 + i;
		const float* w = w_s + g * a.n_splits;
		float v0 = 0.0f, v1 = 0.0f;
		int s = 0;
		for (; s + 1 < a.n_splits; s += 2) {
			v0 = fmaf(w[s], pr[(size_t)s * hd2], v0);
			v1 = fmaf(w[s + 1], pr[(size_t)(s + 1) * hd2], v1);
		}
		if (s < a.n_splits) v0 = fmaf(w[s], pr[(size_t)s * hd2], v0);
		Store<T>::put(ob + (size_t)(kvh * G + g) * hd + i, v0 + v1);
	}
	if (tid == 0) a.counters[b * a.KV + kvh] = 0u;
}

// pages per split that fit the shared-memory budget
inline int attn_decode_max_pages_split(int blk, int hd, size_t esz)
{
	const size_t page = 2 * (size_t)blk * hd * esz;
	return (int)std::min<size_t>(kAttnMaxPagesSplit, std::max<size_t>(1, kAttnSmemBudget / page));
}

inline size_t attn_decode_smem_bytes(int G, int hd, int blk, size_t esz, int max_pages_split, int n_splits)
{
	const int TS = kAttnThreads / G;
	return 2 * (size_t)max_pages_split * blk * hd * esz +
	       sizeof(float) * ((size_t)G * hd + (size_t)G * TS + 3 * G + (size_t)G * n_splits + 2) + 8 +
	       kAttnMaxPagesSplit * sizeof(uint64_t);
}

} // namespace inf
