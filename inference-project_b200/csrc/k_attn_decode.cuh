// Decode attention over the paged KV cache (flash-decoding with a split-K combine).
//
// One query token per sequence (a batch of B tokens, each with its own slot and position).
// Grid (kv_heads, splits, B): a CTA owns one KV head of one token -- the G = H/KV query heads
// that share it (GQA), so every K/V page is read once for the whole group -- and a
// contiguous range of at most max_pages_split pages of the token's context.
//
// It serves batch-1 decode when the context is too long for the cluster kernel
// (k_attn_cluster.cuh) and the stand-alone inf_attn_decode / inf_attn_decode_noalloc entry
// points; batches run the streaming tensor-core kernel (k_attn_decode_mma.cuh).  A layer's
// KV of one token is a few MB, so the kernel is built for latency:
//   * every page of the split is fetched at once with a 1-D bulk copy per K and V block,
//     each page on its own mbarrier; pages older than the current token's page are issued
//     before griddepcontrol.wait (earlier steps wrote them), overlapping the QKV kernel that
//     is still writing this token's K/V;
//   * scores: 8 warps take tokens round-robin, lanes split head_dim, the G queries sit in
//     registers and the G partial dots are reduced with one transposed butterfly;
//   * one softmax pass over all the split's scores (no online rescaling inside a CTA);
//   * P.V: warps again take tokens round-robin and are summed through shared memory;
//   * partial (max, sum, acc) go to scratch and the last CTA of each (token, KV head) --
//     found with an atomic ticket, no spinning -- combines the splits.
// Positions past the context (stale slots in the last page) are masked.
#pragma once

#include "common.cuh"
#include "k_gemv.cuh" // reduce_rows / row_of_lane

namespace inf {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxAcc = 8;          // (G * head_dim) / 256 outputs per thread
constexpr int kAttnMaxPagesSplit = 16;  // mbarriers per CTA
constexpr int kAttnSmemBudget = 96 * 1024; // page buffers of one CTA
constexpr int kAttnTokIlp = 4;          // tokens a warp works on at once

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
	// batched mma kernel: per work unit (token, split | splits << 16); n_splits is then the
	// stride of part (the most splits a token can have)
	const int* units;
};

// head_dim values per lane of a warp
inline int attn_vpl(int hd) { return hd <= 32 ? 1 : hd <= 64 ? 2 : hd <= 128 ? 4 : hd <= 256 ? 8 : 16; }

constexpr size_t kAttnCombineStageMax = 96 * 1024; // larger split partials are combined from global memory

// bytes of one (token, KV head)'s split partials, and whether the combine stages them
__host__ __device__ inline size_t attn_combine_bytes(int G, int hd, int n_splits)
{
	return (size_t)G * n_splits * (hd + 2) * sizeof(float);
}
__host__ __device__ inline bool attn_combine_staged(int G, int hd, int n_splits)
{
	const size_t b = attn_combine_bytes(G, hd, n_splits);
	return b <= kAttnCombineStageMax && (b & 15) == 0;
}

// page buffers, also reused for the P.V reduction and, when staged, the split combine
__host__ __device__ inline size_t attn_region_bytes(int G, int hd, int blk, size_t esz, int max_pages_split, int n_splits)
{
	size_t r = 2 * (size_t)max_pages_split * blk * hd * esz;
	const size_t pv = (size_t)kAttnWarps * G * hd * sizeof(float);
	r = r > pv ? r : pv;
	if (attn_combine_staged(G, hd, n_splits)) {
		const size_t cb = attn_combine_bytes(G, hd, n_splits);
		r = r > cb ? r : cb;
	}
	return (r + 15) & ~(size_t)15;
}

// VPL consecutive head_dim values of one K/V row as floats (lanes past head_dim read nothing)
template <typename T, int VPL>
__device__ __forceinline__ void load_vals(const T* row, int d0, int hd, float (&v)[VPL])
{
#pragma unroll
	for (int j = 0; j < VPL; ++j) v[j] = (d0 + j < hd) ? Store<T>::get(row + d0 + j) : 0.0f;
}

template <typename T, int G, int VPL>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const AttnDecodeArgs a)
{
	extern __shared__ __align__(128) uint8_t sm_raw[];
	const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
	const int hd = a.hd, blk = a.blk;
	const size_t blk_bytes = (size_t)blk * hd * sizeof(T);
	const int max_tok = a.max_pages_split * blk;
	uint8_t* kbuf = sm_raw;                                        // [max_pages_split][blk][hd]
	uint8_t* vbuf = kbuf + (size_t)a.max_pages_split * blk_bytes;
	const size_t region = attn_region_bytes(G, hd, blk, sizeof(T), a.max_pages_split, a.n_splits);
	float* s_s = reinterpret_cast<float*>(sm_raw + region);       // [G][max_tok]
	float* m_s = s_s + G * max_tok;                                // [G]
	float* l_s = m_s + G;                                          // [G]
	float* w_s = l_s + G;                                          // combine weights [G][n_splits]
	uint64_t* bars = reinterpret_cast<uint64_t*>(w_s + G * a.n_splits + 2);
	bars = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(bars) + 7) & ~(uintptr_t)7);
	float* pv_red = reinterpret_cast<float*>(kbuf); // [warps][G*hd], reuses the page buffers after P.V
	__shared__ int last_flag;
	__shared__ int abort_flag;

	const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
	const int d0 = lane * VPL; // this lane's head_dim slice
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
	const int n_tok = np * blk;
	const int tok0 = p_begin * blk;

	if (tid == 0) {
		abort_flag = 0;
		for (int j = 0; j < np; ++j) mbar_init(&bars[j], 1);
		mbar_fence_init();
	}
	__syncthreads();
	// thread j issues page j's two copies (page ids are read in parallel, not one by one)
	auto issue = [&](int j) {
		const int page = a.block_table[(size_t)slot * a.pages_per_seq + p_begin + j];
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

	// the G queries of this KV head, this lane's head_dim slice, in registers
	float qr[G][VPL];
	{
		const T* qb = reinterpret_cast<const T*>(a.q) + (size_t)b * a.H * hd + (size_t)kvh * G * hd;
#pragma unroll
		for (int g = 0; g < G; ++g) load_vals<T, VPL>(qb + (size_t)g * hd, d0, hd, qr[g]);
	}

	// ---- scores
	const int my_g = row_of_lane<G>(lane);
	const bool g_writer = (lane & (32 / G - 1)) == 0;
	// kAttnTokIlp tokens per warp iteration, so their loads, dots and shuffle trees interleave
	int waited = 0;
	for (int t0 = warp * kAttnTokIlp; t0 < n_tok; t0 += kAttnWarps * kAttnTokIlp) {
		for (const int need = min(np, (t0 + kAttnTokIlp - 1) / blk + 1); waited < need; ++waited)
			if (!abort_flag && !mbar_wait(&bars[waited], 0, (volatile int*)&abort_flag, a.err)) abort_flag = 1;
		float kv[kAttnTokIlp][VPL];
#pragma unroll
		for (int u = 0; u < kAttnTokIlp; ++u) {
			const int t = min(t0 + u, n_tok - 1);
			load_vals<T, VPL>(reinterpret_cast<const T*>(kbuf) + (size_t)t * hd, d0, hd, kv[u]);
		}
		float sc[kAttnTokIlp];
#pragma unroll
		for (int u = 0; u < kAttnTokIlp; ++u) {
			float part[G];
#pragma unroll
			for (int g = 0; g < G; ++g) {
				float s = 0.0f;
#pragma unroll
				for (int j = 0; j < VPL; ++j) s = fmaf(qr[g][j], kv[u][j], s);
				part[g] = s;
			}
			sc[u] = reduce_rows<G>(part, lane);
		}
#pragma unroll
		for (int u = 0; u < kAttnTokIlp; ++u) {
			const int t = t0 + u;
			if (g_writer && t < n_tok) s_s[my_g * max_tok + t] = (tok0 + t < ctx && !abort_flag) ? sc[u] * a.scale : -INFINITY;
		}
	}
	// a warp that saw fewer pages than exist must still observe every page before the V pass
	for (; waited < np; ++waited)
		if (!abort_flag && !mbar_wait(&bars[waited], 0, (volatile int*)&abort_flag, a.err)) abort_flag = 1;
	__syncthreads();

	// ---- softmax over the split, one warp per head
	for (int g = warp; g < G; g += kAttnWarps) {
		float mx = -INFINITY;
		for (int t = lane; t < n_tok; t += 32) mx = fmaxf(mx, s_s[g * max_tok + t]);
		mx = warp_max(mx);
		float sum = 0.0f;
		for (int t = lane; t < n_tok; t += 32) {
			const float e = (mx == -INFINITY) ? 0.0f : expf(s_s[g * max_tok + t] - mx);
			s_s[g * max_tok + t] = e;
			sum += e;
		}
		sum = warp_sum(sum);
		if (lane == 0) {
			m_s[g] = mx;
			l_s[g] = sum;
		}
	}
	if (n_tok == 0 && tid < G) {
		m_s[tid] = -INFINITY;
		l_s[tid] = 0.0f;
	}
	__syncthreads();

	// ---- P.V: warps split the tokens, lanes split head_dim
	float acc[G][VPL];
#pragma unroll
	for (int g = 0; g < G; ++g)
#pragma unroll
		for (int j = 0; j < VPL; ++j) acc[g][j] = 0.0f;
	for (int t0 = warp * kAttnTokIlp; t0 < n_tok; t0 += kAttnWarps * kAttnTokIlp) {
		float vv[kAttnTokIlp][VPL], pp[kAttnTokIlp][G];
#pragma unroll
		for (int u = 0; u < kAttnTokIlp; ++u) {
			const bool in = t0 + u < n_tok;
			const int t = in ? t0 + u : n_tok - 1;
			load_vals<T, VPL>(reinterpret_cast<const T*>(vbuf) + (size_t)t * hd, d0, hd, vv[u]);
#pragma unroll
			for (int g = 0; g < G; ++g) pp[u][g] = in ? s_s[g * max_tok + t] : 0.0f;
		}
#pragma unroll
		for (int u = 0; u < kAttnTokIlp; ++u)
#pragma unroll
			for (int g = 0; g < G; ++g)
#pragma unroll
				for (int j = 0; j < VPL; ++j) acc[g][j] = fmaf(pp[u][g], vv[u][j], acc[g][j]);
	}
	// cross-warp sum through shared memory (the page buffers are free once every warp is done)
	__syncthreads();
#pragma unroll
	for (int g = 0; g < G; ++g)
#pragma unroll
		for (int j = 0; j < VPL; ++j)
			if (d0 + j < hd) pv_red[(size_t)warp * G * hd + g * hd + d0 + j] = acc[g][j];
	__syncthreads();

	// partials: [b][h][split][hd + 2] = (acc..., m, l)
	const int hd2 = hd + 2;
	for (int o = tid; o < G * hd; o += kAttnThreads) {
		float v = 0.0f;
#pragma unroll
		for (int w = 0; w < kAttnWarps; ++w) v += pv_red[(size_t)w * G * hd + o];
		const int g = o / hd, i = o % hd;
		a.part[(((size_t)b * a.H + kvh * G + g) * a.n_splits + split) * hd2 + i] = v;
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
	// G * n_splits * (hd + 2) floats.  When it fits the region (sized for it on the host with
	// the same rule) it is copied into the idle page buffers with independent 16-byte loads,
	// eight in flight per thread; otherwise the reduction reads it from global memory.
	const bool staged = attn_combine_staged(G, hd, a.n_splits);
	const float* pc = staged ? reinterpret_cast<const float*>(sm_raw)
	                         : a.part + (((size_t)b * a.H + kvh * G) * a.n_splits) * hd2;
	const size_t n_part = (size_t)G * a.n_splits * hd2;
	if (staged) {
		const float4* src = reinterpret_cast<const float4*>(a.part + (((size_t)b * a.H + kvh * G) * a.n_splits) * hd2);
		float4* dst = reinterpret_cast<float4*>(sm_raw);
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
	}
	__syncthreads();
	// other CTAs wrote the partials: from global memory they are read past L1
	auto rd = [&](const float* p) { return staged ? *p : __ldcg(p); };
	// weights exp(m_s - M) / L once per (head, split)
	for (int g = warp; g < G; g += kAttnWarps) {
		const float* pr = pc + (size_t)g * a.n_splits * hd2;
		float M = -INFINITY;
		for (int s = lane; s < a.n_splits; s += 32) M = fmaxf(M, rd(pr + (size_t)s * hd2 + hd));
		M = warp_max(M);
		float L = 0.0f;
		for (int s = lane; s < a.n_splits; s += 32) {
			const float ms = rd(pr + (size_t)s * hd2 + hd);
			const float w = (ms == -INFINITY) ? 0.0f : expf(ms - M);
			w_s[g * a.n_splits + s] = w;
			L += w * rd(pr + (size_t)s * hd2 + hd + 1);
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
			v0 = fmaf(w[s], rd(pr + (size_t)s * hd2), v0);
			v1 = fmaf(w[s + 1], rd(pr + (size_t)(s + 1) * hd2), v1);
		}
		if (s < a.n_splits) v0 = fmaf(w[s], rd(pr + (size_t)s * hd2), v0);
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

// Splits per (token, KV head): at most one CTA per SM when the context fits (so the next
// kernel's CTA can start beside it), more when a split would exceed the page budget.  The
// page buffers are sized for the pages a split actually needs.
inline void attn_decode_plan(int sms, int kv_heads, int tokens, int pages_per_seq, int blk, int hd, size_t esz,
                             int* splits, int* max_pages_split)
{
	const int budget = attn_decode_max_pages_split(blk, hd, esz);
	int s = std::max(1, sms / std::max(1, kv_heads * tokens));
	s = std::max(s, (pages_per_seq + budget - 1) / budget);
	s = std::min(s, pages_per_seq);
	*splits = s;
	*max_pages_split = (pages_per_seq + s - 1) / s;
}

inline size_t attn_decode_smem_bytes(int G, int hd, int blk, size_t esz, int max_pages_split, int n_splits)
{
	return attn_region_bytes(G, hd, blk, esz, max_pages_split, n_splits) +
	       sizeof(float) * ((size_t)G * max_pages_split * blk + 2 * G + (size_t)G * n_splits + 2) + 8 +
	       kAttnMaxPagesSplit * sizeof(uint64_t);
}

template <typename T>
using AttnKernel = void (*)(AttnDecodeArgs);

// the instantiation for a GQA group G in {1,2,4,8} and head_dim <= 256 (nullptr otherwise)
template <typename T>
inline AttnKernel<T> attn_decode_kernel(int G, int hd)
{
	const int vpl = attn_vpl(hd);
#define INF_ATTN_CASE(g, v) \
	if (G == g && vpl == v) return k_attn_decode<T, g, v>;
#define INF_ATTN_G(g) INF_ATTN_CASE(g, 1) INF_ATTN_CASE(g, 2) INF_ATTN_CASE(g, 4) INF_ATTN_CASE(g, 8)
	INF_ATTN_G(1) INF_ATTN_G(2) INF_ATTN_G(4) INF_ATTN_G(8)
	// head_dim up to 512 (the Gemma-style decoder's global_head_dim) for groups of at most 4
	INF_ATTN_CASE(1, 16) INF_ATTN_CASE(2, 16) INF_ATTN_CASE(4, 16)
#undef INF_ATTN_G
#undef INF_ATTN_CASE
	return nullptr;
}

// whether the split-K kernel serves a GQA group and head_dim
inline bool attn_decode_supported(int G, int hd)
{
	return (G == 1 || G == 2 || G == 4 || G == 8) && hd <= 512 && (hd <= 256 || G <= 4);
}


} // namespace inf
