// Decode attention for batches of tokens (SIMT): the K/V pages of a split are streamed through
// a ring of shared-memory chunks with an online softmax, so a split may cover any number of
// pages and the grid stays a few CTAs per SM.  Batches run the tensor-core kernel of the same
// decomposition (k_attn_decode_mma.cuh) when the pages hold 16 positions and the GQA group and
// head size have an instance there; this kernel serves the other shapes.
//
// Grid (kv_heads, splits, tokens); a CTA owns one KV head of one token (its G query heads)
// and a contiguous range of the token's pages, read in chunks of kStChunkPages pages
// (kStBufs chunks in flight, one 1-D bulk copy per K and V page, one mbarrier per chunk).
// Per chunk: scores for the chunk's positions, the running max / sum per head updated
// (acc rescaled by exp(m_old - m_new)), then acc += P.V.  The split's (max, sum, acc) go to
// scratch and the last CTA of each (token, KV head) -- atomic ticket, no spinning -- combines
// the splits, as in the split-K kernel (k_attn_decode.cuh).  Positions past the context are
// masked; every wait is bounded.
#pragma once

#include "common.cuh"
#include "k_attn_cluster.cuh" // load_vals_vec
#include "k_attn_decode.cuh"  // AttnDecodeArgs, kAttn*, reduce_rows, row_of_lane

namespace inf {

constexpr int kStChunkPages = 4;
constexpr int kStBufs = 3;

__host__ __device__ inline size_t attn_stream_region_bytes(int G, int hd, int blk, size_t esz)
{
	size_t r = (size_t)kStBufs * 2 * kStChunkPages * blk * hd * esz;
	const size_t pv = (size_t)kAttnWarps * G * hd * sizeof(float);
	return ((r > pv ? r : pv) + 127) & ~(size_t)127;
}
inline size_t attn_stream_smem_bytes(int G, int hd, int blk, size_t esz)
{
	return attn_stream_region_bytes(G, hd, blk, esz) + sizeof(float) * ((size_t)G * kStChunkPages * blk + 4 * G) + 16 +
	       kStBufs * sizeof(uint64_t);
}
// splits per (token, KV head): about four CTAs per SM over the whole batch
inline int attn_stream_splits(int sms, int kv_heads, int tokens, int pages_per_seq)
{
	int s = (4 * sms + kv_heads * tokens - 1) / (kv_heads * tokens);
	s = s < 1 ? 1 : s;
	s = s > 32 ? 32 : s;
	return s > pages_per_seq ? pages_per_seq : s;
}

template <typename T, int G, int VPL>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode_stream(const AttnDecodeArgs a)
{
	extern __shared__ __align__(128) uint8_t sm_raw[];
	const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
	const int hd = a.hd, blk = a.blk;
	const int CT = kStChunkPages * blk; // positions per chunk
	const size_t blk_bytes = (size_t)blk * hd * sizeof(T);
	const size_t chunk_bytes = (size_t)kStChunkPages * blk_bytes;
	const size_t region = attn_stream_region_bytes(G, hd, blk, sizeof(T));
	uint8_t* kbuf = sm_raw;                                   // [bufs][pages][blk][hd]
	uint8_t* vbuf = kbuf + (size_t)kStBufs * chunk_bytes;
	float* pv_red = reinterpret_cast<float*>(sm_raw);         // [warps][G*hd] after the last chunk
	float* s_s = reinterpret_cast<float*>(sm_raw + region);  // [G][CT]
	float* m_s = s_s + G * CT;                                // running max per head
	float* l_s = m_s + G;                                     // running sum per head
	float* al_s = l_s + G;                                    // this chunk's rescale factor
	uint64_t* bars = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(al_s + G + 2) + 7) & ~(uintptr_t)7);
	__shared__ int abort_flag;
	__shared__ int last_flag;

	const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
	const int d0 = lane * VPL;
	pdl_wait();
	pdl_trigger();
	const int slot = a.tok_slot[b];
	const int pos = a.tok_pos[b];
	const int ctx = pos + 1;
	const int n_pages = (ctx + blk - 1) / blk;
	const int pps = (n_pages + a.n_splits - 1) / a.n_splits;
	const int p_begin = split * pps;
	const int np = max(0, min(n_pages, p_begin + pps) - p_begin);
	const int n_chunks = (np + kStChunkPages - 1) / kStChunkPages;

	if (tid == 0) {
		abort_flag = 0;
		for (int i = 0; i < kStBufs; ++i) mbar_init(&bars[i], 1);
		mbar_fence_init();
	}
	if (tid < G) {
		m_s[tid] = -INFINITY;
		l_s[tid] = 0.0f;
	}
	__syncthreads();
	// one thread issues a chunk: every valid page's K and V block
	auto issue = [&](int c) {
		const int buf = c % kStBufs;
		const int q0 = c * kStChunkPages, q1 = min(np, q0 + kStChunkPages);
		uint32_t bytes = 0;
		for (int q = q0; q < q1; ++q) {
			const int page = a.block_table[(size_t)slot * a.pages_per_seq + p_begin + q];
			if (page >= 0 && page < a.max_pages) bytes += (uint32_t)(2 * blk_bytes);
		}
		mbar_arrive_expect_tx(&bars[buf], bytes);
		const uint64_t pol = policy_evict_first();
		for (int q = q0; q < q1; ++q) {
			const int page = a.block_table[(size_t)slot * a.pages_per_seq + p_begin + q];
			if (page < 0 || page >= a.max_pages) {
				report_err(a.err, kDevKvRange);
				continue; // its positions are masked below
			}
			const size_t off = (((size_t)page * a.KV + kvh) * blk) * hd;
			uint8_t* kd = kbuf + (size_t)buf * chunk_bytes + (size_t)(q - q0) * blk_bytes;
			uint8_t* vd = vbuf + (size_t)buf * chunk_bytes + (size_t)(q - q0) * blk_bytes;
			bulk_g2s(kd, reinterpret_cast<const T*>(a.kpool) + off, (uint32_t)blk_bytes, &bars[buf], pol);
			bulk_g2s(vd, reinterpret_cast<const T*>(a.vpool) + off, (uint32_t)blk_bytes, &bars[buf], pol);
		}
	};
	if (tid == 0)
		for (int c = 0; c < min(n_chunks, kStBufs); ++c) issue(c);

	float qr[G][VPL];
	{
		const T* qb = reinterpret_cast<const T*>(a.q) + (size_t)b * a.H * hd + (size_t)kvh * G * hd;
#pragma unroll
		for (int g = 0; g < G; ++g) load_vals_vec<T, VPL>(qb + (size_t)g * hd, d0, hd, qr[g]);
	}
	float acc[G][VPL];
#pragma unroll
	for (int g = 0; g < G; ++g)
#pragma unroll
		for (int j = 0; j < VPL; ++j) acc[g][j] = 0.0f;
	const int my_g = row_of_lane<G>(lane);
	const bool g_writer = (lane & (32 / G - 1)) == 0;

	for (int c = 0; c < n_chunks; ++c) {
		const int buf = c % kStBufs;
		if (!abort_flag && !mbar_wait(&bars[buf], (uint32_t)(c / kStBufs) & 1u, (volatile int*)&abort_flag, a.err))
			abort_flag = 1;
		const T* kc = reinterpret_cast<const T*>(kbuf + (size_t)buf * chunk_bytes);
		const T* vc = reinterpret_cast<const T*>(vbuf + (size_t)buf * chunk_bytes);
		const int q0 = c * kStChunkPages;
		const int n_tok = (min(np, q0 + kStChunkPages) - q0) * blk;
		const int tok0 = (p_begin + q0) * blk;
		// scores of the chunk's positions (invalid pages and positions past the context: -inf)
		for (int t0 = warp * kAttnTokIlp; t0 < n_tok; t0 += kAttnWarps * kAttnTokIlp) {
			float kv[kAttnTokIlp][VPL];
#pragma unroll
			for (int u = 0; u < kAttnTokIlp; ++u) load_vals_vec<T, VPL>(kc + (size_t)min(t0 + u, n_tok - 1) * hd, d0, hd, kv[u]);
			float sc[kAttnTokIlp];
#pragma unroll
			for (int u = 0; u < kAttnTokIlp; ++u) {
				float p[G];
#pragma unroll
				for (int g = 0; g < G; ++g) {
					float s = 0.0f;
#pragma unroll
					for (int j = 0; j < VPL; ++j) s = fmaf(qr[g][j], kv[u][j], s);
					p[g] = s;
				}
				sc[u] = reduce_rows<G>(p, lane);
			}
#pragma unroll
			for (int u = 0; u < kAttnTokIlp; ++u) {
				const int t = t0 + u;
				if (g_writer && t < n_tok) {
					const int page = a.block_table[(size_t)slot * a.pages_per_seq + p_begin + q0 + t / blk];
					const bool ok = tok0 + t < ctx && page >= 0 && page < a.max_pages && !abort_flag;
					s_s[my_g * CT + t] = ok ? sc[u] * a.scale : -INFINITY;
				}
			}
		}
		__syncthreads();
		// online softmax over the chunk, one warp per head
		for (int g = warp; g < G; g += kAttnWarps) {
			float mx = -INFINITY;
			for (int t = lane; t < n_tok; t += 32) mx = fmaxf(mx, s_s[g * CT + t]);
			mx = warp_max(mx);
			const float m_old = m_s[g];
			const float m_new = fmaxf(m_old, mx);
			float sum = 0.0f;
			for (int t = lane; t < n_tok; t += 32) {
				const float e = (m_new == -INFINITY) ? 0.0f : expf(s_s[g * CT + t] - m_new);
				s_s[g * CT + t] = e;
				sum += e;
			}
			sum = warp_sum(sum);
			if (lane == 0) {
				const float alpha = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
				al_s[g] = alpha;
				l_s[g] = l_s[g] * alpha + sum;
				m_s[g] = m_new;
			}
		}
		__syncthreads();
		// acc = acc * alpha + P.V over this warp's positions of the chunk
#pragma unroll
		for (int g = 0; g < G; ++g) {
			const float al = al_s[g];
#pragma unroll
			for (int j = 0; j < VPL; ++j) acc[g][j] *= al;
		}
		for (int t0 = warp * kAttnTokIlp; t0 < n_tok; t0 += kAttnWarps * kAttnTokIlp) {
			float vv[kAttnTokIlp][VPL], pp[kAttnTokIlp][G];
#pragma unroll
			for (int u = 0; u < kAttnTokIlp; ++u) {
				const bool in = t0 + u < n_tok;
				const int t = in ? t0 + u : n_tok - 1;
				load_vals_vec<T, VPL>(vc + (size_t)t * hd, d0, hd, vv[u]);
#pragma unroll
				for (int g = 0; g < G; ++g) pp[u][g] = in ? s_s[g * CT + t] : 0.0f;
			}
#pragma unroll
			for (int u = 0; u < kAttnTokIlp; ++u)
#pragma unroll
				for (int g = 0; g < G; ++g)
#pragma unroll
					for (int j = 0; j < VPL; ++j) acc[g][j] = fmaf(pp[u][g], vv[u][j], acc[g][j]);
		}
		__syncthreads(); // the chunk's buffer and the scores are free
		if (tid == 0 && c + kStBufs < n_chunks) issue(c + kStBufs);
	}

	// split partials (cross-warp sum through the idle page buffers)
#pragma unroll
	for (int g = 0; g < G; ++g)
#pragma unroll
		for (int j = 0; j < VPL; ++j)
			if (d0 + j < hd) pv_red[(size_t)warp * G * hd + g * hd + d0 + j] = acc[g][j];
	__syncthreads();
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
	// combine the splits of this (token, KV head): weights exp(m_s - M) / L per head
	T* ob = reinterpret_cast<T*>(a.out) + (size_t)b * a.H * hd;
	for (int o = tid; o < G * hd; o += kAttnThreads) {
		const int g = o / hd, i = o % hd;
		const float* ph = a.part + ((size_t)b * a.H + kvh * G + g) * a.n_splits * hd2;
		float M = -INFINITY;
		for (int s = 0; s < a.n_splits; ++s) M = fmaxf(M, __ldcg(ph + (size_t)s * hd2 + hd));
		float L = 0.0f, v = 0.0f;
		for (int s = 0; s < a.n_splits; ++s) {
			const float ms = __ldcg(ph + (size_t)s * hd2 + hd);
			const float w = (ms == -INFINITY) ? 0.0f : expf(ms - M);
			L = fmaf(w, __ldcg(ph + (size_t)s * hd2 + hd + 1), L);
			v = fmaf(w, __ldcg(ph + (size_t)s * hd2 + i), v);
		}
		Store<T>::put(ob + (size_t)(kvh * G + g) * hd + i, L > 0.0f ? v / L : 0.0f);
	}
	if (tid == 0) a.counters[b * a.KV + kvh] = 0u;
}

template <typename T>
inline AttnKernel<T> attn_decode_stream_kernel(int G, int hd)
{
	const int vpl = attn_vpl(hd);
#define INF_ATTN_CASE(g, v) \
	if (G == g && vpl == v) return k_attn_decode_stream<T, g, v>;
#define INF_ATTN_G(g) INF_ATTN_CASE(g, 1) INF_ATTN_CASE(g, 2) INF_ATTN_CASE(g, 4) INF_ATTN_CASE(g, 8)
	INF_ATTN_G(1) INF_ATTN_G(2) INF_ATTN_G(4) INF_ATTN_G(8)
#undef INF_ATTN_G
#undef INF_ATTN_CASE
	return nullptr;
}

} // namespace inf
