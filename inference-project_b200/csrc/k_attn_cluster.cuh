// Batch-1 decode attention for contexts whose pages fit the shared memory of one thread-block
// cluster (flash-decoding with the split combine in distributed shared memory).
//
// Grid (splits, kv_heads, tokens), cluster (splits, 1, 1): the CTAs of a cluster are the
// splits of one (token, KV head) and each owns a contiguous range of at most max_pages_split
// pages.  Compared with the split-K kernel (k_attn_decode.cuh), whose combine goes through
// global scratch, a fence and an atomic ticket, this kernel keeps every step after the
// dependency wait on chip:
//   * every page of the split -- the current one included -- is fetched with 1-D bulk copies
//     before griddepcontrol.wait.  Only one row of the current page, position pos, is being
//     written by the QKV kernel of this step; after the wait it is replaced with the row read
//     from global memory (256 bytes of K and of V at head_dim 128, an L2 hit);
//   * scores, softmax and P.V as in the split-K kernel, the partial (max, sum, acc) left in
//     shared memory;
//   * one cluster barrier, then CTA r combines its 1/splits share of the G x head_dim outputs
//     by reading every split's partials through distributed shared memory (ld.shared::cluster),
//     and a second barrier keeps each CTA's shared memory alive until its peers are done.
// Positions past the context are masked.  Every CTA reaches both barriers on every path (no
// early return); the page waits are bounded and a timeout only masks the data.
#pragma once

#include "common.cuh"
#include "k_attn_decode.cuh" // AttnDecodeArgs, kAttn* constants, reduce_rows

namespace inf {

constexpr int kAttnClMaxSplits = 16;       // cluster size (16 needs the non-portable opt-in)
constexpr int kAttnClMaxPages = 16;        // mbarriers per CTA
constexpr size_t kAttnClSmemMax = 112 * 1024; // leaves room for a projection CTA on the same SM
static_assert(kAttnClSmemMax + 2 * kSmemReservedPerCta + kGemvSmemFloor <= kSmemPerSm,
              "a cluster-attention CTA and a projection CTA share an SM");

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank)
{
	uint32_t r;
	asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
	return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr)
{
	float v;
	asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
	return v;
}
__device__ __forceinline__ void cluster_sync_all()
{
	asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank()
{
	uint32_t r;
	asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
	return r;
}

// VPL consecutive head_dim values of one row as floats, one vector load when they are whole
template <typename T, int VPL>
__device__ __forceinline__ void load_vals_vec(const T* row, int d0, int hd, float (&v)[VPL])
{
	if (d0 + VPL <= hd) {
		if constexpr (sizeof(T) == 2 && VPL == 2) {
			const uint32_t u = *reinterpret_cast<const uint32_t*>(row + d0);
			v[0] = bf16_lo(u); v[1] = bf16_hi(u);
			return;
		} else if constexpr (sizeof(T) == 2 && VPL == 4) {
			const uint2 u = *reinterpret_cast<const uint2*>(row + d0);
			v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
			return;
		} else if constexpr (sizeof(T) == 2 && VPL == 8) {
			const uint4 u = *reinterpret_cast<const uint4*>(row + d0);
			unpack_unit(u, v, (const bf16*)nullptr);
			return;
		} else if constexpr (sizeof(T) == 4 && VPL == 2) {
			const float2 f = *reinterpret_cast<const float2*>(row + d0);
			v[0] = f.x; v[1] = f.y;
			return;
		} else if constexpr (sizeof(T) == 4 && VPL % 4 == 0) {
#pragma unroll
			for (int j = 0; j < VPL; j += 4) {
				const float4 f = *reinterpret_cast<const float4*>(row + d0 + j);
				v[j] = f.x; v[j + 1] = f.y; v[j + 2] = f.z; v[j + 3] = f.w;
			}
			return;
		}
	}
#pragma unroll
	for (int j = 0; j < VPL; ++j) v[j] = (d0 + j < hd) ? Store<T>::get(row + d0 + j) : 0.0f;
}

// shared-memory layout, host and device alike
struct AttnClLayout {
	size_t region, s_s, part, ml, w, bars, total;
};
__host__ __device__ inline AttnClLayout attn_cl_layout(int G, int hd, int blk, size_t esz, int max_pages_split, int n_splits)
{
	AttnClLayout L;
	size_t r = 2 * (size_t)max_pages_split * blk * hd * esz;
	const size_t pv = (size_t)kAttnWarps * G * hd * sizeof(float);
	L.region = ((r > pv ? r : pv) + 15) & ~(size_t)15;
	L.s_s = L.region;                                                  // [G][max_pages_split * blk]
	L.part = L.s_s + (((size_t)G * max_pages_split * blk * sizeof(float) + 15) & ~(size_t)15); // [G][hd]
	L.ml = L.part + (((size_t)G * hd * sizeof(float) + 15) & ~(size_t)15); // m[G], l[G]
	L.w = L.ml + (((size_t)2 * G * sizeof(float) + 15) & ~(size_t)15); // [G][n_splits]
	L.bars = L.w + (((size_t)G * n_splits * sizeof(float) + 15) & ~(size_t)15);
	L.total = L.bars + kAttnClMaxPages * sizeof(uint64_t);
	return L;
}

template <typename T, int G, int VPL>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode_cl(const AttnDecodeArgs a)
{
	extern __shared__ __align__(128) uint8_t sm_raw[];
	const int kvh = blockIdx.y, b = blockIdx.z;
	const int split = (int)cluster_rank(); // gridDim.x == cluster size == n_splits
	const int CS = a.n_splits;
	const int hd = a.hd, blk = a.blk;
	const size_t blk_bytes = (size_t)blk * hd * sizeof(T);
	const int max_tok = a.max_pages_split * blk;
	const AttnClLayout Ly = attn_cl_layout(G, hd, blk, sizeof(T), a.max_pages_split, CS);
	uint8_t* kbuf = sm_raw;                                  // [max_pages_split][blk][hd]
	uint8_t* vbuf = kbuf + (size_t)a.max_pages_split * blk_bytes;
	float* pv_red = reinterpret_cast<float*>(sm_raw);        // [warps][G*hd] after P.V
	float* s_s = reinterpret_cast<float*>(sm_raw + Ly.s_s);
	float* part_s = reinterpret_cast<float*>(sm_raw + Ly.part);
	float* m_s = reinterpret_cast<float*>(sm_raw + Ly.ml);
	float* l_s = m_s + G;
	float* w_s = reinterpret_cast<float*>(sm_raw + Ly.w);
	uint64_t* bars = reinterpret_cast<uint64_t*>(sm_raw + Ly.bars);
	__shared__ int abort_flag;

	const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
	const int d0 = lane * VPL;
	// slot, position and block table are written by the host before the step
	const int slot = a.tok_slot[b];
	const int pos = a.tok_pos[b];
	const int ctx = pos + 1;
	const int n_pages = (ctx + blk - 1) / blk;
	const int pps = (n_pages + CS - 1) / CS;
	const int p_begin = split * pps;
	const int p_end = min(n_pages, p_begin + pps);
	const int np = max(0, min(p_end - p_begin, a.max_pages_split));
	const int cur_j = pos / blk - p_begin; // index of the current page in this split, if it holds it
	const int n_tok = np * blk;
	const int tok0 = p_begin * blk;

	if (tid == 0) {
		abort_flag = 0;
		for (int j = 0; j < np; ++j) mbar_init(&bars[j], 1);
		mbar_fence_init();
	}
	__syncthreads();
	if (tid < np) {
		const int page = a.block_table[(size_t)slot * a.pages_per_seq + p_begin + tid];
		if (page < 0 || page >= a.max_pages) {
			report_err(a.err, kDevKvRange);
			abort_flag = 1;
			mbar_arrive(&bars[tid]);
		} else {
			const size_t off = (((size_t)page * a.KV + kvh) * blk) * hd;
			mbar_arrive_expect_tx(&bars[tid], (uint32_t)(2 * blk_bytes));
			const uint64_t pol = policy_evict_first();
			bulk_g2s(kbuf + tid * blk_bytes, reinterpret_cast<const T*>(a.kpool) + off, (uint32_t)blk_bytes, &bars[tid], pol);
			bulk_g2s(vbuf + tid * blk_bytes, reinterpret_cast<const T*>(a.vpool) + off, (uint32_t)blk_bytes, &bars[tid], pol);
		}
	}
	pdl_wait();
	pdl_trigger();

	// the row of this step's token, written by the QKV kernel, replaces the early copy's
	if (cur_j >= 0 && cur_j < np && warp == 0) {
		const int page = a.block_table[(size_t)slot * a.pages_per_seq + pos / blk];
		const int r = pos % blk;
		float kr[VPL], vr[VPL];
		const bool good = page >= 0 && page < a.max_pages;
		if (good) {
			const size_t off = ((((size_t)page * a.KV + kvh) * blk) + r) * hd;
			load_vals_vec<T, VPL>(reinterpret_cast<const T*>(a.kpool) + off, d0, hd, kr);
			load_vals_vec<T, VPL>(reinterpret_cast<const T*>(a.vpool) + off, d0, hd, vr);
		}
		if (!mbar_wait(&bars[cur_j], 0, (volatile int*)&abort_flag, a.err)) abort_flag = 1;
		if (good) {
			T* kd = reinterpret_cast<T*>(kbuf + cur_j * blk_bytes) + (size_t)r * hd;
			T* vd = reinterpret_cast<T*>(vbuf + cur_j * blk_bytes) + (size_t)r * hd;
#pragma unroll
			for (int j = 0; j < VPL; ++j)
				if (d0 + j < hd) {
					Store<T>::put(kd + d0 + j, kr[j]);
					Store<T>::put(vd + d0 + j, vr[j]);
				}
		}
	}

	// the G queries of this KV head, this lane's head_dim slice, in registers
	float qr[G][VPL];
	{
		const T* qb = reinterpret_cast<const T*>(a.q) + (size_t)b * a.H * hd + (size_t)kvh * G * hd;
#pragma unroll
		for (int g = 0; g < G; ++g) load_vals_vec<T, VPL>(qb + (size_t)g * hd, d0, hd, qr[g]);
	}
	__syncthreads(); // the patched row is visible to every warp

	// ---- scores
	const int my_g = row_of_lane<G>(lane);
	const bool g_writer = (lane & (32 / G - 1)) == 0;
	int waited = 0;
	for (int t0 = warp * kAttnTokIlp; t0 < n_tok; t0 += kAttnWarps * kAttnTokIlp) {
		for (const int need = min(np, (t0 + kAttnTokIlp - 1) / blk + 1); waited < need; ++waited)
			if (!abort_flag && !mbar_wait(&bars[waited], 0, (volatile int*)&abort_flag, a.err)) abort_flag = 1;
		float kv[kAttnTokIlp][VPL];
#pragma unroll
		for (int u = 0; u < kAttnTokIlp; ++u) {
			const int t = min(t0 + u, n_tok - 1);
			load_vals_vec<T, VPL>(reinterpret_cast<const T*>(kbuf) + (size_t)t * hd, d0, hd, kv[u]);
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
			load_vals_vec<T, VPL>(reinterpret_cast<const T*>(vbuf) + (size_t)t * hd, d0, hd, vv[u]);
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
	__syncthreads(); // every warp is done with the page buffers
#pragma unroll
	for (int g = 0; g < G; ++g)
#pragma unroll
		for (int j = 0; j < VPL; ++j)
			if (d0 + j < hd) pv_red[(size_t)warp * G * hd + g * hd + d0 + j] = acc[g][j];
	__syncthreads();
	for (int o = tid; o < G * hd; o += kAttnThreads) {
		float v = 0.0f;
#pragma unroll
		for (int w = 0; w < kAttnWarps; ++w) v += pv_red[(size_t)w * G * hd + o];
		part_s[o] = v;
	}

	// ---- combine across the cluster: CTA `split` owns outputs [o0, o1) of the G x hd block
	cluster_sync_all();
	const uint32_t ml_addr = smem_addr(m_s), part_addr = smem_addr(part_s);
	for (int g = warp; g < G; g += kAttnWarps) {
		float m = -INFINITY, l = 0.0f;
		if (lane < CS) {
			m = ld_cluster_f32(cluster_map(ml_addr + 4u * g, lane));
			l = ld_cluster_f32(cluster_map(ml_addr + 4u * (G + g), lane));
		}
		const float M = warp_max(m);
		const float w = (m == -INFINITY) ? 0.0f : expf(m - M);
		const float L = warp_sum(w * l);
		if (lane < CS) w_s[g * CS + lane] = L > 0.0f ? w / L : 0.0f;
	}
	__syncthreads();
	const int per = (G * hd + CS - 1) / CS;
	const int o0 = split * per, o1 = min(G * hd, o0 + per);
	T* ob = reinterpret_cast<T*>(a.out) + (size_t)b * a.H * hd + (size_t)kvh * G * hd;
	for (int o = o0 + tid; o < o1; o += kAttnThreads) {
		const int g = o / hd;
		float pv[kAttnClMaxSplits]; // every remote load in flight before the sum
#pragma unroll
		for (int r = 0; r < kAttnClMaxSplits; ++r) pv[r] = r < CS ? ld_cluster_f32(cluster_map(part_addr + 4u * o, r)) : 0.0f;
		float v = 0.0f;
#pragma unroll
		for (int r = 0; r < kAttnClMaxSplits; ++r)
			if (r < CS) v = fmaf(w_s[g * CS + r], pv[r], v);
		Store<T>::put(ob + o, v);
	}
	cluster_sync_all(); // peers may still be reading this CTA's partials
}

// Pages per split when `splits` CTAs (one cluster) cover a context of up to pages_per_seq
// pages, or 0 when a split's pages and partials do not fit the shared-memory limit.
inline int attn_cl_pages_per_split(int splits, int pages_per_seq, int blk, int hd, size_t esz, int G)
{
	const int mp = (pages_per_seq + splits - 1) / splits;
	if (mp > kAttnClMaxPages) return 0;
	if (attn_cl_layout(G, hd, blk, esz, mp, splits).total > kAttnClSmemMax) return 0;
	return mp;
}

template <typename T>
inline AttnKernel<T> attn_decode_cl_kernel(int G, int hd)
{
	const int vpl = attn_vpl(hd);
#define INF_ATTN_CASE(g, v) \
	if (G == g && vpl == v) return k_attn_decode_cl<T, g, v>;
#define INF_ATTN_G(g) INF_ATTN_CASE(g, 1) INF_ATTN_CASE(g, 2) INF_ATTN_CASE(g, 4) INF_ATTN_CASE(g, 8)
	INF_ATTN_G(1) INF_ATTN_G(2) INF_ATTN_G(4) INF_ATTN_G(8)
#undef INF_ATTN_G
#undef INF_ATTN_CASE
	return nullptr;
}

} // namespace inf
