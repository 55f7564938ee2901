// Batch-1 decode attention on the tensor cores: one thread-block cluster per (token, KV head),
// the same split of the context as the SIMT cluster kernel (k_attn_cluster.cuh) -- CTA r of a
// cluster of CS owns pages [r*pps, (r+1)*pps) of the sequence -- with the arithmetic on
// mma.m16n8k16 and a one-barrier combine:
//   * before griddepcontrol.wait, lanes of warp 0 read the split's page ids and load every page
//     of K and V with 4-D TMA boxes (64 head dims x 16 positions x 1 head x 1 page,
//     SWIZZLE_128B, one mbarrier per page), so the fragments come from ldmatrix without bank
//     conflicts;
//   * warp w owns pages w and w + 8 of the split.  After the wait it patches the current
//     position's K and V row (written by this step's QKV kernel after the early copy) into its
//     page, computes S = Q.K^T with the G query heads as the rows of the A tile (rows >= G are
//     zero), the softmax over its positions in log2 units, and O += P.V with P split into three
//     bf16 parts (high, middle, low: three MMAs), so the weights keep the ~24 bits of the fp32
//     weights of the SIMT kernels;
//   * the eight warps merge (max, sum, O) through shared memory into the split's partial;
//   * combine: CTA c owns outputs [c*per, (c+1)*per) of the G x head_dim block.  Every CTA
//     stores each of its partial values straight into the owner's inbox (st.shared::cluster),
//     with the (max, sum) of the heads the owner needs; one release/acquire cluster barrier,
//     then each owner combines from its own shared memory (per-source weights by one warp per
//     head, then eight threads per output).  A relaxed arrive at entry, waited
//     before the first remote store, guarantees every peer is running.
// Positions past the context and pages with invalid ids are masked (the id error is recorded);
// every CTA reaches both barrier phases on every path; the page waits are bounded, and a CTA
// that gave up on a page waits (again bounded) for its copies before it exits.
#pragma once

#include "common.cuh"
#include "k_attn_cluster.cuh"    // cluster helpers, kAttnClMaxSplits, kAttnClSmemMax
#include "k_attn_decode_mma.cuh" // mma_bf16_16816, ldsm_x4(_trans), pack_bf16
#include "k_attn_prefill_tc.cuh" // tma_load_4d

namespace inf {

constexpr int kClTcWarps = 8;
constexpr int kClTcThreads = kClTcWarps * 32;
constexpr int kClTcMaxPages = 2 * kClTcWarps; // pages of 16 positions per split (two per warp)

__device__ __forceinline__ void cluster_arrive_relaxed()
{
	asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release()
{
	asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire()
{
	asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v)
{
	asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Shared-memory layout (offsets from the 1024-byte aligned base), host and device alike.
struct AttnClTcLayout {
	size_t inbox, inbox_ml, bars, total;
};
__host__ __device__ inline size_t attn_cltc_page_bytes(int hd) { return (size_t)(hd / 64) * 2048; }
__host__ __device__ inline int attn_cltc_per(int G, int hd, int cs) { return (G * hd + cs - 1) / cs; }
__host__ __device__ inline AttnClTcLayout attn_cltc_layout(int G, int hd, int max_pages_split, int cs)
{
	AttnClTcLayout L;
	const size_t pages = 2 * (size_t)max_pages_split * attn_cltc_page_bytes(hd);
	const size_t merge = (size_t)kClTcWarps * G * hd * 4 + (size_t)kClTcWarps * G * 2 * 4;
	L.inbox = ((pages > merge ? pages : merge) + 15) & ~(size_t)15;             // [cs][per]
	L.inbox_ml = L.inbox + (((size_t)cs * attn_cltc_per(G, hd, cs) * 4 + 15) & ~(size_t)15); // [cs][G][2]
	L.bars = L.inbox_ml + (((size_t)cs * G * 2 * 4 + 15) & ~(size_t)15);
	L.total = 1024 + L.bars + (size_t)max_pages_split * sizeof(uint64_t); // + alignment slack
	return L;
}

template <int G, int HD>
__global__ void __launch_bounds__(kClTcThreads)
    k_attn_decode_clt(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, const AttnDecodeArgs a)
{
	static_assert(G >= 1 && G <= 8 && (HD == 64 || HD == 128), "rows / head_dim");
	constexpr int kHalves = HD / 64;
	constexpr uint32_t kPageBytes = kHalves * 2048u;
	extern __shared__ __align__(16) uint8_t clt_sm_base[];
	// 1024-byte aligned (the SWIZZLE_128B atoms); the layout's total includes the slack
	uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(clt_sm_base) + 1023) & ~(uintptr_t)1023);
	const int kvh = blockIdx.y, b = blockIdx.z;
	const int split = (int)cluster_rank(); // gridDim.x == cluster size == n_splits
	const int CS = a.n_splits;
	const int mp = a.max_pages_split;
	const AttnClTcLayout Ly = attn_cltc_layout(G, HD, mp, CS);
	uint8_t* kbuf = sm;                                   // [mp][kHalves][16 rows][128 B]
	uint8_t* vbuf = sm + (size_t)mp * kPageBytes;
	float* inbox = reinterpret_cast<float*>(sm + Ly.inbox);
	float* inbox_ml = reinterpret_cast<float*>(sm + Ly.inbox_ml);
	uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ly.bars);
	__shared__ int abort_flag;
	__shared__ int page_ok[kClTcMaxPages];

	const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
	const int gr = lane >> 2, gc = (lane & 3) * 2; // fragment row (query head), column pair
	const int mi = lane >> 3, mr = lane & 7;       // the ldmatrix matrix and row this lane addresses
	// slot, position and block table are written by the host before the step
	const int slot = a.tok_slot[b];
	const int pos = a.tok_pos[b];
	const int ctx = pos + 1;
	const int n_pages = (ctx + 15) >> 4;
	const int pps = (n_pages + CS - 1) / CS;
	const int p_begin = split * pps;
	const int np = max(0, min(min(n_pages, p_begin + pps) - p_begin, min(mp, kClTcMaxPages)));
	const int cur_j = (pos >> 4) - p_begin; // the current page's index in this split, if it holds it

	if (tid == 0) {
		abort_flag = 0;
		for (int j = 0; j < np; ++j) mbar_init(&bars[j], 1);
		mbar_fence_init();
	}
	cluster_arrive_relaxed(); // phase 1: this CTA runs; waited before the first remote store
	__syncthreads();
	if (tid < np) {
		const int pidx = p_begin + tid; // a position past the block-table row is an invalid page
		const int page = pidx < a.pages_per_seq ? a.block_table[(size_t)slot * a.pages_per_seq + pidx] : -1;
		const bool ok = page >= 0 && page < a.max_pages;
		page_ok[tid] = ok;
		if (!ok) {
			report_err(a.err, kDevKvRange);
			mbar_arrive(&bars[tid]);
		} else {
			mbar_arrive_expect_tx(&bars[tid], 2 * kPageBytes);
			const uint64_t pol = policy_evict_first();
#pragma unroll
			for (int h = 0; h < kHalves; ++h) {
				tma_load_4d(kbuf + (size_t)tid * kPageBytes + h * 2048, &tm_k, h * 64, 0, kvh, page, &bars[tid], pol);
				tma_load_4d(vbuf + (size_t)tid * kPageBytes + h * 2048, &tm_v, h * 64, 0, kvh, page, &bars[tid], pol);
			}
		}
	}
	const int cur_page = (cur_j >= 0 && cur_j < np && (pos >> 4) < a.pages_per_seq)
	                         ? a.block_table[(size_t)slot * a.pages_per_seq + (pos >> 4)]
	                         : -1;
	pdl_wait();
	pdl_trigger();

	// the G queries as A fragments: row gr, columns gc.. (a0) and gc+8.. (a2); rows gr + 8 are zero
	uint32_t qa[HD / 16][2];
	{
		const uint32_t* qrow =
		    reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint16_t*>(a.q) + (size_t)b * a.H * HD + ((size_t)kvh * G + gr) * HD);
#pragma unroll
		for (int ks = 0; ks < HD / 16; ++ks) {
			qa[ks][0] = gr < G ? qrow[(ks * 16 + gc) >> 1] : 0u;
			qa[ks][1] = gr < G ? qrow[(ks * 16 + gc + 8) >> 1] : 0u;
		}
	}
	__syncthreads(); // page_ok

	const float sl2 = a.scale * 1.4426950408889634f;
	float s[2][2][2]; // [page of the warp][8-position tile][column]: row gr only
	int mine = 0;     // pages this warp owns
#pragma unroll
	for (int u = 0; u < 2; ++u) {
		const int j = warp + u * kClTcWarps;
		if (j >= np) break;
		mine = u + 1;
		if (!abort_flag && !mbar_wait(&bars[j], 0, (volatile int*)&abort_flag, a.err)) abort_flag = 1;
		uint8_t* kp = kbuf + (size_t)j * kPageBytes;
		if (j == cur_j && cur_page >= 0 && cur_page < a.max_pages && page_ok[j]) {
			// 8 bytes of the row per lane: byte b8 = lane * 8 of the K and of the V row
			const int r = pos & 15, b8 = lane * 8;
			if (b8 < HD * 2) {
				const size_t off = ((((size_t)cur_page * a.KV + kvh) * 16) + r) * HD * 2 + b8;
				const uint2 kr = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(a.kpool) + off);
				const uint2 vr = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(a.vpool) + off);
				const uint32_t o = page_sw_off(r, (b8 & 127) >> 4, b8 >> 7) + (b8 & 15);
				*reinterpret_cast<uint2*>(kp + o) = kr;
				*reinterpret_cast<uint2*>(vbuf + (size_t)j * kPageBytes + o) = vr;
			}
			__syncwarp();
		}
		float acc[2][4];
#pragma unroll
		for (int nt = 0; nt < 2; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
		const uint32_t kc = smem_u32(kp);
		const int krow = (mi >> 1) * 8 + mr;
#pragma unroll
		for (int ks = 0; ks < HD / 16; ++ks) {
			uint32_t b00, b01, b10, b11;
			ldsm_x4(kc + page_sw_off(krow, (ks & 3) * 2 + (mi & 1), ks >> 2), b00, b01, b10, b11);
			const uint32_t af[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
			mma_bf16_16816(acc[0], af, b00, b01);
			mma_bf16_16816(acc[1], af, b10, b11);
		}
		const int tok0 = (p_begin + j) * 16;
		const bool pg = page_ok[j] && !abort_flag;
#pragma unroll
		for (int nt = 0; nt < 2; ++nt)
#pragma unroll
			for (int c = 0; c < 2; ++c)
				s[u][nt][c] = (pg && tok0 + nt * 8 + gc + c < ctx) ? acc[nt][c] * sl2 : -INFINITY;
	}
	// the row's max over the warp's positions (the four lanes of a quad share a row)
	float mx = -INFINITY;
#pragma unroll
	for (int u = 0; u < 2; ++u)
		if (u < mine)
#pragma unroll
			for (int nt = 0; nt < 2; ++nt) mx = fmaxf(mx, fmaxf(s[u][nt][0], s[u][nt][1]));
	mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
	mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));

	float o[HD / 8][4];
#pragma unroll
	for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
	float l = 0.0f;
#pragma unroll
	for (int u = 0; u < 2; ++u) {
		if (u >= mine) break;
		const int j = warp + u * kClTcWarps;
		float p[2][2];
#pragma unroll
		for (int nt = 0; nt < 2; ++nt)
#pragma unroll
			for (int c = 0; c < 2; ++c) {
				p[nt][c] = (mx == -INFINITY) ? 0.0f : exp2f(s[u][nt][c] - mx);
				l += p[nt][c];
			}
		// P = hi + mid + lo, each bf16 (the remainder of the previous parts, rounded): ~24 bits,
		// the fp32 weights of the SIMT kernels.  The A fragments of one 16-position step (rows
		// gr + 8 zero).
		uint32_t ph[4] = {0u, 0u, 0u, 0u}, pm[4] = {0u, 0u, 0u, 0u}, pl[4] = {0u, 0u, 0u, 0u};
#pragma unroll
		for (int nt = 0; nt < 2; ++nt) {
			const float x0 = p[nt][0], x1 = p[nt][1];
			const uint32_t hi = pack_bf16(x0, x1);
			const float r0 = x0 - __uint_as_float(hi << 16), r1 = x1 - __uint_as_float(hi & 0xFFFF0000u);
			const uint32_t mid = pack_bf16(r0, r1);
			ph[2 * nt] = hi;
			pm[2 * nt] = mid;
			pl[2 * nt] = pack_bf16(r0 - __uint_as_float(mid << 16), r1 - __uint_as_float(mid & 0xFFFF0000u));
		}
		const uint32_t vc = smem_u32(vbuf + (size_t)j * kPageBytes);
		const int vrow = (mi & 1) * 8 + mr;
#pragma unroll
		for (int dt = 0; dt < HD / 8; dt += 2) {
			const int d16 = dt + (mi >> 1); // 8-dim chunk over head_dim
			uint32_t b0, b1, c0, c1;
			ldsm_x4_trans(vc + page_sw_off(vrow, d16 & 7, d16 >> 3), b0, b1, c0, c1);
			mma_bf16_16816(o[dt], pl, b0, b1); // smallest part first
			mma_bf16_16816(o[dt + 1], pl, c0, c1);
			mma_bf16_16816(o[dt], pm, b0, b1);
			mma_bf16_16816(o[dt + 1], pm, c0, c1);
			mma_bf16_16816(o[dt], ph, b0, b1);
			mma_bf16_16816(o[dt + 1], ph, c0, c1);
		}
	}
	l += __shfl_xor_sync(0xFFFFFFFFu, l, 1);
	l += __shfl_xor_sync(0xFFFFFFFFu, l, 2);

	// a CTA that gave up on a page lets its copies land before the page region is reused
	if (abort_flag && tid < np) {
		const uint64_t t0 = global_timer_ns();
		while (!mbar_try_wait(&bars[tid], 0) && global_timer_ns() - t0 < kWaitLimitNs) {
		}
	}
	__syncthreads(); // every warp is done with the page buffers

	// merge the warps: (max, sum, O) of each row through shared memory
	float* mo = reinterpret_cast<float*>(sm);       // [warps][G][HD]
	float* mlw = mo + (size_t)kClTcWarps * G * HD;   // [warps][G][2]
	if (gr < G) {
		float* row = mo + ((size_t)warp * G + gr) * HD + gc;
#pragma unroll
		for (int dt = 0; dt < HD / 8; ++dt) {
			row[dt * 8] = o[dt][0];
			row[dt * 8 + 1] = o[dt][1];
		}
		if ((lane & 3) == 0) {
			mlw[((size_t)warp * G + gr) * 2] = mx;
			mlw[((size_t)warp * G + gr) * 2 + 1] = l;
		}
	}
	__syncthreads();

	// the split's partial, pushed into the owners' inboxes
	cluster_wait_acquire(); // phase 1: every peer is running
	const int per = attn_cltc_per(G, HD, CS);
	const uint32_t inbox_a = smem_u32(inbox), inbox_ml_a = smem_u32(inbox_ml);
	for (int e = tid; e < G * HD; e += kClTcThreads) {
		const int g = e / HD, i = e - g * HD;
		float M = -INFINITY;
#pragma unroll
		for (int w = 0; w < kClTcWarps; ++w) M = fmaxf(M, mlw[((size_t)w * G + g) * 2]);
		float v = 0.0f, L = 0.0f;
#pragma unroll
		for (int w = 0; w < kClTcWarps; ++w) {
			const float mw = mlw[((size_t)w * G + g) * 2];
			const float wt = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
			v = fmaf(wt, mo[((size_t)w * G + g) * HD + i], v);
			L = fmaf(wt, mlw[((size_t)w * G + g) * 2 + 1], L);
		}
		const int c = e / per, k = e - c * per;
		st_cluster_f32(cluster_map(inbox_a + 4u * (uint32_t)(split * per + k), (uint32_t)c), v);
		if (k == 0 || i == 0) { // the first output of head g in c's range: g's (max, sum)
			st_cluster_f32(cluster_map(inbox_ml_a + 4u * (uint32_t)((split * G + g) * 2), (uint32_t)c), M);
			st_cluster_f32(cluster_map(inbox_ml_a + 4u * (uint32_t)((split * G + g) * 2 + 1), (uint32_t)c), L);
		}
	}
	cluster_arrive_release(); // phase 2: every partial is in its owner's inbox
	cluster_wait_acquire();

	// this CTA's outputs, combined from its own shared memory: first every source's weight for
	// the heads the CTA owns (one warp per head, lane r = source r), then 8 threads per output
	// sum every 8th source
	bf16* ob = reinterpret_cast<bf16*>(a.out) + (size_t)b * a.H * HD + (size_t)kvh * G * HD;
	const int e0 = split * per, e1 = min(G * HD, e0 + per);
	const int g0 = e0 / HD;
	const int nh = e1 > e0 ? (e1 - 1) / HD - g0 + 1 : 0;
	float* wts = mo; // [nh][CS]; the merge region is free after the barrier
	for (int gl = warp; gl < nh; gl += kClTcWarps) {
		const int g = g0 + gl;
		const float m = lane < CS ? inbox_ml[(lane * G + g) * 2] : -INFINITY;
		const float ls = lane < CS ? inbox_ml[(lane * G + g) * 2 + 1] : 0.0f;
		const float M = warp_max(m);
		const float w = (m == -INFINITY) ? 0.0f : exp2f(m - M);
		const float L = warp_sum(w * ls);
		if (lane < CS) wts[gl * CS + lane] = L > 0.0f ? w / L : 0.0f;
	}
	__syncthreads();
	constexpr int kTpo = 8; // threads per output
	const int sub = tid & (kTpo - 1);
	for (int base = 0; base < per; base += kClTcThreads / kTpo) {
		const int e = e0 + base + tid / kTpo;
		const bool in = e < e1;
		float v = 0.0f;
		if (in) {
			const int gl = e / HD - g0, k = e - e0;
			for (int r = sub; r < CS; r += kTpo) v = fmaf(wts[gl * CS + r], inbox[r * per + k], v);
		}
		v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
		v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
		v += __shfl_xor_sync(0xFFFFFFFFu, v, 4);
		if (in && sub == 0) Store<bf16>::put(ob + e, v);
	}
}

typedef void (*AttnClTcKernel)(CUtensorMap, CUtensorMap, AttnDecodeArgs);

// the instantiation for GQA group G (<= 8) and head_dim 64 / 128 (nullptr otherwise)
inline AttnClTcKernel attn_decode_cltc_kernel(int G, int hd)
{
#define INF_CT_CASE(g)                                               \
	if (G == g && hd == 64) return k_attn_decode_clt<g, 64>;     \
	if (G == g && hd == 128) return k_attn_decode_clt<g, 128>;
	INF_CT_CASE(1) INF_CT_CASE(2) INF_CT_CASE(4) INF_CT_CASE(8)
#undef INF_CT_CASE
	return nullptr;
}

// Pages per split when `splits` CTAs cover a context of up to pages_per_seq pages of 16
// positions, or 0 when a split's pages do not fit the shared-memory budget or the two pages per
// warp.
inline int attn_cltc_pages_per_split(int splits, int pages_per_seq, int hd, int G)
{
	const int mp = (pages_per_seq + splits - 1) / splits;
	if (mp > kClTcMaxPages) return 0;
	if (attn_cltc_layout(G, hd, mp, splits).total > kAttnClSmemMax) return 0;
	return mp;
}

} // namespace inf
