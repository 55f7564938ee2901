// Decode attention for batches of tokens on the tensor cores (bf16, head_dim 64 or 128).
//
// Grid (kv_heads, splits, tokens), or (kv_heads, 1, work units) where the host lists each unit's
// (token, split, splits of the token) (a page budget per unit, longest contexts first, so the
// CTAs that start last are short); a CTA covers a contiguous range of one token's pages.  Thread
// 0-127 read the split's page ids into shared memory once; then each of the four warps streams
// its own pages (q = warp, warp + 4, ...) through its own ring of kStBufs stages (one page of K
// and of V per stage, one mbarrier per stage, 4-D TMA boxes of 64 head dims x 16 positions x 1
// head x 1 page into SWIZZLE_128B atoms, so the K and V fragments come from ldmatrix (.x4 for
// K, .x4.trans for V) without bank conflicts); lane 0 refills a stage as soon as its warp is
// done with it, so no CTA-wide barrier paces the stream.  Pages of 16 positions only.
// The arithmetic is warp-level mma.m16n8k16 (bf16 in, fp32 out): the G query heads of the KV
// head are the rows of a 16-row A tile (rows >= G are zero); per page a warp computes S = Q.K^T
// (2 x head_dim/16 MMAs), keeps a per-row running max / sum (online softmax on the accumulator
// fragments; O is rescaled only when some row's max grew), turns its S fragments into the bf16
// A fragments of P (the C layout of two 8-column tiles is the A layout of one 16-deep step) and
// accumulates O += P.V (head_dim/8 MMAs).  At the end the four warps' (max, sum, O) are merged
// through shared memory into the split's partial, and the last CTA of each (token, KV head)
// combines the splits (atomic ticket, no spinning).
// P is rounded to bf16 for the P.V product (the SIMT kernels keep it in fp32).
#pragma once

#include "common.cuh"
#include "k_attn_decode.cuh"        // AttnDecodeArgs, AttnKernel, attn_vpl
#include "k_attn_decode_stream.cuh" // kStChunkPages, kStBufs, attn_stream_splits
#include "k_attn_prefill_tc.cuh"    // tma_load_4d (4-D boxes of the paged K/V pool)

namespace inf {

constexpr int kAmThreads = 128; // 4 warps, each streaming every 4th page of the split
constexpr int kAmUnitPagesMin = 16;  // pages of a work unit at least (host work list)
constexpr int kAmUnitSplitsMax = 32; // splits of one token at most (host work list)
static_assert(kAmThreads / 32 == kStChunkPages, "the region holds kStBufs pages of K and V per warp");

__host__ __device__ inline size_t attn_mma_region_bytes(int hd, int blk)
{
	const size_t ring = (size_t)kStBufs * 2 * kStChunkPages * blk * hd * 2;
	const size_t merge = (size_t)4 * 16 * hd * 4 + 4 * 16 * 2 * 4; // O, then (m, l) of every warp
	return ((ring > merge ? ring : merge) + 127) & ~(size_t)127;
}
// region, the split's page ids (at most pages_per_seq), one mbarrier per stage of each warp
inline size_t attn_mma_smem_bytes(int hd, int blk, int pages_per_seq)
{
	return 1024 + attn_mma_region_bytes(hd, blk) + (((size_t)pages_per_seq * 4 + 15) & ~(size_t)15) +
	       (kAmThreads / 32) * kStBufs * sizeof(uint64_t);
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
	asm volatile(
	    "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
	    : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
	    : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi)
{
	const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
	return *reinterpret_cast<const uint32_t*>(&b);
}
__device__ __forceinline__ uint32_t pack_raw_bf16(uint16_t lo, uint16_t hi) { return (uint32_t)lo | ((uint32_t)hi << 16); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3)
{
	asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
	             : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
	             : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3)
{
	asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
	             : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
	             : "r"(addr));
}
// Byte offset of 16-byte chunk c16 of row r (position) in half h of one page of K or V in
// shared memory: [head_dim / 64 halves][16 positions][128 bytes], each half two SWIZZLE_128B
// atoms (8 positions x 128 bytes) as the TMA box writes it.
__device__ __forceinline__ uint32_t page_sw_off(int r, int c16, int h)
{
	return (uint32_t)h * 2048u + (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c16 ^ (r & 7)) << 4));
}

template <int G, int HD>
__global__ void __launch_bounds__(kAmThreads)
    k_attn_decode_mma(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, const AttnDecodeArgs a)
{
	static_assert(G >= 1 && G <= 16 && (HD == 64 || HD == 128), "rows / head_dim");
	extern __shared__ __align__(1024) uint8_t sm_base[];
	// 1024-byte aligned: the TMA boxes are SWIZZLE_128B atoms
	uint8_t* sm_raw = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_base) + 1023) & ~(uintptr_t)1023);
	const int kvh = blockIdx.x;
	// (token, split, splits of that token): from the grid, or from the host's work list
	int b = blockIdx.z, split = blockIdx.y, ns = a.n_splits;
	if (a.units) {
		const int2 u = reinterpret_cast<const int2*>(a.units)[blockIdx.z];
		b = u.x;
		split = u.y & 0xFFFF;
		ns = u.y >> 16;
	}
	const int blk = a.blk; // 16 (the host checks)
	int* pg_s = reinterpret_cast<int*>(sm_raw + attn_mma_region_bytes(HD, blk)); // this split's page ids
	uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(pg_s) + (((size_t)a.pages_per_seq * 4 + 15) & ~(size_t)15));
	__shared__ int abort_flag;
	__shared__ int last_flag;

	const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
	const int gr = lane >> 2, gc = (lane & 3) * 2; // fragment row (and row + 8), column pair
	pdl_wait();
	pdl_trigger();
	const int slot = a.tok_slot[b];
	const int pos = a.tok_pos[b];
	const int ctx = pos + 1;
	const int n_pages = (ctx + blk - 1) / blk;
	const int pps = (n_pages + ns - 1) / ns;
	const int p_begin = split * pps;
	const int np = max(0, min(n_pages, p_begin + pps) - p_begin);

	if (tid == 0) {
		abort_flag = 0;
		for (int i = 0; i < (kAmThreads / 32) * kStBufs; ++i) mbar_init(&bars[i], 1);
		mbar_fence_init();
	}
	// page ids once into shared memory (invalid ids as -1): the chunk issue and the mask read them
	for (int q = tid; q < np; q += kAmThreads) {
		const int page = a.block_table[(size_t)slot * a.pages_per_seq + p_begin + q];
		const bool ok = page >= 0 && page < a.max_pages;
		if (!ok) report_err(a.err, kDevKvRange); // masked below
		pg_s[q] = ok ? page : -1;
	}
	__syncthreads();
	// this warp's pages q = warp + 4 i, i < n_mine, through its own ring
	constexpr uint32_t kPage = (HD / 64) * 2048u; // one page of K (or V)
	const int n_mine = np > warp ? (np - warp + 3) / 4 : 0;
	uint8_t* ring = sm_raw + (size_t)warp * kStBufs * 2 * kPage;
	uint64_t* wbar = bars + warp * kStBufs;
	auto issue = [&](int i) { // lane 0
		const int st = i % kStBufs;
		const int page = pg_s[warp + 4 * i];
		if (page < 0) {
			mbar_arrive(&wbar[st]);
			return;
		}
		mbar_arrive_expect_tx(&wbar[st], 2 * kPage);
		const uint64_t pol = policy_evict_first();
		uint8_t* dst = ring + (size_t)st * 2 * kPage;
#pragma unroll
		for (int h = 0; h < HD / 64; ++h) {
			tma_load_4d(dst + h * 2048, &tm_k, h * 64, 0, kvh, page, &wbar[st], pol);
			tma_load_4d(dst + kPage + h * 2048, &tm_v, h * 64, 0, kvh, page, &wbar[st], pol);
		}
	};
	int issued = 0;
	if (lane == 0)
		for (; issued < min(n_mine, kStBufs); ++issued) issue(issued);

	// Q as A fragments (rows gr and gr + 8; rows >= G are zero)
	uint32_t qa[HD / 16][4];
	{
		const uint16_t* qb = reinterpret_cast<const uint16_t*>(a.q) + (size_t)b * a.H * HD + (size_t)kvh * G * HD;
#pragma unroll
		for (int ks = 0; ks < HD / 16; ++ks) {
			const int c0 = ks * 16 + gc;
			const uint16_t* r0 = qb + (size_t)gr * HD;
			const uint16_t* r1 = qb + (size_t)(gr + 8) * HD;
			const bool v0 = gr < G, v1 = gr + 8 < G;
			qa[ks][0] = v0 ? pack_raw_bf16(r0[c0], r0[c0 + 1]) : 0u;
			qa[ks][1] = v1 ? pack_raw_bf16(r1[c0], r1[c0 + 1]) : 0u;
			qa[ks][2] = v0 ? pack_raw_bf16(r0[c0 + 8], r0[c0 + 9]) : 0u;
			qa[ks][3] = v1 ? pack_raw_bf16(r1[c0 + 8], r1[c0 + 9]) : 0u;
		}
	}
	float o[HD / 8][4];
#pragma unroll
	for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
	float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f; // rows gr, gr + 8 (l: this thread's share)
	const float sl2 = a.scale * 1.4426950408889634f;
	const int mi = lane >> 3, mr = lane & 7; // the ldmatrix matrix and row this lane addresses

	for (int i = 0; i < n_mine; ++i) {
		const int st = i % kStBufs;
		if (!abort_flag && !mbar_wait(&wbar[st], (uint32_t)(i / kStBufs) & 1u, (volatile int*)&abort_flag, a.err))
			abort_flag = 1;
		const int q = warp + 4 * i;
		const uint32_t kc = smem_u32(ring + (size_t)st * 2 * kPage), vc = kc + kPage;
		// S = Q.K^T for the page's 16 positions (two 8-position tiles); ldmatrix x4: matrices
		// (tile 0, dims +0..7), (tile 0, +8..15), (tile 1, +0..7), (tile 1, +8..15)
		float s[2][4];
#pragma unroll
		for (int nt = 0; nt < 2; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
		const int krow = (mi >> 1) * 8 + mr;
#pragma unroll
		for (int ks = 0; ks < HD / 16; ++ks) {
			uint32_t b00, b01, b10, b11;
			ldsm_x4(kc + page_sw_off(krow, (ks & 3) * 2 + (mi & 1), ks >> 2), b00, b01, b10, b11);
			mma_bf16_16816(s[0], qa[ks], b00, b01);
			mma_bf16_16816(s[1], qa[ks], b10, b11);
		}
		// scale (log2 units) and mask positions past the context or on invalid pages
		const int tok0 = (p_begin + q) * blk;
		const bool pg_ok = pg_s[q] >= 0 && !abort_flag;
		float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
		for (int nt = 0; nt < 2; ++nt)
#pragma unroll
			for (int j = 0; j < 2; ++j) {
				const bool ok = pg_ok && tok0 + nt * 8 + gc + j < ctx;
				s[nt][j] = ok ? s[nt][j] * sl2 : -INFINITY;
				s[nt][2 + j] = ok ? s[nt][2 + j] * sl2 : -INFINITY;
				mx0 = fmaxf(mx0, s[nt][j]);
				mx1 = fmaxf(mx1, s[nt][2 + j]);
			}
		// the row's max over the quad (the four lanes that hold one row)
		mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, 1));
		mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, 2));
		mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, 1));
		mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, 2));
		const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
		const float al0 = (m0 == -INFINITY) ? 0.0f : exp2f(m0 - n0);
		const float al1 = (m1 == -INFINITY) ? 0.0f : exp2f(m1 - n1);
		m0 = n0;
		m1 = n1;
		float ps[2][4];
#pragma unroll
		for (int nt = 0; nt < 2; ++nt)
#pragma unroll
			for (int j = 0; j < 2; ++j) {
				ps[nt][j] = (n0 == -INFINITY) ? 0.0f : exp2f(s[nt][j] - n0);
				ps[nt][2 + j] = (n1 == -INFINITY) ? 0.0f : exp2f(s[nt][2 + j] - n1);
			}
		uint32_t pa[4];
		pa[0] = pack_bf16(ps[0][0], ps[0][1]);
		pa[1] = pack_bf16(ps[0][2], ps[0][3]);
		pa[2] = pack_bf16(ps[1][0], ps[1][1]);
		pa[3] = pack_bf16(ps[1][2], ps[1][3]);
		// the sums add the rounded values, the weights the MMA applies
		float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
		for (int k = 0; k < 4; k += 2) {
			sum0 += __uint_as_float(pa[k] << 16) + __uint_as_float(pa[k] & 0xFFFF0000u);
			sum1 += __uint_as_float(pa[k + 1] << 16) + __uint_as_float(pa[k + 1] & 0xFFFF0000u);
		}
		l0 = l0 * al0 + sum0;
		l1 = l1 * al1 + sum1;
		// O = O * alpha (only when some row's max grew) + P.V; ldmatrix x4 trans: matrices
		// (positions +0..7, dims dt), (+8..15, dt), (+0..7, dt+1), (+8..15, dt+1) are the B
		// fragments of two 8-dim output tiles
		if (__any_sync(0xFFFFFFFFu, al0 != 1.0f || al1 != 1.0f)) {
#pragma unroll
			for (int dt = 0; dt < HD / 8; ++dt) {
				o[dt][0] *= al0;
				o[dt][1] *= al0;
				o[dt][2] *= al1;
				o[dt][3] *= al1;
			}
		}
		const int vrow = (mi & 1) * 8 + mr;
#pragma unroll
		for (int dt = 0; dt < HD / 8; dt += 2) {
			const int d16 = dt + (mi >> 1); // 8-dim chunk index over head_dim
			uint32_t b0, b1, c0, c1;
			ldsm_x4_trans(vc + page_sw_off(vrow, d16 & 7, d16 >> 3), b0, b1, c0, c1);
			mma_bf16_16816(o[dt], pa, b0, b1);
			mma_bf16_16816(o[dt + 1], pa, c0, c1);
		}
		__syncwarp(); // every lane is done with the stage
		if (lane == 0 && issued < n_mine && !abort_flag) issue(issued++);
	}
	// a warp that gave up lets its copies in flight land before the ring is reused
	if (abort_flag && lane == 0) {
		for (int k = max(0, issued - kStBufs); k < issued; ++k) {
			const uint64_t t0 = global_timer_ns();
			while (!mbar_try_wait(&wbar[k % kStBufs], (uint32_t)(k / kStBufs) & 1u) && global_timer_ns() - t0 < kWaitLimitNs) {
			}
		}
	}
	__syncthreads(); // every warp is done with its ring

	// merge the four warps: (m, l, O) per row through shared memory (the ring is idle now)
	float* mo = reinterpret_cast<float*>(sm_raw);       // [warps][16][HD]
	float* ml = mo + 4 * 16 * HD;                        // [warps][16][2]
	l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 1);
	l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 2);
	l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 1);
	l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 2);
#pragma unroll
	for (int dt = 0; dt < HD / 8; ++dt) {
		float* r0 = mo + ((size_t)warp * 16 + gr) * HD + dt * 8 + gc;
		float* r1 = mo + ((size_t)warp * 16 + gr + 8) * HD + dt * 8 + gc;
		r0[0] = o[dt][0];
		r0[1] = o[dt][1];
		r1[0] = o[dt][2];
		r1[1] = o[dt][3];
	}
	if ((lane & 3) == 0) {
		ml[((size_t)warp * 16 + gr) * 2 + 0] = m0;
		ml[((size_t)warp * 16 + gr) * 2 + 1] = l0;
		ml[((size_t)warp * 16 + gr + 8) * 2 + 0] = m1;
		ml[((size_t)warp * 16 + gr + 8) * 2 + 1] = l1;
	}
	__syncthreads();
	// split partial: acc (unnormalised, against the max M in natural-log units), M, L
	const int hd2 = HD + 2;
	const float ln2 = 0.6931471805599453f;
	for (int e = tid; e < G * HD; e += kAmThreads) {
		const int g = e / HD, i = e % HD;
		float M = -INFINITY;
#pragma unroll
		for (int w = 0; w < 4; ++w) M = fmaxf(M, ml[((size_t)w * 16 + g) * 2]);
		float v = 0.0f, L = 0.0f;
#pragma unroll
		for (int w = 0; w < 4; ++w) {
			const float mw = ml[((size_t)w * 16 + g) * 2];
			const float wgt = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
			v = fmaf(wgt, mo[((size_t)w * 16 + g) * HD + i], v);
			L = fmaf(wgt, ml[((size_t)w * 16 + g) * 2 + 1], L);
		}
		float* pr = a.part + (((size_t)b * a.H + kvh * G + g) * a.n_splits + split) * hd2;
		pr[i] = v;
		if (i == 0) {
			pr[HD] = M == -INFINITY ? -INFINITY : M * ln2; // the combine works in natural-log units
			pr[HD + 1] = L;
		}
	}
	__threadfence();
	__syncthreads();
	if (tid == 0) {
		const unsigned t = atomicAdd(&a.counters[b * a.KV + kvh], 1u);
		last_flag = (t == (unsigned)ns - 1);
	}
	__syncthreads();
	if (!last_flag) return;
	__threadfence();
	bf16* ob = reinterpret_cast<bf16*>(a.out) + (size_t)b * a.H * HD;
	for (int e = tid; e < G * HD; e += kAmThreads) {
		const int g = e / HD, i = e % HD;
		const float* ph = a.part + ((size_t)b * a.H + kvh * G + g) * a.n_splits * hd2;
		float M = -INFINITY;
		for (int s = 0; s < ns; ++s) M = fmaxf(M, __ldcg(ph + (size_t)s * hd2 + HD));
		float L = 0.0f, v = 0.0f;
		for (int s = 0; s < ns; ++s) {
			const float ms = __ldcg(ph + (size_t)s * hd2 + HD);
			const float w = (ms == -INFINITY) ? 0.0f : expf(ms - M);
			L = fmaf(w, __ldcg(ph + (size_t)s * hd2 + HD + 1), L);
			v = fmaf(w, __ldcg(ph + (size_t)s * hd2 + i), v);
		}
		Store<bf16>::put(ob + (size_t)(kvh * G + g) * HD + i, L > 0.0f ? v / L : 0.0f);
	}
	if (tid == 0) a.counters[b * a.KV + kvh] = 0u;
}

typedef void (*AttnMmaKernel)(CUtensorMap, CUtensorMap, AttnDecodeArgs);

// the instantiation for GQA group G (<= 8) and head_dim 64 / 128 (nullptr otherwise)
inline AttnMmaKernel attn_decode_mma_kernel(int G, int hd)
{
#define INF_AM_CASE(g)                                               \
	if (G == g && hd == 64) return k_attn_decode_mma<g, 64>;     \
	if (G == g && hd == 128) return k_attn_decode_mma<g, 128>;
	INF_AM_CASE(1) INF_AM_CASE(2) INF_AM_CASE(4) INF_AM_CASE(8)
#undef INF_AM_CASE
	return nullptr;
}

} // namespace inf
