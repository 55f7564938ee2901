// Causal prefill attention on the 5th-generation tensor cores (bf16, head_dim 64 or 128).
//
// Flash attention over the paged KV cache.  A CTA owns 128 query rows: 128/G consecutive
// tokens of one sequence times the G query heads that share one KV head, so each K/V tile is
// read once for the whole GQA group.  Row r = tq * G + g.  Per tile of 128 keys (8 pages of 16):
//   warp 0      loads the tile's K and V pages with 4-D TMA (SWIZZLE_128B boxes of 64 head dims
//               x 16 keys x 8 consecutive pages, or one page per box when the ids are not
//               consecutive; no multicast) into 2-stage K and V rings;
//   warp 1      allocates TMEM (S: 128 columns, O: head_dim columns) and issues, from one
//               thread, S = Q.K^T (both operands K-major) and O += P.V (P K-major from shared
//               memory, V MN-major: the page rows are keys, contiguous along head_dim);
//   warps 2..9  load Q once (swizzled by hand), then per tile read S from TMEM -- two warps
//               per TMEM lane quarter, each on half of a row's 128 scores, the halves' maxima
//               exchanged through shared memory -- mask keys past the row's position, keep the
//               running max and sum, write P = exp(S - max) as bf16 in the swizzled K-major
//               layout, and rescale their half of O in TMEM when the max grows by more than
//               2^8; at the end O / sum is stored as bf16.
// Rounding: S and O accumulate in fp32, P is rounded to bf16 for the second MMA (the SIMT
// kernel k_attn_prefill.cuh keeps P in fp32).  Every wait is bounded; on a timeout the
// kernel records kDevTimeout, lets its copies and MMAs drain, frees TMEM and returns.
#pragma once

#include "k_attn_prefill.cuh" // AttnPrefillArgs
#include "k_gemm_tc.cuh"      // tma_load_2d, umma_bf16, umma_commit, tmem_ld_32cols, fences

namespace inf {

constexpr int kPtRows = 128;       // query rows per CTA (MMA M)
constexpr int kPtKeys = 128;       // keys per tile (MMA N of S, K of P.V)
constexpr int kPtStages = 2;
constexpr int kPtThreads = 320; // TMA warp, MMA warp, 8 softmax warps
constexpr uint32_t kPtAtom = 128 * 64 * 2; // one [128 x 64] bf16 SWIZZLE_128B block: 16 KB

// shared-memory descriptor with explicit leading / stride byte offsets (SWIZZLE_128B)
__device__ __forceinline__ uint64_t umma_desc_sw128_lbo(uint32_t smem_addr, uint32_t lbo, uint32_t sbo)
{
	uint64_t d = 0;
	d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
	d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
	d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
	d |= (uint64_t)1u << 46;
	d |= (uint64_t)2u << 61;
	return d;
}

// tcgen05.ld of 32 columns without the wait (several loads, then one tcgen05.wait::ld)
__device__ __forceinline__ void tmem_ld_32cols_nowait(uint32_t taddr, float* v)
{
	uint32_t r[32];
	asm volatile(
	    "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
	    "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
	    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
	    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
	      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
	      "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
	      "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
	    : "r"(taddr));
#pragma unroll
	for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st_32cols(uint32_t taddr, const float (&v)[32])
{
	uint32_t r[32];
#pragma unroll
	for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
	asm volatile(
	    "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
	    "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
	    "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
	    "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
	    "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
	    "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
	    "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
	    : "memory");
	asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 4-D tiled TMA load (head_dim, row in page, KV head, page) of the paged K/V pool
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint64_t* bar,
                                            uint64_t policy)
{
	asm volatile(
	    "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
	    " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
	    "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
	    : "memory");
}

// byte offset of 16-byte chunk c (0..7) of row r inside a SWIZZLE_128B block of 128-byte rows
__device__ __forceinline__ uint32_t sw128_off(int r, int c)
{
	return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

struct PtLayout {
	size_t q, k, v, p, bars, total;
	uint32_t tile_bytes, halves; // one K or V tile: halves x 16 KB
};
__host__ __device__ inline PtLayout pt_layout(int hd)
{
	PtLayout L;
	L.halves = (uint32_t)(hd / 64);
	L.tile_bytes = L.halves * kPtAtom;
	L.q = 0;
	L.k = L.q + L.tile_bytes;
	L.v = L.k + (size_t)kPtStages * L.tile_bytes;
	L.p = L.v + (size_t)kPtStages * L.tile_bytes;
	L.bars = L.p + 2 * (size_t)2 * kPtAtom; // two P buffers of [128 rows x 128 keys]
	L.total = L.bars + 256 + 2 * 128 * 4; // barriers, flags, the halves' row maxima [2][128]
	return L;
}
inline size_t attn_prefill_tc_smem_bytes(int hd) { return 1024 + pt_layout(hd).total; }

__device__ __forceinline__ float ex2_approx(float x)
{
	float y;
	asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
	return y;
}

// Largest growth of the running max (log2 units) absorbed without rescaling O: P values up to
// 2^8 stay exact enough in bf16 and fp32, and O / l is unchanged in exact arithmetic.
constexpr float kPtRescaleLog2 = 8.0f;

__global__ void __launch_bounds__(kPtThreads, 1)
    k_attn_prefill_tc(const __grid_constant__ CUtensorMap tm_k8, const __grid_constant__ CUtensorMap tm_k1,
                      const __grid_constant__ CUtensorMap tm_v8, const __grid_constant__ CUtensorMap tm_v1,
                      const AttnPrefillArgs a)
{
	extern __shared__ __align__(1024) uint8_t smem_raw[];
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
	const int hd = a.hd, G = a.H / a.KV, blk = a.blk;
	const PtLayout Ly = pt_layout(hd);
	uint8_t* q_s = smem + Ly.q;
	uint8_t* k_s = smem + Ly.k;
	uint8_t* v_s = smem + Ly.v;
	uint8_t* p_s = smem + Ly.p;
	uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Ly.bars);
	uint64_t* k_full = bars;       // [2] TMA -> MMA
	uint64_t* k_empty = bars + 2;  // [2] S MMA done with the K tile
	uint64_t* v_full = bars + 4;   // [2]
	uint64_t* v_empty = bars + 6;  // [2] P.V MMA done with the V tile
	uint64_t* s_full = bars + 8;   // [2] S buffer b ready (MMA -> softmax)
	uint64_t* p_free = bars + 10;  // [2] P buffer b read by its P.V MMA
	uint64_t* bar_p = bars + 12;   // P of tile j written, its S consumed (256 arrivals)
	uint64_t* bar_o = bars + 13;   // P.V of tile j done
	uint64_t* bar_q = bars + 14;   // Q staged (256 arrivals)
	uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
	volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int kvh = blockIdx.x;
	const int tq_per = kPtRows / G;
	// causal work grows with the token index: the last tokens' tiles are scheduled first
	const int t0 = (gridDim.y - 1 - blockIdx.y) * tq_per;
	const int n_tok = min(tq_per, a.T - t0);
	const int slot = a.tok_slot[t0];
	const int last_pos = a.tok_pos[t0 + n_tok - 1];
	const int n_tiles = last_pos / kPtKeys + 1;
	const int pages_tile = kPtKeys / blk;

	if (threadIdx.x == 0) {
		for (int i = 0; i < 12; ++i) mbar_init(&bars[i], 1);
		mbar_init(bar_p, 256);
		mbar_init(bar_o, 1);
		mbar_init(bar_q, 256);
		*abort_flag = 0;
		mbar_fence_init();
	}
	if (warp == 1) {
		asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
		             "r"(512)
		             : "memory");
		asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = *tmem_slot;
	const uint32_t tmem_o = tmem + 2 * kPtKeys; // S buffers at columns 0 and 128
	pdl_wait(); // queries and this chunk's keys come from the QKV kernel before it
	pdl_trigger();

	if (warp == 0) {
		// ---------------- TMA producer: the K pages, then the V pages, of each tile
		if (lane == 0) {
			const uint64_t pol = policy_evict_last(); // the tile is re-read by the next query tiles
			const int* bt = a.block_table + (size_t)slot * a.pages_per_seq;
			int first = bt[0];
			if (first < 0 || first >= a.max_pages) first = 0;
			// A tile whose pages have consecutive ids (a sequence prefilled into a fresh cache) is
			// one box of pages_tile pages per 64 head dims; otherwise one box per page.
			auto load = [&](const CUtensorMap* tm8, const CUtensorMap* tm1, uint8_t* dst, uint64_t* bar, int j) {
				mbar_arrive_expect_tx(bar, Ly.tile_bytes);
				const int p0 = j * pages_tile;
				bool contig = p0 + pages_tile <= a.pages_per_seq;
				const int id0 = contig ? bt[p0] : -1;
				contig = contig && id0 >= 0 && id0 + pages_tile <= a.max_pages;
				for (int pg = 1; contig && pg < pages_tile; ++pg) contig = bt[p0 + pg] == id0 + pg;
				if (contig) {
					for (uint32_t h = 0; h < Ly.halves; ++h) tma_load_4d(dst + h * kPtAtom, tm8, (int)h * 64, 0, kvh, id0, bar, pol);
					return;
				}
				for (int pg = 0; pg < pages_tile; ++pg) {
					const int pidx = p0 + pg;
					int page = first; // pages past the context hold finite data that the mask drops
					if (pidx * blk <= last_pos) {
						page = bt[pidx];
						if (page < 0 || page >= a.max_pages) {
							report_err(a.err, kDevKvRange);
							page = first;
						}
					}
					for (uint32_t h = 0; h < Ly.halves; ++h)
						tma_load_4d(dst + h * kPtAtom + pg * blk * 128, tm1, (int)h * 64, 0, kvh, page, bar, pol);
				}
			};
			int kiss = 0, viss = 0;
			for (int j = 0; j < n_tiles; ++j) {
				const int s = j % kPtStages;
				const uint32_t par = (uint32_t)((j / kPtStages) - 1) & 1u;
				if (j >= kPtStages && !mbar_wait(&k_empty[s], par, abort_flag, a.err)) break;
				load(&tm_k8, &tm_k1, k_s + (size_t)s * Ly.tile_bytes, &k_full[s], j);
				++kiss;
				if (j >= kPtStages && !mbar_wait(&v_empty[s], par, abort_flag, a.err)) break;
				load(&tm_v8, &tm_v1, v_s + (size_t)s * Ly.tile_bytes, &v_full[s], j);
				++viss;
			}
			// never leave the CTA with copies in flight
			for (int i = max(0, kiss - kPtStages); i < kiss; ++i) {
				const uint64_t tw = global_timer_ns();
				while (!mbar_try_wait(&k_full[i % kPtStages], (uint32_t)(i / kPtStages) & 1u))
					if (global_timer_ns() - tw > kWaitLimitNs) break;
			}
			for (int i = max(0, viss - kPtStages); i < viss; ++i) {
				const uint64_t tw = global_timer_ns();
				while (!mbar_try_wait(&v_full[i % kPtStages], (uint32_t)(i / kPtStages) & 1u))
					if (global_timer_ns() - tw > kWaitLimitNs) break;
			}
		}
	} else if (warp == 1) {
		// ---------------- MMA issuer: S(j+2) runs while the softmax warps work on S(j+1)
		if (lane == 0) {
			const uint32_t idesc_s = umma_idesc_bf16(kPtRows, kPtKeys);
			const uint32_t idesc_o = umma_idesc_bf16(kPtRows, hd) | (1u << 16); // B (V) MN-major
			const uint32_t qa = smem_u32(q_s);
			const int ksteps_s = hd / 16;
			auto issue_s = [&](int j) -> bool {
				const int s = j % kPtStages;
				if (!mbar_wait(&k_full[s], (uint32_t)(j / kPtStages) & 1u, abort_flag, a.err)) return false;
				tc_fence_after();
				const uint32_t ka = smem_u32(k_s + (size_t)s * Ly.tile_bytes);
				const uint32_t ts = tmem + (uint32_t)(j & 1) * kPtKeys;
				for (int k = 0; k < ksteps_s; ++k) {
					const uint32_t off = (uint32_t)(k >> 2) * kPtAtom + (uint32_t)(k & 3) * 32;
					umma_bf16(ts, umma_desc_sw128(qa + off), umma_desc_sw128(ka + off), idesc_s, k > 0 ? 1u : 0u);
				}
				umma_commit(&s_full[j & 1]);
				umma_commit(&k_empty[s]);
				return true;
			};
			bool ok = mbar_wait(bar_q, 0, abort_flag, a.err);
			ok = ok && issue_s(0);
			if (ok && n_tiles > 1) ok = issue_s(1);
			for (int j = 0; ok && j < n_tiles; ++j) {
				if (!mbar_wait(bar_p, (uint32_t)j & 1u, abort_flag, a.err)) break;
				const int s = j % kPtStages;
				if (!mbar_wait(&v_full[s], (uint32_t)(j / kPtStages) & 1u, abort_flag, a.err)) break;
				tc_fence_after();
				const uint32_t va = smem_u32(v_s + (size_t)s * Ly.tile_bytes);
				const uint32_t pa = smem_u32(p_s + (size_t)(j & 1) * 2 * kPtAtom);
				for (int k = 0; k < kPtKeys / 16; ++k) {
					const uint32_t poff = (uint32_t)(k >> 2) * kPtAtom + (uint32_t)(k & 3) * 32;
					umma_bf16(tmem_o, umma_desc_sw128(pa + poff), umma_desc_sw128_lbo(va + (uint32_t)k * 2048u, kPtAtom, 1024u),
					          idesc_o, (j > 0 || k > 0) ? 1u : 0u);
				}
				umma_commit(bar_o);
				umma_commit(&p_free[j & 1]);
				umma_commit(&v_empty[s]);
				if (j + 2 < n_tiles && !issue_s(j + 2)) break;
			}
		}
	} else {
		// ---------------- softmax / epilogue: eight warps, two per TMEM lane quarter; a row's
		// 128 scores are split in halves (warps 2-5: keys 0-63, warps 6-9: keys 64-127), the
		// halves exchange their maxima through shared memory, and each half rescales and
		// stores its half of the O columns
		const int quarter = warp & 3, half = (warp - 2) >> 2;
		const int r = quarter * 32 + lane;
		const int tq = r / G, g = r % G;
		const bool valid = tq < n_tok;
		const int pos = valid ? a.tok_pos[t0 + tq] : -1;
		const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
		float* xmax = reinterpret_cast<float*>(smem + Ly.bars + 256); // [2 halves][128 rows]
		constexpr int kHalfKeys = kPtKeys / 2;
		const int hd_half = hd / 2;
		// Q row -> shared memory, swizzled (K-major SWIZZLE_128B, one block per 64 head dims);
		// each half loads half of the row's 16-byte chunks
		{
			const uint4* src = reinterpret_cast<const uint4*>(
			    reinterpret_cast<const bf16*>(a.q) + ((size_t)(t0 + (valid ? tq : 0)) * a.H + kvh * G + g) * hd);
			const int nc = hd / 8;
			for (int c = half * (nc / 2); c < (half + 1) * (nc / 2); ++c) {
				const uint4 v = valid ? src[c] : make_uint4(0, 0, 0, 0);
				*reinterpret_cast<uint4*>(q_s + (size_t)(c >> 3) * kPtAtom + sw128_off(r, c & 7)) = v;
			}
			asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
			mbar_arrive(bar_q);
		}
		const float sl2 = a.scale * 1.4426950408889634f; // scores in log2 units
		// waits are voted warp-wide so that the warp stays converged for tcgen05.ld/st
		auto wait_all = [&](uint64_t* bar, uint32_t par) {
			const bool w = mbar_wait(bar, par, abort_flag, a.err);
			return __all_sync(0xFFFFFFFFu, w);
		};
		float m = -INFINITY, l = 0.0f; // m: the max the P values are taken against; l: this half's sum
		bool ok = true;
		// every softmax thread reaches both named barriers of every tile (no early exit)
		for (int j = 0; j < n_tiles; ++j) {
			ok = ok && wait_all(&s_full[j & 1], (uint32_t)(j >> 1) & 1u);
			const int kbase = j * kPtKeys + half * kHalfKeys;
			float v[kHalfKeys];
			float mt = -INFINITY;
			if (ok) {
				tc_fence_after();
				const uint32_t ts = tmem + (uint32_t)(j & 1) * kPtKeys + (uint32_t)(half * kHalfKeys) + lane_off;
				const bool masked = kbase + kHalfKeys - 1 > pos; // the diagonal tile (or an invalid row)
#pragma unroll
				for (int c = 0; c < kHalfKeys; c += 32) tmem_ld_32cols_nowait(ts + (uint32_t)c, v + c);
				asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
				// raw scores: the scale is applied to the max here and inside the exponent's FMA
				// below (rounding is monotonic, so the max equals the max of the scaled scores)
				if (masked) {
#pragma unroll
					for (int i = 0; i < kHalfKeys; ++i)
						if (kbase + i > pos) v[i] = -INFINITY;
				}
				// four independent max chains (the max is exact, so the order does not matter)
				float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
				for (int i = 0; i < kHalfKeys; ++i) m4[i & 3] = fmaxf(m4[i & 3], v[i]);
				mt = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * sl2;
			}
			// the exchange is between the two warps of this TMEM lane quarter only (rows r):
			// one 64-thread named barrier per quarter
			xmax[half * kPtRows + r] = mt;
			named_bar_sync(1 + quarter, 64);
			mt = fmaxf(mt, xmax[(half ^ 1) * kPtRows + r]);
			named_bar_sync(1 + quarter, 64); // both halves have read before the next tile's writes
			// rescale only when the max grows by more than 2^8 (or on the first finite max);
			// both halves of a row take the same decision
			const bool grow = mt > m + kPtRescaleLog2 || (m == -INFINITY && mt != -INFINITY);
			const float mn = grow ? mt : m;
			if (ok && __any_sync(0xFFFFFFFFu, grow) && j > 0) {
				// O must hold every earlier P.V before it is rescaled
				ok = wait_all(bar_o, (uint32_t)(j - 1) & 1u);
				if (ok) {
					tc_fence_after();
					const float alpha = grow && m != -INFINITY ? ex2_approx(m - mn) : 1.0f;
#pragma unroll 1
					for (int c = half * hd_half; c < (half + 1) * hd_half; c += 32) {
						float o[32];
						tmem_ld_32cols(tmem_o + lane_off + (uint32_t)c, o);
#pragma unroll
						for (int i = 0; i < 32; ++i) o[i] *= alpha;
						tmem_st_32cols(tmem_o + lane_off + (uint32_t)c, o);
					}
				}
			}
			if (grow && m != -INFINITY) l *= ex2_approx(m - mn);
			m = mn;
			// P buffer j&1 was last read by the P.V of tile j-2
			if (ok && j >= 2) ok = wait_all(&p_free[j & 1], (uint32_t)((j >> 1) - 1) & 1u);
			if (ok) {
				uint8_t* pb = p_s + (size_t)(j & 1) * 2 * kPtAtom + (size_t)half * kPtAtom; // this half's 64 keys
				float sums[4] = {0.0f, 0.0f, 0.0f, 0.0f}; // four independent add chains
#pragma unroll
				for (int c = 0; c < kHalfKeys; c += 8) {
					uint32_t pk[4];
#pragma unroll
					for (int i = 0; i < 8; i += 2) {
						const float p0 = m == -INFINITY ? 0.0f : ex2_approx(fmaf(v[c + i], sl2, -m));
						const float p1 = m == -INFINITY ? 0.0f : ex2_approx(fmaf(v[c + i + 1], sl2, -m));
						const __nv_bfloat162 b = __floats2bfloat162_rn(p0, p1);
						// the row sum adds the rounded values, the weights the MMA applies
						sums[i >> 1] += __low2float(b) + __high2float(b);
						pk[i >> 1] = *reinterpret_cast<const uint32_t*>(&b);
					}
					*reinterpret_cast<uint4*>(pb + sw128_off(r, c >> 3)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
				}
				l += (sums[0] + sums[1]) + (sums[2] + sums[3]);
				asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
				tc_fence_before();
				mbar_arrive(bar_p);
			}
		}
		// the row's sum: both halves
		xmax[half * kPtRows + r] = l;
		named_bar_sync(1 + quarter, 64);
		const float lt = l + xmax[(half ^ 1) * kPtRows + r];
		if (ok && wait_all(bar_o, (uint32_t)(n_tiles - 1) & 1u)) {
			tc_fence_after();
			const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
			bf16* dst = reinterpret_cast<bf16*>(a.out) + (size_t)(t0 + (valid ? tq : 0)) * a.H * hd + (size_t)(kvh * G + g) * hd;
#pragma unroll 1
			for (int c = half * hd_half; c < (half + 1) * hd_half; c += 32) {
				float o[32];
				tmem_ld_32cols(tmem_o + lane_off + (uint32_t)c, o);
				if (valid) {
					uint32_t pk[16];
#pragma unroll
					for (int i = 0; i < 32; i += 2)
						pk[i >> 1] = (uint32_t)f32_to_bf16_bits(o[i] * inv) | ((uint32_t)f32_to_bf16_bits(o[i + 1] * inv) << 16);
#pragma unroll
					for (int u = 0; u < 4; ++u)
						reinterpret_cast<uint4*>(dst + c)[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
				}
			}
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 1) {
		if (*abort_flag) {
			// let every issued MMA finish before TMEM is freed
			const uint64_t tw = global_timer_ns();
			while (!mbar_try_wait(bar_o, (uint32_t)(n_tiles - 1) & 1u))
				if (global_timer_ns() - tw > kWaitLimitNs) break;
		}
		tc_fence_after();
		asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
	}
}

} // namespace inf
