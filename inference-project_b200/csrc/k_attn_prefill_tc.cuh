// Causal prefill attention on the 5th-generation tensor cores (bf16, head_dim 64 or 128).
//
// Flash attention over the paged KV cache.  A CTA owns 128 query rows: 128/G consecutive
// tokens of one sequence times the G query heads that share one KV head, so each K/V tile is
// read once for the whole GQA group.  Row r = tq * G + g.  Per tile of 128 keys (8 pages of 16):
//   warp 0      loads the tile's K and V pages with 2-D TMA (SWIZZLE_128B boxes of 16 keys x 64
//               head dims, no multicast) into a 2-stage ring;
//   warp 1      allocates TMEM (S: 128 columns, O: head_dim columns) and issues, from one
//               thread, S = Q.K^T (both operands K-major) and O += P.V (P K-major from shared
//               memory, V MN-major: the page rows are keys, contiguous along head_dim);
//   warps 2..5  load Q once (swizzled by hand), then per tile read their row of S from TMEM,
//               mask keys past the row's position, keep the running max and sum, write
//               P = exp(S - max) as bf16 in the swizzled K-major layout, and rescale O in TMEM
//               when the max grows; at the end O / sum is stored as bf16.
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
constexpr int kPtThreads = 192;
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

// byte offset of 16-byte chunk c (0..7) of row r inside a SWIZZLE_128B block of 128-byte rows
__device__ __forceinline__ uint32_t sw128_off(int r, int c)
{
	return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

struct PtLayout {
	size_t q, kv, p, bars, total;
	uint32_t stage_bytes, halves;
};
__host__ __device__ inline PtLayout pt_layout(int hd)
{
	PtLayout L;
	L.halves = (uint32_t)(hd / 64);
	L.stage_bytes = 2 * L.halves * kPtAtom; // K then V
	L.q = 0;
	L.kv = L.q + (size_t)L.halves * kPtAtom;
	L.p = L.kv + (size_t)kPtStages * L.stage_bytes;
	L.bars = L.p + 2 * (size_t)kPtAtom;
	L.total = L.bars + 128;
	return L;
}
inline size_t attn_prefill_tc_smem_bytes(int hd) { return 1024 + pt_layout(hd).total; }

__global__ void __launch_bounds__(kPtThreads, 1)
    k_attn_prefill_tc(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const AttnPrefillArgs a)
{
	extern __shared__ __align__(1024) uint8_t smem_raw[];
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
	const int hd = a.hd, G = a.H / a.KV, blk = a.blk;
	const PtLayout Ly = pt_layout(hd);
	uint8_t* q_s = smem + Ly.q;
	uint8_t* kv_s = smem + Ly.kv;
	uint8_t* p_s = smem + Ly.p;
	uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + Ly.bars);
	uint64_t* kv_empty = kv_full + kPtStages;
	uint64_t* bar_s = kv_empty + kPtStages;  // S ready (MMA -> softmax)
	uint64_t* bar_p = bar_s + 1;             // P written, S consumed (softmax -> MMA), 128 arrivals
	uint64_t* bar_o = bar_p + 1;             // P.V done (MMA -> softmax)
	uint64_t* bar_q = bar_o + 1;             // Q staged, 128 arrivals
	uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_q + 1);
	volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int kvh = blockIdx.x;
	const int tq_per = kPtRows / G;
	const int t0 = blockIdx.y * tq_per;
	const int n_tok = min(tq_per, a.T - t0);
	const int slot = a.tok_slot[t0];
	const int last_pos = a.tok_pos[t0 + n_tok - 1];
	const int n_tiles = last_pos / kPtKeys + 1;
	const int pages_tile = kPtKeys / blk;

	if (threadIdx.x == 0) {
		for (int s = 0; s < kPtStages; ++s) {
			mbar_init(&kv_full[s], 1);
			mbar_init(&kv_empty[s], 1);
		}
		mbar_init(bar_s, 1);
		mbar_init(bar_p, 128);
		mbar_init(bar_o, 1);
		mbar_init(bar_q, 128);
		*abort_flag = 0;
		mbar_fence_init();
	}
	if (warp == 1) {
		asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
		             "r"(256)
		             : "memory");
		asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = *tmem_slot;
	const uint32_t tmem_s = tmem, tmem_o = tmem + kPtKeys;
	pdl_wait(); // queries and this chunk's keys come from the QKV kernel before it
	pdl_trigger();

	if (warp == 0) {
		// ---------------- TMA producer: K and V pages of each tile
		if (lane == 0) {
			const uint64_t pol = policy_evict_last(); // the tile is re-read by the next query tiles
			const int* bt = a.block_table + (size_t)slot * a.pages_per_seq;
			int first = bt[0];
			if (first < 0 || first >= a.max_pages) first = 0;
			int issued = 0;
			for (int j = 0; j < n_tiles; ++j) {
				const int s = j % kPtStages;
				if (j >= kPtStages && !mbar_wait(&kv_empty[s], (uint32_t)((j / kPtStages) - 1) & 1u, abort_flag, a.err)) break;
				uint8_t* ks = kv_s + (size_t)s * Ly.stage_bytes;
				uint8_t* vs = ks + (size_t)Ly.halves * kPtAtom;
				mbar_arrive_expect_tx(&kv_full[s], Ly.stage_bytes);
				for (int pg = 0; pg < pages_tile; ++pg) {
					const int pidx = j * pages_tile + pg;
					int page = first; // pages past the context hold finite data that the mask drops
					if (pidx * blk <= last_pos) {
						page = bt[pidx];
						if (page < 0 || page >= a.max_pages) {
							report_err(a.err, kDevKvRange);
							page = first;
						}
					}
					const int y = (page * a.KV + kvh) * blk;
					for (uint32_t h = 0; h < Ly.halves; ++h) {
						tma_load_2d(ks + h * kPtAtom + pg * blk * 128, &tm_k, (int)h * 64, y, &kv_full[s], pol);
						tma_load_2d(vs + h * kPtAtom + pg * blk * 128, &tm_v, (int)h * 64, y, &kv_full[s], pol);
					}
				}
				++issued;
			}
			for (int i = max(0, issued - kPtStages); i < issued; ++i) {
				const uint64_t t0n = global_timer_ns();
				while (!mbar_try_wait(&kv_full[i % kPtStages], (uint32_t)(i / kPtStages) & 1u))
					if (global_timer_ns() - t0n > kWaitLimitNs) {
						report_err(a.err, kDevTimeout);
						break;
					}
			}
		}
	} else if (warp == 1) {
		// ---------------- MMA issuer
		if (lane == 0) {
			const uint32_t idesc_s = umma_idesc_bf16(kPtRows, kPtKeys);
			const uint32_t idesc_o = umma_idesc_bf16(kPtRows, hd) | (1u << 16); // B (V) MN-major
			const uint32_t qa = smem_u32(q_s), pa = smem_u32(p_s);
			const int ksteps_s = hd / 16;
			bool ok = mbar_wait(bar_q, 0, abort_flag, a.err);
			auto issue_s = [&](int j) {
				const uint32_t ka = smem_u32(kv_s + (size_t)(j % kPtStages) * Ly.stage_bytes);
				for (int k = 0; k < ksteps_s; ++k) {
					const uint32_t off = (uint32_t)(k >> 2) * kPtAtom + (uint32_t)(k & 3) * 32;
					umma_bf16(tmem_s, umma_desc_sw128(qa + off), umma_desc_sw128(ka + off), idesc_s, k > 0 ? 1u : 0u);
				}
				umma_commit(bar_s);
			};
			if (ok && mbar_wait(&kv_full[0], 0, abort_flag, a.err)) {
				tc_fence_after();
				issue_s(0);
			} else {
				ok = false;
			}
			for (int j = 0; ok && j < n_tiles; ++j) {
				if (!mbar_wait(bar_p, (uint32_t)j & 1u, abort_flag, a.err)) break;
				tc_fence_after();
				const uint32_t va =
				    smem_u32(kv_s + (size_t)(j % kPtStages) * Ly.stage_bytes + (size_t)Ly.halves * kPtAtom);
				for (int k = 0; k < kPtKeys / 16; ++k) {
					const uint32_t poff = (uint32_t)(k >> 2) * kPtAtom + (uint32_t)(k & 3) * 32;
					umma_bf16(tmem_o, umma_desc_sw128(pa + poff), umma_desc_sw128_lbo(va + (uint32_t)k * 2048u, kPtAtom, 1024u),
					          idesc_o, (j > 0 || k > 0) ? 1u : 0u);
				}
				umma_commit(bar_o);
				umma_commit(&kv_empty[j % kPtStages]);
				if (j + 1 < n_tiles) {
					if (!mbar_wait(&kv_full[(j + 1) % kPtStages], (uint32_t)((j + 1) / kPtStages) & 1u, abort_flag, a.err))
						break;
					tc_fence_after();
					issue_s(j + 1);
				}
			}
		}
	} else {
		// ---------------- softmax / epilogue: TMEM lane quarter = warp % 4, one row per thread
		const int quarter = warp & 3;
		const int r = quarter * 32 + lane;
		const int tq = r / G, g = r % G;
		const bool valid = tq < n_tok;
		const int pos = valid ? a.tok_pos[t0 + tq] : -1;
		const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
		// Q row -> shared memory, swizzled (K-major SWIZZLE_128B, one block per 64 head dims)
		{
			const uint4* src = reinterpret_cast<const uint4*>(
			    reinterpret_cast<const bf16*>(a.q) + ((size_t)(t0 + (valid ? tq : 0)) * a.H + kvh * G + g) * hd);
			for (int c = 0; c < hd / 8; ++c) {
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
		float m = -INFINITY, l = 0.0f;
		bool ok = true;
		for (int j = 0; j < n_tiles; ++j) {
			if (!wait_all(bar_s, (uint32_t)j & 1u)) {
				ok = false;
				break;
			}
			tc_fence_after();
			const int kbase = j * kPtKeys;
			float mt = -INFINITY;
#pragma unroll 1
			for (int c = 0; c < kPtKeys; c += 32) {
				float v[32];
				tmem_ld_32cols(tmem_s + lane_off + (uint32_t)c, v);
#pragma unroll
				for (int i = 0; i < 32; ++i)
					if (kbase + c + i <= pos) mt = fmaxf(mt, v[i] * sl2);
			}
			const float mn = fmaxf(m, mt);
			const float alpha = (m == -INFINITY) ? 1.0f : exp2f(m - mn);
			// P.V of the previous tile has to finish before P is overwritten and O rescaled
			if (j > 0) {
				if (!wait_all(bar_o, (uint32_t)(j - 1) & 1u)) {
					ok = false;
					break;
				}
				tc_fence_after();
				if (__any_sync(0xFFFFFFFFu, alpha != 1.0f)) {
#pragma unroll 1
					for (int c = 0; c < hd; c += 32) {
						float o[32];
						tmem_ld_32cols(tmem_o + lane_off + (uint32_t)c, o);
#pragma unroll
						for (int i = 0; i < 32; ++i) o[i] *= alpha;
						tmem_st_32cols(tmem_o + lane_off + (uint32_t)c, o);
					}
				}
			}
			float sum = 0.0f;
#pragma unroll 1
			for (int c = 0; c < kPtKeys; c += 32) {
				float v[32];
				tmem_ld_32cols(tmem_s + lane_off + (uint32_t)c, v);
				uint32_t pk[16];
#pragma unroll
				for (int i = 0; i < 32; i += 2) {
					const float p0 = (kbase + c + i <= pos && mn != -INFINITY) ? exp2f(v[i] * sl2 - mn) : 0.0f;
					const float p1 = (kbase + c + i + 1 <= pos && mn != -INFINITY) ? exp2f(v[i + 1] * sl2 - mn) : 0.0f;
					const uint32_t b0 = f32_to_bf16_bits(p0), b1 = f32_to_bf16_bits(p1);
					// the sum uses the rounded values, the ones the MMA sees
					sum += __uint_as_float(b0 << 16) + __uint_as_float(b1 << 16);
					pk[i >> 1] = b0 | (b1 << 16);
				}
				uint8_t* blkp = p_s + (size_t)(c >> 6) * kPtAtom;
				const int c0 = (c & 63) >> 3;
#pragma unroll
				for (int u = 0; u < 4; ++u)
					*reinterpret_cast<uint4*>(blkp + sw128_off(r, c0 + u)) =
					    make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
			}
			l = l * alpha + sum;
			m = mn;
			asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
			tc_fence_before();
			mbar_arrive(bar_p);
		}
		if (ok && wait_all(bar_o, (uint32_t)(n_tiles - 1) & 1u)) {
			tc_fence_after();
			const float inv = l > 0.0f ? 1.0f / l : 0.0f;
			bf16* dst = reinterpret_cast<bf16*>(a.out) + (size_t)(t0 + (valid ? tq : 0)) * a.H * hd + (size_t)(kvh * G + g) * hd;
#pragma unroll 1
			for (int c = 0; c < hd; c += 32) {
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
			const uint64_t t0n = global_timer_ns();
			while (!mbar_try_wait(bar_o, (uint32_t)(n_tiles - 1) & 1u))
				if (global_timer_ns() - t0n > kWaitLimitNs) break;
		}
		tc_fence_after();
		asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
	}
}

} // namespace inf
