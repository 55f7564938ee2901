// Prefill / multi-token projections on the 5th-generation tensor cores (sm_100a).
//
// D[T x N] = X[T x K] . W[N x K]^T, bf16 inputs, fp32 accumulation in tensor memory.
// A persistent CTA per SM loops over 128 x 256 output tiles (M tiles fastest):
//   warp 0      TMA producer: 2-D tiled bulk tensor loads (SWIZZLE_128B, no multicast) of
//               X[128 x 64] and W[256 x 64] per stage into a 4-stage shared-memory ring that
//               runs on across tiles
//   warp 1      allocates 512 TMEM columns (two 256-column accumulators); one elected lane
//               issues tcgen05.mma (kind::f16, M=128, N=256, K=16; both operands K-major);
//               tcgen05.commit frees each stage and signals each finished accumulator
//   warps 2..9  epilogue, overlapping the next tile's MMAs (two warps per TMEM lane quarter,
//               128 columns each): tcgen05.ld 32x32b (row = TMEM lane = token), a transpose
//               through shared memory, then the fused epilogues (store, residual add, RoPE +
//               KV-cache write, SwiGLU on adjacent column pairs, fp32 logits with a per-row
//               greedy argmax folded in by a 64-bit atomicMax of a (value, column) key) along
//               rows, so stores are row segments
// When the output has too few tiles to fill the SMs (a batch of decode tokens), K is split
// across CTAs; each split writes fp32 partials and k_gemm_splitk_reduce (or, for a residual
// projection followed by an RMSNorm, k_gemm_splitk_resid_norm) sums them and runs the epilogue.
// Every wait is bounded; on a timeout the kernel records kDevTimeout, lets its copies and
// MMAs drain, frees TMEM and returns.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace inf {

constexpr int kTcBM = 128;
constexpr int kTcBN = 256;
constexpr int kTcBK = 64; // 128 bytes of bf16: one SWIZZLE_128B atom row
constexpr int kTcStages = 4;
constexpr int kTcThreads = 320;
constexpr uint32_t kTcStageA = kTcBM * kTcBK * 2;
constexpr uint32_t kTcStageB = kTcBN * kTcBK * 2;
constexpr uint32_t kTcStageBytes = kTcStageA + kTcStageB;
constexpr int kTcAccBufs = 2;
constexpr int kTcTmemCols = kTcAccBufs * kTcBN;
constexpr int kTcEpiWarps = 8; // two per TMEM lane quarter, each 128 of the 256 columns
constexpr size_t kTcKeepXBytes = 48u << 20; // activations up to this size stay in L2 (evict_last)
constexpr uint32_t kTcOutStageBytes = kTcEpiWarps * 32 * 33 * 4; // per epilogue warp a 32 x 33 fp32 transpose

enum TcEpi : int { kTcStore = 0, kTcStoreF32 = 1, kTcResid = 2, kTcQkv = 3, kTcSwiglu = 4, kTcLogitsArgmax = 5 };

struct TcArgs {
	int T, N, K;
	int epi;
	void* out;               // store: bf16 [T x N]; f32 store: f32 [T x N]; swiglu: bf16 [T x N/2]; qkv: q bf16 [T x Hq*hd]
	float* resid;            // resid: f32 [T x N]
	void* kpool;             // qkv: this layer's pages [pages][KV][blk][hd]
	void* vpool;
	const int* block_table;
	int pages_per_seq, max_pages, max_seq;
	const int* tok_pos;      // [T] position of each row
	const int* tok_slot;     // [T] sequence slot of each row
	const float* rope_cos;
	const float* rope_sin;
	int head_dim, n_q_heads, n_kv_heads, kv_block;
	int* err;
	// split-K (few output tiles, e.g. a 64-token batch): CTA z of k_splits sums its share of
	// the K blocks into partial [k_splits][T][N] fp32; k_gemm_splitk_reduce adds the shares
	// in z order and runs the epilogue
	int k_splits;
	float* partial;
	// kTcLogitsArgmax: f32 logits to out and, per row, the max (value, column + col_base) key
	// folded into best_keys[row] with a 64-bit atomicMax (ties -> lowest column)
	unsigned long long* best_keys;
	uint32_t col_base;
	// N tile width (a multiple of 16, 16 .. 256; 0: 256): narrower tiles when 256-wide ones
	// would leave SMs idle
	int bn;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar, uint64_t policy)
{
	asm volatile(
	    "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
	    " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
	    "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
	    : "memory");
}

// K-major operand in the canonical SWIZZLE_128B layout: 8-row atoms of 1024 bytes stacked
// along M/N (stride byte offset 1024), version 1 (sm_100), layout type 2 (128B swizzle).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr)
{
	uint64_t d = 0;
	d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
	d |= (uint64_t)1u << 16;               // leading byte offset (unused for swizzled K-major): 16 B
	d |= (uint64_t)(1024u >> 4) << 32;     // stride byte offset: 1024 B between 8-row atoms
	d |= (uint64_t)1u << 46;               // descriptor version for sm_100
	d |= (uint64_t)2u << 61;               // SWIZZLE_128B
	return d;
}

// kind::f16 instruction descriptor: D f32, A/B bf16, both K-major, M = 128, N = 256.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N)
{
	return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate)
{
	asm volatile(
	    "{\n\t.reg .pred p;\n\t"
	    "setp.ne.b32 p, %4, 0;\n\t"
	    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
	    "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
	    : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
	asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
	             : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, float (&v)[32])
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
	asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
	for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// The fused epilogues, one output column per lane: the whole warp calls it for token row t
// and columns n = n0 + lane (n0 a multiple of 32).  The column pairs of the
// RoPE and SwiGLU epilogues are (even lane, odd lane); the argmax key of the 32 columns is
// the warp's maximum, folded into the row's key by lane 0.
__device__ __forceinline__ void tc_epilogue_lane(const TcArgs& a, int t, int n, float v, int n_lim)
{
	const int lane = threadIdx.x & 31;
	const float v1 = __shfl_down_sync(0xffffffffu, v, 1); // the odd partner of an even lane
	if (a.epi == kTcStoreF32 || a.epi == kTcLogitsArgmax) {
		unsigned long long k = 0ull;
		if (n < n_lim) {
			reinterpret_cast<float*>(a.out)[(size_t)t * a.N + n] = v;
			k = argmax_key(v, (uint32_t)n + a.col_base);
		}
		if (a.epi == kTcLogitsArgmax) {
#pragma unroll
			for (int o = 16; o > 0; o >>= 1) {
				const unsigned long long p = __shfl_xor_sync(0xffffffffu, k, o);
				k = p > k ? p : k;
			}
			if (lane == 0) atomicMax(a.best_keys + t, k);
		}
	} else if (a.epi == kTcStore) {
		if (n < n_lim) Store<bf16>::put(reinterpret_cast<bf16*>(a.out) + (size_t)t * a.N + n, v);
	} else if (a.epi == kTcResid) {
		if (n < n_lim) a.resid[(size_t)t * a.N + n] += v;
	} else if (a.epi == kTcSwiglu) {
		if (!(lane & 1) && n + 1 < n_lim)
			Store<bf16>::put(reinterpret_cast<bf16*>(a.out) + (size_t)t * (a.N >> 1) + (n >> 1), __fmul_rn(silu(v), v1));
	} else if (a.epi == kTcQkv) {
		if ((lane & 1) || n >= n_lim) return;
		const int hd = a.head_dim, half = hd >> 1;
		const int pos = a.tok_pos[t], slot = a.tok_slot[t];
		const int head = n / hd, dim = (n % hd) >> 1;
		float o0 = v, o1 = v1;
		if (head < a.n_q_heads + a.n_kv_heads) {
			const float c = a.rope_cos[(size_t)pos * half + dim];
			const float s = a.rope_sin[(size_t)pos * half + dim];
			o0 = __fsub_rn(__fmul_rn(v, c), __fmul_rn(v1, s));
			o1 = __fadd_rn(__fmul_rn(v1, c), __fmul_rn(v, s));
		}
		if (head < a.n_q_heads) {
			bf16* q = reinterpret_cast<bf16*>(a.out) + ((size_t)t * a.n_q_heads + head) * hd;
			Store<bf16>::put(q + dim, o0);
			Store<bf16>::put(q + dim + half, o1);
			return;
		}
		const int page = (pos >= 0 && pos < a.max_seq) ? a.block_table[(size_t)slot * a.pages_per_seq + pos / a.kv_block] : -1;
		if (page < 0 || page >= a.max_pages) {
			report_err(a.err, kDevKvRange);
			return;
		}
		const bool is_k = head < a.n_q_heads + a.n_kv_heads;
		const int kvh = head - a.n_q_heads - (is_k ? 0 : a.n_kv_heads);
		bf16* base = reinterpret_cast<bf16*>(is_k ? a.kpool : a.vpool) +
		             (((size_t)page * a.n_kv_heads + kvh) * a.kv_block + (pos % a.kv_block)) * hd;
		Store<bf16>::put(base + dim, o0);
		Store<bf16>::put(base + dim + half, o1);
	}
}

// The fused epilogues for one 32-column chunk (columns n0 .. n0 + 31) of a warp's token rows
// t0 .. t0 + rows - 1, the values v(r, c) = st[r * 33 + c] (transposed through shared memory).
// Column epilogues (store, residual add, f32 logits + argmax) take lane = column, one row per
// step, the residual loaded 8 rows at a time so the latencies overlap.  Pair epilogues (SwiGLU,
// RoPE + KV write) take lane = (row parity lane / 16, pair lane % 16): two rows of 16 adjacent
// column pairs per step, every lane busy; the QKV epilogue's position and KV page of row r are
// row_pos / row_page of lane r.  Same arithmetic per element as tc_epilogue_lane.
constexpr int kTcEpiRowGroup = 8;
__device__ __forceinline__ void tc_epilogue_rows(const TcArgs& a, int t0, int rows, int n0, const float* st, int row_pos,
                                                 int row_page, int n_lim)
{
	const int lane = threadIdx.x & 31;
	if (a.epi == kTcResid) {
		const int n = n0 + lane;
		float* rp = a.resid + (size_t)t0 * a.N + n;
		for (int r0 = 0; r0 < rows; r0 += kTcEpiRowGroup) {
			float old[kTcEpiRowGroup];
#pragma unroll
			for (int j = 0; j < kTcEpiRowGroup; ++j)
				old[j] = (r0 + j < rows && n < n_lim) ? rp[(size_t)(r0 + j) * a.N] : 0.0f;
#pragma unroll
			for (int j = 0; j < kTcEpiRowGroup; ++j)
				if (r0 + j < rows && n < n_lim) rp[(size_t)(r0 + j) * a.N] = old[j] + st[(r0 + j) * 33 + lane];
		}
	} else if (a.epi == kTcSwiglu) {
		const int p = lane & 15, n = n0 + 2 * p;
		bf16* o = reinterpret_cast<bf16*>(a.out) + (n >> 1);
		if (n + 1 < n_lim)
			for (int r = lane >> 4; r < rows; r += 2)
				Store<bf16>::put(o + (size_t)(t0 + r) * (a.N >> 1), __fmul_rn(silu(st[r * 33 + 2 * p]), st[r * 33 + 2 * p + 1]));
	} else if (a.epi == kTcQkv) {
		const int hd = a.head_dim, half = hd >> 1;
		const int p = lane & 15, n = n0 + 2 * p;
		const int head = n / hd, dim = (n % hd) >> 1;
		const bool ok = n < n_lim;
		const bool rope = head < a.n_q_heads + a.n_kv_heads; // q and k heads
		const bool is_k = head >= a.n_q_heads && rope;
		const int kvh = head - a.n_q_heads - (is_k ? 0 : a.n_kv_heads);
		// steps of two rows: row r = 2 * i + lane / 16
		for (int i0 = 0; 2 * i0 < rows; i0 += kTcEpiRowGroup) {
			float cs[kTcEpiRowGroup], sn[kTcEpiRowGroup];
#pragma unroll
			for (int j = 0; j < kTcEpiRowGroup; ++j) {
				const int r = 2 * (i0 + j) + (lane >> 4);
				const int pos = __shfl_sync(0xffffffffu, row_pos, r & 31);
				cs[j] = sn[j] = 0.0f;
				if (ok && rope && r < rows) {
					cs[j] = a.rope_cos[(size_t)pos * half + dim];
					sn[j] = a.rope_sin[(size_t)pos * half + dim];
				}
			}
#pragma unroll
			for (int j = 0; j < kTcEpiRowGroup; ++j) {
				const int r = 2 * (i0 + j) + (lane >> 4);
				const int pos = __shfl_sync(0xffffffffu, row_pos, r & 31);
				const int page = __shfl_sync(0xffffffffu, row_page, r & 31);
				if (!ok || r >= rows) continue;
				const float v = st[r * 33 + 2 * p], v1 = st[r * 33 + 2 * p + 1];
				float o0 = v, o1 = v1;
				if (rope) {
					o0 = __fsub_rn(__fmul_rn(v, cs[j]), __fmul_rn(v1, sn[j]));
					o1 = __fadd_rn(__fmul_rn(v1, cs[j]), __fmul_rn(v, sn[j]));
				}
				if (head < a.n_q_heads) {
					bf16* q = reinterpret_cast<bf16*>(a.out) + ((size_t)(t0 + r) * a.n_q_heads + head) * hd;
					Store<bf16>::put(q + dim, o0);
					Store<bf16>::put(q + dim + half, o1);
				} else if (page < 0 || page >= a.max_pages) {
					report_err(a.err, kDevKvRange);
				} else {
					bf16* base = reinterpret_cast<bf16*>(is_k ? a.kpool : a.vpool) +
					             (((size_t)page * a.n_kv_heads + kvh) * a.kv_block + (pos % a.kv_block)) * hd;
					Store<bf16>::put(base + dim, o0);
					Store<bf16>::put(base + dim + half, o1);
				}
			}
		}
	} else {
		// store / f32 store / logits with argmax: nothing to load per row
		for (int r = 0; r < rows; ++r) tc_epilogue_lane(a, t0 + r, n0 + lane, st[r * 33 + lane], n_lim);
	}
}

// Persistent tensor-core GEMM.  Work units are (M tile, N tile, K split) triples, M fastest
// (the CTAs working at the same time share each weight tile through L2); CTA b takes units
// b, b + gridDim.x, ...  Two 256-column TMEM accumulators let the MMAs of a CTA's next unit
// run while the epilogue warps drain the previous one.
__global__ void __launch_bounds__(kTcThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, const TcArgs a)
{
	extern __shared__ __align__(1024) uint8_t smem_raw[];
	// 1024-byte aligned tile area (SWIZZLE_128B atoms)
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
	uint8_t* tiles = smem;
	float* stage_out = reinterpret_cast<float*>(smem + kTcStages * kTcStageBytes); // [4 warps][32][33]
	uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes + kTcOutStageBytes);
	uint64_t* empty = full + kTcStages;
	uint64_t* acc_full = empty + kTcStages;  // [kTcAccBufs]
	uint64_t* acc_empty = acc_full + kTcAccBufs;
	uint64_t* drained = acc_empty + kTcAccBufs;
	uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);
	volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int BN = a.bn > 0 ? a.bn : kTcBN;
	const int m_tiles = (a.T + kTcBM - 1) / kTcBM, n_tiles = (a.N + BN - 1) / BN;
	const uint32_t stage_tx = kTcStageA + (uint32_t)BN * kTcBK * 2; // full boxes, out-of-range rows zero-filled
	const int n_kb_all = (a.K + kTcBK - 1) / kTcBK;
	const int S = a.k_splits > 1 ? a.k_splits : 1;
	const int units = m_tiles * n_tiles * S;

	if (threadIdx.x == 0) {
		for (int s = 0; s < kTcStages; ++s) {
			mbar_init(&full[s], 1);
			mbar_init(&empty[s], 1);
		}
		for (int b = 0; b < kTcAccBufs; ++b) {
			mbar_init(&acc_full[b], 1);
			mbar_init(&acc_empty[b], kTcEpiWarps);
		}
		mbar_init(drained, 1);
		*abort_flag = 0;
		mbar_fence_init();
	}
	if (warp == 1) {
		asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
		             "r"(kTcTmemCols)
		             : "memory");
		asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem_d = *tmem_slot;
	pdl_trigger();

	if (warp == 0) {
		if (lane == 0) {
			// weights: streamed once when one M tile covers every token (decode batches), else
			// shared by the CTAs of one N tile's M tiles; the activation tile is kept in L2 for
			// the other N tiles while it fits there comfortably
			const uint64_t pol_w = m_tiles > 1 ? policy_evict_normal() : policy_evict_first();
			const uint64_t pol_x = (size_t)a.T * a.K * 2 <= kTcKeepXBytes ? policy_evict_last() : policy_evict_normal();
			int it = 0; // k blocks issued so far (ring position)
			bool waited = false;
			for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
				const int m_tile = u % m_tiles, n_tile = (u / m_tiles) % n_tiles, z = u / (m_tiles * n_tiles);
				const int kb0 = (int)(((long long)z * n_kb_all) / S);
				const int n_kb = (int)(((long long)(z + 1) * n_kb_all) / S) - kb0;
				int kb = 0;
				if (!waited) {
					// the first unit's first weight tiles before the dependency wait (W is never
					// written by a kernel of the step); their X tiles, which the previous kernel
					// writes, after it
					const int pre = min(n_kb, kTcStages);
					for (; kb < pre; ++kb) {
						mbar_arrive_expect_tx(&full[kb], stage_tx);
						tma_load_2d(tiles + (size_t)kb * kTcStageBytes + kTcStageA, &tm_w, (kb0 + kb) * kTcBK,
						            n_tile * BN, &full[kb], pol_w);
					}
					pdl_wait();
					waited = true;
					for (int i = 0; i < pre; ++i)
						tma_load_2d(tiles + (size_t)i * kTcStageBytes, &tm_x, (kb0 + i) * kTcBK, m_tile * kTcBM, &full[i],
						            pol_x);
					it = pre;
				}
				for (; kb < n_kb; ++kb, ++it) {
					const int s = it % kTcStages;
					if (it >= kTcStages && !mbar_wait(&empty[s], ((it / kTcStages) - 1) & 1, abort_flag, a.err)) break;
					uint8_t* sa = tiles + (size_t)s * kTcStageBytes;
					mbar_arrive_expect_tx(&full[s], stage_tx);
					tma_load_2d(sa, &tm_x, (kb0 + kb) * kTcBK, m_tile * kTcBM, &full[s], pol_x);
					tma_load_2d(sa + kTcStageA, &tm_w, (kb0 + kb) * kTcBK, n_tile * BN, &full[s], pol_w);
				}
			}
			if (!waited) pdl_wait();
			// the loads still in flight land before the CTA may exit (only the last ring-full can be)
			for (int i = max(0, it - kTcStages); i < it; ++i) {
				const int s = i % kTcStages;
				const uint64_t t0 = global_timer_ns();
				while (!mbar_try_wait(&full[s], (i / kTcStages) & 1))
					if (global_timer_ns() - t0 > kWaitLimitNs) {
						report_err(a.err, kDevTimeout);
						break;
					}
			}
		}
	} else if (warp == 1) {
		if (lane == 0) {
			const uint32_t idesc = umma_idesc_bf16(kTcBM, BN);
			int it = 0, ub = 0;
			for (int u = blockIdx.x; u < units; u += gridDim.x, ++ub) {
				const int z = u / (m_tiles * n_tiles);
				const int n_kb = (int)(((long long)(z + 1) * n_kb_all) / S) - (int)(((long long)z * n_kb_all) / S);
				const int b = ub & 1;
				// the epilogue has drained this accumulator's previous unit
				if (ub >= kTcAccBufs && !mbar_wait(&acc_empty[b], ((ub >> 1) - 1) & 1, abort_flag, a.err)) break;
				tc_fence_after();
				const uint32_t acc = tmem_d + (uint32_t)(b * kTcBN);
				bool ok = true;
				for (int kb = 0; kb < n_kb; ++kb, ++it) {
					const int s = it % kTcStages;
					if (!mbar_wait(&full[s], (it / kTcStages) & 1, abort_flag, a.err)) {
						ok = false;
						break;
					}
					tc_fence_after();
					const uint32_t sa = smem_u32(tiles + (size_t)s * kTcStageBytes);
					const uint32_t sb = sa + kTcStageA;
#pragma unroll
					for (int k = 0; k < kTcBK / 16; ++k)
						umma_bf16(acc, umma_desc_sw128(sa + k * 32), umma_desc_sw128(sb + k * 32), idesc,
						          (kb > 0 || k > 0) ? 1u : 0u);
					umma_commit(&empty[s]); // stage free once these MMAs have read it
				}
				if (!ok) break;
				umma_commit(&acc_full[b]); // accumulator complete once every MMA above has finished
			}
			umma_commit(drained); // always: completes when every MMA this thread issued has finished
		}
	} else {
		// epilogue warps 2..9: TMEM lane quarter = warp % 4 (token rows t0 .. t0 + 31 of the
		// tile); warps 2..5 take columns 0..127 of the tile, warps 6..9 columns 128..255
		const int quarter = warp & 3, c_begin = ((warp - 2) >> 2) * (kTcBN / 2), c_end = min(c_begin + kTcBN / 2, BN);
		float* st = stage_out + (warp - 2) * (32 * 33);
		int ub = 0;
		for (int u = blockIdx.x; u < units; u += gridDim.x, ++ub) {
			const int m_tile = u % m_tiles, n_tile = (u / m_tiles) % n_tiles, z = u / (m_tiles * n_tiles);
			const int b = ub & 1;
			if (!mbar_wait(&acc_full[b], (ub >> 1) & 1, abort_flag, a.err)) break;
			tc_fence_after();
			const int t0 = m_tile * kTcBM + quarter * 32;
			if (t0 < a.T) {
				const int rows = min(32, a.T - t0);
				// QKV: lane r holds the position and KV page of token row t0 + r
				int row_pos = 0, row_page = -1;
				if (a.epi == kTcQkv && S == 1 && lane < rows) {
					row_pos = a.tok_pos[t0 + lane];
					if (row_pos >= 0 && row_pos < a.max_seq)
						row_page = a.block_table[(size_t)a.tok_slot[t0 + lane] * a.pages_per_seq + row_pos / a.kv_block];
				}
				// columns of this tile and half: n0 .. n_lim - 1 (the last chunk may be 16 wide)
				const int n_lim = min(a.N, n_tile * BN + c_end);
				for (int c = c_begin; c < c_end; c += 32) {
					const int n0 = n_tile * BN + c;
					if (n0 >= n_lim) break;
					float v[32];
					tmem_ld_32cols(tmem_d + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * kTcBN + c), v);
					// transpose through shared memory: lane = column, one row per step
#pragma unroll
					for (int i = 0; i < 32; ++i) st[lane * 33 + i] = v[i];
					__syncwarp();
					if (S > 1) {
						float* pp = a.partial + ((size_t)z * a.T + t0) * a.N + n0 + lane;
						if (n0 + lane < n_lim)
							for (int r = 0; r < rows; ++r) pp[(size_t)r * a.N] = st[r * 33 + lane];
					} else {
						tc_epilogue_rows(a, t0, rows, n0, st, row_pos, row_page, n_lim);
					}
					__syncwarp();
				}
			}
			tc_fence_before();
			__syncwarp();
			if (lane == 0) mbar_arrive(&acc_empty[b]);
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 1) {
		// the last commit's arrival (every MMA has finished; also after a wait gave up) before
		// TMEM is freed and the CTA's shared memory can be reused
		{
			const uint64_t t0 = global_timer_ns();
			while (!mbar_try_wait(drained, 0))
				if (global_timer_ns() - t0 > kWaitLimitNs) break;
		}
		tc_fence_after();
		asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kTcTmemCols) : "memory");
	}
}

// Sum of the split-K shares in split order, then the GEMM's epilogue.  A warp takes one
// (token row, 32 columns) group: lane i sums column n0 + i over the splits (coalesced, read
// from L2 where the GEMM left them) and runs the epilogue on that column.
__global__ void __launch_bounds__(256) k_gemm_splitk_reduce(const TcArgs a)
{
	pdl_wait();
	pdl_trigger();
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int groups = (a.N + 31) / 32;
	const int gw = blockIdx.x * 8 + warp;
	if (gw >= a.T * groups) return;
	const int t = gw / groups, n = (gw % groups) * 32 + lane;
	float v = 0.0f;
	if (n < a.N) {
		const float* p = a.partial + (size_t)t * a.N + n;
		const size_t zs = (size_t)a.T * a.N;
#pragma unroll 4
		for (int z = 0; z < a.k_splits; ++z) v += __ldcg(p + z * zs);
	}
	tc_epilogue_lane(a, t, n, v, a.N);
}

// A residual projection's split-K sum (O or down, kTcResid) added to the residual row, then
// the RMSNorm of the updated row into the next projection's bf16 input: the work of
// k_gemm_splitk_reduce and k_rmsnorm_rows in one launch of one CTA per token row, with the
// same fp32 operations in the same order (thread j owns columns j, j + 256, ..., the shares
// are added in split order, the squares summed as k_rmsnorm_rows sums them).
constexpr int kResNormThreads = 256;
constexpr int kResNormMaxCols = 32; // columns per thread: rows of up to 8192
template <int PER>
__global__ void __launch_bounds__(kResNormThreads) k_gemm_splitk_resid_norm(const TcArgs a, bf16* __restrict__ y,
                                                                            const bf16* __restrict__ gain, float eps)
{
	pdl_wait();
	pdl_trigger();
	const int t = blockIdx.x;
	if (t >= a.T) return;
	float* xr = a.resid + (size_t)t * a.N;
	const float* p = a.partial + (size_t)t * a.N + threadIdx.x;
	const size_t zs = (size_t)a.T * a.N;
	float r[PER];
#pragma unroll
	for (int j = 0; j < PER; ++j) r[j] = 0.0f;
	// U splits' loads in flight per round, added in split order
	constexpr int U = 64 / PER;
	int z = 0;
	for (; z + U <= a.k_splits; z += U) {
		float v[U][PER];
#pragma unroll
		for (int q = 0; q < U; ++q)
#pragma unroll
			for (int j = 0; j < PER; ++j)
				v[q][j] = threadIdx.x + j * kResNormThreads < a.N ? __ldcg(p + (z + q) * zs + j * kResNormThreads) : 0.0f;
#pragma unroll
		for (int q = 0; q < U; ++q)
#pragma unroll
			for (int j = 0; j < PER; ++j) r[j] += v[q][j];
	}
	for (; z < a.k_splits; ++z)
#pragma unroll
		for (int j = 0; j < PER; ++j)
			if (threadIdx.x + j * kResNormThreads < a.N) r[j] += __ldcg(p + z * zs + j * kResNormThreads);
	float ss = 0.0f;
#pragma unroll
	for (int j = 0; j < PER; ++j) {
		const int i = threadIdx.x + j * kResNormThreads;
		if (i < a.N) {
			r[j] = xr[i] + r[j];
			xr[i] = r[j];
			ss += r[j] * r[j];
		}
	}
	__shared__ float red[32];
	ss = warp_sum(ss);
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	if (lane == 0) red[warp] = ss;
	__syncthreads();
	if (warp == 0) {
		float v = lane < kResNormThreads / 32 ? red[lane] : 0.0f;
		v = warp_sum(v);
		if (lane == 0) red[0] = v;
	}
	__syncthreads();
	const float inv = 1.0f / sqrtf(__fdiv_rn(red[0], (float)a.N) + eps);
	bf16* yr = y + (size_t)t * a.N;
#pragma unroll
	for (int j = 0; j < PER; ++j) {
		const int i = threadIdx.x + j * kResNormThreads;
		if (i < a.N) Store<bf16>::put(yr + i, __fmul_rn(__fmul_rn(r[j], inv), Store<bf16>::get(gain + i)));
	}
}

// token ids from the argmax keys of kTcLogitsArgmax; the keys are cleared for the next use
__global__ void k_keys_to_ids(unsigned long long* keys, int n, uint32_t* ids)
{
	pdl_wait();
	pdl_trigger();
	const int i = blockIdx.x * blockDim.x + threadIdx.x;
	if (i < n) {
		ids[i] = argmax_key_index(keys[i]);
		keys[i] = 0ull;
	}
}

inline size_t gemm_tc_smem_bytes() { return 1024 + (size_t)kTcStages * kTcStageBytes + kTcOutStageBytes + 256; }
static_assert(kTcThreads == 64 + 32 * kTcEpiWarps, "producer, MMA and epilogue warps");
static_assert(1024 + (size_t)kTcStages * kTcStageBytes + kTcOutStageBytes + 256 <= 227 * 1024, "shared memory per CTA");

} // namespace inf
