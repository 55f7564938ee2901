// Prefill / multi-token projections on the 5th-generation tensor cores (sm_100a).
//
// D[T x N] = X[T x K] . W[N x K]^T, bf16 inputs, fp32 accumulation in tensor memory.
// One CTA computes one 128 x 256 output tile:
//   warp 0      TMA producer: 2-D tiled bulk tensor loads (SWIZZLE_128B, no multicast) of
//               X[128 x 64] and W[256 x 64] per stage into a 4-stage shared-memory ring
//   warp 1      allocates 256 TMEM columns; one elected lane issues tcgen05.mma
//               (kind::f16, M=128, N=256, K=16; both operands K-major) and tcgen05.commit
//               frees each stage and finally signals the accumulator
//   warps 2..5  epilogue: tcgen05.ld 32x32b (row = TMEM lane = token) and the same fused
//               epilogues as the decode GEMV (store, residual add, RoPE + KV-cache write,
//               SwiGLU) on adjacent column pairs, or fp32 logits with a per-row greedy
//               argmax folded in (atomicMax of a (value, column) key)
// When the output has too few tiles to fill the SMs (a batch of decode tokens), blockIdx.z
// splits the K blocks; each split writes fp32 partials and k_gemm_splitk_reduce sums them
// and runs the epilogue.
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
constexpr int kTcThreads = 192;
constexpr uint32_t kTcStageA = kTcBM * kTcBK * 2;
constexpr uint32_t kTcStageB = kTcBN * kTcBK * 2;
constexpr uint32_t kTcStageBytes = kTcStageA + kTcStageB;
constexpr int kTcTmemCols = 256;

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

// Epilogue for one token row and 32 consecutive output columns n0 .. n0+31.
__device__ __forceinline__ void tc_epilogue_row(const TcArgs& a, int t, int n0, const float (&v)[32])
{
	if (a.epi == kTcStoreF32 || a.epi == kTcLogitsArgmax) {
		float* o = reinterpret_cast<float*>(a.out) + (size_t)t * a.N;
		unsigned long long best = 0ull;
#pragma unroll
		for (int i = 0; i < 32; ++i)
			if (n0 + i < a.N) {
				o[n0 + i] = v[i];
				const unsigned long long k = argmax_key(v[i], (uint32_t)(n0 + i) + a.col_base);
				best = k > best ? k : best;
			}
		if (a.epi == kTcLogitsArgmax) atomicMax(a.best_keys + t, best);
	} else if (a.epi == kTcStore) {
		bf16* o = reinterpret_cast<bf16*>(a.out) + (size_t)t * a.N;
#pragma unroll
		for (int i = 0; i < 32; ++i)
			if (n0 + i < a.N) Store<bf16>::put(o + n0 + i, v[i]);
	} else if (a.epi == kTcResid) {
		float* r = a.resid + (size_t)t * a.N;
#pragma unroll
		for (int i = 0; i < 32; ++i)
			if (n0 + i < a.N) r[n0 + i] += v[i];
	} else if (a.epi == kTcSwiglu) {
		bf16* o = reinterpret_cast<bf16*>(a.out) + (size_t)t * (a.N >> 1);
#pragma unroll
		for (int i = 0; i < 32; i += 2)
			if (n0 + i + 1 < a.N) Store<bf16>::put(o + ((n0 + i) >> 1), __fmul_rn(silu(v[i]), v[i + 1]));
	} else if (a.epi == kTcQkv) {
		const int hd = a.head_dim, half = hd >> 1;
		const int pos = a.tok_pos[t], slot = a.tok_slot[t];
		int page = -1;
		if (pos >= 0 && pos < a.max_seq) page = a.block_table[(size_t)slot * a.pages_per_seq + pos / a.kv_block];
#pragma unroll
		for (int i = 0; i < 32; i += 2) {
			const int row = n0 + i;
			if (row >= a.N) continue;
			const int head = row / hd, dim = (row % hd) >> 1;
			const float d0 = v[i], d1 = v[i + 1];
			float o0 = d0, o1 = d1;
			if (head < a.n_q_heads + a.n_kv_heads) {
				const float c = a.rope_cos[(size_t)pos * half + dim];
				const float s = a.rope_sin[(size_t)pos * half + dim];
				o0 = __fsub_rn(__fmul_rn(d0, c), __fmul_rn(d1, s));
				o1 = __fadd_rn(__fmul_rn(d1, c), __fmul_rn(d0, s));
			}
			if (head < a.n_q_heads) {
				bf16* q = reinterpret_cast<bf16*>(a.out) + ((size_t)t * a.n_q_heads + head) * hd;
				Store<bf16>::put(q + dim, o0);
				Store<bf16>::put(q + dim + half, o1);
			} else if (page < 0 || page >= a.max_pages) {
				report_err(a.err, kDevKvRange);
			} else {
				const bool is_k = head < a.n_q_heads + a.n_kv_heads;
				const int kvh = head - a.n_q_heads - (is_k ? 0 : a.n_kv_heads);
				bf16* base = reinterpret_cast<bf16*>(is_k ? a.kpool : a.vpool) +
				             (((size_t)page * a.n_kv_heads + kvh) * a.kv_block + (pos % a.kv_block)) * hd;
				Store<bf16>::put(base + dim, o0);
				Store<bf16>::put(base + dim + half, o1);
			}
		}
	}
}

__global__ void __launch_bounds__(kTcThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, const TcArgs a)
{
	extern __shared__ __align__(1024) uint8_t smem_raw[];
	// 1024-byte aligned tile area (SWIZZLE_128B atoms)
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
	uint8_t* tiles = smem;
	uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes);
	uint64_t* empty = full + kTcStages;
	uint64_t* acc_full = empty + kTcStages;
	uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
	volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int n_tile = blockIdx.x, m_tile = blockIdx.y;
	const int n_kb_all = (a.K + kTcBK - 1) / kTcBK;
	const int S = a.k_splits > 1 ? a.k_splits : 1;
	const int kb0 = (int)(((long long)blockIdx.z * n_kb_all) / S);
	const int n_kb = (int)(((long long)(blockIdx.z + 1) * n_kb_all) / S) - kb0;

	if (threadIdx.x == 0) {
		for (int s = 0; s < kTcStages; ++s) {
			mbar_init(&full[s], 1);
			mbar_init(&empty[s], 1);
		}
		mbar_init(acc_full, 1);
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
			const uint64_t pol_w = policy_evict_first();
			const uint64_t pol_x = policy_evict_last();
			// the first stages' weight tiles before the dependency wait (W is never written by a
			// kernel of the step); their X tiles, which the previous kernel writes, after it
			const int pre = min(n_kb, kTcStages);
			for (int kb = 0; kb < pre; ++kb) {
				mbar_arrive_expect_tx(&full[kb], kTcStageBytes);
				tma_load_2d(tiles + (size_t)kb * kTcStageBytes + kTcStageA, &tm_w, (kb0 + kb) * kTcBK, n_tile * kTcBN,
				            &full[kb], pol_w);
			}
			pdl_wait();
			for (int kb = 0; kb < pre; ++kb)
				tma_load_2d(tiles + (size_t)kb * kTcStageBytes, &tm_x, (kb0 + kb) * kTcBK, m_tile * kTcBM, &full[kb], pol_x);
			int issued = pre;
			for (int kb = pre; kb < n_kb; ++kb) {
				const int s = kb % kTcStages;
				if (kb >= kTcStages && !mbar_wait(&empty[s], ((kb / kTcStages) - 1) & 1, abort_flag, a.err)) break;
				uint8_t* sa = tiles + (size_t)s * kTcStageBytes;
				mbar_arrive_expect_tx(&full[s], kTcStageBytes);
				tma_load_2d(sa, &tm_x, (kb0 + kb) * kTcBK, m_tile * kTcBM, &full[s], pol_x);
				tma_load_2d(sa + kTcStageA, &tm_w, (kb0 + kb) * kTcBK, n_tile * kTcBN, &full[s], pol_w);
				++issued;
			}
			for (int i = max(0, issued - kTcStages); i < issued; ++i) {
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
			constexpr uint32_t idesc = umma_idesc_bf16(kTcBM, kTcBN);
			for (int kb = 0; kb < n_kb; ++kb) {
				const int s = kb % kTcStages;
				if (!mbar_wait(&full[s], (kb / kTcStages) & 1, abort_flag, a.err)) break;
				tc_fence_after();
				const uint32_t sa = smem_u32(tiles + (size_t)s * kTcStageBytes);
				const uint32_t sb = sa + kTcStageA;
#pragma unroll
				for (int k = 0; k < kTcBK / 16; ++k)
					umma_bf16(tmem_d, umma_desc_sw128(sa + k * 32), umma_desc_sw128(sb + k * 32), idesc,
					          (kb > 0 || k > 0) ? 1u : 0u);
				umma_commit(&empty[s]); // stage free once these MMAs have read it
			}
			umma_commit(acc_full); // always: completes when every issued MMA has finished
		}
	} else {
		// epilogue warps 2..5: TMEM lane quarter = warp % 4
		const int quarter = warp & 3;
		const bool ok = mbar_wait(acc_full, 0, abort_flag, a.err);
		tc_fence_after();
		const int t = m_tile * kTcBM + quarter * 32 + lane;
		if (ok && !*abort_flag) {
			for (int c = 0; c < kTcBN; c += 32) {
				const int n0 = n_tile * kTcBN + c;
				if (n0 >= a.N) break;
				float v[32];
				tmem_ld_32cols(tmem_d + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c, v);
				if (t < a.T) {
					if (S > 1) {
						float* pp = a.partial + ((size_t)blockIdx.z * a.T + t) * a.N;
#pragma unroll
						for (int i = 0; i < 32; ++i)
							if (n0 + i < a.N) pp[n0 + i] = v[i];
					} else {
						tc_epilogue_row(a, t, n0, v);
					}
				}
			}
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 1) {
		// MMAs have all completed (acc_full) unless the wait timed out; wait for them once more
		if (*abort_flag) {
			const uint64_t t0 = global_timer_ns();
			while (!mbar_try_wait(acc_full, 0))
				if (global_timer_ns() - t0 > kWaitLimitNs) break;
		}
		tc_fence_after();
		asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kTcTmemCols) : "memory");
	}
}

// Sum of the split-K shares in split order, then the GEMM's epilogue.  A warp takes one
// (token row, 32 columns) group: lane i sums column n0 + i over the splits (coalesced), and
// lane 0 runs the epilogue on the 32 sums.
__global__ void __launch_bounds__(256) k_gemm_splitk_reduce(const TcArgs a)
{
	pdl_wait();
	pdl_trigger();
	__shared__ float st[8][32];
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int groups = (a.N + 31) / 32;
	const int gw = blockIdx.x * 8 + warp;
	if (gw >= a.T * groups) return;
	const int t = gw / groups, n0 = (gw % groups) * 32;
	float v = 0.0f;
	if (n0 + lane < a.N)
		for (int z = 0; z < a.k_splits; ++z) v += a.partial[((size_t)z * a.T + t) * a.N + n0 + lane];
	st[warp][lane] = v;
	__syncwarp();
	if (lane == 0) {
		float vals[32];
#pragma unroll
		for (int i = 0; i < 32; ++i) vals[i] = st[warp][i];
		tc_epilogue_row(a, t, n0, vals);
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

inline size_t gemm_tc_smem_bytes() { return 1024 + (size_t)kTcStages * kTcStageBytes + 256; }

} // namespace inf
