// Tensor-parallel exchange over NVLink peer memory (one process per GPU, buffers of the
// peers' arenas mapped with CUDA IPC).  No TMA, no multicast: plain stores to peer memory,
// a system-scope release store of a round number as the flag, an acquire load to wait.
//
// Round numbers are shared by all ranks without communication: every rank runs the same
// steps, so round = (epoch + 1) * kTpRoundsPerStep + index, where epoch advances once per decode
// step (by the LM-head kernel) and index is fixed per call site (2 * layer + {0, 1} for the
// two all-reduces of a layer, kTpRoundLm for the argmax).
#pragma once

#include "common.cuh"

namespace inf {

constexpr int kTpMax = 8;
constexpr int kTpMaxCtas = 256;
constexpr int kTpRoundsPerStep = 256;
constexpr int kTpRoundLm = 255;
constexpr int kTpMaxRowsCta = 256; // rows a GEMV CTA may own when it exchanges them

struct TpComm {
	int rank, size;
	const uint32_t* epoch;                 // device counter, +1 per decode step
	// decode-step all-reduce of [dim] fp32 partials, double-buffered by round parity; each
	// slot is one 8-byte store of (value bits, round) so it carries its own flag
	unsigned long long* inbox[kTpMax];     // rank k's inbox base: [2][size][dim]
	// greedy argmax across vocabulary shards
	unsigned long long* am_inbox[kTpMax];  // rank k's: [2][size]
	unsigned* am_flags[kTpMax];            // rank k's: [size]
	// multi-token all-reduce of [T x dim] (two-shot: reduce-scatter, then all-gather)
	float* part[kTpMax];                   // rank k's partial sums [chunk x dim]
	float* red[kTpMax];                    // rank k's reduced copy [chunk x dim]
	unsigned* ready[kTpMax];               // rank k's: [size]
	unsigned* done[kTpMax];                // rank k's: [size][kTpMaxCtas]
	int dim;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v)
{
	asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v)
{
	asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p)
{
	unsigned long long v;
	asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
	return v;
}
__device__ __forceinline__ unsigned long long ll_pack(float v, unsigned round)
{
	return ((unsigned long long)round << 32) | __float_as_uint(v);
}

// Bounded wait until an (value, round) slot carries `round`; returns the value (0 and
// kDevTimeout if the peer never writes it).
__device__ __forceinline__ float ll_wait(const unsigned long long* slot, unsigned round, int* err, bool* ok)
{
	unsigned long long v = ld_relaxed_sys_u64(slot);
	if ((unsigned)(v >> 32) != round) {
		const uint64_t t0 = global_timer_ns();
		while ((unsigned)((v = ld_relaxed_sys_u64(slot)) >> 32) != round) {
			if (global_timer_ns() - t0 > kWaitLimitNs) {
				report_err(err, kDevTimeout);
				*ok = false;
				return 0.0f;
			}
		}
	}
	return __uint_as_float((unsigned)v);
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p)
{
	unsigned v;
	asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
	return v;
}

// Bounded wait until *flag has reached `round` (flags only move forward).  Returns false
// and records kDevTimeout if a peer never arrives.
__device__ __forceinline__ bool tp_wait_flag(const unsigned* flag, unsigned round, int* err)
{
	if ((int)(ld_acquire_sys(flag) - round) >= 0) return true;
	const uint64_t t0 = global_timer_ns();
	while ((int)(ld_acquire_sys(flag) - round) < 0) {
		if (global_timer_ns() - t0 > kWaitLimitNs) {
			report_err(err, kDevTimeout);
			return false;
		}
	}
	return true;
}

// never 0: exchange buffers start zeroed, and a zero round would look complete
__device__ __forceinline__ unsigned tp_round(const TpComm& c, int index) { return (*c.epoch + 1u) * kTpRoundsPerStep + index; }

// Two-shot all-reduce of part[0..n) across ranks, added into dst (every rank ends with the
// same dst: slices are reduced in rank order and the reduced values are copied, not
// re-summed).  Grid: any number of CTAs <= kTpMaxCtas; launched right after the kernel
// that wrote `part`.
__global__ void __launch_bounds__(256) k_tp_allreduce_add(TpComm c, int n, unsigned round_index, float* dst, int* err)
{
	pdl_wait();
	pdl_trigger();
	const unsigned round = tp_round(c, (int)round_index);
	const int me = c.rank, N = c.size, g = blockIdx.x, G = gridDim.x;
	__shared__ int ok;
	if (threadIdx.x == 0) {
		ok = 1;
		// my partials are complete (kernel boundary): tell every rank
		for (int k = 0; k < N; ++k) st_release_sys(c.ready[k] + me, round);
		for (int k = 0; k < N; ++k)
			if (!tp_wait_flag(c.ready[me] + k, round, err)) ok = 0;
	}
	__syncthreads();
	// reduce-scatter: rank `me` owns slice [s0, s1); CTA g a contiguous piece of it
	const int s0 = (int)((long long)n * me / N), s1 = (int)((long long)n * (me + 1) / N);
	const int p0 = s0 + (int)((long long)(s1 - s0) * g / G), p1 = s0 + (int)((long long)(s1 - s0) * (g + 1) / G);
	if (ok) {
		for (int i = p0 + threadIdx.x; i < p1; i += blockDim.x) {
			float v = 0.0f;
			for (int k = 0; k < N; ++k) v += __ldcv(c.part[k] + i);
			for (int k = 0; k < N; ++k) c.red[k][i] = v;
		}
	}
	__syncthreads(); // orders every thread's peer stores before thread 0's fence and release
	if (threadIdx.x == 0) {
		__threadfence_system();
		for (int k = 0; k < N; ++k) st_release_sys(c.done[k] + me * kTpMaxCtas + g, round);
		for (int k = 0; k < N; ++k)
			if (!tp_wait_flag(c.done[me] + k * kTpMaxCtas + g, round, err)) ok = 0;
	}
	__syncthreads();
	if (!ok) return;
	// all-gather done: piece g of every rank's slice is in my `red`
	for (int k = 0; k < N; ++k) {
		const int t0 = (int)((long long)n * k / N), t1 = (int)((long long)n * (k + 1) / N);
		const int q0 = t0 + (int)((long long)(t1 - t0) * g / G), q1 = t0 + (int)((long long)(t1 - t0) * (g + 1) / G);
		for (int i = q0 + threadIdx.x; i < q1; i += blockDim.x) dst[i] += __ldcv(c.red[me] + i);
	}
}

} // namespace inf
