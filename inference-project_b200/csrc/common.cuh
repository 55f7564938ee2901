// Device-side building blocks shared by every kernel of libinf.so (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/inf.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libinf.so is built for sm_100a only"
#endif

typedef __nv_bfloat16 bf16;

namespace inf {

constexpr int kWarp = 32;

// device error word codes (written with atomicCAS so the first failure wins)
enum DevErr : int {
	kDevOk = 0,
	kDevTimeout = 1,
	kDevTokenRange = 2,
	kDevKvRange = 3,
};

// A bounded wait gives up after this long; the kernel then records kDevTimeout and
// finishes without touching the data it was waiting for.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ void report_err(int* err, int code)
{
	if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint64_t global_timer_ns()
{
	uint64_t t;
	asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
	return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
	return (uint32_t)__cvta_generic_to_shared(p);
}

// ---- bf16 <-> f32 (bit-level, round to nearest even) ----------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__host__ __device__ __forceinline__ uint16_t f32_to_bf16_bits(float x)
{
#if defined(__CUDA_ARCH__)
	uint32_t u = __float_as_uint(x);
#else
	uint32_t u;
	memcpy(&u, &x, 4);
#endif
	if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)0x7FC0u;
	u += 0x7FFFu + ((u >> 16) & 1u);
	return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float round_bf16(float x) { return __uint_as_float((uint32_t)f32_to_bf16_bits(x) << 16); }

// storage element traits: the type values are stored in between kernels
template <typename T> struct Store;
template <> struct Store<float> {
	static constexpr int kVec = 4; // elements per 16-byte unit
	__device__ static __forceinline__ float round(float x) { return x; }
	__device__ static __forceinline__ void put(float* p, float x) { *p = x; }
	__device__ static __forceinline__ float get(const float* p) { return *p; }
};
template <> struct Store<bf16> {
	static constexpr int kVec = 8;
	__device__ static __forceinline__ float round(float x) { return round_bf16(x); }
	__device__ static __forceinline__ void put(bf16* p, float x)
	{
		*reinterpret_cast<uint16_t*>(p) = f32_to_bf16_bits(x);
	}
	__device__ static __forceinline__ float get(const bf16* p)
	{
		return __uint_as_float((uint32_t)(*reinterpret_cast<const uint16_t*>(p)) << 16);
	}
};

// unpack one 16-byte unit into floats
__device__ __forceinline__ void unpack_unit(const uint4& u, float* out, const bf16*)
{
	out[0] = bf16_lo(u.x); out[1] = bf16_hi(u.x);
	out[2] = bf16_lo(u.y); out[3] = bf16_hi(u.y);
	out[4] = bf16_lo(u.z); out[5] = bf16_hi(u.z);
	out[6] = bf16_lo(u.w); out[7] = bf16_hi(u.w);
}
__device__ __forceinline__ void unpack_unit(const uint4& u, float* out, const float*)
{
	out[0] = __uint_as_float(u.x); out[1] = __uint_as_float(u.y);
	out[2] = __uint_as_float(u.z); out[3] = __uint_as_float(u.w);
}

// ---- programmatic dependent launch ----------------------------------------------------
// Pre-wait code may only read memory that no kernel of the same step writes (weights).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- mbarrier + bulk copy (no multicast anywhere in this library) ----------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
	asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
	asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
	             : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
	asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
	uint32_t ok;
	asm volatile(
	    "{\n\t.reg .pred p;\n\t"
	    "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
	    "selp.u32 %0, 1, 0, p;\n\t}"
	    : "=r"(ok)
	    : "r"(smem_u32(bar)), "r"(parity)
	    : "memory");
	return ok != 0;
}
// Bounded wait on an mbarrier phase.  Returns false (and records kDevTimeout once) if the
// phase did not complete within kWaitLimitNs, or immediately if *abort is already set.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err)
{
	if (mbar_try_wait(bar, parity)) return true;
	const uint64_t t0 = global_timer_ns();
	for (uint32_t it = 1;; ++it) {
		if (mbar_try_wait(bar, parity)) return true;
		if ((it & 63u) == 0) {
			if (*abort) return false;
			if (global_timer_ns() - t0 > kWaitLimitNs) {
				*abort = 1;
				report_err(err, kDevTimeout);
				return false;
			}
		}
	}
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes multiple of 16,
// both addresses 16-byte aligned).  evict_first: weights are streamed once per step.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy)
{
	asm volatile(
	    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
	        smem_u32(dst)),
	    "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
	    : "memory");
}
// Bulk prefetch of a global range into L2 (no shared memory, no completion tracking).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes)
{
	asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first()
{
	uint64_t p;
	asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
	return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal()
{
	uint64_t p;
	asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
	return p;
}
__device__ __forceinline__ uint64_t policy_evict_last()
{
	uint64_t p;
	asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
	return p;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads)
{
	asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
	for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
	return v;
}
__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
	for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
	return v;
}

// (value, index) packed so that an unsigned max picks the largest value and, among equal
// values, the lowest index.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx)
{
	uint32_t u = __float_as_uint(v);
	u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
	return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long k) { return 0xFFFFFFFFu - (uint32_t)k; }

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }
// GELU, tanh approximation: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
__device__ __forceinline__ float gelu_tanh(float x)
{
	return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

} // namespace inf
