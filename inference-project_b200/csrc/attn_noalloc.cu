// Decode attention for callers that cannot allocate device memory.
//
// inf_attn_decode needs a scratch buffer (the split-K partial results, the per-head tickets
// and an error word) that its caller provides.  Some callers cannot provide one: a serving
// loop in the middle of a step cannot call cudaMalloc/cudaFree, which synchronize the whole
// device and stall every other stream; a runtime whose device memory is entirely committed
// to a pre-sized arena (as this library's DevArena and the reference's are) has nothing left
// to allocate from; a host framework that owns all device memory through its own allocator
// may forbid allocations outside it.  inf_attn_decode_noalloc serves them from a scratch
// array that is part of the library image itself.
#include <mutex>

#include "../../include/inf.h"
#include "runtime.h"

namespace {

// Largest scratch one call may use.  Batch-1 decode of the Llama-3-8B shape needs ~0.3 MiB
// at 3k positions and ~2.9 MiB at the 32k-token maximum context.
constexpr u64 kNoAllocScratchBytes = 4ull << 20;
constexpr int kNoAllocMaxDevices = 64;

// Every GPU that loads this library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_addr[kNoAllocMaxDevices] = {};

// Device address of g_attn_scratch on the current device.  In host code the array's name
// is only a host-side stand-in, so the address comes from cudaGetSymbolAddress, once per
// device, with that device current.  The address is kept for the life of the process: a
// cudaDeviceReset (which unloads this module from the device) invalidates it, so the library
// must not be used on a device after that device was reset.
Error_t scratch_address(void** out)
{
	int dev = 0;
	INF_CUDA_TRY(cudaGetDevice(&dev));
	if (dev < 0 || dev >= kNoAllocMaxDevices) return inf::fail(ErrorUnsupported, "device %d beyond %d", dev, kNoAllocMaxDevices);
	std::lock_guard<std::mutex> lk(g_setup_mutex);
	if (!g_scratch_addr[dev]) {
		void* p = nullptr;
		const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
		if (e != cudaSuccess || !p)
			return inf::fail(ErrorCuda, "cudaGetSymbolAddress(no-alloc attention scratch): %s", cudaGetErrorString(e));
		g_scratch_addr[dev] = p;
	}
	*out = g_scratch_addr[dev];
	return Success;
}

} // namespace

extern "C" Error_t inf_attn_decode_noalloc(const void* d_q, const void* d_kpool, const void* d_vpool,
                                           const i32* d_block_table, u32 pages_per_seq, u32 n_pages,
                                           const i32* d_tok_slot, const i32* d_tok_pos, u32 n_tokens, u32 n_heads,
                                           u32 n_kv_heads, u32 head_dim, u32 kv_block, u32 dtype, void* d_out,
                                           void* stream)
{
	const u64 need = inf_attn_decode_scratch_bytes(n_tokens, n_heads, n_kv_heads, head_dim, kv_block, pages_per_seq, dtype);
	if (need > kNoAllocScratchBytes)
		return inf::fail(ErrorInvalidValue,
		                 "inf_attn_decode_noalloc: this shape needs %llu bytes of scratch, above the built-in %llu; "
		                 "use inf_attn_decode with caller-provided scratch",
		                 (unsigned long long)need, (unsigned long long)kNoAllocScratchBytes);
	void* scratch = nullptr;
	INF_TRY(scratch_address(&scratch));
	// need == 0: a shape the attention cannot serve; inf_attn_decode's own checks report why
	// (the same error the scratch-taking entry point gives), before anything is launched
	// inf_attn_decode clears the tickets and the error word on the stream before the kernel,
	// so what a previous call left in the array does not matter
	return inf_attn_decode(d_q, d_kpool, d_vpool, d_block_table, pages_per_seq, n_pages, d_tok_slot, d_tok_pos, n_tokens,
	                       n_heads, n_kv_heads, head_dim, kv_block, dtype, d_out, scratch, kNoAllocScratchBytes, stream);
}
