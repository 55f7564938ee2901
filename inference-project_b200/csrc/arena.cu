// Execution context, host and device arenas, checked copies and error strings.
//
// Semantics follow the reference (src/allocator.c:53-188, src/cuda/api/cuda_allocator.cu:4-68,
// src/cuda/api/cuda_mem_wrapper.cu:9-70) with three deliberate differences: nothing aborts
// (every failure returns an Error_t), device pushes are 256-byte aligned (the reference's
// 8-byte alignment, defect D9, breaks vector loads and bulk copies), and the host arena
// commits exactly the pages it grows into (defect D11).
#include <sys/mman.h>
#include <unistd.h>

#include <cstring>

#include "runtime.h"

namespace inf {

static thread_local char g_detail[512] = "";

Error_t fail(Error_t err, const char* fmt, ...)
{
	va_list ap;
	va_start(ap, fmt);
	vsnprintf(g_detail, sizeof g_detail, fmt, ap);
	va_end(ap);
	return err;
}

bool is_device_ptr(const void* p)
{
	if (!p) return false;
	cudaPointerAttributes a;
	if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
		cudaGetLastError();
		return false;
	}
	return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

} // namespace inf

using inf::fail;

static inline u64 pad_pow2(u64 n, u64 p) { return (p - (n & (p - 1))) & (p - 1); }

extern "C" {

const char* inf_error_string(Error_t err)
{
	switch (err) {
	case Success: return "Success";
	case ErrorMemoryAllocation: return "ErrorMemoryAllocation";
	case ErrorArenaOutOfMemory: return "ErrorArenaOutOfMemory";
	case ErrorAlreadyInitialized: return "ErrorAlreadyInitialized";
	case ErrorInvalidValue: return "ErrorInvalidValue";
	case ErrorInvalidHostPtr: return "ErrorInvalidHostPtr";
	case ErrorInvalidDevPtr: return "ErrorInvalidDevPtr";
	case ErrorGeneric: return "ErrorGeneric";
	case ErrorCuda: return "ErrorCuda";
	case ErrorBadConfig: return "ErrorBadConfig";
	case ErrorTokenOutOfRange: return "ErrorTokenOutOfRange";
	case ErrorKvOutOfRange: return "ErrorKvOutOfRange";
	case ErrorNccl: return "ErrorNccl";
	case ErrorTimeout: return "ErrorTimeout";
	case ErrorIo: return "ErrorIo";
	case ErrorUnsupported: return "ErrorUnsupported";
	}
	return "unknown Error_t";
}

const char* inf_last_error_detail(void) { return inf::g_detail; }

/* ---- host arena: reserve address space, commit in commit_size steps ---------------- */

Error_t arena_host_create(HostArena** const arena, const u64 reserve_size, const u64 commit_size)
{
	if (!arena || reserve_size == 0 || commit_size == 0 || commit_size > reserve_size)
		return fail(ErrorInvalidValue, "arena_host_create: bad sizes");
	const u64 page = (u64)sysconf(_SC_PAGESIZE);
	const u64 reserve = reserve_size + pad_pow2(reserve_size, page);
	const u64 commit = commit_size + pad_pow2(commit_size, page);
	void* p = mmap(NULL, reserve, PROT_NONE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
	if (p == MAP_FAILED) return fail(ErrorMemoryAllocation, "arena_host_create: mmap failed");
	if (mprotect(p, commit, PROT_READ | PROT_WRITE) != 0) {
		munmap(p, reserve);
		return fail(ErrorMemoryAllocation, "arena_host_create: commit failed");
	}
	HostArena* a = (HostArena*)p;
	a->reserve_size = reserve;
	a->commit_size = commit;
	a->commit_pos = commit;
	a->pos = sizeof *a;
	*arena = a;
	return Success;
}

Error_t arena_host_destroy(HostArena* arena)
{
	if (!arena) return fail(ErrorInvalidValue, "arena_host_destroy: NULL");
	if (munmap(arena, arena->reserve_size) != 0) return fail(ErrorMemoryAllocation, "arena_host_destroy: munmap");
	return Success;
}

Error_t arena_host_push(HostArena* const arena, const u64 req_size, void** ptr_out)
{
	if (!arena || !ptr_out) return fail(ErrorInvalidValue, "arena_host_push: NULL");
	const u64 aligned = arena->pos + pad_pow2(arena->pos, sizeof(void*));
	const u64 new_pos = aligned + req_size;
	if (new_pos > arena->reserve_size) return fail(ErrorArenaOutOfMemory, "arena_host_push: %llu bytes", (unsigned long long)req_size);
	if (new_pos > arena->commit_pos) {
		u64 target = new_pos + arena->commit_size - 1;
		target -= target % arena->commit_size;
		if (target > arena->reserve_size) target = arena->reserve_size;
		if (mprotect((u8*)arena + arena->commit_pos, target - arena->commit_pos, PROT_READ | PROT_WRITE) != 0)
			return fail(ErrorMemoryAllocation, "arena_host_push: commit failed");
		arena->commit_pos = target;
	}
	*ptr_out = (u8*)arena + aligned;
	arena->pos = new_pos;
	return Success;
}

void arena_host_pop(HostArena* const arena, u64 size)
{
	if (!arena) return;
	const u64 avail = arena->pos - sizeof *arena;
	arena->pos -= size < avail ? size : avail;
}

void arena_host_pop_at(HostArena* const arena, u64 pos)
{
	if (!arena) return;
	arena_host_pop(arena, pos < arena->pos ? arena->pos - pos : 0);
}

u64 mem_arena_host_pos_get(const HostArena* const arena) { return arena ? arena->pos : 0; }

/* ---- execution context: lives at the start of its own host arena (src/allocator.c:53-71) */

Error_t exec_ctx_create(ExecCtx** ctx)
{
	if (!ctx) return fail(ErrorInvalidValue, "exec_ctx_create: NULL");
	if (*ctx) return fail(ErrorAlreadyInitialized, "exec_ctx_create: context exists");
	HostArena* ha = NULL;
	Error_t e = arena_host_create(&ha, 1ull << 30, 1ull << 20);
	if (e != Success) return e;
	// the ExecCtx header occupies the arena's own bookkeeping plus the DevArena after it
	void* dev = NULL;
	e = arena_host_push(ha, sizeof(DevArena), &dev);
	if (e != Success) {
		arena_host_destroy(ha);
		return e;
	}
	ExecCtx* c = (ExecCtx*)ha;
	c->dev_arena._d_ptr = NULL;
	c->dev_arena.size = 0;
	c->dev_arena.pos = 0;
	*ctx = c;
	return Success;
}

Error_t exec_ctx_destroy(ExecCtx** ctx)
{
	if (!ctx || !*ctx) return fail(ErrorInvalidValue, "exec_ctx_destroy: no context");
	if ((*ctx)->dev_arena._d_ptr) {
		Error_t e = arena_dev_destroy(&(*ctx)->dev_arena);
		if (e != Success) return e;
	}
	Error_t e = arena_host_destroy(&(*ctx)->host_arena);
	if (e != Success) return e;
	*ctx = NULL;
	return Success;
}

/* ---- device arena: one cudaMalloc slab, 256-byte aligned bump pushes ----------------- */

Error_t arena_dev_create(DevArena* const arena, const u64 bsize)
{
	if (!arena || bsize == 0) return fail(ErrorInvalidValue, "arena_dev_create: bad arguments");
	if (arena->_d_ptr) return fail(ErrorAlreadyInitialized, "arena_dev_create: arena exists");
	void* p = NULL;
	cudaError_t ce = cudaMalloc(&p, bsize);
	if (ce != cudaSuccess) {
		cudaGetLastError();
		return fail(ErrorMemoryAllocation, "arena_dev_create: cudaMalloc(%llu): %s", (unsigned long long)bsize,
		            cudaGetErrorString(ce));
	}
	arena->_d_ptr = (u8*)p;
	arena->size = bsize;
	arena->pos = 0;
	return Success;
}

Error_t arena_dev_destroy(DevArena* arena)
{
	if (!arena || !arena->_d_ptr) return fail(ErrorInvalidValue, "arena_dev_destroy: no arena");
	cudaError_t ce = cudaFree(arena->_d_ptr);
	arena->_d_ptr = NULL;
	arena->size = arena->pos = 0;
	if (ce != cudaSuccess) return fail(ErrorCuda, "arena_dev_destroy: %s", cudaGetErrorString(ce));
	return Success;
}

Error_t arena_dev_push(DevArena* const arena, const u64 bsize, void** ptr_out)
{
	if (!arena || !ptr_out || !arena->_d_ptr) return fail(ErrorInvalidValue, "arena_dev_push: no arena");
	const u64 aligned = arena->pos + pad_pow2(arena->pos, 256);
	const u64 new_pos = aligned + bsize;
	if (new_pos > arena->size)
		return fail(ErrorArenaOutOfMemory, "arena_dev_push: %llu bytes at %llu of %llu", (unsigned long long)bsize,
		            (unsigned long long)aligned, (unsigned long long)arena->size);
	*ptr_out = arena->_d_ptr + aligned;
	arena->pos = new_pos;
	return Success;
}

void arena_dev_pop(DevArena* const arena, u64 bsize)
{
	if (!arena) return;
	arena->pos -= bsize < arena->pos ? bsize : arena->pos;
}

void arena_dev_pop_at(DevArena* const arena, u64 pos)
{
	if (!arena) return;
	arena_dev_pop(arena, pos < arena->pos ? arena->pos - pos : 0);
}

u64 arena_dev_pos_get(const DevArena* const arena) { return arena ? arena->pos : 0; }

/* ---- CUDA memory wrappers (src/cuda/api/cuda_mem_wrapper.cu:10-87) --------------------
 * Same names and return conventions as the reference: the b32 wrappers return 1 on success
 * and 0 on failure, the Error_t ones Success or a code.  Unlike the reference nothing aborts: a
 * failing CUDA call returns 0 (or ErrorCuda) and inf_last_error_detail() says which call and
 * why, as does a rejected pointer. */

b32 cu_malloc(void** dev_ptr, const u64 bsize)
{
	// The reference takes the pointer by value and checks that it is already device memory
	// before allocating, so the allocation never reaches its caller (defect D10).  Here the
	// caller's pointer receives the allocation.
	if (!dev_ptr) {
		(void)fail(ErrorInvalidValue, "cu_malloc: NULL out pointer");
		return 0;
	}
	*dev_ptr = nullptr;
	const cudaError_t e = cudaMalloc(dev_ptr, bsize);
	if (e != cudaSuccess) {
		(void)cudaGetLastError();
		*dev_ptr = nullptr;
		(void)fail(ErrorMemoryAllocation, "cu_malloc: cudaMalloc(%llu): %s", (unsigned long long)bsize,
		           cudaGetErrorString(e));
		return 0;
	}
	return 1;
}

b32 cu_free(void* dev_ptr)
{
	if (!inf::is_device_ptr(dev_ptr)) {
		(void)fail(ErrorInvalidDevPtr, "cu_free: not device memory");
		return 0;
	}
	const cudaError_t e = cudaFree(dev_ptr);
	if (e != cudaSuccess) {
		(void)fail(ErrorCuda, "cu_free: %s", cudaGetErrorString(e));
		return 0;
	}
	return 1;
}

Error_t cu_memcpy_htd(void* dst, const void* src, const u64 bsize)
{
	if (!inf::is_device_ptr(dst)) return fail(ErrorInvalidDevPtr, "cu_memcpy_htd: dst is not device memory");
	INF_CUDA_TRY(cudaMemcpy(dst, src, bsize, cudaMemcpyHostToDevice));
	return Success;
}

b32 cu_memcpy_htd_async(void* dst, const void* src, const u64 bsize, void* stream)
{
	if (!inf::is_device_ptr(dst)) {
		(void)fail(ErrorInvalidDevPtr, "cu_memcpy_htd_async: dst is not device memory");
		return 0;
	}
	const cudaError_t e = cudaMemcpyAsync(dst, src, bsize, cudaMemcpyHostToDevice, (cudaStream_t)stream);
	if (e != cudaSuccess) {
		(void)fail(ErrorCuda, "cu_memcpy_htd_async: %s", cudaGetErrorString(e));
		return 0;
	}
	return 1;
}

Error_t cu_memcpy_dth(void* dst, const void* src, const u64 bsize)
{
	// the reference answers a source that is not device memory with ErrorInvalidHostPtr
	// (src/cuda/api/cuda_mem_wrapper.cu:65-67); kept, so its callers' checks still match
	if (!inf::is_device_ptr(src)) return fail(ErrorInvalidHostPtr, "cu_memcpy_dth: src is not device memory");
	INF_CUDA_TRY(cudaMemcpy(dst, src, bsize, cudaMemcpyDeviceToHost));
	return Success;
}

b32 cu_host_register_read_only(void* ptr, const u64 bsize)
{
	if (!ptr || inf::is_device_ptr(ptr)) {
		(void)fail(ErrorInvalidHostPtr, "cu_host_register_read_only: not host memory");
		return 0;
	}
	const cudaError_t e = cudaHostRegister(ptr, bsize, cudaHostRegisterReadOnly);
	if (e != cudaSuccess) {
		(void)cudaGetLastError();
		(void)fail(ErrorCuda, "cu_host_register_read_only: %s", cudaGetErrorString(e));
		return 0;
	}
	return 1;
}

b32 cu_memset(void* s, i32 c, u64 n)
{
	if (!inf::is_device_ptr(s)) {
		(void)fail(ErrorInvalidDevPtr, "cu_memset: not device memory");
		return 0;
	}
	const cudaError_t e = cudaMemset(s, c, n);
	if (e != cudaSuccess) {
		(void)fail(ErrorCuda, "cu_memset: %s", cudaGetErrorString(e));
		return 0;
	}
	return 1;
}

} // extern "C"
