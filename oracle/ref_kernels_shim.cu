// Test infrastructure: launchers for the reference's own kernels, compiled from the
// reference sources in place (REF_ROOT).  Used only by the GPU tests that pin the
// oracle's gather and RMSNorm to the reference.
//
// k_fetch_input_embeddings  src/cuda/kernels/input_embeddings.cu:23-34, launched as
//                           src/main.cu:396-404 (grid = tokens, block = dim/4).
// k_rmsnorm                 src/cuda/kernels/rmsnorm.cu:11-59.  It is only launched on
//                           the domain where it is well defined: one row (its gain
//                           indexing is row-major, rmsnorm.cu:54), dim a multiple of 128
//                           with dim/128 a power of two <= 16 (rmsnorm.cu:38-47), and
//                           with one f32 of shared memory per warp (the shipped launch,
//                           src/main.cu:409, sizes it in bytes instead).
#include "input_embeddings.cu"
#include "rmsnorm.cu"

extern "C" int ref_fetch_input_embeddings(const unsigned* d_ids, unsigned long long n, unsigned dim,
                                          const void* d_table, void* d_out, void* stream)
{
	if (n == 0 || dim % 4 != 0 || dim / 4 > 1024) return -1;
	const dim3 block(dim / 4);
	const dim3 grid((unsigned)n);
	k_fetch_input_embeddings<<<grid, block, 0, (cudaStream_t)stream>>>(d_ids, n, dim, (const bf16*)d_table,
	                                                                   (bf16*)d_out);
	return (int)cudaGetLastError();
}

extern "C" int ref_rmsnorm_row0(void* d_x, unsigned dim, const void* d_gain, void* stream)
{
	if (dim % 128 != 0) return -1;
	const unsigned threads = dim / 4, warps = threads / 32;
	if (warps == 0 || warps > 16 || (warps & (warps - 1)) != 0) return -1;
	k_rmsnorm<<<1, threads, warps * sizeof(float), (cudaStream_t)stream>>>((bf16*)d_x, dim, (const bf16*)d_gain);
	return (int)cudaGetLastError();
}
