// Embedding gather and row RMSNorm.
//
// k_embed replaces the reference's k_fetch_input_embeddings
// (src/cuda/kernels/input_embeddings.cu:23-34): out[t,:] = table[ids[t],:].  It copies
// 16-byte units, works for any dim that is a multiple of the unit, checks ids against the
// vocabulary (the reference does not, defect D12) and can widen rows to the fp32 residual.
//
// k_rmsnorm_rows replaces k_rmsnorm (src/cuda/kernels/rmsnorm.cu:11-59): fp32 sum of
// squares, y = x * g / sqrt(mean(x^2) + eps), one gain vector for every row, any dim.
#pragma once

#include "common.cuh"

namespace inf {

template <typename T, typename OutT>
__global__ void k_embed(const uint32_t* __restrict__ ids, int n_tokens, int dim, uint32_t vocab,
                        const T* __restrict__ table, OutT* __restrict__ out, int* err)
{
	pdl_wait();
	pdl_trigger();
	const int t = blockIdx.y;
	if (t >= n_tokens) return;
	const uint32_t id = ids[t];
	const bool bad = id >= vocab;
	if (bad && threadIdx.x == 0 && blockIdx.x == 0) report_err(err, kDevTokenRange);
	const T* src = table + (uint64_t)(bad ? 0u : id) * dim;
	OutT* dst = out + (uint64_t)t * dim;
	for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
		const float v = bad ? 0.0f : Store<T>::get(src + i);
		Store<OutT>::put(dst + i, v);
	}
}

// bit-exact row copy for same-typed gather (16-byte units when dim allows)
template <typename T>
__global__ void k_embed_copy(const uint32_t* __restrict__ ids, int n_tokens, int dim, uint32_t vocab,
                             const T* __restrict__ table, T* __restrict__ out, int* err)
{
	const int t = blockIdx.y;
	if (t >= n_tokens) return;
	const uint32_t id = ids[t];
	const bool bad = id >= vocab;
	if (bad && threadIdx.x == 0 && blockIdx.x == 0) report_err(err, kDevTokenRange);
	const size_t row_bytes = (size_t)dim * sizeof(T);
	const uint8_t* src = reinterpret_cast<const uint8_t*>(table) + (uint64_t)(bad ? 0u : id) * row_bytes;
	uint8_t* dst = reinterpret_cast<uint8_t*>(out) + (uint64_t)t * row_bytes;
	if ((row_bytes & 15) == 0 && ((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 15) == 0) {
		const int units = (int)(row_bytes >> 4);
		for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < units; i += gridDim.x * blockDim.x) {
			uint4 v = bad ? make_uint4(0, 0, 0, 0) : reinterpret_cast<const uint4*>(src)[i];
			reinterpret_cast<uint4*>(dst)[i] = v;
		}
	} else {
		for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
			out[(uint64_t)t * dim + i] = bad ? T() : table[(uint64_t)id * dim + i];
	}
}

// one CTA per row; InT is the stored row type (float residual or T), OutT the output.
template <typename InT, typename OutT, typename GT>
__global__ void k_rmsnorm_rows(const InT* x, OutT* y, int rows, int dim,
                               const GT* __restrict__ gain, float eps)
{
	pdl_wait();
	pdl_trigger();
	const int r = blockIdx.x;
	if (r >= rows) return;
	const InT* xr = x + (uint64_t)r * dim;
	float ss = 0.0f;
	for (int i = threadIdx.x; i < dim; i += blockDim.x) {
		const float v = Store<InT>::get(xr + i);
		ss += v * v;
	}
	__shared__ float red[32];
	ss = warp_sum(ss);
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	if (lane == 0) red[warp] = ss;
	__syncthreads();
	if (warp == 0) {
		const int nw = (blockDim.x + 31) >> 5;
		float v = lane < nw ? red[lane] : 0.0f;
		v = warp_sum(v);
		if (lane == 0) red[0] = v;
	}
	__syncthreads();
	const float inv = 1.0f / sqrtf(__fdiv_rn(red[0], (float)dim) + eps);
	OutT* yr = y + (uint64_t)r * dim;
	for (int i = threadIdx.x; i < dim; i += blockDim.x) {
		const float v = __fmul_rn(__fmul_rn(Store<InT>::get(xr + i), inv), Store<GT>::get(gain + i));
		Store<OutT>::put(yr + i, v);
	}
}

// Greedy argmax of each row of a [rows x n] fp32 matrix (ties -> lowest index), one CTA per
// row; the token id is the column index plus col_base (vocabulary shard offset).
__global__ void k_argmax_rows(const float* __restrict__ x, int n, uint32_t col_base, uint32_t* __restrict__ out)
{
	pdl_wait();
	pdl_trigger();
	const float* row = x + (size_t)blockIdx.x * n;
	unsigned long long best = 0ull;
	for (int i = threadIdx.x; i < n; i += blockDim.x) {
		const unsigned long long k = argmax_key(row[i], (uint32_t)i + col_base);
		best = k > best ? k : best;
	}
#pragma unroll
	for (int o = 16; o > 0; o >>= 1) {
		const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, best, o);
		best = other > best ? other : best;
	}
	__shared__ unsigned long long red[32];
	if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
	__syncthreads();
	if (threadIdx.x == 0) {
		for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
		best = red[0] > best ? red[0] : best;
		out[blockIdx.x] = argmax_key_index(best);
	}
}

} // namespace inf
