// Synthetic seeded weights, generated on the device directly in the device layout.
//
// Definition (identical bits on host and device): element idx of the tensor with stream
// id s draws Philox4x32-10 (Salmon et al., SC'11) at counter (idx_lo, idx_hi, 0, 0) with
// key = SplitMix64(SplitMix64(seed) ^ s); the four words' top 22 bits are summed, centred
// (an exact fp32 integer) and multiplied once by std*sqrt(3)/2^22 (Irwin-Hall(4) ~ N(0,std)),
// then rounded to bf16 (RNE) for bf16 models.  Stream ids: ((layer+1) << 8) | kind.
#pragma once

#include "common.cuh"

namespace inf {

enum TensorKind : uint32_t {
	kEmbed = 0, kLmHead = 1, kFinalNorm = 2,
	kEmbedPle = 3, kPleModelProj = 4, kPleProjNorm = 5, // Gemma-style models
	kWq = 8, kWk = 9, kWv = 10, kWo = 11, kWgate = 12, kWup = 13, kWdown = 14, kAttnNorm = 15, kFfnNorm = 16,
	kQNorm = 17, kKNorm = 18, kPostAttnNorm = 19, kPostFfnNorm = 20, kPleGate = 21, kPleProj = 22, kPlePostNorm = 23,
};

__host__ __device__ inline uint64_t splitmix64(uint64_t x)
{
	uint64_t z = x + 0x9E3779B97F4A7C15ull;
	z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
	z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
	return z ^ (z >> 31);
}

__host__ __device__ inline uint64_t tensor_stream(int layer, uint32_t kind)
{
	return ((uint64_t)(int64_t)(layer + 1) << 8) | kind;
}

struct PhiloxKey {
	uint32_t k0, k1;
};

__host__ __device__ inline PhiloxKey stream_key(uint64_t seed, uint64_t stream)
{
	const uint64_t k = splitmix64(splitmix64(seed) ^ stream);
	return PhiloxKey{(uint32_t)k, (uint32_t)(k >> 32)};
}

__device__ __forceinline__ uint4 philox10(uint64_t idx, PhiloxKey key)
{
	uint32_t c0 = (uint32_t)idx, c1 = (uint32_t)(idx >> 32), c2 = 0, c3 = 0;
	uint32_t k0 = key.k0, k1 = key.k1;
#pragma unroll
	for (int r = 0; r < 10; ++r) {
		const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
		const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
		c0 = hi1 ^ c1 ^ k0;
		c1 = lo1;
		c2 = hi0 ^ c3 ^ k1;
		c3 = lo0;
		k0 += 0x9E3779B9u;
		k1 += 0xBB67AE85u;
	}
	return make_uint4(c0, c1, c2, c3);
}

__device__ __forceinline__ float synth_normal(uint64_t idx, PhiloxKey key, float scale)
{
	const uint4 w = philox10(idx, key);
	const int32_t s = (int32_t)((w.x >> 10) + (w.y >> 10) + (w.z >> 10) + (w.w >> 10)) - (1 << 23);
	return __fmul_rn((float)s, scale);
}

inline float synth_scale(float std) { return (float)((double)std * 1.7320508075688772 / 4194304.0); }

// How a device row maps to (tensor, canonical row).
enum RowMap : int {
	kMapPlain = 0,  // one tensor, device row == canonical row (+ row_offset)
	kMapQkv = 1,    // fused [q heads | k heads | v heads], each head's rows ordered (i, i+hd/2) pairs
	kMapGateUp = 2, // rows alternate gate_j, up_j
};

struct SynthArgs {
	void* dst;
	uint64_t rows, cols;      // device shape
	uint64_t canon_cols;      // columns of the canonical tensor (full, before a column shard)
	uint64_t col_offset;      // first canonical column of this shard
	int map;
	PhiloxKey key[3];         // plain: key[0]; qkv: q,k,v; gate/up: gate, up
	float scale;
	// qkv geometry (heads local to this shard, first global head of each kind)
	int head_dim, n_q_heads, n_kv_heads, q_head0, kv_head0;
	uint64_t row_offset;      // plain / gate-up: first canonical row of this shard
	int ones;                 // gains: every element 1.0
};

template <typename T>
__global__ void k_synth(SynthArgs a)
{
	const uint64_t n = a.rows * a.cols;
	for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (uint64_t)gridDim.x * blockDim.x) {
		const uint64_t r = e / a.cols, c = e % a.cols;
		float v = 1.0f;
		if (!a.ones) {
			uint64_t crow;
			PhiloxKey key;
			if (a.map == kMapQkv) {
				const uint64_t hd = (uint64_t)a.head_dim;
				const uint64_t head = r / hd, rr = r % hd;
				const uint64_t dim = (rr & 1) ? (rr >> 1) + hd / 2 : (rr >> 1);
				if (head < (uint64_t)a.n_q_heads) {
					key = a.key[0];
					crow = (a.q_head0 + head) * hd + dim;
				} else if (head < (uint64_t)(a.n_q_heads + a.n_kv_heads)) {
					key = a.key[1];
					crow = (a.kv_head0 + head - a.n_q_heads) * hd + dim;
				} else {
					key = a.key[2];
					crow = (a.kv_head0 + head - a.n_q_heads - a.n_kv_heads) * hd + dim;
				}
			} else if (a.map == kMapGateUp) {
				key = a.key[r & 1];
				crow = a.row_offset + (r >> 1);
			} else {
				key = a.key[0];
				crow = a.row_offset + r;
			}
			v = synth_normal(crow * a.canon_cols + a.col_offset + c, key, a.scale);
		}
		Store<T>::put(reinterpret_cast<T*>(a.dst) + e, v);
	}
}

} // namespace inf
