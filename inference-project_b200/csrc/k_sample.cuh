// Sampling beyond greedy for the decode loop: temperature, top-k and top-p over the logits
// the LM head wrote, one CTA of 1024 threads, after the LM head in the decode step.
//
// Definition (the oracle restates it exactly; everything after the exponential is integer):
//   m    = max_i logits_i
//   w_i  = expf((logits_i - m) * inv_temp)                   fp32, in (0, 1]
//   q_i  = min(floor(w_i * 2^32), 2^32 - 1)                  32-bit fixed-point weight
//   t_k  = largest t with #{q_i >= t} >= top_k               (top_k 0 or >= V: t_k = 0)
//   Z_k  = sum of q_i over q_i >= t_k
//   t_p  = largest t with sum{q_i : q_i >= t, q_i >= t_k} >= ceil(top_p * Z_k)   (in double)
//   kept = {i : q_i >= t_p},  Z = sum of kept q_i
//   r    = 64-bit Philox4x32-10 draw (words y:x) keyed by SplitMix64(SplitMix64(seed) ^ 0x3000000)
//          at counter (position of the new token, sequence slot)
//   s    = floor(r * Z / 2^64);  id = the first kept index (ascending) whose inclusive prefix
//          sum of kept q exceeds s
// Ties at a threshold are all kept.  Both thresholds come from a 4-pass radix select on 8-bit
// digits with per-warp shared-memory histograms of counts or 64-bit masses: integer atomics, so
// the result does not depend on the order threads add.  The weights q are kept in global scratch
// (L2-resident: 4 bytes x V) between passes; every pass reads them with 16-byte loads, two in
// flight per thread, and the draw gives each warp a contiguous range that the warp holding s
// searches row by row with warp scans.  One CTA makes every pass, so the kernel is bound by its
// own instruction stream (about 0.2 ms per token at V = 128256).
#pragma once

#include "common.cuh"
#include "synth.cuh"

namespace inf {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kSampleSubStride = 257; // u64 per warp histogram: 256 bins + 1 to skew banks across warps
constexpr size_t kSampleSmem = (size_t)kSampleWarps * kSampleSubStride * sizeof(unsigned long long);
constexpr uint64_t kSampleStream = 0x3000000;

struct SampleArgs {
	const float* logits; // [V]
	uint32_t* q;         // [V] scratch: fixed-point weights
	int V;
	float inv_temp;
	float top_p;
	uint32_t top_k;
	PhiloxKey key;
	uint32_t* cur_id;    // overwritten with the sampled id
	uint32_t* out_ids;   // out_ids[*step - 1] overwritten (the LM head already advanced step)
	const uint32_t* step;
	const int* pos;      // position of the new token (already advanced by the LM head)
	const int* slot;
	int max_out;
	uint32_t* row_id;    // non-null: the id goes here only (a row of the batched step)
};

// One row of the batched decode step: its sequence's settings and the draw's counter.
struct SampleRow {
	float inv_temp;
	float top_p;
	uint32_t top_k;
	uint32_t on;         // 0: keep the row's greedy id
	int pos_new;         // position of the token being chosen
	int slot;            // the draw counter's high word
	PhiloxKey key;
};

struct SampleRowsArgs {
	const float* logits; // [rows][V]
	uint32_t* q;         // [rows][V] scratch
	int V;               // multiple of 4 (16-byte aligned rows)
	const SampleRow* rows;
	uint32_t* ids;       // [rows]: greedy ids in, sampled ids out where on
};

__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v)
{
#pragma unroll
	for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
	return v;
}

// Calls f(q_i) for the indices this thread owns in a strided pass over [0, V): 16-byte loads,
// two in flight per thread (one CTA makes every pass, so each pass is load-latency bound), then
// the ragged tail one by one.  p must be 16-byte aligned.
template <typename T, typename F>
__device__ __forceinline__ void sample_visit(const T* p, int V, F f)
{
	static_assert(sizeof(T) == 4, "4-byte elements");
	const int n4 = V >> 2;
	const uint4* p4 = reinterpret_cast<const uint4*>(p);
	int i = threadIdx.x;
	for (; i + kSampleThreads < n4; i += 2 * kSampleThreads) {
		const uint4 x = p4[i], y = p4[i + kSampleThreads];
		f(i * 4 + 0, x.x); f(i * 4 + 1, x.y); f(i * 4 + 2, x.z); f(i * 4 + 3, x.w);
		const int j = (i + kSampleThreads) * 4;
		f(j + 0, y.x); f(j + 1, y.y); f(j + 2, y.z); f(j + 3, y.w);
	}
	if (i < n4) {
		const uint4 x = p4[i];
		f(i * 4 + 0, x.x); f(i * 4 + 1, x.y); f(i * 4 + 2, x.z); f(i * 4 + 3, x.w);
	}
	for (int k = n4 * 4 + (int)threadIdx.x; k < V; k += kSampleThreads) f(k, reinterpret_cast<const uint32_t*>(p)[k]);
}

// Largest t such that the weight of {i : q_i >= t, q_i >= floor_t} reaches target, where an
// element weighs 1 (by_mass false) or q_i.  Every thread returns the same t.  Each warp counts
// into its own histogram in `sub` (logits put most tokens in a few bins, and one shared
// histogram serialised every update on them), and a thread adds runs of equal bins in a
// register before it touches shared memory; the warp histograms are then summed per bin.
__device__ uint32_t sample_radix_select(const SampleArgs& a, uint32_t floor_t, bool by_mass, uint64_t target,
                                        unsigned long long* hist, unsigned long long* sub, unsigned long long* sh_acc,
                                        uint32_t* sh_prefix)
{
	const int tid = threadIdx.x;
	unsigned long long* mine = sub + (size_t)(tid >> 5) * kSampleSubStride;
	uint32_t prefix = 0;
	uint64_t acc = 0; // weight of the elements above the current bucket
	for (int shift = 24; shift >= 0; shift -= 8) {
		for (int b = tid; b < kSampleWarps * kSampleSubStride; b += kSampleThreads) sub[b] = 0ull;
		__syncthreads();
		const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
		uint32_t cb = 0xFFFFFFFFu; // the bin of the run in the register
		unsigned long long cw = 0ull;
		sample_visit(a.q, a.V, [&](int, uint32_t q) {
			if (q < floor_t || (q & hi_mask) != (prefix & hi_mask)) return;
			const uint32_t bin = (q >> shift) & 255u;
			const unsigned long long w = by_mass ? (unsigned long long)q : 1ull;
			if (bin == cb) {
				cw += w;
			} else {
				if (cw) atomicAdd(&mine[cb], cw);
				cb = bin;
				cw = w;
			}
		});
		if (cw) atomicAdd(&mine[cb], cw);
		__syncthreads();
		for (int b = tid; b < 256; b += kSampleThreads) {
			unsigned long long h = 0ull;
			for (int w = 0; w < kSampleWarps; ++w) h += sub[(size_t)w * kSampleSubStride + b];
			hist[b] = h;
		}
		__syncthreads();
		if (tid < 32) {
			// the highest bin d whose weight, added to everything above it, reaches target (bin 0
			// if none does): lane l holds bins 255 - 8l .. 248 - 8l, a scan over the lanes gives
			// the weight above each lane's bins, the first lane to reach target takes it
			const int lane = tid;
			unsigned long long h[8], own = 0ull;
#pragma unroll
			for (int j = 0; j < 8; ++j) {
				h[j] = hist[255 - 8 * lane - j];
				own += h[j];
			}
			unsigned long long incl = own;
#pragma unroll
			for (int o = 1; o < 32; o <<= 1) {
				const unsigned long long v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
				if (lane >= o) incl += v;
			}
			unsigned long long c = acc + (incl - own);
			int hit = -1;
#pragma unroll
			for (int j = 0; j < 8; ++j) {
				if (hit < 0) {
					if (c + h[j] >= target || (lane == 31 && j == 7)) hit = j;
					else c += h[j];
				}
			}
			const unsigned first = __ffs(__ballot_sync(0xFFFFFFFFu, hit >= 0)) - 1;
			if (lane == (int)first) {
				*sh_prefix = prefix | ((uint32_t)(255 - 8 * lane - hit) << shift);
				*sh_acc = c;
			}
		}
		__syncthreads();
		prefix = *sh_prefix;
		acc = *sh_acc;
		__syncthreads();
	}
	return prefix;
}

// The whole draw of one token by one CTA of kSampleThreads threads (sub: the dynamic shared
// memory of kSampleSmem bytes).
__device__ __forceinline__ void sample_token(const SampleArgs& a, unsigned long long* sub)
{
	__shared__ unsigned long long hist[256];
	__shared__ unsigned long long red[kSampleThreads / 32];
	__shared__ float redf[kSampleThreads / 32];
	__shared__ unsigned long long sh_acc;
	__shared__ uint32_t sh_prefix;
	const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

	// max logit
	float m = -INFINITY;
	sample_visit(a.logits, a.V, [&](int, uint32_t bits) { m = fmaxf(m, __uint_as_float(bits)); });
	m = warp_max(m);
	if (lane == 0) redf[warp] = m;
	__syncthreads();
	if (warp == 0) {
		float v = redf[lane];
		v = warp_max(v);
		if (lane == 0) redf[0] = v;
	}
	__syncthreads();
	m = redf[0];

	// fixed-point weights
	sample_visit(a.logits, a.V, [&](int i, uint32_t bits) {
		const float w = expf((__uint_as_float(bits) - m) * a.inv_temp);
		const float s = w * 4294967296.0f; // exact: a power-of-two scale
		a.q[i] = s >= 4294967295.0f ? 0xFFFFFFFFu : (uint32_t)s;
	});
	__syncthreads(); // q is read back by other threads (global, same CTA)

	// top-k threshold, then the mass it keeps
	uint32_t tk = 0;
	if (a.top_k > 0 && a.top_k < (uint32_t)a.V) tk = sample_radix_select(a, 0u, false, a.top_k, hist, sub, &sh_acc, &sh_prefix);
	uint64_t zk = 0;
	sample_visit(a.q, a.V, [&](int, uint32_t q) {
		if (q >= tk) zk += q;
	});
	zk = warp_sum_u64(zk);
	if (lane == 0) red[warp] = zk;
	__syncthreads();
	if (tid == 0) {
		uint64_t z = 0;
		for (int w = 0; w < kSampleThreads / 32; ++w) z += red[w];
		sh_acc = z;
	}
	__syncthreads();
	zk = sh_acc;
	__syncthreads();

	// top-p threshold
	uint32_t tp = tk;
	if (a.top_p < 1.0f && zk > 0) {
		double tgt = ceil((double)a.top_p * (double)zk);
		if (tgt < 1.0) tgt = 1.0;
		if (tgt > (double)zk) tgt = (double)zk;
		tp = sample_radix_select(a, tk, true, (uint64_t)tgt, hist, sub, &sh_acc, &sh_prefix);
		if (tp < tk) tp = tk;
	}

	// the draw: first kept index whose inclusive prefix mass exceeds s.  Warp w owns the
	// contiguous elements [w * E, (w + 1) * E), read in rows of 128 (one 16-byte load per lane,
	// coalesced); the warp holding s then walks its rows with warp scans.
	const int rows = (a.V + kSampleWarps * 128 - 1) / (kSampleWarps * 128);
	const int wbase = warp * rows * 128;
	auto lane_row = [&](int r, uint32_t (&v)[4]) { // this lane's 4 elements of row r (0 past V)
		const int i = wbase + r * 128 + lane * 4;
		if (i + 4 <= a.V) {
			const uint4 x = *reinterpret_cast<const uint4*>(a.q + i);
			v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
		} else {
#pragma unroll
			for (int k = 0; k < 4; ++k) v[k] = i + k < a.V ? a.q[i + k] : 0u;
		}
#pragma unroll
		for (int k = 0; k < 4; ++k) v[k] = (v[k] >= tp && i + k < a.V) ? v[k] : 0u; // kept mass only
	};
	uint64_t mine = 0;
	for (int r = 0; r < rows; ++r) {
		uint32_t v[4];
		lane_row(r, v);
		mine += (uint64_t)v[0] + v[1] + v[2] + v[3];
	}
	mine = warp_sum_u64(mine);
	if (lane == 0) red[warp] = mine;
	__syncthreads();
	if (warp == 0) {
		const uint64_t v = red[lane];
		uint64_t t = v;
#pragma unroll
		for (int o = 1; o < 32; o <<= 1) {
			const uint64_t u = __shfl_up_sync(0xFFFFFFFFu, t, o);
			if (lane >= o) t += u;
		}
		red[lane] = t - v;          // exclusive prefix of the warps
		if (lane == 31) sh_acc = t; // total kept mass
	}
	__syncthreads();
	const uint64_t total = sh_acc;
	const uint64_t ctr = (uint64_t)(uint32_t)*a.pos | ((uint64_t)(uint32_t)*a.slot << 32);
	const uint4 wds = philox10(ctr, a.key);
	const uint64_t r64 = ((uint64_t)wds.y << 32) | wds.x;
	const uint64_t s = __umul64hi(r64, total);
	uint64_t c = red[warp];
	if (total == 0 || s < c || s >= c + mine) return; // another warp's range (warp-uniform)
	for (int r = 0; r < rows; ++r) {
		uint32_t v[4];
		lane_row(r, v);
		const uint64_t own = (uint64_t)v[0] + v[1] + v[2] + v[3];
		uint64_t incl = own;
#pragma unroll
		for (int o = 1; o < 32; o <<= 1) {
			const uint64_t u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
			if (lane >= o) incl += u;
		}
		const uint64_t row = __shfl_sync(0xFFFFFFFFu, incl, 31);
		if (c + row <= s) {
			c += row;
			continue;
		}
		const unsigned hit = __ballot_sync(0xFFFFFFFFu, c + incl > s);
		if (lane == (int)(__ffs(hit) - 1)) {
			uint64_t cc = c + incl - own;
#pragma unroll
			for (int k = 0; k < 4; ++k) {
				cc += v[k];
				if (cc > s) {
					const uint32_t id = (uint32_t)(wbase + r * 128 + lane * 4 + k);
					if (a.row_id) {
						*a.row_id = id;
					} else {
						*a.cur_id = id;
						const uint32_t st = *a.step;
						if (st >= 1 && (int)(st - 1) < a.max_out) a.out_ids[st - 1] = id;
					}
					break;
				}
			}
		}
		break;
	}
}

__global__ void __launch_bounds__(kSampleThreads) k_sample(const SampleArgs a)
{
	pdl_wait();
	pdl_trigger();
	extern __shared__ unsigned long long sample_sub[]; // [kSampleWarps][kSampleSubStride]
	sample_token(a, sample_sub);
}

// One CTA per row of the batched decode step: rows with sampling on replace their greedy id
// by a draw under their sequence's settings, the counter being (position of the new token,
// SampleRow::slot) -- the engine passes 0, so a sequence draws what the batch-1 decode of slot 0
// would, whichever slot it runs in.
__global__ void __launch_bounds__(kSampleThreads) k_sample_rows(const SampleRowsArgs ra)
{
	pdl_wait();
	pdl_trigger();
	extern __shared__ unsigned long long sample_sub[];
	const SampleRow& r = ra.rows[blockIdx.x];
	if (!r.on) return;
	SampleArgs a;
	a.logits = ra.logits + (size_t)blockIdx.x * ra.V;
	a.q = ra.q + (size_t)blockIdx.x * ra.V;
	a.V = ra.V;
	a.inv_temp = r.inv_temp;
	a.top_p = r.top_p;
	a.top_k = r.top_k;
	a.key = r.key;
	a.cur_id = nullptr;
	a.out_ids = nullptr;
	a.step = nullptr;
	a.pos = &r.pos_new;
	a.slot = &r.slot;
	a.max_out = 0;
	a.row_id = ra.ids + blockIdx.x;
	sample_token(a, sample_sub);
}

} // namespace inf
