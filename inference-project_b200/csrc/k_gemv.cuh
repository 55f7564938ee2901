// Batch-1 decode projections: y = W.x over a row-major [N x K] weight, HBM-bound.
//
// One CTA per SM.  A producer warp streams the CTA's contiguous row range through a ring
// of shared-memory stages with 1-D bulk copies (cp.async.bulk, evict_first), issuing the
// first stages before griddepcontrol.wait so the weight stream of kernel n+1 overlaps the
// tail of kernel n (programmatic dependent launch).  Sixteen consumer warps hold the
// activation vector in registers (each lane owns 16-byte units u*512 + lane_id), dot every
// staged row against it, reduce across warps and run a fused epilogue:
//   kEpiStore   y[row] = round(dot)
//   kEpiResid   r[row] += dot                           (O-proj and down-proj + residual)
//   kEpiQkv     RoPE on (i, i+hd/2) row pairs, q -> buffer, k/v -> paged KV cache
//   kEpiSwiglu  h[j] = round(silu(gate_j) * up_j) on (gate_j, up_j) row pairs
//   kEpiLogits  logits[row] = dot (soft-capped when softcap > 0), then a grid-wide greedy argmax
//               (ties -> lowest index)
//   kEpiStoreF32  y[row] = dot in fp32 (raw projections of the Gemma-style decoder)
//   kEpiGeglu   h[j] = round(gelu_tanh(gate_j) * up_j) on (gate_j, up_j) row pairs
//   kEpiPleGate y[row] = round(gelu_tanh(dot) * ple[row]) (the per-layer-embedding gate)
// The prologue either normalises the fp32 residual with the layer's RMSNorm gain
// (src/cuda/kernels/rmsnorm.cu:11-59 semantics, with eps) or loads a stored vector.  For the
// Gemma-style decoder it can first fold a pending projection output into the residual,
// r' = r + (p * rsqrt(mean(p^2) + eps)) * (1 + g_p), written to a second residual buffer by
// CTA 0 (every CTA computes the same r'), scale the gains by (1 + w), or skip the
// normalisation (x = round(r')).
#pragma once

#include "common.cuh"
#include "k_tp.cuh"

namespace inf {

constexpr int kGemvConsumerWarps = 16;
constexpr int kGemvConsumers = kGemvConsumerWarps * 32;
constexpr int kGemvThreads = kGemvConsumers + 32;
constexpr int kGemvRingBytes = 96 * 1024;
constexpr int kGemvMaxStages = 8;
constexpr int kGemvPrefetch = 2;    // chunks prefetched into L2 beyond the ring
constexpr int kGemvFlushRows = 128; // rows per deferred-epilogue window
constexpr uint32_t kGemvNextPrefetch = 192 * 1024; // bytes of the next projection warmed per CTA

enum EpiKind : int {
	kEpiStore = 0, kEpiResid = 1, kEpiQkv = 2, kEpiSwiglu = 3, kEpiLogits = 4,
	kEpiStoreF32 = 5, kEpiGeglu = 6, kEpiPleGate = 7,
};

template <int EPI> struct EpiTraits {
	static constexpr bool kPaired = (EPI == kEpiQkv || EPI == kEpiSwiglu || EPI == kEpiGeglu);
	static constexpr bool kNorm = (EPI == kEpiQkv || EPI == kEpiSwiglu || EPI == kEpiLogits || EPI == kEpiGeglu);
	// the prologue is chosen at run time (norm when resid_in is set, else the stored vector)
	static constexpr bool kRuntimeProlog = (EPI == kEpiStoreF32 || EPI == kEpiPleGate);
	// the Gemma-style prologue features (pending add, (1 + w) gains, no-norm) are compiled in
	static constexpr bool kGemma = (EPI == kEpiStoreF32 || EPI == kEpiGeglu || EPI == kEpiPleGate || EPI == kEpiLogits);
};

template <int UPL, int EPI> struct GemvShape {
	// rows per chunk so that a chunk is ~32 KB: 2048 units of 16 bytes over the consumer lanes
	static constexpr int kRpcBase = (2048 / (UPL * kGemvConsumers)) < 1 ? 1 : (2048 / (UPL * kGemvConsumers));
	static constexpr int kRpc = (EpiTraits<EPI>::kPaired && kRpcBase < 2) ? 2 : kRpcBase; // rows per chunk
};

struct GemvArgs {
	const void* W;
	int N, K;
	int stages;
	uint32_t stage_bytes;
	// prologue
	const float* resid_in;  // norm prologue: fp32 [K]
	const void* gain;       // norm gain [K]
	float eps;
	const void* xin;        // plain prologue: [K]
	// epilogue
	void* out;              // store: [N]; swiglu: [N/2]; qkv: q [n_q_heads*hd]
	float* resid;           // resid: fp32 [N]
	void* kpool;            // qkv: this layer's K pages [pages][kv][blk][hd]
	void* vpool;
	const int* block_table; // [slots][pages_per_seq]
	int pages_per_seq, max_pages;
	const int* pos;         // device position of the token
	const int* slot;        // device slot of the token
	const float* rope_cos;  // [max_seq][hd/2]
	const float* rope_sin;
	int head_dim, n_q_heads, n_kv_heads, kv_block, max_seq;
	float* logits;                // logits: fp32 [N]
	unsigned long long* best;     // logits: grid argmax key
	unsigned* counter;            // logits: finished CTAs
	uint32_t* cur_id;             // logits: next input id
	uint32_t* out_ids;            // logits: generated ids [max_out]
	uint32_t* step;               // logits: index into out_ids
	int* pos_rw;                  // logits: position advanced after the step
	int max_out;
	float softcap;                // logits: c * tanh(logit / c) when c > 0
	// Gemma-style prologue
	const float* pend;            // pending projection output fp32 [K] folded into the residual first
	const void* pend_gain;        // its RMSNorm gain [K] (scaled by 1 + w)
	float* resid_out;             // r + normed(pend), written by CTA 0
	int gain_plus1;               // the prologue's gains scale by (1 + w)
	int no_norm;                  // x = round(r) instead of the RMSNorm
	const void* ple;              // kEpiPleGate: this layer's per-layer input [N]
	int* err;
	// tensor parallelism: tp.size > 1 turns kEpiResid into a fused all-reduce of the rows'
	// partial sums and kEpiLogits into a cross-shard argmax (logit row + row_base = token id)
	TpComm tp;
	int tp_round_index;
	int row_base;
	// the next projection of the step: once its last chunk is issued, the producer warms L2
	// with the head of the slice that the same CTA index owns there.  Two projection CTAs do
	// not always fit on one SM, so the next kernel's own stream may only start when this
	// kernel's CTAs leave; the warm-up keeps HBM busy across that boundary.
	const void* nx_W;
	int nx_N, nx_K, nx_unit_rows, nx_grid;
	uint32_t nx_bytes; // multiple of 16
};

// Sum of RPC per-lane row partials across the warp, transposed: at the first log2(RPC)
// butterfly levels each lane keeps half of its rows and hands the other half to its partner,
// so one value per lane survives; after the remaining levels lane l holds the full sum of
// row row_of_lane<RPC>(l).  6 shuffles for 4 rows instead of 20.
template <int RPC>
__device__ __forceinline__ int row_of_lane(int lane)
{
	if constexpr (RPC == 8) return ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
	else if constexpr (RPC == 4) return ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
	else if constexpr (RPC == 2) return (lane >> 4) & 1;
	else return 0;
}

template <int RPC>
__device__ __forceinline__ float reduce_rows(const float (&p)[RPC], int lane)
{
	constexpr unsigned kFull = 0xFFFFFFFFu;
	if constexpr (RPC == 1) {
		return warp_sum(p[0]);
	} else if constexpr (RPC == 2) {
		const bool b16 = lane & 16;
		float s = (b16 ? p[1] : p[0]) + __shfl_xor_sync(kFull, b16 ? p[0] : p[1], 16);
#pragma unroll
		for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
		return s;
	} else if constexpr (RPC == 4) {
		const bool b16 = lane & 16, b8 = lane & 8;
		float q[2];
#pragma unroll
		for (int j = 0; j < 2; ++j) q[j] = (b16 ? p[2 + j] : p[j]) + __shfl_xor_sync(kFull, b16 ? p[j] : p[2 + j], 16);
		float s = (b8 ? q[1] : q[0]) + __shfl_xor_sync(kFull, b8 ? q[0] : q[1], 8);
#pragma unroll
		for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
		return s;
	} else {
		static_assert(RPC == 8, "rows per chunk");
		const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
		float q[4], r[2];
#pragma unroll
		for (int j = 0; j < 4; ++j) q[j] = (b16 ? p[4 + j] : p[j]) + __shfl_xor_sync(kFull, b16 ? p[j] : p[4 + j], 16);
#pragma unroll
		for (int j = 0; j < 2; ++j) r[j] = (b8 ? q[2 + j] : q[j]) + __shfl_xor_sync(kFull, b8 ? q[j] : q[2 + j], 8);
		float s = (b4 ? r[1] : r[0]) + __shfl_xor_sync(kFull, b4 ? r[0] : r[1], 4);
		s += __shfl_xor_sync(kFull, s, 2);
		s += __shfl_xor_sync(kFull, s, 1);
		return s;
	}
}

// One row's dot product over this lane's units, already in registers (zero units contribute nothing).
template <typename T, int UPL>
__device__ __forceinline__ float gemv_unit_dot(const uint4 (&w)[UPL], const float (&xh)[UPL][Store<T>::kVec])
{
	constexpr int VEC = Store<T>::kVec;
	float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
	for (int u = 0; u < UPL; ++u) {
		float wf[VEC];
		unpack_unit(w[u], wf, (const T*)nullptr);
#pragma unroll
		for (int v = 0; v < VEC; v += 2) {
			a0 = fmaf(wf[v], xh[u][v], a0);
			a1 = fmaf(wf[v + 1], xh[u][v + 1], a1);
		}
	}
	return a0 + a1;
}

template <typename T, int UPL, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) k_gemv(const GemvArgs a)
{
	constexpr int VEC = Store<T>::kVec;
	constexpr int RPC = GemvShape<UPL, EPI>::kRpc;
	constexpr bool PAIRED = EpiTraits<EPI>::kPaired;
	constexpr int UNIT_ROWS = PAIRED ? 2 : 1;

	extern __shared__ __align__(1024) uint8_t smem[];
	uint8_t* ring = smem;
	uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGemvRingBytes);
	uint64_t* empty = full + kGemvMaxStages;
	float* wpart = reinterpret_cast<float*>(empty + kGemvMaxStages);    // [warps][kGemvFlushRows]
	float* red_ss = wpart + kGemvConsumerWarps * kGemvFlushRows;          // [warps]
	unsigned long long* red_best = reinterpret_cast<unsigned long long*>(red_ss + kGemvConsumerWarps + 8);
	volatile int* abort_flag = reinterpret_cast<volatile int*>(red_best + kGemvConsumerWarps);
	float* tp_stage = reinterpret_cast<float*>(red_best + kGemvConsumerWarps + 2); // [kTpMaxRowsCta]
	const bool tp_on = a.tp.size > 1;

	const int tid = threadIdx.x;
	const int warp = tid >> 5, lane = tid & 31;
	const int S = a.stages;

	// balanced contiguous row range of this CTA (whole pairs for paired epilogues)
	const int total_units = a.N / UNIT_ROWS;
	const int r0 = (int)(((long long)blockIdx.x * total_units) / gridDim.x) * UNIT_ROWS;
	const int r1 = (int)(((long long)(blockIdx.x + 1) * total_units) / gridDim.x) * UNIT_ROWS;
	const int n_rows = r1 - r0;
	const int n_chunks = (n_rows + RPC - 1) / RPC;
	const size_t row_bytes = (size_t)a.K * sizeof(T);

	if (tid == 0) {
		for (int s = 0; s < S; ++s) {
			mbar_init(&full[s], 1);
			mbar_init(&empty[s], kGemvConsumerWarps);
		}
		*abort_flag = 0;
		mbar_fence_init();
	}
	__syncthreads();
	pdl_trigger();

	if (warp == kGemvConsumerWarps) {
		// ---------------- producer ----------------
		if (lane == 0) {
			const uint64_t pol = policy_evict_first();
			const uint8_t* wbase = reinterpret_cast<const uint8_t*>(a.W) + (size_t)r0 * row_bytes;
			auto chunk_bytes = [&](int i) { return (uint32_t)(min(RPC, n_rows - i * RPC) * row_bytes); };
			// L2 prefetch runs kGemvPrefetch chunks ahead of the shared-memory ring, so each SM
			// has more bytes in flight than its ring holds
			const int pf_end0 = min(n_chunks, S + kGemvPrefetch);
			for (int i = S; i < pf_end0; ++i) bulk_prefetch_l2(wbase + (size_t)i * RPC * row_bytes, chunk_bytes(i));
			int issued = 0;
			for (int i = 0; i < n_chunks; ++i) {
				const int s = i % S;
				if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1, abort_flag, a.err)) break;
				const uint32_t bytes = chunk_bytes(i);
				mbar_arrive_expect_tx(&full[s], bytes);
				bulk_g2s(ring + (size_t)s * a.stage_bytes, wbase + (size_t)i * RPC * row_bytes, bytes, &full[s], pol);
				const int pf = i + S + kGemvPrefetch;
				if (pf < n_chunks) bulk_prefetch_l2(wbase + (size_t)pf * RPC * row_bytes, chunk_bytes(pf));
				++issued;
			}
			if (a.nx_W && issued == n_chunks && (int)blockIdx.x < a.nx_grid) {
				const int tu = a.nx_N / a.nx_unit_rows;
				const int q0 = (int)(((long long)blockIdx.x * tu) / a.nx_grid) * a.nx_unit_rows;
				const int q1 = (int)(((long long)(blockIdx.x + 1) * tu) / a.nx_grid) * a.nx_unit_rows;
				const size_t nrb = (size_t)a.nx_K * sizeof(T);
				const uint8_t* p = reinterpret_cast<const uint8_t*>(a.nx_W) + (size_t)q0 * nrb;
				size_t left = min((size_t)(q1 - q0) * nrb, (size_t)a.nx_bytes);
				while (left > 0) {
					const uint32_t n = (uint32_t)min(left, (size_t)32768);
					bulk_prefetch_l2(p, n);
					p += n;
					left -= n;
				}
			}
			// never leave the CTA with bulk copies in flight: wait for the last stages to land
			for (int i = max(0, issued - S); i < issued; ++i) {
				const int s = i % S;
				const uint64_t t0 = global_timer_ns();
				while (!mbar_try_wait(&full[s], (i / S) & 1)) {
					if (global_timer_ns() - t0 > kWaitLimitNs) {
						report_err(a.err, kDevTimeout);
						break;
					}
				}
			}
		}
		return;
	}

	// ---------------- consumers ----------------
	const int ct = tid; // 0..255
	const int units_per_row = (int)(row_bytes >> 4);
	// the norm gain is a weight: with at most two units a lane it is read before the dependency
	// wait, taking a cold HBM read off the prologue (more units would spill registers)
	constexpr bool kEarlyGain = UPL <= 2;
	uint4 graw[UPL];
	if constexpr (kEarlyGain) {
		bool norm_early = EpiTraits<EPI>::kNorm;
		if constexpr (EpiTraits<EPI>::kRuntimeProlog) norm_early = a.resid_in != nullptr;
		const T* g = reinterpret_cast<const T*>(a.gain);
#pragma unroll
		for (int u = 0; u < UPL; ++u) {
			const int unit = u * kGemvConsumers + ct;
			graw[u] = (norm_early && g && unit < units_per_row) ? *reinterpret_cast<const uint4*>(g + (size_t)unit * VEC)
			                                                  : make_uint4(0, 0, 0, 0);
		}
	}
	pdl_wait();
	// kEpiResid on one GPU with the CTA's rows in one window: this thread's residual row, read now
	// so that the epilogue adds to a register instead of waiting on L2 after the last chunk
	const bool res_pre = EPI == kEpiResid && !tp_on && n_rows <= kGemvFlushRows;
	float res_row = 0.0f;
	if (res_pre && ct < n_rows) res_row = a.resid[r0 + ct];

	float xh[UPL][VEC];
	bool norm_prolog = EpiTraits<EPI>::kNorm;
	if constexpr (EpiTraits<EPI>::kRuntimeProlog) norm_prolog = a.resid_in != nullptr;
	if (norm_prolog) {
		float ss = 0.0f;
#pragma unroll
		for (int u = 0; u < UPL; ++u) {
			const int unit = u * kGemvConsumers + ct;
#pragma unroll
			for (int v = 0; v < VEC; ++v) xh[u][v] = 0.0f;
			if (unit < units_per_row) {
				const float* src = a.resid_in + (size_t)unit * VEC;
#pragma unroll
				for (int v = 0; v < VEC; v += 4) {
					const float4 f = *reinterpret_cast<const float4*>(src + v);
					xh[u][v] = f.x; xh[u][v + 1] = f.y; xh[u][v + 2] = f.z; xh[u][v + 3] = f.w;
				}
#pragma unroll
				for (int v = 0; v < VEC; ++v) ss = fmaf(xh[u][v], xh[u][v], ss);
			}
		}
		if constexpr (EpiTraits<EPI>::kGemma) {
			if (a.pend) {
				// r' = r + (p * rsqrt(mean(p^2) + eps)) * (1 + g_p)
				float pv[UPL][VEC];
				float sp = 0.0f;
#pragma unroll
				for (int u = 0; u < UPL; ++u) {
					const int unit = u * kGemvConsumers + ct;
#pragma unroll
					for (int v = 0; v < VEC; ++v) pv[u][v] = 0.0f;
					if (unit < units_per_row) {
						const float* src = a.pend + (size_t)unit * VEC;
#pragma unroll
						for (int v = 0; v < VEC; v += 4) {
							const float4 f = *reinterpret_cast<const float4*>(src + v);
							pv[u][v] = f.x; pv[u][v + 1] = f.y; pv[u][v + 2] = f.z; pv[u][v + 3] = f.w;
						}
#pragma unroll
						for (int v = 0; v < VEC; ++v) sp = fmaf(pv[u][v], pv[u][v], sp);
					}
				}
				sp = warp_sum(sp);
				if (lane == 0) red_ss[warp] = sp;
				named_bar_sync(1, kGemvConsumers);
				float tp_ = 0.0f;
#pragma unroll
				for (int w = 0; w < kGemvConsumerWarps; ++w) tp_ += red_ss[w];
				named_bar_sync(1, kGemvConsumers); // red_ss is reused below
				const float invp = 1.0f / sqrtf(__fdiv_rn(tp_, (float)a.K) + a.eps);
				const T* gp = reinterpret_cast<const T*>(a.pend_gain);
				ss = 0.0f;
#pragma unroll
				for (int u = 0; u < UPL; ++u) {
					const int unit = u * kGemvConsumers + ct;
					if (unit < units_per_row) {
						const uint4 gw = *reinterpret_cast<const uint4*>(gp + (size_t)unit * VEC);
						float gf[VEC];
						unpack_unit(gw, gf, (const T*)nullptr);
#pragma unroll
						for (int v = 0; v < VEC; ++v)
							xh[u][v] = __fadd_rn(xh[u][v], __fmul_rn(__fmul_rn(pv[u][v], invp), __fadd_rn(1.0f, gf[v])));
						if (blockIdx.x == 0 && a.resid_out) {
							float* dst = a.resid_out + (size_t)unit * VEC;
#pragma unroll
							for (int v = 0; v < VEC; v += 4)
								*reinterpret_cast<float4*>(dst + v) = make_float4(xh[u][v], xh[u][v + 1], xh[u][v + 2], xh[u][v + 3]);
						}
#pragma unroll
						for (int v = 0; v < VEC; ++v) ss = fmaf(xh[u][v], xh[u][v], ss);
					}
				}
			}
		}
		bool skip_norm = false;
		if constexpr (EpiTraits<EPI>::kGemma) skip_norm = a.no_norm != 0;
		if (skip_norm) {
#pragma unroll
			for (int u = 0; u < UPL; ++u)
#pragma unroll
				for (int v = 0; v < VEC; ++v) xh[u][v] = Store<T>::round(xh[u][v]);
		} else {
			ss = warp_sum(ss);
			if (lane == 0) red_ss[warp] = ss;
			named_bar_sync(1, kGemvConsumers);
			float tot = 0.0f;
#pragma unroll
			for (int w = 0; w < kGemvConsumerWarps; ++w) tot += red_ss[w];
			const float inv = 1.0f / sqrtf(__fdiv_rn(tot, (float)a.K) + a.eps);
			const T* g = reinterpret_cast<const T*>(a.gain);
			bool plus1 = false;
			if constexpr (EpiTraits<EPI>::kGemma) plus1 = a.gain_plus1 != 0;
#pragma unroll
			for (int u = 0; u < UPL; ++u) {
				const int unit = u * kGemvConsumers + ct;
				if (unit < units_per_row) {
					uint4 gw;
					if constexpr (kEarlyGain) gw = graw[u];
					else gw = *reinterpret_cast<const uint4*>(g + (size_t)unit * VEC);
					float gf[VEC];
					unpack_unit(gw, gf, (const T*)nullptr);
					if (plus1) {
#pragma unroll
						for (int v = 0; v < VEC; ++v) gf[v] = __fadd_rn(1.0f, gf[v]);
					}
#pragma unroll
					for (int v = 0; v < VEC; ++v) xh[u][v] = Store<T>::round(__fmul_rn(__fmul_rn(xh[u][v], inv), gf[v]));
				}
			}
		}
	} else {
		const T* x = reinterpret_cast<const T*>(a.xin);
#pragma unroll
		for (int u = 0; u < UPL; ++u) {
			const int unit = u * kGemvConsumers + ct;
			if (unit < units_per_row) {
				const uint4 xw = *reinterpret_cast<const uint4*>(x + (size_t)unit * VEC);
				unpack_unit(xw, xh[u], (const T*)nullptr);
			} else {
#pragma unroll
				for (int v = 0; v < VEC; ++v) xh[u][v] = 0.0f;
			}
		}
	}

	unsigned long long best = 0ull;
	int pos = 0, slot = 0;
	if constexpr (EPI == kEpiQkv) {
		pos = *a.pos;
		slot = *a.slot;
	}

	// Each warp reduces its RPC row partials across lanes (transposed butterfly: one value
	// per lane survives) and parks them in wpart; the cross-warp sum and the epilogue run
	// for a window of kGemvFlushRows rows at a time, so chunks flow without a block barrier.
	constexpr int kChunksPerFlush = kGemvFlushRows / RPC;
	const int my_row = row_of_lane<RPC>(lane);
	const bool row_writer = (lane & (32 / RPC - 1)) == 0;
	int w0 = 0; // first CTA-local row of the current window
	for (int i = 0; i < n_chunks; ++i) {
		const int s = i % S;
		const bool ok = mbar_wait(&full[s], (i / S) & 1, abort_flag, a.err);
		const int rows = min(RPC, n_rows - i * RPC);
		const uint8_t* stage = ring + (size_t)s * a.stage_bytes;
		// this lane's units of the chunk into registers, then the slot goes back to the producer
		// at once: the unpacking, FMAs and reductions below run while the next copy is in flight
		uint4 wreg[RPC][UPL];
#pragma unroll
		for (int r = 0; r < RPC; ++r)
#pragma unroll
			for (int u = 0; u < UPL; ++u) {
				const int unit = u * kGemvConsumers + ct;
				wreg[r][u] = (ok && r < rows && unit < units_per_row)
				                 ? *reinterpret_cast<const uint4*>(stage + (size_t)r * row_bytes + (size_t)unit * 16)
				                 : make_uint4(0, 0, 0, 0);
			}
		__syncwarp();
		if (lane == 0) mbar_arrive(&empty[s]);
		float part[RPC];
#pragma unroll
		for (int r = 0; r < RPC; ++r) part[r] = gemv_unit_dot<T, UPL>(wreg[r], xh);
		const float v = reduce_rows<RPC>(part, lane);
		if (row_writer && my_row < rows) wpart[warp * kGemvFlushRows + (i * RPC - w0) + my_row] = v;
		if ((i + 1) % kChunksPerFlush != 0 && i + 1 != n_chunks) continue;

		// ---- flush: epilogue of window rows [w0, w0 + nw)
		const int nw = min(n_rows, (i + 1) * RPC) - w0;
		named_bar_sync(1, kGemvConsumers);
		for (int e = ct; e < nw / UNIT_ROWS; e += kGemvConsumers) {
			const int lr = e * UNIT_ROWS;
			const int row = r0 + w0 + lr;
			float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
			for (int w = 0; w < kGemvConsumerWarps; ++w) {
				d0 += wpart[w * kGemvFlushRows + lr];
				if (PAIRED) d1 += wpart[w * kGemvFlushRows + lr + 1];
			}
			if constexpr (EPI == kEpiStore) {
				Store<T>::put(reinterpret_cast<T*>(a.out) + row, d0);
			} else if constexpr (EPI == kEpiResid) {
				if (tp_on) tp_stage[row - r0] = d0;
				else if (res_pre) a.resid[row] = res_row + d0; // row == r0 + ct (one window)
				else a.resid[row] += d0;
			} else if constexpr (EPI == kEpiSwiglu) {
				Store<T>::put(reinterpret_cast<T*>(a.out) + (row >> 1), __fmul_rn(silu(d0), d1));
			} else if constexpr (EPI == kEpiLogits) {
				if (a.softcap > 0.0f) d0 = __fmul_rn(a.softcap, tanhf(__fdiv_rn(d0, a.softcap)));
				a.logits[row] = d0;
				const unsigned long long key = argmax_key(d0, (uint32_t)(row + a.row_base));
				best = key > best ? key : best;
			} else if constexpr (EPI == kEpiStoreF32) {
				reinterpret_cast<float*>(a.out)[row] = d0;
			} else if constexpr (EPI == kEpiGeglu) {
				Store<T>::put(reinterpret_cast<T*>(a.out) + (row >> 1), __fmul_rn(gelu_tanh(d0), d1));
			} else if constexpr (EPI == kEpiPleGate) {
				Store<T>::put(reinterpret_cast<T*>(a.out) + row,
				              __fmul_rn(gelu_tanh(d0), Store<T>::get(reinterpret_cast<const T*>(a.ple) + row)));
			} else if constexpr (EPI == kEpiQkv) {
				const int hd = a.head_dim, half = hd >> 1;
				const int head = row / hd;
				const int dim = (row % hd) >> 1; // pair (dim, dim + half)
				float o0 = d0, o1 = d1;
				if (head < a.n_q_heads + a.n_kv_heads) {
					const float c = a.rope_cos[(size_t)pos * half + dim];
					const float sn = a.rope_sin[(size_t)pos * half + dim];
					o0 = __fsub_rn(__fmul_rn(d0, c), __fmul_rn(d1, sn));
					o1 = __fadd_rn(__fmul_rn(d1, c), __fmul_rn(d0, sn));
				}
				if (head < a.n_q_heads) {
					T* q = reinterpret_cast<T*>(a.out) + (size_t)head * hd;
					Store<T>::put(q + dim, o0);
					Store<T>::put(q + dim + half, o1);
				} else {
					const bool is_k = head < a.n_q_heads + a.n_kv_heads;
					const int kvh = head - a.n_q_heads - (is_k ? 0 : a.n_kv_heads);
					const int page = a.block_table[(size_t)slot * a.pages_per_seq + pos / a.kv_block];
					if (page < 0 || page >= a.max_pages || pos >= a.max_seq) {
						report_err(a.err, kDevKvRange);
					} else {
						T* base = reinterpret_cast<T*>(is_k ? a.kpool : a.vpool) +
						          (((size_t)page * a.n_kv_heads + kvh) * a.kv_block + (pos % a.kv_block)) * hd;
						Store<T>::put(base + dim, o0);
						Store<T>::put(base + dim + half, o1);
					}
				}
			}
		}
		named_bar_sync(1, kGemvConsumers); // the window buffer is reused by the next chunks
		w0 += nw;
	}

	if constexpr (EPI == kEpiResid) {
		if (tp_on) {
			// fused all-reduce: every rank's partials for this CTA's rows go to every rank as
			// (value, round) slots; each rank sums the ranks' values in rank order (identical on
			// all ranks).  No flag and no fence: a slot is complete when it carries the round.
			const TpComm& c = a.tp;
			const unsigned round = tp_round(c, a.tp_round_index);
			const int par = (int)(round & 1u);
			named_bar_sync(1, kGemvConsumers);
			for (int i = ct; i < n_rows * c.size; i += kGemvConsumers) {
				const int k = i / n_rows, r = i % n_rows;
				st_relaxed_sys_u64(c.inbox[k] + ((size_t)par * c.size + c.rank) * c.dim + r0 + r, ll_pack(tp_stage[r], round));
			}
			// collect: thread i waits for (rank k, row r); the sums are formed in rank order
			float* recv = wpart; // the epilogue window is idle now: [size][n_rows]
			bool ok = true;
			for (int i = ct; i < n_rows * c.size; i += kGemvConsumers) {
				const int k = i / n_rows, r = i % n_rows;
				recv[i] = ll_wait(c.inbox[c.rank] + ((size_t)par * c.size + k) * c.dim + r0 + r, round, a.err, &ok);
			}
			if (!ok) *abort_flag = 1;
			named_bar_sync(1, kGemvConsumers);
			if (!*abort_flag) {
				for (int r = ct; r < n_rows; r += kGemvConsumers) {
					float v = 0.0f;
					for (int k = 0; k < c.size; ++k) v += recv[k * n_rows + r];
					a.resid[r0 + r] += v;
				}
			}
		}
	}

	if constexpr (EPI == kEpiLogits) {
		// CTA max, then grid max through one atomic; the last CTA publishes the token.
#pragma unroll
		for (int o = 16; o > 0; o >>= 1) {
			const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, best, o);
			best = other > best ? other : best;
		}
		if (lane == 0) red_best[warp] = best;
		named_bar_sync(1, kGemvConsumers);
		if (ct == 0) {
			unsigned long long b = 0ull;
			for (int w = 0; w < kGemvConsumerWarps; ++w) b = red_best[w] > b ? red_best[w] : b;
			atomicMax(a.best, b);
			__threadfence();
			const unsigned done = atomicAdd(a.counter, 1u);
			if (done == gridDim.x - 1) {
				__threadfence();
				unsigned long long fin = atomicAdd(a.best, 0ull);
				if (tp_on) {
					// cross-shard argmax: every rank publishes its best key, takes the max of all
					const TpComm& c = a.tp;
					const unsigned round = tp_round(c, kTpRoundLm);
					const int par = (int)(*c.epoch & 1u);
					// one thread: its key stores are ordered before its own release stores
					for (int k = 0; k < c.size; ++k) c.am_inbox[k][par * c.size + c.rank] = fin;
					for (int k = 0; k < c.size; ++k) st_release_sys(c.am_flags[k] + c.rank, round);
					bool ok = true;
					for (int k = 0; k < c.size; ++k) ok = tp_wait_flag(c.am_flags[c.rank] + k, round, a.err) && ok;
					if (ok)
						for (int k = 0; k < c.size; ++k) {
							const unsigned long long o = *(volatile unsigned long long*)&c.am_inbox[c.rank][par * c.size + k];
							fin = o > fin ? o : fin;
						}
				}
				const uint32_t id = argmax_key_index(fin);
				*a.cur_id = id;
				const uint32_t st = *a.step;
				if ((int)st < a.max_out) a.out_ids[st] = id;
				*a.step = st + 1;
				*a.pos_rw = *a.pos_rw + 1;
				*a.best = 0ull;
				*a.counter = 0u;
				if (tp_on) *(uint32_t*)a.tp.epoch = *a.tp.epoch + 1u;
			}
		}
	}
}

// Shared memory of one SM on sm_100 and the part the hardware reserves per CTA.
constexpr size_t kSmemPerSm = 228 * 1024;
constexpr size_t kSmemReservedPerCta = 1024;
// A projection CTA takes just over half of an SM's shared memory, whatever its own needs, so
// two of them never share an SM: with programmatic dependent launch the block scheduler
// otherwise doubles up the CTAs of a low-register projection (the O-proj) on some SMs and
// lets the next projection's early CTAs stream their ring on the SMs left free, and the
// doubled-up CTAs finish ~3 us after the others.  A decode-attention CTA still fits beside one.
constexpr size_t kGemvSmemFloor = kSmemPerSm / 2 - kSmemReservedPerCta + 512;

constexpr size_t gemv_smem_need()
{
	return (size_t)kGemvRingBytes + 2 * kGemvMaxStages * sizeof(uint64_t) +
	       (kGemvConsumerWarps * kGemvFlushRows + kGemvConsumerWarps + 8) * sizeof(float) +
	       kGemvConsumerWarps * sizeof(unsigned long long) + 16 + kTpMaxRowsCta * sizeof(float);
}
static_assert(gemv_smem_need() <= kGemvSmemFloor, "projection shared memory above the floor");
static_assert(2 * (kGemvSmemFloor + kSmemReservedPerCta) > kSmemPerSm, "two projection CTAs fit on one SM");

inline size_t gemv_smem_bytes() { return kGemvSmemFloor; }

} // namespace inf
