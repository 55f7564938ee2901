// Engine: model build (model_build, src/main.cu:200-352), forward and generate for the
// decoder token loop, and the stand-alone kernels of the C ABI (include/inf.h).
//
// Device memory is one arena slab (src/cuda/api/cuda_allocator.cu:4-19) holding, in
// order: weights in the device layout, RoPE tables, the paged KV cache, block tables,
// activations and decode scratch.  The batch-1 decode step is one CUDA graph whose
// kernels read the token id and position from device memory and advance them, so
// replays chain without the host.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <utility>
#include <vector>

#include "common.cuh"
#include "k_attn_decode.cuh"
#include "k_attn_decode_stream.cuh"
#include "k_attn_decode_mma.cuh"
#include "k_attn_cluster.cuh"
#include "k_attn_cluster_tc.cuh"
#include "k_gemv.cuh"
#include "k_gemma.cuh"
#include "k_attn_prefill.cuh"
#include "k_attn_prefill_tc.cuh"
#include "k_gemm_tc.cuh"
#include "k_sample.cuh"
#include "k_small.cuh"
#include "loader.h"
#include "runtime.h"
#include "synth.cuh"

using namespace inf;

struct LayerW {
	void* wqkv;      // [(Hl + 2 KVl) hd x d], rows of each head in (i, i+hd/2) pairs
	void* wo;        // [d x Hl hd]
	void* wgu;       // [2 Fl x d], rows alternate gate_j / up_j
	void* wd;        // [d x Fl]
	void* attn_norm; // [d]
	void* ffn_norm;  // [d]
	void* kpool;     // [pages][KVl][blk][hd]
	void* vpool;
	// Gemma-style decoder
	void* q_norm;        // [hd]
	void* k_norm;        // [hd]
	void* post_attn;     // [d]
	void* post_ffn;      // [d]
	void* ple_gate;      // [P x d]
	void* ple_proj;      // [d x P]
	void* ple_post;      // [d]
};

struct InfEngine {
	InfConfig cfg;
	ExecCtx* ctx = nullptr;
	int device = 0;
	int sm_count = 148;
	cudaStream_t stream = nullptr;
	size_t esz = 2; // bytes of the storage dtype
	// local (per tensor-parallel rank) shapes
	int Hl = 0, KVl = 0, Fl = 0, Vl = 0;
	// weights
	void* embed = nullptr;
	void* lm_head = nullptr;
	void* final_norm = nullptr;
	std::vector<LayerW> layers;
	u64 weight_bytes = 0;
	float* rope_cos = nullptr;
	float* rope_sin = nullptr;
	// paged KV
	int pages_per_seq = 0, n_pages = 0;
	int* block_table = nullptr;             // device [max_batch][pages_per_seq]
	std::vector<int> h_block_table;         // host mirror
	std::vector<std::vector<int>> seq_pages;
	std::vector<int> free_pages;
	// activations / scratch (batch-1 decode)
	float* resid = nullptr;
	void* q = nullptr;
	void* attn = nullptr;
	void* h = nullptr;
	float* logits = nullptr;
	int* ctl = nullptr; // [kCtlWords]: id, pos, slot, step, err (one H2D / one D2H per token)
	uint32_t* cur_id = nullptr;
	int* pos = nullptr;
	int* slot = nullptr;
	uint32_t* out_ids = nullptr;
	uint32_t* step = nullptr;
	unsigned long long* best = nullptr;
	unsigned* lm_counter = nullptr;
	float* attn_part = nullptr;  // split partials, sized for the larger of batch 1 and max_batch
	int attn_splits_batch = 1;    // splits when max_batch tokens share one launch
	int attn_max_pages_split_batch = 1;
	// batched mma attention work list: (token, split | splits << 16) per unit, longest first
	int* attn_units = nullptr;    // [max_batch * attn_unit_splits] int2
	int* h_units = nullptr;       // pinned staging
	int attn_unit_splits = 1;     // the most splits of one token (stride of the split partials)
	int n_attn_units = 0;         // units of the batched step being enqueued (0: no list)
	u64 h2d_bytes = 0;            // bytes staged host -> device by the batched step
	float* logits_p = nullptr;    // [max_batch][Vl] batched-decode logits
	uint32_t* argmax_p = nullptr; // [max_batch]
	unsigned long long* batch_keys = nullptr; // [max_batch] argmax keys, zero between steps
	unsigned* attn_counters = nullptr;
	int* err = nullptr;
	uint32_t* d_ids = nullptr; // staged ids [max_seq]
	int max_out = 0;
	int attn_splits = 1;
	int attn_max_pages_split = 1;
	bool pf_tc = false;           // prefill attention on the tensor cores (k_attn_prefill_tc.cuh)
	float* gemm_part = nullptr;   // split-K shares of the tensor-core GEMM
	u64 gemm_part_bytes = 0;
	bool gemm_split = false;      // split-K allowed (batched decode; prefill keeps one K pass per tile)
	int attn_cl_splits = 0;       // batch-1 decode attention as one cluster per KV head (0: split-K)
	int attn_cl_pages = 0;
	int attn_cl_tc = 0;           // ... on the tensor cores (k_attn_decode_clt)
	// multi-token (prefill) buffers, prefill_chunk rows each
	int chunk = 0;
	float* resid_p = nullptr;  // [chunk][d] f32
	void* xhat_p = nullptr;    // [chunk][d]
	void* q_p = nullptr;       // [chunk][Hl*hd]
	void* attn_p = nullptr;    // [chunk][Hl*hd]
	void* h_p = nullptr;       // [chunk][Fl]
	int* tok_pos = nullptr;    // [chunk]
	int* tok_slot = nullptr;   // [chunk]
	int* h_tok = nullptr;      // pinned [2 * chunk]
	// pinned host staging
	uint32_t* h_pin = nullptr; // [max_seq + 16]
	int* h_ctl = nullptr;      // [2 * kCtlWords]: staging in, staging out
	// decode graph
	cudaGraphExec_t decode_exec = nullptr;
	InfSampling samp = {};      // temperature 0: greedy
	bool sampling = false;
	uint32_t* sample_q = nullptr; // [Vl] fixed-point weights of the sampler
	// per-slot sampling of the batched step and the server (inf_set_slot_sampling)
	std::vector<InfSampling> slot_samp; // [max_batch], temperature 0: greedy
	SampleRow* rows_d = nullptr;        // [max_batch] the rows' settings on the device
	SampleRow* rows_h = nullptr;        // [max_batch] pinned staging
	uint32_t* sample_q_rows = nullptr;  // [max_batch][Vl] fixed-point weights of the rows
	int graph_kernels = 0;
	u64 launches = 0;
	bool profiling = false;
	bool dry = false; // walk the launch sequence without launching (sets kernel attributes)
	// Gemma-style decoder (cfg.arch == InfArchGemma)
	bool gemma = false;
	void* embed_ple = nullptr;      // [V][L * P]
	void* ple_model_proj = nullptr; // [L * P][d]
	void* ple_proj_norm = nullptr;  // [P]
	float* resid2 = nullptr;        // the second residual buffer (pending adds write the other one)
	float* raw = nullptr;           // fp32 raw projection output: qkv [(H + 2 KV) hd], or o / down / PLE [d]
	float* pend = nullptr;          // fp32 [d] projection output waiting for its norm and residual add
	void* xb = nullptr;             // bf16 [d] rounded embedding (per-layer-input projection)
	float* pm = nullptr;            // fp32 [L * P]
	void* ple = nullptr;            // bf16 [L][P] per-layer inputs of the token
	void* ple_y = nullptr;          // bf16 [P]
	float* resid_final = nullptr;   // the residual buffer the LM head's prologue wrote
	// tensor parallelism over peer memory (tp_size > 1)
	TpComm tpc;                        // size 1 until inf_tp_connect
	u64 comm_off = 0;                  // offset of this rank's comm region in its arena
	std::vector<void*> peer_bases;     // opened IPC mappings (nullptr for self)
	unsigned pf_round = 0;             // multi-token all-reduce rounds issued so far
	cudaEvent_t prof_ev[2] = {nullptr, nullptr};
	float prof_ms[InfKNumKinds] = {};
};

namespace {

enum CtlWord { kCtlId = 0, kCtlPos = 1, kCtlSlot = 2, kCtlStep = 3, kCtlErr = 4, kCtlEpoch = 5, kCtlWords = 8 };

std::mutex g_attr_mutex;

Error_t map_dev_err(int v)
{
	switch (v) {
	case kDevOk: return Success;
	case kDevTimeout: return fail(ErrorTimeout, "a bounded device wait expired");
	case kDevTokenRange: return fail(ErrorTokenOutOfRange, "token id >= vocab_size");
	case kDevKvRange: return fail(ErrorKvOutOfRange, "KV position or page outside the cache");
	default: return fail(ErrorGeneric, "device error word %d", v);
	}
}

Error_t check_dev_err(InfEngine* e)
{
	int v = 0;
	INF_CUDA_TRY(cudaMemcpyAsync(&v, e->err, sizeof v, cudaMemcpyDeviceToHost, e->stream));
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	if (v == kDevOk) return Success;
	INF_CUDA_TRY(cudaMemsetAsync(e->err, 0, sizeof(int), e->stream));
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	return map_dev_err(v);
}

template <typename... KArgs, typename... Args>
cudaError_t launch(InfEngine* e, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args)
{
	cudaLaunchConfig_t lc = {};
	lc.gridDim = grid;
	lc.blockDim = block;
	lc.dynamicSmemBytes = smem;
	lc.stream = e->stream;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;
	lc.attrs = attr;
	lc.numAttrs = e->profiling ? 0 : 1;
	if (e->dry) return cudaSuccess;
	e->launches++;
	return cudaLaunchKernelEx(&lc, kern, std::forward<Args>(args)...);
}

// Raises a kernel's dynamic shared-memory ceiling to `bytes` if it is below it (models of
// different shapes in one process need different sizes for the same kernel), and asks for
// the largest shared-memory carveout: the driver otherwise sizes an SM's carveout for the
// kernel that occupies it (a projection CTA alone gets too little room for an attention CTA
// beside it, so the next kernel's CTAs could not start before the dependency resolves).
template <typename K>
cudaError_t set_smem(K kern, size_t bytes)
{
	static std::unordered_map<const void*, size_t> set_to;
	std::lock_guard<std::mutex> lk(g_attr_mutex);
	size_t& cur = set_to[reinterpret_cast<const void*>(kern)];
	if (bytes <= cur) return cudaSuccess;
	cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
	if (e == cudaSuccess)
		e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
	if (e == cudaSuccess) cur = bytes;
	return e;
}

// --------------------------------------------------------------------------- GEMV
template <typename T, int UPL, int EPI>
Error_t launch_gemv_u(InfEngine* e, GemvArgs a)
{
	constexpr int RPC = GemvShape<UPL, EPI>::kRpc;
	const size_t row_bytes = (size_t)a.K * sizeof(T);
	a.stage_bytes = (uint32_t)(RPC * row_bytes);
	a.stages = std::min<int>(kGemvMaxStages, (int)(kGemvRingBytes / a.stage_bytes));
	if (a.stages < 2) return fail(ErrorUnsupported, "gemv: row of %zu bytes too long", row_bytes);
	const int unit_rows = EpiTraits<EPI>::kPaired ? 2 : 1;
	const int grid = std::max(1, std::min(e->sm_count, a.N / unit_rows));
	const size_t smem = gemv_smem_bytes();
	INF_CUDA_TRY(set_smem(k_gemv<T, UPL, EPI>, smem));
	INF_CUDA_TRY(launch(e, k_gemv<T, UPL, EPI>, dim3(grid), dim3(kGemvThreads), smem, a));
	return Success;
}

template <typename T, int EPI>
Error_t launch_gemv(InfEngine* e, const GemvArgs& a)
{
	const size_t row_bytes = (size_t)a.K * sizeof(T);
	if (row_bytes % 16 != 0) return fail(ErrorUnsupported, "gemv: K*%zu not a multiple of 16 bytes", sizeof(T));
	const int units = (int)(row_bytes / 16);
	const int upl = (units + kGemvConsumers - 1) / kGemvConsumers;
	if (upl <= 1) return launch_gemv_u<T, 1, EPI>(e, a);
	if (upl <= 2) return launch_gemv_u<T, 2, EPI>(e, a);
	if (upl <= 4) return launch_gemv_u<T, 4, EPI>(e, a);
	return fail(ErrorUnsupported, "gemv: K=%d too long", a.K);
}

// the projection that follows in the decode step, for the producer's L2 warm-up
void gemv_next(InfEngine* e, GemvArgs& a, const void* W, int N, int K, bool paired)
{
	a.nx_W = W;
	a.nx_N = N;
	a.nx_K = K;
	a.nx_unit_rows = paired ? 2 : 1;
	a.nx_grid = std::max(1, std::min(e->sm_count, N / a.nx_unit_rows));
	a.nx_bytes = kGemvNextPrefetch;
}

GemvArgs gemv_base(InfEngine* e, const void* W, int N, int K)
{
	GemvArgs a;
	memset(&a, 0, sizeof a);
	a.W = W;
	a.N = N;
	a.K = K;
	a.eps = e->cfg.norm_eps;
	a.err = e->err;
	a.tp = e->tpc;
	return a;
}

// --------------------------------------------------------------------------- cluster attention
// Whether a cluster of cs CTAs (mp pages each) of the batch-1 attention kernel fits one GPU.
template <typename T>
Error_t attn_cl_fit(int G, int hd, int blk, int kv_heads, int cs, int mp, bool* ok)
{
	*ok = false;
	const AttnKernel<T> k = attn_decode_cl_kernel<T>(G, hd);
	if (!k) return Success;
	const size_t smem = attn_cl_layout(G, hd, blk, sizeof(T), mp, cs).total;
	INF_CUDA_TRY(set_smem(k, smem));
	if (cs > 8) INF_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
	cudaLaunchConfig_t lc = {};
	lc.gridDim = dim3(cs, kv_heads, 1);
	lc.blockDim = dim3(kAttnThreads);
	lc.dynamicSmemBytes = smem;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeClusterDimension;
	attr[0].val.clusterDim.x = cs;
	attr[0].val.clusterDim.y = 1;
	attr[0].val.clusterDim.z = 1;
	lc.attrs = attr;
	lc.numAttrs = 1;
	int n = 0;
	if (cudaOccupancyMaxActiveClusters(&n, k, &lc) != cudaSuccess) {
		(void)cudaGetLastError(); // not placeable: use the split-K kernel
		return Success;
	}
	*ok = n >= 1;
	return Success;
}

// The batch-1 decode attention plan: one cluster per KV head, the largest cluster (16, then 8
// CTAs) whose split of a pages_per_seq-page context fits the shared-memory budget and that the
// GPU can place.  *splits = 0 when none does (the split-K kernel serves the shape).
Error_t attn_cl_plan(int G, int hd, int blk, size_t esz, int pages_per_seq, int kv_heads, int* splits, int* pages)
{
	*splits = 0;
	*pages = 0;
	for (int cs = kAttnClMaxSplits; cs >= 8; cs >>= 1) {
		const int mp = attn_cl_pages_per_split(cs, pages_per_seq, blk, hd, esz, G);
		if (mp == 0) continue;
		bool ok = false;
		if (esz == 2) INF_TRY(attn_cl_fit<bf16>(G, hd, blk, kv_heads, cs, mp, &ok));
		else INF_TRY(attn_cl_fit<float>(G, hd, blk, kv_heads, cs, mp, &ok));
		if (!ok) continue;
		*splits = cs;
		*pages = mp;
		return Success;
	}
	return Success;
}

// The same plan for the tensor-core cluster kernel (bf16, 16-position pages, head_dim 64 or
// 128, G <= 8): *splits = 0 when it does not apply or fit.
Error_t attn_cltc_plan(int G, int hd, int blk, size_t esz, int pages_per_seq, int kv_heads, int* splits, int* pages)
{
	*splits = 0;
	*pages = 0;
	const AttnClTcKernel k = attn_decode_cltc_kernel(G, hd);
	if (esz != 2 || blk != 16 || !k) return Success;
	for (int cs = kAttnClMaxSplits; cs >= 8; cs >>= 1) {
		const int mp = attn_cltc_pages_per_split(cs, pages_per_seq, hd, G);
		if (mp == 0) continue;
		const size_t smem = attn_cltc_layout(G, hd, mp, cs).total;
		INF_CUDA_TRY(set_smem(k, smem));
		if (cs > 8) INF_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
		cudaLaunchConfig_t lc = {};
		lc.gridDim = dim3(cs, kv_heads, 1);
		lc.blockDim = dim3(kClTcThreads);
		lc.dynamicSmemBytes = smem;
		cudaLaunchAttribute attr[1];
		attr[0].id = cudaLaunchAttributeClusterDimension;
		attr[0].val.clusterDim.x = cs;
		attr[0].val.clusterDim.y = 1;
		attr[0].val.clusterDim.z = 1;
		lc.attrs = attr;
		lc.numAttrs = 1;
		int n = 0;
		if (cudaOccupancyMaxActiveClusters(&n, k, &lc) != cudaSuccess) {
			(void)cudaGetLastError();
			continue;
		}
		if (n < 1) continue;
		*splits = cs;
		*pages = mp;
		return Success;
	}
	return Success;
}

Error_t attn_cl_choose(InfEngine* e, int G, int hd)
{
	INF_TRY(attn_cltc_plan(G, hd, (int)e->cfg.kv_block, e->esz, e->pages_per_seq, e->KVl, &e->attn_cl_splits,
	                       &e->attn_cl_pages));
	e->attn_cl_tc = e->attn_cl_splits > 0;
	if (e->attn_cl_tc) return Success;
	return attn_cl_plan(G, hd, (int)e->cfg.kv_block, e->esz, e->pages_per_seq, e->KVl, &e->attn_cl_splits,
	                    &e->attn_cl_pages);
}

Error_t tensor_map_kv(CUtensorMap* m, const void* base, u32 hd, u32 blk, u32 kv, u32 pages, u32 box_pages);

// launch with a cluster of cluster_x CTAs along x and the programmatic-dependency edge
template <typename... KArgs, typename... Args>
cudaError_t launch_cluster(InfEngine* e, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster_x,
                           Args&&... args)
{
	cudaLaunchConfig_t lc = {};
	lc.gridDim = grid;
	lc.blockDim = block;
	lc.dynamicSmemBytes = smem;
	lc.stream = e->stream;
	cudaLaunchAttribute attr[2];
	attr[0].id = cudaLaunchAttributeClusterDimension;
	attr[0].val.clusterDim.x = cluster_x;
	attr[0].val.clusterDim.y = 1;
	attr[0].val.clusterDim.z = 1;
	attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[1].val.programmaticStreamSerializationAllowed = 1;
	lc.attrs = attr;
	lc.numAttrs = e->profiling ? 1 : 2;
	if (e->dry) return cudaSuccess;
	e->launches++;
	return cudaLaunchKernelEx(&lc, kern, std::forward<Args>(args)...);
}

// --------------------------------------------------------------------------- decode step
Error_t prof_begin(InfEngine* e)
{
	if (e->profiling) INF_CUDA_TRY(cudaEventRecord(e->prof_ev[0], e->stream));
	return Success;
}
Error_t prof_end(InfEngine* e, int kind)
{
	if (!e->profiling) return Success;
	INF_CUDA_TRY(cudaEventRecord(e->prof_ev[1], e->stream));
	INF_CUDA_TRY(cudaEventSynchronize(e->prof_ev[1]));
	float ms = 0.f;
	INF_CUDA_TRY(cudaEventElapsedTime(&ms, e->prof_ev[0], e->prof_ev[1]));
	e->prof_ms[kind] += ms;
	return Success;
}

Error_t enqueue_sample(InfEngine* e);

// Batch-1 decode attention of one layer over the paged cache (q in e->q, output e->attn): one
// cluster per KV head when the plan fits, else the split-K kernel.
template <typename T>
Error_t enqueue_attention(InfEngine* e, const LayerW& L)
{
	const InfConfig& c = e->cfg;
	const int hd = (int)c.head_dim;
	AttnDecodeArgs a;
	memset(&a, 0, sizeof a);
	a.q = e->q;
	a.kpool = L.kpool;
	a.vpool = L.vpool;
	a.block_table = e->block_table;
	a.pages_per_seq = e->pages_per_seq;
	a.max_pages = e->n_pages;
	a.tok_slot = e->slot;
	a.tok_pos = e->pos;
	a.H = e->Hl;
	a.KV = e->KVl;
	a.hd = hd;
	a.blk = (int)c.kv_block;
	a.n_splits = e->attn_splits;
	a.max_pages_split = e->attn_max_pages_split;
	a.scale = (float)(1.0 / std::sqrt((double)hd));
	a.part = e->attn_part;
	a.counters = e->attn_counters;
	a.out = e->attn;
	a.err = e->err;
	if (e->attn_cl_splits > 0 && e->attn_cl_tc) {
		a.n_splits = e->attn_cl_splits;
		a.max_pages_split = e->attn_cl_pages;
		const int cs = e->attn_cl_splits, G = e->Hl / e->KVl;
		const size_t smem = attn_cltc_layout(G, hd, e->attn_cl_pages, cs).total;
		const AttnClTcKernel ak = attn_decode_cltc_kernel(G, hd);
		if (!ak) return fail(ErrorUnsupported, "attention: GQA group %d, head_dim %d", G, hd);
		CUtensorMap tk, tv; // one page (16 positions x 64 head dims) per box
		INF_TRY(tensor_map_kv(&tk, L.kpool, (u32)hd, c.kv_block, (u32)e->KVl, (u32)e->n_pages, 1));
		INF_TRY(tensor_map_kv(&tv, L.vpool, (u32)hd, c.kv_block, (u32)e->KVl, (u32)e->n_pages, 1));
		INF_CUDA_TRY(set_smem(ak, smem));
		INF_TRY(prof_begin(e));
		INF_CUDA_TRY(launch_cluster(e, ak, dim3(cs, e->KVl, 1), dim3(kClTcThreads), smem, cs, tk, tv, a));
		INF_TRY(prof_end(e, InfKAttn));
	} else if (e->attn_cl_splits > 0) {
		a.n_splits = e->attn_cl_splits;
		a.max_pages_split = e->attn_cl_pages;
		const int cs = e->attn_cl_splits;
		const size_t smem = attn_cl_layout(e->Hl / e->KVl, hd, (int)c.kv_block, sizeof(T), e->attn_cl_pages, cs).total;
		const AttnKernel<T> ak = attn_decode_cl_kernel<T>(e->Hl / e->KVl, hd);
		if (!ak) return fail(ErrorUnsupported, "attention: GQA group %d, head_dim %d", e->Hl / e->KVl, hd);
		INF_CUDA_TRY(set_smem(ak, smem));
		INF_TRY(prof_begin(e));
		INF_CUDA_TRY(launch_cluster(e, ak, dim3(cs, e->KVl, 1), dim3(kAttnThreads), smem, cs, a));
		INF_TRY(prof_end(e, InfKAttn));
	} else {
		const size_t smem = attn_decode_smem_bytes(e->Hl / e->KVl, hd, (int)c.kv_block, sizeof(T),
		                                           e->attn_max_pages_split, e->attn_splits);
		const AttnKernel<T> ak = attn_decode_kernel<T>(e->Hl / e->KVl, hd);
		if (!ak) return fail(ErrorUnsupported, "attention: GQA group %d, head_dim %d", e->Hl / e->KVl, hd);
		INF_CUDA_TRY(set_smem(ak, smem));
		INF_TRY(prof_begin(e));
		INF_CUDA_TRY(launch(e, ak, dim3(e->KVl, e->attn_splits, 1), dim3(kAttnThreads), smem, a));
		INF_TRY(prof_end(e, InfKAttn));
	}
	return Success;
}

template <typename T>
Error_t enqueue_decode_step(InfEngine* e)
{
	const InfConfig& c = e->cfg;
	const int d = (int)c.dim, hd = (int)c.head_dim;
	const int kernels_before = (int)e->launches;

	INF_TRY(prof_begin(e));
	INF_CUDA_TRY(launch(e, k_embed<T, float>, dim3((d + 255) / 256, 1), dim3(256), 0, (const uint32_t*)e->cur_id, 1, d,
	                    c.vocab_size, (const T*)e->embed, e->resid, e->err));
	INF_TRY(prof_end(e, InfKEmbed));

	for (u32 l = 0; l < c.n_layers; ++l) {
		const LayerW& L = e->layers[l];
		// QKV + RoPE + KV write, RMSNorm fused in front
		{
			GemvArgs a = gemv_base(e, L.wqkv, (e->Hl + 2 * e->KVl) * hd, d);
			a.resid_in = e->resid;
			a.gain = L.attn_norm;
			a.out = e->q;
			a.kpool = L.kpool;
			a.vpool = L.vpool;
			a.block_table = e->block_table;
			a.pages_per_seq = e->pages_per_seq;
			a.max_pages = e->n_pages;
			a.pos = e->pos;
			a.slot = e->slot;
			a.rope_cos = e->rope_cos;
			a.rope_sin = e->rope_sin;
			a.head_dim = hd;
			a.n_q_heads = e->Hl;
			a.n_kv_heads = e->KVl;
			a.kv_block = (int)c.kv_block;
			a.max_seq = (int)c.max_seq;
			INF_TRY(prof_begin(e));
			INF_TRY((launch_gemv<T, kEpiQkv>(e, a)));
			INF_TRY(prof_end(e, InfKQkv));
		}
		// attention
		INF_TRY(enqueue_attention<T>(e, L));
		// O-proj + residual
		{
			GemvArgs a = gemv_base(e, L.wo, d, e->Hl * hd);
			a.tp_round_index = 2 * (int)l;
			a.xin = e->attn;
			a.resid = e->resid;
			gemv_next(e, a, L.wgu, 2 * e->Fl, d, true);
			INF_TRY(prof_begin(e));
			INF_TRY((launch_gemv<T, kEpiResid>(e, a)));
			INF_TRY(prof_end(e, InfKO));
		}
		// gate/up + SwiGLU, RMSNorm fused in front
		{
			GemvArgs a = gemv_base(e, L.wgu, 2 * e->Fl, d);
			a.resid_in = e->resid;
			a.gain = L.ffn_norm;
			a.out = e->h;
			gemv_next(e, a, L.wd, d, e->Fl, false);
			INF_TRY(prof_begin(e));
			INF_TRY((launch_gemv<T, kEpiSwiglu>(e, a)));
			INF_TRY(prof_end(e, InfKGateUp));
		}
		// down + residual
		{
			GemvArgs a = gemv_base(e, L.wd, d, e->Fl);
			a.tp_round_index = 2 * (int)l + 1;
			a.xin = e->h;
			a.resid = e->resid;
			if (l + 1 < c.n_layers) gemv_next(e, a, e->layers[l + 1].wqkv, (e->Hl + 2 * e->KVl) * hd, d, true);
			else gemv_next(e, a, e->lm_head, e->Vl, d, false);
			INF_TRY(prof_begin(e));
			INF_TRY((launch_gemv<T, kEpiResid>(e, a)));
			INF_TRY(prof_end(e, InfKDown));
		}
	}
	// final norm + LM head + greedy argmax; advances id, position and step
	{
		GemvArgs a = gemv_base(e, e->lm_head, e->Vl, d);
		a.row_base = (int)e->cfg.tp_rank * e->Vl;
		a.resid_in = e->resid;
		a.gain = e->final_norm;
		a.logits = e->logits;
		a.best = e->best;
		a.counter = e->lm_counter;
		a.cur_id = e->cur_id;
		a.out_ids = e->out_ids;
		a.step = e->step;
		a.pos_rw = e->pos;
		a.max_out = e->max_out;
		INF_TRY(prof_begin(e));
		INF_TRY((launch_gemv<T, kEpiLogits>(e, a)));
		INF_TRY(enqueue_sample(e)); // timed with the LM head when profiling
		INF_TRY(prof_end(e, InfKLmHead));
	}
	e->graph_kernels = (int)e->launches - kernels_before;
	return Success;
}

// The constants of the Gemma-style decoder, rounded to bf16 from double as the model dtype holds
// them: the embedding scale sqrt(dim), and sqrt(ple_dim), dim^-1/2 and 2^-1/2 of the per-layer
// inputs.
float gemma_const(double v)
{
	const uint32_t u = (uint32_t)f32_to_bf16_bits((float)v) << 16;
	float f;
	memcpy(&f, &u, 4);
	return f;
}

// One decode step of the Gemma-style decoder (bf16, one GPU).  Every projection stores its raw
// fp32 output; the RMSNorm that follows it (q/k norms, post-attention, post-FFN, post-PLE) runs in
// the next kernel: a separate kernel for the per-head q/k norms (with RoPE and the KV write), the
// next projection's prologue for the others, which folds the normalised output into the residual.
// The residual alternates between two buffers: a prologue that folds reads one and writes the
// other (from CTA 0), so no CTA of the same kernel reads a half-updated residual.
Error_t enqueue_decode_step_gemma(InfEngine* e)
{
	const InfConfig& c = e->cfg;
	const int d = (int)c.dim, hd = (int)c.head_dim, P = (int)c.ple_dim, L = (int)c.n_layers;
	const int H = e->Hl, KV = e->KVl;
	const int kernels_before = (int)e->launches;
	float* rbuf[2] = {e->resid, e->resid2};
	int cur = 0;                     // rbuf[cur] holds the residual
	const void* pend_gain = nullptr; // gain of the output waiting in e->pend (none: nullptr)
	auto fold = [&](GemvArgs& a) {
		a.resid_in = rbuf[cur];
		if (pend_gain) {
			a.pend = e->pend;
			a.pend_gain = pend_gain;
			a.resid_out = rbuf[cur ^ 1];
			cur ^= 1;
			pend_gain = nullptr;
		}
	};
	auto round32 = [](int n) { return (n + 31) / 32 * 32; };

	// embedding * bf16(sqrt(dim)) and, with per-layer embeddings, the token's per-layer inputs
	INF_TRY(prof_begin(e));
	{
		GemmaEmbedArgs a;
		a.id = e->cur_id;
		a.vocab = c.vocab_size;
		a.dim = d;
		a.table = (const bf16*)e->embed;
		a.scale = gemma_const(std::sqrt((double)d));
		a.resid = rbuf[0];
		a.xb = P ? (bf16*)e->xb : nullptr;
		a.err = e->err;
		INF_CUDA_TRY(launch(e, k_gemma_embed, dim3((d + 255) / 256), dim3(256), 0, a));
	}
	if (P) {
		GemvArgs a = gemv_base(e, e->ple_model_proj, L * P, d);
		a.xin = e->xb;
		a.out = e->pm;
		INF_TRY((launch_gemv<bf16, kEpiStoreF32>(e, a)));
		PleCombineArgs pa;
		pa.id = e->cur_id;
		pa.vocab = c.vocab_size;
		pa.L = L;
		pa.P = P;
		pa.pm = e->pm;
		pa.embed_ple = (const bf16*)e->embed_ple;
		pa.norm_gain = (const bf16*)e->ple_proj_norm;
		pa.s_ple = gemma_const(std::sqrt((double)P));
		pa.s_proj = gemma_const(1.0 / std::sqrt((double)d));
		pa.s_sum = gemma_const(1.0 / std::sqrt(2.0));
		pa.eps = c.norm_eps;
		pa.ple = (bf16*)e->ple;
		INF_CUDA_TRY(launch(e, k_ple_combine, dim3(L), dim3(round32(P)), 0, pa));
	}
	INF_TRY(prof_end(e, InfKEmbed));

	for (int l = 0; l < L; ++l) {
		const LayerW& W = e->layers[l];
		// QKV (raw), then per-head q/k RMSNorm + RoPE + KV write
		INF_TRY(prof_begin(e));
		{
			GemvArgs a = gemv_base(e, W.wqkv, (H + 2 * KV) * hd, d);
			fold(a);
			a.gain = W.attn_norm;
			a.gain_plus1 = 1;
			a.out = e->raw;
			INF_TRY((launch_gemv<bf16, kEpiStoreF32>(e, a)));
			QkNormArgs q;
			q.raw = e->raw;
			q.H = H;
			q.KV = KV;
			q.hd = hd;
			q.q_gain = (const bf16*)W.q_norm;
			q.k_gain = (const bf16*)W.k_norm;
			q.eps = c.norm_eps;
			q.rope_cos = e->rope_cos;
			q.rope_sin = e->rope_sin;
			q.pos = e->pos;
			q.slot = e->slot;
			q.q_out = (bf16*)e->q;
			q.kpool = (bf16*)W.kpool;
			q.vpool = (bf16*)W.vpool;
			q.block_table = e->block_table;
			q.pages_per_seq = e->pages_per_seq;
			q.max_pages = e->n_pages;
			q.kv_block = (int)c.kv_block;
			q.max_seq = (int)c.max_seq;
			q.err = e->err;
			INF_CUDA_TRY(launch(e, k_qk_norm_rope, dim3(H + 2 * KV), dim3(round32(hd / 2)), 0, q));
		}
		INF_TRY(prof_end(e, InfKQkv));
		INF_TRY(enqueue_attention<bf16>(e, W));
		// O (raw) -> pending, post-attention norm
		INF_TRY(prof_begin(e));
		{
			GemvArgs a = gemv_base(e, W.wo, d, H * hd);
			a.xin = e->attn;
			a.out = e->pend;
			INF_TRY((launch_gemv<bf16, kEpiStoreF32>(e, a)));
			pend_gain = W.post_attn;
		}
		INF_TRY(prof_end(e, InfKO));
		// residual += post-attention norm, pre-FFN norm, gate/up + GELU-tanh
		INF_TRY(prof_begin(e));
		{
			GemvArgs a = gemv_base(e, W.wgu, 2 * e->Fl, d);
			fold(a);
			a.gain = W.ffn_norm;
			a.gain_plus1 = 1;
			a.out = e->h;
			INF_TRY((launch_gemv<bf16, kEpiGeglu>(e, a)));
		}
		INF_TRY(prof_end(e, InfKGateUp));
		// down (raw) -> pending, post-FFN norm; the per-layer-embedding block
		INF_TRY(prof_begin(e));
		{
			GemvArgs a = gemv_base(e, W.wd, d, e->Fl);
			a.xin = e->h;
			a.out = e->pend;
			INF_TRY((launch_gemv<bf16, kEpiStoreF32>(e, a)));
			pend_gain = W.post_ffn;
		}
		if (P) {
			GemvArgs a = gemv_base(e, W.ple_gate, P, d);
			fold(a);
			a.no_norm = 1;
			a.ple = (const bf16*)e->ple + (size_t)l * P;
			a.out = e->ple_y;
			INF_TRY((launch_gemv<bf16, kEpiPleGate>(e, a)));
			a = gemv_base(e, W.ple_proj, d, P);
			a.xin = e->ple_y;
			a.out = e->pend;
			INF_TRY((launch_gemv<bf16, kEpiStoreF32>(e, a)));
			pend_gain = W.ple_post;
		}
		INF_TRY(prof_end(e, InfKDown));
	}
	// residual += the last pending output, final norm, LM head (the embedding), soft-cap, argmax
	{
		GemvArgs a = gemv_base(e, e->lm_head, e->Vl, d);
		fold(a);
		a.gain = e->final_norm;
		a.gain_plus1 = 1;
		a.softcap = c.final_softcap;
		a.logits = e->logits;
		a.best = e->best;
		a.counter = e->lm_counter;
		a.cur_id = e->cur_id;
		a.out_ids = e->out_ids;
		a.step = e->step;
		a.pos_rw = e->pos;
		a.max_out = e->max_out;
		INF_TRY(prof_begin(e));
		INF_TRY((launch_gemv<bf16, kEpiLogits>(e, a)));
		INF_TRY(enqueue_sample(e));
		INF_TRY(prof_end(e, InfKLmHead));
	}
	e->resid_final = rbuf[cur];
	e->graph_kernels = (int)e->launches - kernels_before;
	return Success;
}

Error_t enqueue_step(InfEngine* e)
{
	if (e->gemma) return enqueue_decode_step_gemma(e);
	return e->cfg.dtype == InfBF16 ? enqueue_decode_step<bf16>(e) : enqueue_decode_step<float>(e);
}

// --------------------------------------------------------------------------- prefill
constexpr u64 kGemmPartBytes = 16ull << 20; // split-K scratch of the tensor-core GEMM
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

Error_t tensor_map_2d(CUtensorMap* m, const void* base, u64 rows, u64 cols, u32 box_rows)
{
	if (!g_encode) {
		cudaDriverEntryPointQueryResult q;
		void* fn = nullptr;
		INF_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
		if (q != cudaDriverEntryPointSuccess || !fn) return fail(ErrorCuda, "cuTensorMapEncodeTiled unavailable");
		g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
	}
	const cuuint64_t dims[2] = {cols, rows};
	const cuuint64_t strides[1] = {cols * 2};
	const cuuint32_t box[2] = {(cuuint32_t)kTcBK, box_rows};
	const cuuint32_t estr[2] = {1, 1};
	const CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
	                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
	                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
	if (r != CUDA_SUCCESS) return fail(ErrorCuda, "cuTensorMapEncodeTiled failed (%d)", (int)r);
	return Success;
}

// A layer's paged K or V pool [pages][KV][blk][hd] as a 4-D tensor (hd, row, head, page) with
// boxes of 64 head dims x blk rows x 1 head x box_pages pages, SWIZZLE_128B.
Error_t tensor_map_kv(CUtensorMap* m, const void* base, u32 hd, u32 blk, u32 kv, u32 pages, u32 box_pages)
{
	CUtensorMap dummy;
	INF_TRY(tensor_map_2d(&dummy, base, 8, 64, 8)); // resolves the driver entry point
	const cuuint64_t dims[4] = {hd, blk, kv, pages};
	const cuuint64_t strides[3] = {(cuuint64_t)hd * 2, (cuuint64_t)blk * hd * 2, (cuuint64_t)kv * blk * hd * 2};
	const cuuint32_t box[4] = {64, blk, 1, box_pages};
	const cuuint32_t estr[4] = {1, 1, 1, 1};
	const CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
	                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
	                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
	if (r != CUDA_SUCCESS) return fail(ErrorCuda, "cuTensorMapEncodeTiled (K/V pool) failed (%d)", (int)r);
	return Success;
}

// The RMSNorm that follows a residual projection (its gain, bf16 output and epsilon); when the
// projection is split across K the norm runs inside the split-K sum (k_gemm_splitk_resid_norm)
// and *done is set, otherwise the caller launches k_rmsnorm_rows.
struct NormNext {
	const void* gain;
	void* out;
	float eps;
	bool* done;
};

// N tile width of a GEMM: 256, or, when the 256-wide tiles come to fewer than two waves over
// the SMs and K is not going to be split (a split fills the SMs by itself), the multiple of 16
// in 128 .. 256 whose tiles fill the waves best (ties: the wider).  The 64-token batched
// gate/up projection (N 28672): 112 tiles of 256 fill 76% of 148 SMs, 138 tiles of 208 fill 93%.
int gemm_tile_width(int T, int N, int sms, bool may_split)
{
	const int m_tiles = (T + kTcBM - 1) / kTcBM;
	const int tiles256 = m_tiles * ((N + kTcBN - 1) / kTcBN);
	if (tiles256 >= 2 * sms || (may_split && tiles256 * 2 <= sms)) return kTcBN;
	int best = kTcBN;
	double best_fill = 0.0;
	for (int bn = kTcBN; bn >= 128; bn -= 16) {
		const int units = m_tiles * ((N + bn - 1) / bn);
		const int waves = (units + sms - 1) / sms;
		const double fill = (double)m_tiles * N / bn / ((double)waves * sms);
		if (fill > best_fill + 1e-9) {
			best_fill = fill;
			best = bn;
		}
	}
	return best;
}

// D[T x N] = X[T x K] . W[N x K]^T on the tensor cores, fused epilogue a.epi
Error_t launch_gemm_tc(InfEngine* e, const void* X, const void* W, TcArgs a, const NormNext* nn = nullptr)
{
	if (nn) *nn->done = false;
	if (a.K % 8 != 0) return fail(ErrorUnsupported, "gemm: K %% 8 != 0");
	a.bn = gemm_tile_width(a.T, a.N, std::max(e->sm_count, 1), e->gemm_split && e->gemm_part);
	CUtensorMap tx, tw;
	INF_TRY(tensor_map_2d(&tx, X, (u64)a.T, (u64)a.K, kTcBM));
	INF_TRY(tensor_map_2d(&tw, W, (u64)a.N, (u64)a.K, (u32)a.bn));
	const size_t smem = gemm_tc_smem_bytes();
	INF_CUDA_TRY(set_smem(k_gemm_tc, smem));
	a.err = e->err;
	// too few output tiles to stream the weights on every SM: split K across CTAs
	const int tiles = ((a.N + a.bn - 1) / a.bn) * ((a.T + kTcBM - 1) / kTcBM), n_kb = (a.K + kTcBK - 1) / kTcBK;
	int splits = 1;
	if (e->gemm_split && e->gemm_part && tiles * 2 <= e->sm_count) {
		splits = std::min(e->sm_count / tiles, n_kb / 2);
		const u64 per_split = (u64)a.T * a.N * 4;
		splits = (int)std::min<u64>((u64)splits, e->gemm_part_bytes / std::max<u64>(per_split, 1));
	}
	if (splits >= 2) {
		a.k_splits = splits;
		a.partial = e->gemm_part;
		// persistent CTAs over the (tile, split) units, at most one per SM
		INF_CUDA_TRY(launch(e, k_gemm_tc, dim3(std::min(tiles * splits, std::max(e->sm_count, 1))), dim3(kTcThreads), smem,
		                    tx, tw, a));
		if (nn && a.epi == kTcResid && a.N <= kResNormThreads * kResNormMaxCols) {
			const auto kn = a.N <= kResNormThreads * 16 ? k_gemm_splitk_resid_norm<16> : k_gemm_splitk_resid_norm<kResNormMaxCols>;
			INF_CUDA_TRY(launch(e, kn, dim3(a.T), dim3(kResNormThreads), 0, a, (bf16*)nn->out, (const bf16*)nn->gain, nn->eps));
			*nn->done = true;
			return Success;
		}
		const int groups = a.T * ((a.N + 31) / 32);
		INF_CUDA_TRY(launch(e, k_gemm_splitk_reduce, dim3((groups + 7) / 8), dim3(256), 0, a));
		return Success;
	}
	a.k_splits = 1;
	INF_CUDA_TRY(launch(e, k_gemm_tc, dim3(std::min(tiles, std::max(e->sm_count, 1))), dim3(kTcThreads), smem, tx, tw, a));
	return Success;
}

// Row-parallel projection + residual: local GEMM into the fp32 partial buffer, then the
// two-shot peer-memory all-reduce adds the sum over ranks into the residual.
Error_t launch_gemm_resid_tp(InfEngine* e, const void* X, const void* W, TcArgs a, const NormNext* nn = nullptr);

TcArgs tc_base(InfEngine* e, int T, int N, int K, int epi)
{
	TcArgs a;
	memset(&a, 0, sizeof a);
	a.T = T;
	a.N = N;
	a.K = K;
	a.epi = epi;
	a.err = e->err;
	return a;
}

Error_t launch_gemm_resid_tp(InfEngine* e, const void* X, const void* W, TcArgs a, const NormNext* nn)
{
	if (e->tpc.size <= 1) return launch_gemm_tc(e, X, W, a, nn);
	if (nn) *nn->done = false;
	float* resid = a.resid;
	a.epi = kTcStoreF32;
	a.out = e->tpc.part[e->tpc.rank];
	INF_TRY(launch_gemm_tc(e, X, W, a));
	const int n = a.T * a.N;
	const int grid = std::min(kTpMaxCtas, std::max(1, std::min(e->sm_count, (n + 4095) / 4096)));
	const unsigned round = ++e->pf_round;
	INF_CUDA_TRY(launch(e, k_tp_allreduce_add, dim3(grid), dim3(256), 0, e->tpc, n, round, resid, e->err));
	return Success;
}

// One chunk of T tokens of one sequence (positions and slots already in tok_pos/tok_slot),
// all layers on the tensor cores; leaves the residual of every token in resid_p.
Error_t enqueue_prefill_layers(InfEngine* e, int T)
{
	const InfConfig& c = e->cfg;
	const int d = (int)c.dim, hd = (int)c.head_dim, G = e->Hl / e->KVl;
	INF_CUDA_TRY(launch(e, k_embed<bf16, float>, dim3((d + 255) / 256, T), dim3(256), 0, (const uint32_t*)e->d_ids, T, d,
	                    c.vocab_size, (const bf16*)e->embed, e->resid_p, e->err));
	const size_t pf_smem = e->pf_tc ? attn_prefill_tc_smem_bytes(hd) : attn_prefill_smem_bytes(G, hd, (int)c.kv_block);
	if (e->pf_tc) INF_CUDA_TRY(set_smem(k_attn_prefill_tc, pf_smem));
	else INF_CUDA_TRY(set_smem(k_attn_prefill<bf16>, pf_smem));
	bool normed = false; // xhat_p already holds the norm that the next projection reads
	for (u32 l = 0; l < c.n_layers; ++l) {
		const LayerW& L = e->layers[l];
		if (!normed)
			INF_CUDA_TRY(launch(e, k_rmsnorm_rows<float, bf16, bf16>, dim3(T), dim3(256), 0, (const float*)e->resid_p,
			                    (bf16*)e->xhat_p, T, d, (const bf16*)L.attn_norm, c.norm_eps));
		{
			TcArgs a = tc_base(e, T, (e->Hl + 2 * e->KVl) * hd, d, kTcQkv);
			a.out = e->q_p;
			a.kpool = L.kpool;
			a.vpool = L.vpool;
			a.block_table = e->block_table;
			a.pages_per_seq = e->pages_per_seq;
			a.max_pages = e->n_pages;
			a.max_seq = (int)c.max_seq;
			a.tok_pos = e->tok_pos;
			a.tok_slot = e->tok_slot;
			a.rope_cos = e->rope_cos;
			a.rope_sin = e->rope_sin;
			a.head_dim = hd;
			a.n_q_heads = e->Hl;
			a.n_kv_heads = e->KVl;
			a.kv_block = (int)c.kv_block;
			INF_TRY(launch_gemm_tc(e, e->xhat_p, L.wqkv, a));
		}
		{
			AttnPrefillArgs a;
			memset(&a, 0, sizeof a);
			a.q = e->q_p;
			a.kpool = L.kpool;
			a.vpool = L.vpool;
			a.block_table = e->block_table;
			a.pages_per_seq = e->pages_per_seq;
			a.max_pages = e->n_pages;
			a.tok_pos = e->tok_pos;
			a.tok_slot = e->tok_slot;
			a.T = T;
			a.H = e->Hl;
			a.KV = e->KVl;
			a.hd = hd;
			a.blk = (int)c.kv_block;
			a.scale = (float)(1.0 / std::sqrt((double)hd));
			a.out = e->attn_p;
			a.err = e->err;
			if (e->pf_tc) {
				// the layer's K and V pools, boxes of one tile's pages and of one page
				const u32 bp = kPtKeys / c.kv_block;
				CUtensorMap tk8, tk1, tv8, tv1;
				INF_TRY(tensor_map_kv(&tk8, L.kpool, (u32)hd, c.kv_block, (u32)e->KVl, (u32)e->n_pages, bp));
				INF_TRY(tensor_map_kv(&tk1, L.kpool, (u32)hd, c.kv_block, (u32)e->KVl, (u32)e->n_pages, 1));
				INF_TRY(tensor_map_kv(&tv8, L.vpool, (u32)hd, c.kv_block, (u32)e->KVl, (u32)e->n_pages, bp));
				INF_TRY(tensor_map_kv(&tv1, L.vpool, (u32)hd, c.kv_block, (u32)e->KVl, (u32)e->n_pages, 1));
				const int tq = kPtRows / G;
				INF_CUDA_TRY(launch(e, k_attn_prefill_tc, dim3(e->KVl, (T + tq - 1) / tq), dim3(kPtThreads), pf_smem, tk8, tk1,
				                    tv8, tv1, a));
			} else {
				INF_CUDA_TRY(launch(e, k_attn_prefill<bf16>, dim3(e->KVl, (T + kPfTq - 1) / kPfTq), dim3(kPfThreads), pf_smem, a));
			}
		}
		{
			TcArgs a = tc_base(e, T, d, e->Hl * hd, kTcResid);
			a.resid = e->resid_p;
			const NormNext nn{L.ffn_norm, e->xhat_p, c.norm_eps, &normed};
			INF_TRY(launch_gemm_resid_tp(e, e->attn_p, L.wo, a, &nn));
		}
		if (!normed)
			INF_CUDA_TRY(launch(e, k_rmsnorm_rows<float, bf16, bf16>, dim3(T), dim3(256), 0, (const float*)e->resid_p,
			                    (bf16*)e->xhat_p, T, d, (const bf16*)L.ffn_norm, c.norm_eps));
		{
			TcArgs a = tc_base(e, T, 2 * e->Fl, d, kTcSwiglu);
			a.out = e->h_p;
			INF_TRY(launch_gemm_tc(e, e->xhat_p, L.wgu, a));
		}
		{
			TcArgs a = tc_base(e, T, d, e->Fl, kTcResid);
			a.resid = e->resid_p;
			// the next layer's attention norm (the last layer's residual goes to the LM head row)
			const NormNext nn{l + 1 < c.n_layers ? e->layers[l + 1].attn_norm : nullptr, e->xhat_p, c.norm_eps, &normed};
			INF_TRY(launch_gemm_resid_tp(e, e->h_p, L.wd, a, l + 1 < c.n_layers ? &nn : nullptr));
			if (l + 1 == c.n_layers) normed = false;
		}
	}
	return Success;
}

// With sampling on, replaces the id the LM head chose (greedy) by a draw from the
// temperature / top-k / top-p distribution of its logits (k_sample.cuh).
Error_t enqueue_sample(InfEngine* e)
{
	if (!e->sampling) return Success;
	SampleArgs a;
	a.logits = e->logits;
	a.q = e->sample_q;
	a.V = e->Vl;
	a.inv_temp = (float)(1.0 / (double)e->samp.temperature);
	a.top_p = e->samp.top_p;
	a.top_k = e->samp.top_k;
	a.key = stream_key(e->samp.seed, kSampleStream);
	a.cur_id = e->cur_id;
	a.out_ids = e->out_ids;
	a.step = e->step;
	a.pos = e->pos;
	a.slot = e->slot;
	a.max_out = e->max_out;
	INF_CUDA_TRY(set_smem(k_sample, kSampleSmem));
	INF_CUDA_TRY(launch(e, k_sample, dim3(1), dim3(kSampleThreads), kSampleSmem, a));
	return Success;
}

// Rows of logits [n][Vl] whose slot samples (inf_set_slot_sampling) replace their greedy id in
// ids_dev by a draw, one sampler CTA per row, the counter (pos_new[i], 0).  The caller
// has synchronised the stream since the last use of the pinned row staging.
Error_t enqueue_sample_rows(InfEngine* e, int n, const float* logits, const u32* slots, const u32* pos_new,
                            uint32_t* ids_dev)
{
	bool any = false;
	for (int i = 0; i < n; ++i) {
		const InfSampling& s = e->slot_samp[slots[i]];
		SampleRow& r = e->rows_h[i];
		r.on = s.temperature > 0.0f;
		r.inv_temp = r.on ? (float)(1.0 / (double)s.temperature) : 0.0f;
		r.top_p = s.top_p;
		r.top_k = s.top_k;
		r.pos_new = (int)pos_new[i];
		r.slot = 0; // the counter's high word: draws do not depend on which slot a sequence runs in
		r.key = stream_key(s.seed, kSampleStream);
		any = any || r.on;
	}
	if (!any) return Success;
	INF_CUDA_TRY(cudaMemcpyAsync(e->rows_d, e->rows_h, sizeof(SampleRow) * n, cudaMemcpyHostToDevice, e->stream));
	SampleRowsArgs a;
	a.logits = logits;
	a.q = e->sample_q_rows;
	a.V = e->Vl;
	a.rows = e->rows_d;
	a.ids = ids_dev;
	INF_CUDA_TRY(set_smem(k_sample_rows, kSampleSmem));
	INF_CUDA_TRY(launch(e, k_sample_rows, dim3(n), dim3(kSampleThreads), kSampleSmem, a));
	return Success;
}

// Final norm + LM head + argmax of one residual row (the decode GEMV); advances the ctl
// block exactly like a decode step (pos += 1, id = argmax, or the sampled id).
Error_t enqueue_lm_head_row(InfEngine* e, const float* resid_row)
{
	GemvArgs a = gemv_base(e, e->lm_head, e->Vl, (int)e->cfg.dim);
	a.row_base = (int)e->cfg.tp_rank * e->Vl;
	a.resid_in = resid_row;
	a.gain = e->final_norm;
	a.logits = e->logits;
	a.best = e->best;
	a.counter = e->lm_counter;
	a.cur_id = e->cur_id;
	a.out_ids = e->out_ids;
	a.step = e->step;
	a.pos_rw = e->pos;
	a.max_out = e->max_out;
	INF_TRY((e->cfg.dtype == InfBF16 ? launch_gemv<bf16, kEpiLogits>(e, a) : launch_gemv<float, kEpiLogits>(e, a)));
	return enqueue_sample(e);
}

// Prefill of n tokens (already in d_ids) of one slot from start: chunks of e->chunk tokens
// on the tensor cores, then the LM head of the last token.  Leaves ctl = (argmax, start+n, slot).
Error_t run_prefill(InfEngine* e, u32 n, u32 start, u32 slot)
{
	for (u32 c0 = 0; c0 < n; c0 += (u32)e->chunk) {
		const int T = (int)std::min<u32>((u32)e->chunk, n - c0);
		INF_CUDA_TRY(cudaStreamSynchronize(e->stream)); // h_tok reuse
		for (int t = 0; t < T; ++t) {
			e->h_tok[t] = (int)(start + c0 + t);
			e->h_tok[e->chunk + t] = (int)slot;
		}
		INF_CUDA_TRY(cudaMemcpyAsync(e->tok_pos, e->h_tok, sizeof(int) * T, cudaMemcpyHostToDevice, e->stream));
		INF_CUDA_TRY(cudaMemcpyAsync(e->tok_slot, e->h_tok + e->chunk, sizeof(int) * T, cudaMemcpyHostToDevice, e->stream));
		if (c0 > 0)
			INF_CUDA_TRY(cudaMemcpyAsync(e->d_ids, e->d_ids + c0, sizeof(u32) * T, cudaMemcpyDeviceToDevice, e->stream));
		INF_TRY(enqueue_prefill_layers(e, T));
		if (c0 + (u32)T == n) {
			int* in = e->h_ctl;
			in[kCtlPos] = (int)(start + n - 1);
			in[kCtlSlot] = (int)slot;
			INF_CUDA_TRY(cudaMemcpyAsync(e->pos, &in[kCtlPos], 2 * sizeof(int), cudaMemcpyHostToDevice, e->stream));
			INF_TRY(enqueue_lm_head_row(e, e->resid_p + (size_t)(T - 1) * e->cfg.dim));
		}
	}
	return Success;
}

bool use_tc_prefill(const InfEngine* e, u32 n) { return e->cfg.dtype == InfBF16 && e->chunk > 0 && n > 1; }

// Work list of the batched mma attention into h_units: each token's pages in units of about P
// pages, P chosen for about kAttnUnitCtasPerSm CTAs per SM over the KV heads (at least
// kAmUnitPagesMin pages), the units in decreasing page count, so the CTAs that start last are
// the short ones.  Returns the number of units.  Measured on 64 sequences of 512-4096 positions
// (Llama-3-8B shape): 2 CTAs per SM (every sequence one unit) 7.88 ms per step, 4 -> 8.20,
// 8 -> 8.41, the grid of two splits per sequence in batch order 8.54.
constexpr int kAttnUnitCtasPerSm = 2;
int build_attn_units(InfEngine* e, const u32* positions, u32 n)
{
	const u32 blk = e->cfg.kv_block;
	std::vector<int> np(n);
	u64 total = 0;
	for (u32 i = 0; i < n; ++i) {
		np[i] = (int)((positions[i] + blk) / blk); // pages of positions 0 .. positions[i]
		total += (u64)np[i];
	}
	const u64 target = std::max<u64>(1, (u64)kAttnUnitCtasPerSm * e->sm_count / (u64)std::max(1, e->KVl));
	const int P = (int)std::max<u64>((u64)kAmUnitPagesMin, (total + target - 1) / target);
	struct Unit {
		int pages, b, code;
	};
	std::vector<Unit> list;
	for (u32 i = 0; i < n; ++i) {
		const int ns = std::min(e->attn_unit_splits, std::max(1, (np[i] + P - 1) / P));
		const int pps = (np[i] + ns - 1) / ns;
		for (int sp = 0; sp < ns; ++sp)
			list.push_back({std::max(0, std::min(np[i], (sp + 1) * pps) - sp * pps), (int)i, sp | (ns << 16)});
	}
	std::stable_sort(list.begin(), list.end(), [](const Unit& x, const Unit& y) { return x.pages > y.pages; });
	for (size_t k = 0; k < list.size(); ++k) {
		e->h_units[2 * k] = list[k].b;
		e->h_units[2 * k + 1] = list[k].code;
	}
	return (int)list.size();
}

// One decode token for each of B sequences (ids in d_ids, slots/positions in tok_slot/tok_pos):
// the projections run once for all B tokens on the tensor cores (split-K when there are few
// output tiles), attention is the streaming mma kernel with one grid slice per token, the LM
// head is a GEMM whose epilogue folds the greedy argmax of every row.
Error_t enqueue_decode_batch(InfEngine* e, int B)
{
	const InfConfig& c = e->cfg;
	const int d = (int)c.dim, hd = (int)c.head_dim;
	INF_CUDA_TRY(launch(e, k_embed<bf16, float>, dim3((d + 255) / 256, B), dim3(256), 0, (const uint32_t*)e->d_ids, B, d,
	                    c.vocab_size, (const bf16*)e->embed, e->resid_p, e->err));
	bool normed = false; // xhat_p already holds the norm that the next projection reads
	for (u32 l = 0; l < c.n_layers; ++l) {
		const LayerW& L = e->layers[l];
		if (!normed)
			INF_CUDA_TRY(launch(e, k_rmsnorm_rows<float, bf16, bf16>, dim3(B), dim3(256), 0, (const float*)e->resid_p,
			                    (bf16*)e->xhat_p, B, d, (const bf16*)L.attn_norm, c.norm_eps));
		{
			TcArgs a = tc_base(e, B, (e->Hl + 2 * e->KVl) * hd, d, kTcQkv);
			a.out = e->q_p;
			a.kpool = L.kpool;
			a.vpool = L.vpool;
			a.block_table = e->block_table;
			a.pages_per_seq = e->pages_per_seq;
			a.max_pages = e->n_pages;
			a.max_seq = (int)c.max_seq;
			a.tok_pos = e->tok_pos;
			a.tok_slot = e->tok_slot;
			a.rope_cos = e->rope_cos;
			a.rope_sin = e->rope_sin;
			a.head_dim = hd;
			a.n_q_heads = e->Hl;
			a.n_kv_heads = e->KVl;
			a.kv_block = (int)c.kv_block;
			INF_TRY(launch_gemm_tc(e, e->xhat_p, L.wqkv, a));
		}
		{
			AttnDecodeArgs a;
			memset(&a, 0, sizeof a);
			a.q = e->q_p;
			a.kpool = L.kpool;
			a.vpool = L.vpool;
			a.block_table = e->block_table;
			a.pages_per_seq = e->pages_per_seq;
			a.max_pages = e->n_pages;
			a.tok_slot = e->tok_slot;
			a.tok_pos = e->tok_pos;
			a.H = e->Hl;
			a.KV = e->KVl;
			a.hd = hd;
			a.blk = (int)c.kv_block;
			a.n_splits = e->attn_splits_batch;
			a.max_pages_split = 0;
			a.scale = (float)(1.0 / std::sqrt((double)hd));
			a.part = e->attn_part;
			a.counters = e->attn_counters;
			a.out = e->attn_p;
			a.err = e->err;
			// tensor-core (mma) scores and P.V where the shape allows, else the SIMT streaming kernel
			const AttnMmaKernel am = attn_decode_mma_kernel(e->Hl / e->KVl, hd);
			if (am && c.kv_block == 16) { // 64-position chunks = 8 KB per 64 head dims
				const size_t smem = attn_mma_smem_bytes(hd, (int)c.kv_block, e->pages_per_seq);
				CUtensorMap tk, tv; // one page (blk positions x 64 head dims) per box
				INF_TRY(tensor_map_kv(&tk, L.kpool, (u32)hd, c.kv_block, (u32)e->KVl, (u32)e->n_pages, 1));
				INF_TRY(tensor_map_kv(&tv, L.vpool, (u32)hd, c.kv_block, (u32)e->KVl, (u32)e->n_pages, 1));
				INF_CUDA_TRY(set_smem(am, smem));
				if (e->n_attn_units > 0) {
					a.units = e->attn_units;
					a.n_splits = e->attn_unit_splits;
					INF_CUDA_TRY(launch(e, am, dim3(e->KVl, 1, e->n_attn_units), dim3(kAmThreads), smem, tk, tv, a));
				} else {
					INF_CUDA_TRY(launch(e, am, dim3(e->KVl, e->attn_splits_batch, B), dim3(kAmThreads), smem, tk, tv, a));
				}
			} else {
				const size_t smem = attn_stream_smem_bytes(e->Hl / e->KVl, hd, (int)c.kv_block, 2);
				const AttnKernel<bf16> ak = attn_decode_stream_kernel<bf16>(e->Hl / e->KVl, hd);
				if (!ak) return fail(ErrorUnsupported, "attention: GQA group %d, head_dim %d", e->Hl / e->KVl, hd);
				INF_CUDA_TRY(set_smem(ak, smem));
				INF_CUDA_TRY(launch(e, ak, dim3(e->KVl, e->attn_splits_batch, B), dim3(kAttnThreads), smem, a));
			}
		}
		{
			TcArgs a = tc_base(e, B, d, e->Hl * hd, kTcResid);
			a.resid = e->resid_p;
			const NormNext nn{L.ffn_norm, e->xhat_p, c.norm_eps, &normed};
			INF_TRY(launch_gemm_resid_tp(e, e->attn_p, L.wo, a, &nn));
		}
		if (!normed)
			INF_CUDA_TRY(launch(e, k_rmsnorm_rows<float, bf16, bf16>, dim3(B), dim3(256), 0, (const float*)e->resid_p,
			                    (bf16*)e->xhat_p, B, d, (const bf16*)L.ffn_norm, c.norm_eps));
		{
			TcArgs a = tc_base(e, B, 2 * e->Fl, d, kTcSwiglu);
			a.out = e->h_p;
			INF_TRY(launch_gemm_tc(e, e->xhat_p, L.wgu, a));
		}
		{
			TcArgs a = tc_base(e, B, d, e->Fl, kTcResid);
			a.resid = e->resid_p;
			// the next layer's attention norm, or the final norm before the LM head
			const NormNext nn{l + 1 < c.n_layers ? e->layers[l + 1].attn_norm : e->final_norm, e->xhat_p, c.norm_eps,
			                  &normed};
			INF_TRY(launch_gemm_resid_tp(e, e->h_p, L.wd, a, &nn));
		}
	}
	if (!normed)
		INF_CUDA_TRY(launch(e, k_rmsnorm_rows<float, bf16, bf16>, dim3(B), dim3(256), 0, (const float*)e->resid_p,
		                    (bf16*)e->xhat_p, B, d, (const bf16*)e->final_norm, c.norm_eps));
	{
		// logits and the greedy argmax of every row in the GEMM's epilogue
		TcArgs a = tc_base(e, B, e->Vl, d, kTcLogitsArgmax);
		a.out = e->logits_p;
		a.best_keys = e->batch_keys;
		a.col_base = (uint32_t)(c.tp_rank * (u32)e->Vl);
		INF_TRY(launch_gemm_tc(e, e->xhat_p, e->lm_head, a));
	}
	INF_CUDA_TRY(launch(e, k_keys_to_ids, dim3((B + 255) / 256), dim3(256), 0, e->batch_keys, B, e->argmax_p));
	return Success;
}

Error_t build_decode_graph(InfEngine* e)
{
	cudaGraph_t g = nullptr;
	e->dry = true; // shared-memory attributes are set outside the capture
	const Error_t dr = enqueue_step(e);
	e->dry = false;
	INF_TRY(dr);
	INF_CUDA_TRY(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
	const u64 before = e->launches;
	Error_t r = enqueue_step(e);
	cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
	e->launches = before;
	if (r != Success) {
		if (g) cudaGraphDestroy(g);
		return r;
	}
	if (ce != cudaSuccess) return fail(ErrorCuda, "graph capture: %s", cudaGetErrorString(ce));
	ce = cudaGraphInstantiate(&e->decode_exec, g, 0);
	cudaGraphDestroy(g);
	if (ce != cudaSuccess) return fail(ErrorCuda, "graph instantiate: %s", cudaGetErrorString(ce));
	return Success;
}

Error_t launch_decode_graph(InfEngine* e)
{
	INF_CUDA_TRY(cudaGraphLaunch(e->decode_exec, e->stream));
	e->launches += (u64)e->graph_kernels;
	return Success;
}

// --------------------------------------------------------------------------- pages
Error_t ensure_pages(InfEngine* e, u32 slot, u32 n_positions)
{
	const u32 blk = e->cfg.kv_block;
	const u32 need = (n_positions + blk - 1) / blk;
	if (need > (u32)e->pages_per_seq) return fail(ErrorKvOutOfRange, "sequence needs %u pages > %d", need, e->pages_per_seq);
	std::vector<int>& pg = e->seq_pages[slot];
	bool changed = false;
	while (pg.size() < need) {
		if (e->free_pages.empty()) return fail(ErrorArenaOutOfMemory, "KV cache out of pages");
		const int p = e->free_pages.back();
		e->free_pages.pop_back();
		e->h_block_table[(size_t)slot * e->pages_per_seq + pg.size()] = p;
		pg.push_back(p);
		changed = true;
	}
	if (changed) {
		// pageable source: the copy is staged before the call returns, ordered on the stream
		INF_CUDA_TRY(cudaMemcpyAsync(e->block_table + (size_t)slot * e->pages_per_seq,
		                             e->h_block_table.data() + (size_t)slot * e->pages_per_seq,
		                             sizeof(int) * e->pages_per_seq, cudaMemcpyHostToDevice, e->stream));
	}
	return Success;
}

Error_t release_pages(InfEngine* e, u32 slot)
{
	std::vector<int>& pg = e->seq_pages[slot];
	for (int p : pg) e->free_pages.push_back(p);
	// lowest ids are handed out first, so a sequence gets consecutive pages again (the prefill
	// attention loads a tile of consecutive pages with one copy)
	std::sort(e->free_pages.begin(), e->free_pages.end(), std::greater<int>());
	pg.clear();
	std::fill(e->h_block_table.begin() + (size_t)slot * e->pages_per_seq,
	          e->h_block_table.begin() + (size_t)(slot + 1) * e->pages_per_seq, -1);
	INF_CUDA_TRY(cudaMemcpyAsync(e->block_table + (size_t)slot * e->pages_per_seq,
	                             e->h_block_table.data() + (size_t)slot * e->pages_per_seq, sizeof(int) * e->pages_per_seq,
	                             cudaMemcpyHostToDevice, e->stream));
	return Success;
}

// --------------------------------------------------------------------------- build
Error_t validate(const InfConfig& c)
{
	if (c.vocab_size == 0 || c.dim == 0 || c.n_layers == 0 || c.n_heads == 0 || c.n_kv_heads == 0 || c.head_dim == 0 ||
	    c.ffn_dim == 0 || c.max_seq == 0 || c.max_batch == 0 || c.kv_block == 0)
		return fail(ErrorBadConfig, "zero-sized config field");
	if (c.dtype != InfF32 && c.dtype != InfBF16) return fail(ErrorBadConfig, "dtype %u", c.dtype);
	if (c.n_heads % c.n_kv_heads) return fail(ErrorBadConfig, "n_heads %% n_kv_heads != 0");
	if (c.head_dim % 2) return fail(ErrorBadConfig, "head_dim must be even");
	const u32 tp = c.tp_size ? c.tp_size : 1;
	if (c.tp_rank >= tp) return fail(ErrorBadConfig, "tp_rank >= tp_size");
	if (c.n_kv_heads % tp || c.ffn_dim % tp || c.vocab_size % tp) return fail(ErrorBadConfig, "shapes not divisible by tp_size");
	const u32 vec = c.dtype == InfBF16 ? 8 : 4;
	if (c.dim % vec || c.ffn_dim / tp % vec || (c.n_heads / tp * c.head_dim) % vec)
		return fail(ErrorBadConfig, "dim, ffn_dim and heads*head_dim must be multiples of %u", vec);
	if (c.arch != InfArchGemma && (c.n_heads / c.n_kv_heads) * c.head_dim * kPfTq > (u32)(kPfThreads * kPfMaxAcc))
		return fail(ErrorUnsupported, "GQA group x head_dim above %d", kPfThreads * kPfMaxAcc / kPfTq);
	if (c.arch > InfArchGemma) return fail(ErrorBadConfig, "arch %u", c.arch);
	{
		const u32 G = c.n_heads / c.n_kv_heads;
		if (G != 1 && G != 2 && G != 4 && G != 8) return fail(ErrorUnsupported, "GQA group %u (1, 2, 4 or 8)", G);
		if (c.arch == InfArchGemma) {
			if (!attn_decode_supported((int)G, (int)c.head_dim))
				return fail(ErrorUnsupported, "head_dim %u with GQA group %u (up to 512 for groups of at most 4)", c.head_dim, G);
		} else if (c.head_dim > 256) {
			return fail(ErrorUnsupported, "head_dim above 256");
		}
	}
	if (c.arch == InfArchGemma) {
		if (c.dtype != InfBF16) return fail(ErrorUnsupported, "Gemma-style models are bf16");
		if (tp > 1) return fail(ErrorUnsupported, "Gemma-style models run on one GPU");
		if (c.head_dim / 2 > 1024) return fail(ErrorUnsupported, "head_dim");
		if (c.ple_dim % 8 || c.ple_dim > 1024) return fail(ErrorUnsupported, "ple_dim must be a multiple of 8, at most 1024");
		if (!(c.final_softcap >= 0.0f)) return fail(ErrorBadConfig, "final_softcap");
	} else if (c.ple_dim || c.final_softcap != 0.0f) {
		return fail(ErrorBadConfig, "ple_dim and final_softcap belong to Gemma-style models");
	}
	if ((c.n_heads / c.n_kv_heads) * c.head_dim > (u32)(kAttnThreads * kAttnMaxAcc))
		return fail(ErrorUnsupported, "GQA group x head_dim above %d", kAttnThreads * kAttnMaxAcc);
	const u32 max_k = c.dtype == InfBF16 ? 16384 : 8192; // one 16-byte unit per consumer lane and 4 per row
	if (c.dim > max_k || c.ffn_dim / tp > max_k || (c.n_heads / tp) * c.head_dim > max_k)
		return fail(ErrorUnsupported, "dim, ffn_dim or heads*head_dim above %u", max_k);
	if (tp > (u32)kTpMax) return fail(ErrorUnsupported, "tp_size above %d", kTpMax);
	if (!(c.norm_eps >= 0.0f) || !(c.rope_theta > 0.0f)) return fail(ErrorBadConfig, "eps/theta");
	return Success;
}

struct Pusher {
	DevArena* a;
	Error_t err = Success;
	template <typename P>
	void push(P** out, u64 bytes)
	{
		if (err != Success) return;
		void* p = nullptr;
		err = arena_dev_push(a, bytes, &p);
		*out = (P*)p;
	}
};

template <typename T>
Error_t synth(InfEngine* e, void* dst, u64 rows, u64 cols, SynthArgs a)
{
	a.dst = dst;
	a.rows = rows;
	a.cols = cols;
	const u64 n = rows * cols;
	const int grid = (int)std::min<u64>((n + 255) / 256, (u64)e->sm_count * 16);
	k_synth<T><<<grid, 256, 0, e->stream>>>(a);
	INF_CUDA_TRY(cudaGetLastError());
	return Success;
}

template <typename T>
Error_t generate_weights(InfEngine* e, u64 seed)
{
	const InfConfig& c = e->cfg;
	const u64 d = c.dim, hd = c.head_dim;
	const u32 rk = c.tp_rank;
	const float scale = synth_scale(c.init_std);
	auto base = [&](int layer, uint32_t kind) {
		SynthArgs a;
		memset(&a, 0, sizeof a);
		a.key[0] = stream_key(seed, tensor_stream(layer, kind));
		a.scale = scale;
		a.map = kMapPlain;
		return a;
	};
	// norm gains: 1.0 for Llama; Gemma-style models scale by (1 + w), so their w are drawn
	auto norm = [&](int layer, uint32_t kind, void* dst, u64 n) {
		SynthArgs a = base(layer, kind);
		a.ones = e->gemma ? 0 : 1;
		a.canon_cols = n;
		return synth<T>(e, dst, 1, n, a);
	};
	// embedding: full table on every rank; LM head: vocab rows split across ranks (the
	// embedding itself for Gemma-style models)
	{
		SynthArgs a = base(-1, kEmbed);
		a.canon_cols = d;
		INF_TRY(synth<T>(e, e->embed, c.vocab_size, d, a));
	}
	if (!e->gemma) {
		SynthArgs a = base(-1, kLmHead);
		a.canon_cols = d;
		a.row_offset = (u64)rk * e->Vl;
		INF_TRY(synth<T>(e, e->lm_head, e->Vl, d, a));
	}
	INF_TRY(norm(-1, kFinalNorm, e->final_norm, d));
	const u64 P = c.ple_dim;
	if (e->gemma && P) {
		SynthArgs a = base(-1, kEmbedPle);
		a.canon_cols = c.n_layers * P;
		INF_TRY(synth<T>(e, e->embed_ple, c.vocab_size, c.n_layers * P, a));
		a = base(-1, kPleModelProj);
		a.canon_cols = d;
		INF_TRY(synth<T>(e, e->ple_model_proj, c.n_layers * P, d, a));
		INF_TRY(norm(-1, kPleProjNorm, e->ple_proj_norm, P));
	}
	for (u32 l = 0; l < c.n_layers; ++l) {
		const LayerW& L = e->layers[l];
		{
			SynthArgs a = base((int)l, kWq);
			a.map = kMapQkv;
			a.key[1] = stream_key(seed, tensor_stream((int)l, kWk));
			a.key[2] = stream_key(seed, tensor_stream((int)l, kWv));
			a.canon_cols = d;
			a.head_dim = (int)hd;
			a.n_q_heads = e->Hl;
			a.n_kv_heads = e->KVl;
			a.q_head0 = (int)rk * e->Hl;
			a.kv_head0 = (int)rk * e->KVl;
			INF_TRY(synth<T>(e, L.wqkv, (u64)(e->Hl + 2 * e->KVl) * hd, d, a));
		}
		{
			SynthArgs a = base((int)l, kWo); // columns split across ranks (row-parallel)
			a.canon_cols = (u64)c.n_heads * hd;
			a.col_offset = (u64)rk * e->Hl * hd;
			INF_TRY(synth<T>(e, L.wo, d, (u64)e->Hl * hd, a));
		}
		{
			SynthArgs a = base((int)l, kWgate);
			a.map = kMapGateUp;
			a.key[1] = stream_key(seed, tensor_stream((int)l, kWup));
			a.canon_cols = d;
			a.row_offset = (u64)rk * e->Fl;
			INF_TRY(synth<T>(e, L.wgu, 2 * (u64)e->Fl, d, a));
		}
		{
			SynthArgs a = base((int)l, kWdown);
			a.canon_cols = c.ffn_dim;
			a.col_offset = (u64)rk * e->Fl;
			INF_TRY(synth<T>(e, L.wd, d, e->Fl, a));
		}
		if (e->gemma) {
			INF_TRY(norm((int)l, kAttnNorm, L.attn_norm, d));
			INF_TRY(norm((int)l, kFfnNorm, L.ffn_norm, d));
			INF_TRY(norm((int)l, kQNorm, L.q_norm, hd));
			INF_TRY(norm((int)l, kKNorm, L.k_norm, hd));
			INF_TRY(norm((int)l, kPostAttnNorm, L.post_attn, d));
			INF_TRY(norm((int)l, kPostFfnNorm, L.post_ffn, d));
			if (P) {
				SynthArgs a = base((int)l, kPleGate);
				a.canon_cols = d;
				INF_TRY(synth<T>(e, L.ple_gate, P, d, a));
				a = base((int)l, kPleProj);
				a.canon_cols = P;
				INF_TRY(synth<T>(e, L.ple_proj, d, P, a));
				INF_TRY(norm((int)l, kPlePostNorm, L.ple_post, d));
			}
		} else {
			// both Llama gains are 1.0 (one stream: the values do not depend on it)
			SynthArgs a = base((int)l, kAttnNorm);
			a.ones = 1;
			a.canon_cols = d;
			INF_TRY(synth<T>(e, L.attn_norm, 1, d, a));
			INF_TRY(synth<T>(e, L.ffn_norm, 1, d, a));
		}
	}
	return Success;
}

void rope_tables(const InfConfig& c, std::vector<float>& cs, std::vector<float>& sn)
{
	const u32 half = c.head_dim / 2;
	cs.resize((size_t)c.max_seq * half);
	sn.resize(cs.size());
	for (u32 p = 0; p < c.max_seq; ++p)
		for (u32 i = 0; i < half; ++i) {
			const double inv_freq = std::pow((double)c.rope_theta, -2.0 * (double)i / (double)c.head_dim);
			const double ang = (double)p * inv_freq;
			cs[(size_t)p * half + i] = (float)std::cos(ang);
			sn[(size_t)p * half + i] = (float)std::sin(ang);
		}
}

Error_t engine_build(InfEngine* e, u64 seed, const Checkpoint* ck)
{
	InfConfig& c = e->cfg;
	if (c.kv_block == 0) c.kv_block = 16;
	if (c.tp_size == 0) c.tp_size = 1;
	INF_TRY(validate(c));
	if (ck) INF_TRY(checkpoint_check(*ck, c)); // every tensor present, dtypes and shapes, before the device is touched
	INF_CUDA_TRY(cudaGetDevice(&e->device));
	INF_CUDA_TRY(cudaDeviceGetAttribute(&e->sm_count, cudaDevAttrMultiProcessorCount, e->device));
	INF_CUDA_TRY(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
	INF_CUDA_TRY(cudaEventCreate(&e->prof_ev[0]));
	INF_CUDA_TRY(cudaEventCreate(&e->prof_ev[1]));
	e->esz = c.dtype == InfBF16 ? 2 : 4;
	e->gemma = c.arch == InfArchGemma;
	const u32 tp = c.tp_size;
	e->Hl = (int)(c.n_heads / tp);
	e->KVl = (int)(c.n_kv_heads / tp);
	e->Fl = (int)(c.ffn_dim / tp);
	e->Vl = (int)(c.vocab_size / tp);
	const u64 d = c.dim, hd = c.head_dim, es = e->esz, L = c.n_layers;
	e->pages_per_seq = (int)((c.max_seq + c.kv_block - 1) / c.kv_block);
	e->n_pages = c.kv_pages ? (int)c.kv_pages : (int)(c.max_batch * (u32)e->pages_per_seq);
	e->max_out = (int)c.max_seq;
	const int G = e->Hl / e->KVl;
	// split-K attention at batch 1: about one CTA per SM over the KV heads, each split within
	// the shared-memory budget; batches stream their pages (a few CTAs per SM over the batch)
	attn_decode_plan(e->sm_count, e->KVl, 1, e->pages_per_seq, (int)c.kv_block, (int)hd, e->esz, &e->attn_splits,
	                 &e->attn_max_pages_split);
	e->attn_splits_batch = attn_stream_splits(e->sm_count, e->KVl, (int)c.max_batch, e->pages_per_seq);
	e->attn_max_pages_split_batch = 0;
	e->attn_unit_splits = std::min(kAmUnitSplitsMax, (e->pages_per_seq + kAmUnitPagesMin - 1) / kAmUnitPagesMin);
	// batch-1 decode: one cluster per KV head when the longest context fits its shared memory
	// and the GPU can place a cluster of that size
	INF_TRY(attn_cl_choose(e, G, (int)hd));
	e->pf_tc = c.dtype == InfBF16 && c.prefill_attention == InfPrefillAttnAuto && (hd == 64 || hd == 128) &&
	           kPtRows % G == 0 && c.kv_block % 8 == 0 && kPtKeys % c.kv_block == 0;
	const u64 part_floats =
	    std::max((u64)e->Hl * e->attn_splits, (u64)c.max_batch * e->Hl * std::max(e->attn_splits_batch, e->attn_unit_splits)) *
	    (hd + 2);
	// multi-token passes run on the tensor cores (bf16 Llama models); fp32 and Gemma-style models
	// feed tokens one by one through the decode step
	e->chunk = c.dtype == InfBF16 && !e->gemma
	               ? (int)(c.prefill_chunk ? std::min(c.prefill_chunk, c.max_seq) : std::min(c.max_seq, 4096u))
	               : 0;

	// ---- sizes
	const u64 w_layer = ((u64)(e->Hl + 2 * e->KVl) * hd * d + d * e->Hl * hd + 2ull * e->Fl * d + d * e->Fl + 2 * d) * es;
	const u64 pl = c.ple_dim;
	const u64 w_gemma_layer = e->gemma ? (2 * hd + 3 * d + 2 * pl * d) * es + 6 * 256 : 0;
	const u64 w_gemma = e->gemma ? ((u64)c.vocab_size * L * pl + L * pl * d + pl) * es + 3 * 256 : 0;
	// embed is full, LM head is a shard (Gemma: the embedding is the LM head)
	const u64 w_total = ((e->gemma ? 1ull : 2ull) * c.vocab_size * d) * es + d * es + L * (w_layer + w_gemma_layer) + w_gemma;
	const u64 page_elems = (u64)e->KVl * c.kv_block * hd;
	const u64 kv_total = 2ull * L * e->n_pages * page_elems * es;
	const u64 comm = c.tp_size > 1 ? (2ull * c.tp_size * d * 8 + 2ull * c.tp_size * kTpMaxCtas * 4 + 64ull * c.tp_size +
	                                   (e->chunk > 0 ? 2ull * (u64)(c.prefill_chunk ? c.prefill_chunk : 4096) * d * 4 : 0) + 8 * 256)
	                                : 0;
	const u64 batch_bufs = c.max_batch > 1 ? (u64)c.max_batch * ((u64)e->Vl * 4 + 4 + 8) + 768 : 0;
	const u64 act = comm + batch_bufs + (c.dtype == InfBF16 ? kGemmPartBytes + 256 : 0) + d * 4 + (u64)e->Hl * hd * es * 2 + (u64)e->Fl * es + (u64)e->Vl * 4 + part_floats * 4 +
	                (u64)e->chunk * (d * 4 + d * es + 2ull * e->Hl * hd * es + (u64)e->Fl * es + 8) + 16 * 256;
	const u64 gemma_act = e->gemma ? (d * 4 + std::max<u64>((u64)(e->Hl + 2 * e->KVl) * hd, d) * 4 + d * 4 + d * es +
	                                  L * pl * 4 + L * pl * es + pl * es + 8 * 256)
	                               : 0;
	const u64 slack = (u64)(64 + 16 * L) * 256 + 64ull * 1024 * 1024 + gemma_act;
	const u64 total = w_total + kv_total + act + (u64)c.max_seq * hd * 4 + (u64)c.max_batch * e->pages_per_seq * 4 +
	                  (u64)c.max_seq * 8 + slack;

	if (!e->ctx) INF_TRY(exec_ctx_create(&e->ctx));
	INF_TRY(arena_dev_create(&e->ctx->dev_arena, total));
	Pusher P{&e->ctx->dev_arena};
	const u64 w_begin = arena_dev_pos_get(&e->ctx->dev_arena);
	P.push(&e->embed, (u64)c.vocab_size * d * es);
	if (e->gemma && c.ple_dim) {
		P.push(&e->embed_ple, (u64)c.vocab_size * L * c.ple_dim * es);
		P.push(&e->ple_model_proj, (u64)L * c.ple_dim * d * es);
		P.push(&e->ple_proj_norm, (u64)c.ple_dim * es);
	}
	e->layers.resize(L);
	for (u32 l = 0; l < L; ++l) {
		LayerW& Ly = e->layers[l];
		P.push(&Ly.wqkv, (u64)(e->Hl + 2 * e->KVl) * hd * d * es);
		P.push(&Ly.wo, d * e->Hl * hd * es);
		P.push(&Ly.wgu, 2ull * e->Fl * d * es);
		P.push(&Ly.wd, d * e->Fl * es);
		P.push(&Ly.attn_norm, d * es);
		P.push(&Ly.ffn_norm, d * es);
		if (e->gemma) {
			P.push(&Ly.q_norm, hd * es);
			P.push(&Ly.k_norm, hd * es);
			P.push(&Ly.post_attn, d * es);
			P.push(&Ly.post_ffn, d * es);
			if (c.ple_dim) {
				P.push(&Ly.ple_gate, (u64)c.ple_dim * d * es);
				P.push(&Ly.ple_proj, d * c.ple_dim * es);
				P.push(&Ly.ple_post, d * es);
			}
		}
	}
	P.push(&e->final_norm, d * es);
	if (e->gemma) e->lm_head = e->embed;
	else P.push(&e->lm_head, (u64)e->Vl * d * es);
	e->weight_bytes = arena_dev_pos_get(&e->ctx->dev_arena) - w_begin;
	P.push(&e->rope_cos, (u64)c.max_seq * (hd / 2) * 4);
	P.push(&e->rope_sin, (u64)c.max_seq * (hd / 2) * 4);
	for (u32 l = 0; l < L; ++l) {
		P.push(&e->layers[l].kpool, e->n_pages * page_elems * es);
		P.push(&e->layers[l].vpool, e->n_pages * page_elems * es);
	}
	P.push(&e->block_table, (u64)c.max_batch * e->pages_per_seq * 4);
	P.push(&e->resid, d * 4);
	P.push(&e->q, (u64)e->Hl * hd * es);
	P.push(&e->attn, (u64)e->Hl * hd * es);
	P.push(&e->h, (u64)e->Fl * es);
	P.push(&e->logits, (u64)e->Vl * 4);
	P.push(&e->ctl, kCtlWords * sizeof(int));
	P.push(&e->best, 16);
	P.push(&e->lm_counter, 16);
	P.push(&e->sample_q, (u64)e->Vl * 4);
	P.push(&e->rows_d, (u64)c.max_batch * sizeof(SampleRow));
	P.push(&e->sample_q_rows, (u64)c.max_batch * e->Vl * 4);
	P.push(&e->out_ids, (u64)e->max_out * 4);
	P.push(&e->d_ids, (u64)c.max_seq * 4);
	P.push(&e->attn_part, part_floats * 4);
	P.push(&e->attn_counters, (u64)c.max_batch * e->KVl * 4);
	P.push(&e->attn_units, (u64)c.max_batch * e->attn_unit_splits * 8);
	if (c.dtype == InfBF16) {
		e->gemm_part_bytes = kGemmPartBytes;
		P.push(&e->gemm_part, kGemmPartBytes);
	}
	if (e->gemma) {
		P.push(&e->resid2, d * 4);
		P.push(&e->raw, std::max<u64>((u64)(e->Hl + 2 * e->KVl) * hd, d) * 4);
		P.push(&e->pend, d * 4);
		P.push(&e->xb, d * es);
		if (c.ple_dim) {
			P.push(&e->pm, (u64)L * c.ple_dim * 4);
			P.push(&e->ple, (u64)L * c.ple_dim * es);
			P.push(&e->ple_y, (u64)c.ple_dim * es);
		}
	}
	if (c.max_batch > 1) {
		P.push(&e->logits_p, (u64)c.max_batch * e->Vl * 4);
		P.push(&e->argmax_p, (u64)c.max_batch * 4);
		P.push(&e->batch_keys, (u64)c.max_batch * 8);
	}
	if (e->chunk > 0) {
		P.push(&e->resid_p, (u64)e->chunk * d * 4);
		P.push(&e->xhat_p, (u64)e->chunk * d * es);
		P.push(&e->q_p, (u64)e->chunk * e->Hl * hd * es);
		P.push(&e->attn_p, (u64)e->chunk * e->Hl * hd * es);
		P.push(&e->h_p, (u64)e->chunk * e->Fl * es);
		P.push(&e->tok_pos, (u64)e->chunk * 4);
		P.push(&e->tok_slot, (u64)e->chunk * 4);
	}
	if (c.tp_size > 1) {
		// peer-visible region, same offsets on every rank (identical shapes, deterministic layout)
		e->comm_off = arena_dev_pos_get(&e->ctx->dev_arena);
		TpComm& t = e->tpc;
		memset(&t, 0, sizeof t);
		t.rank = (int)c.tp_rank;
		t.size = 1; // becomes tp_size in inf_tp_connect
		t.dim = (int)d;
		const int r = (int)c.tp_rank, N = (int)c.tp_size;
		P.push(&t.inbox[r], 2ull * N * d * 8);
		P.push(&t.am_inbox[r], 2ull * N * 8);
		P.push(&t.am_flags[r], (u64)N * 4);
		P.push(&t.ready[r], (u64)N * 4);
		P.push(&t.done[r], (u64)N * kTpMaxCtas * 4);
		if (e->chunk > 0) {
			P.push(&t.part[r], (u64)e->chunk * d * 4);
			P.push(&t.red[r], (u64)e->chunk * d * 4);
		}
	}
	if (P.err != Success) return P.err;
	e->cur_id = reinterpret_cast<uint32_t*>(e->ctl + kCtlId);
	e->pos = e->ctl + kCtlPos;
	e->slot = e->ctl + kCtlSlot;
	e->step = reinterpret_cast<uint32_t*>(e->ctl + kCtlStep);
	e->err = e->ctl + kCtlErr;
	e->tpc.epoch = reinterpret_cast<const uint32_t*>(e->ctl + kCtlEpoch);
	if (c.tp_size <= 1) {
		e->tpc.size = 1;
		e->tpc.rank = 0;
	}

	INF_CUDA_TRY(cudaMemsetAsync(e->ctx->dev_arena._d_ptr + w_begin + e->weight_bytes, 0,
	                             arena_dev_pos_get(&e->ctx->dev_arena) - w_begin - e->weight_bytes, e->stream));
	if (ck) {
		std::vector<WeightDst> w;
		w.push_back({0, InfWEmbed, e->embed});
		for (u32 l = 0; l < L; ++l) {
			const LayerW& Ly = e->layers[l];
			const int li = (int)l;
			w.push_back({li, InfWQkv, Ly.wqkv});
			w.push_back({li, InfWO, Ly.wo});
			w.push_back({li, InfWGateUp, Ly.wgu});
			w.push_back({li, InfWDown, Ly.wd});
			w.push_back({li, InfWAttnNorm, Ly.attn_norm});
			w.push_back({li, InfWFfnNorm, Ly.ffn_norm});
		}
		w.push_back({0, InfWFinalNorm, e->final_norm});
		if (!e->gemma) w.push_back({0, InfWLmHead, e->lm_head}); // Gemma: the embedding
		if (e->gemma) {
			for (u32 l = 0; l < L; ++l) {
				const LayerW& Ly = e->layers[l];
				const int li = (int)l;
				w.push_back({li, InfWQNorm, Ly.q_norm});
				w.push_back({li, InfWKNorm, Ly.k_norm});
				w.push_back({li, InfWPostAttnNorm, Ly.post_attn});
				w.push_back({li, InfWPostFfnNorm, Ly.post_ffn});
				if (c.ple_dim) {
					w.push_back({li, InfWPleGate, Ly.ple_gate});
					w.push_back({li, InfWPleProj, Ly.ple_proj});
					w.push_back({li, InfWPlePostNorm, Ly.ple_post});
				}
			}
			if (c.ple_dim) {
				w.push_back({0, InfWEmbedPle, e->embed_ple});
				w.push_back({0, InfWPleModelProj, e->ple_model_proj});
				w.push_back({0, InfWPleProjNorm, e->ple_proj_norm});
			}
		}
		INF_TRY(checkpoint_upload(*ck, c, w, e->stream));
	} else if (c.dtype == InfBF16) {
		INF_TRY(generate_weights<bf16>(e, seed));
	} else {
		INF_TRY(generate_weights<float>(e, seed));
	}

	std::vector<float> cs, sn;
	rope_tables(c, cs, sn);
	INF_CUDA_TRY(cudaMemcpyAsync(e->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, e->stream));
	INF_CUDA_TRY(cudaMemcpyAsync(e->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, e->stream));
	e->h_block_table.assign((size_t)c.max_batch * e->pages_per_seq, -1);
	INF_CUDA_TRY(cudaMemcpyAsync(e->block_table, e->h_block_table.data(), e->h_block_table.size() * 4,
	                             cudaMemcpyHostToDevice, e->stream));
	e->seq_pages.assign(c.max_batch, {});
	e->free_pages.clear();
	for (int p = e->n_pages - 1; p >= 0; --p) e->free_pages.push_back(p);
	INF_CUDA_TRY(cudaMallocHost(&e->h_pin, sizeof(uint32_t) * (c.max_seq + 16)));
	INF_CUDA_TRY(cudaMallocHost(&e->h_ctl, sizeof(int) * 2 * kCtlWords));
	if (e->chunk > 0) INF_CUDA_TRY(cudaMallocHost(&e->h_tok, sizeof(int) * 2 * e->chunk));
	INF_CUDA_TRY(cudaMallocHost(&e->h_units, (size_t)c.max_batch * e->attn_unit_splits * 8));
	INF_CUDA_TRY(cudaMallocHost(&e->rows_h, sizeof(SampleRow) * c.max_batch));
	e->slot_samp.assign(c.max_batch, InfSampling{});
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	INF_TRY(build_decode_graph(e));
	return Success;
}

void engine_free(InfEngine* e)
{
	if (!e) return;
	if (e->stream) cudaStreamSynchronize(e->stream);
	if (e->decode_exec) cudaGraphExecDestroy(e->decode_exec);
	for (void* p : e->peer_bases)
		if (p) cudaIpcCloseMemHandle(p);
	if (e->h_pin) cudaFreeHost(e->h_pin);
	if (e->h_ctl) cudaFreeHost(e->h_ctl);
	if (e->h_tok) cudaFreeHost(e->h_tok);
	if (e->rows_h) cudaFreeHost(e->rows_h);
	if (e->h_units) cudaFreeHost(e->h_units);
	for (auto& ev : e->prof_ev)
		if (ev) cudaEventDestroy(ev);
	if (e->stream) cudaStreamDestroy(e->stream);
	delete e;
}

Error_t copy_in_ids(InfEngine* e, const u32* ids, u32 n)
{
	if (is_device_ptr(ids)) {
		INF_CUDA_TRY(cudaMemcpyAsync(e->d_ids, ids, (size_t)n * 4, cudaMemcpyDeviceToDevice, e->stream));
	} else {
		for (u32 i = 0; i < n; ++i)
			if (ids[i] >= e->cfg.vocab_size) return fail(ErrorTokenOutOfRange, "id %u at %u >= vocab %u", ids[i], i, e->cfg.vocab_size);
		INF_CUDA_TRY(cudaStreamSynchronize(e->stream)); // h_pin may still feed an earlier copy
		memcpy(e->h_pin, ids, (size_t)n * 4);
		INF_CUDA_TRY(cudaMemcpyAsync(e->d_ids, e->h_pin, (size_t)n * 4, cudaMemcpyHostToDevice, e->stream));
	}
	return Success;
}

Error_t set_scalars(InfEngine* e, int slot, int pos)
{
	int v[2] = {slot, pos};
	INF_CUDA_TRY(cudaMemcpyAsync(e->slot, &v[0], 4, cudaMemcpyHostToDevice, e->stream));
	INF_CUDA_TRY(cudaMemcpyAsync(e->pos, &v[1], 4, cudaMemcpyHostToDevice, e->stream));
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	return Success;
}

// Feeds ids[0..n) (already in d_ids) through the decode graph at consecutive positions.
Error_t run_tokens(InfEngine* e, u32 n)
{
	for (u32 t = 0; t < n; ++t) {
		INF_CUDA_TRY(cudaMemcpyAsync(e->cur_id, e->d_ids + t, 4, cudaMemcpyDeviceToDevice, e->stream));
		INF_TRY(launch_decode_graph(e));
	}
	return Success;
}

Error_t copy_out(InfEngine* e, void* dst, const void* src, size_t bytes)
{
	const cudaMemcpyKind k = is_device_ptr(dst) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
	INF_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, k, e->stream));
	return Success;
}

// One host token: one 12-byte H2D of (id, pos, slot) from pinned memory, one graph launch,
// one 20-byte D2H of (argmax, ..., err) -- the per-token cost of the public API.
Error_t forward_one(InfEngine* e, u32 id, u32 pos, u32 slot, f32* logits_out, u32* argmax_out)
{
	if (id >= e->cfg.vocab_size) return fail(ErrorTokenOutOfRange, "id %u >= vocab %u", id, e->cfg.vocab_size);
	int* in = e->h_ctl;
	int* out = e->h_ctl + kCtlWords;
	in[kCtlId] = (int)id;
	in[kCtlPos] = (int)pos;
	in[kCtlSlot] = (int)slot;
	INF_CUDA_TRY(cudaMemcpyAsync(e->ctl, in, 3 * sizeof(int), cudaMemcpyHostToDevice, e->stream));
	INF_TRY(launch_decode_graph(e));
	INF_CUDA_TRY(cudaMemcpyAsync(out, e->ctl, (kCtlErr + 1) * sizeof(int), cudaMemcpyDeviceToHost, e->stream));
	if (logits_out) INF_TRY(copy_out(e, logits_out, e->logits, sizeof(float) * e->Vl));
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	if (out[kCtlErr] != kDevOk) {
		INF_CUDA_TRY(cudaMemsetAsync(e->err, 0, sizeof(int), e->stream));
		INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
		return map_dev_err(out[kCtlErr]);
	}
	if (argmax_out) {
		if (is_device_ptr(argmax_out)) INF_CUDA_TRY(cudaMemcpy(argmax_out, &out[kCtlId], 4, cudaMemcpyHostToDevice));
		else *argmax_out = (u32)out[kCtlId];
	}
	return Success;
}

} // namespace

// =============================================================================== C ABI
bool inf::model_sampling_on(const Model* m) { return m && m->engine && m->engine->sampling; }

extern "C" {

Error_t inf_config_preset(u32 preset, InfConfig* out)
{
	if (!out) return fail(ErrorInvalidValue, "inf_config_preset: NULL");
	InfConfig c;
	memset(&c, 0, sizeof c);
	c.kv_block = 16;
	c.max_batch = 1;
	c.norm_eps = 1e-5f;
	c.init_std = 0.02f;
	c.tp_size = 1;
	switch (preset) {
	case 1:
		c.vocab_size = 32000; c.dim = 288; c.n_layers = 6; c.n_heads = 6; c.n_kv_heads = 6; c.head_dim = 48;
		c.ffn_dim = 768; c.max_seq = 256; c.dtype = InfF32; c.rope_theta = 10000.0f;
		break;
	case 2:
		c.vocab_size = 32000; c.dim = 2048; c.n_layers = 22; c.n_heads = 32; c.n_kv_heads = 4; c.head_dim = 64;
		c.ffn_dim = 5632; c.max_seq = 1024; c.dtype = InfBF16; c.rope_theta = 10000.0f;
		break;
	case 3: case 4: case 5:
		c.vocab_size = 128256; c.dim = 4096; c.n_layers = 32; c.n_heads = 32; c.n_kv_heads = 8; c.head_dim = 128;
		c.ffn_dim = 14336; c.dtype = InfBF16; c.rope_theta = 500000.0f;
		c.max_seq = preset == 3 ? 3072 : preset == 4 ? 4352 : 32896;
		c.max_batch = preset == 4 ? 64 : 1;
		break;
	case 6: // the Gemma-4-E2B shape of the reference's comments (src/model.cuh:9-14)
		c.arch = InfArchGemma;
		c.vocab_size = 262144; c.dim = 1536; c.n_layers = 35; c.n_heads = 8; c.n_kv_heads = 2; c.head_dim = 512;
		c.ffn_dim = 6144; c.ple_dim = 256; c.max_seq = 4096; c.dtype = InfBF16; c.rope_theta = 1000000.0f;
		c.norm_eps = 1e-6f; c.final_softcap = 30.0f;
		break;
	default:
		return fail(ErrorInvalidValue, "unknown preset %u", preset);
	}
	*out = c;
	return Success;
}

Error_t inf_model_build(ExecCtx** ctx, Model* model, const InfConfig* config, const char* weights_path, u64 seed)
{
	if (!ctx || !model || !config) return fail(ErrorInvalidValue, "inf_model_build: NULL argument");
	std::unique_ptr<Checkpoint> ck;
	if (weights_path) { // opened and indexed before any device work
		ck.reset(new (std::nothrow) Checkpoint());
		if (!ck) return fail(ErrorMemoryAllocation, "checkpoint");
		INF_TRY(checkpoint_open(weights_path, ck.get()));
	}
	InfEngine* e = new (std::nothrow) InfEngine();
	if (!e) return fail(ErrorMemoryAllocation, "engine");
	e->cfg = *config;
	e->ctx = *ctx;
	Error_t r = engine_build(e, seed, ck.get());
	if (r != Success) {
		ExecCtx* c = e->ctx;
		engine_free(e);
		if (c && !*ctx) exec_ctx_destroy(&c); // created here: undo
		else if (c && c->dev_arena._d_ptr) arena_dev_destroy(&c->dev_arena);
		return r;
	}
	*ctx = e->ctx;
	model->config = e->cfg;
	model->data = e->embed;
	model->model_bsize = e->weight_bytes;
	model->engine = e;
	return Success;
}

Error_t inf_config_from_json(const char* config_path, InfConfig* inout) { return config_from_json(config_path, inout); }

// the config as engine_build sees it: defaults filled in, shape rules checked
static Error_t checkpoint_config(const InfConfig* config, InfConfig* c)
{
	if (!config) return fail(ErrorInvalidValue, "NULL config");
	*c = *config;
	if (c->kv_block == 0) c->kv_block = 16;
	if (c->tp_size == 0) c->tp_size = 1;
	return validate(*c);
}

Error_t inf_safetensors_check(const char* weights_path, const InfConfig* config)
{
	InfConfig c;
	INF_TRY(checkpoint_config(config, &c));
	Checkpoint ck;
	INF_TRY(checkpoint_open(weights_path, &ck));
	return checkpoint_check(ck, c);
}

Error_t inf_safetensors_read(const char* weights_path, const InfConfig* config, u32 layer, u32 kind, void* out, u64 out_bytes)
{
	InfConfig c;
	INF_TRY(checkpoint_config(config, &c));
	if (!out) return fail(ErrorInvalidValue, "inf_safetensors_read: NULL out");
	const bool per_layer = kind != InfWEmbed && kind != InfWLmHead && kind != InfWFinalNorm && kind != InfWEmbedPle &&
	                       kind != InfWPleModelProj && kind != InfWPleProjNorm;
	if (per_layer && layer >= c.n_layers) return fail(ErrorInvalidValue, "layer %u of %u", layer, c.n_layers);
	u64 rows, cols;
	weight_dims(c, kind, &rows, &cols);
	const u64 need = rows * cols * (c.dtype == InfBF16 ? 2 : 4);
	if (out_bytes < need) return fail(ErrorInvalidValue, "out holds %llu bytes, the weight needs %llu", (unsigned long long)out_bytes, (unsigned long long)need);
	Checkpoint ck;
	INF_TRY(checkpoint_open(weights_path, &ck));
	return weight_rows_parallel(ck, c, per_layer ? (int)layer : 0, kind, 0, rows, out);
}

Error_t inf_model_destroy(ExecCtx** ctx, Model* model)
{
	if (!model || !model->engine) return fail(ErrorInvalidValue, "inf_model_destroy: no model");
	engine_free(model->engine);
	model->engine = nullptr;
	model->data = nullptr;
	if (ctx && *ctx) return exec_ctx_destroy(ctx);
	return Success;
}

Error_t inf_forward(Model* model, const u32* ids, u32 n_tokens, u32 start_pos, u32 seq_slot, f32* logits_out,
                    u32* argmax_out)
{
	if (!model || !model->engine || !ids || n_tokens == 0) return fail(ErrorInvalidValue, "inf_forward: bad arguments");
	InfEngine* e = model->engine;
	if (seq_slot >= e->cfg.max_batch) return fail(ErrorInvalidValue, "slot %u >= max_batch", seq_slot);
	if ((u64)start_pos + n_tokens > e->cfg.max_seq) return fail(ErrorKvOutOfRange, "positions beyond max_seq");
	INF_TRY(ensure_pages(e, seq_slot, start_pos + n_tokens));
	if (n_tokens == 1 && !is_device_ptr(ids)) return forward_one(e, ids[0], start_pos, seq_slot, logits_out, argmax_out);
	INF_TRY(copy_in_ids(e, ids, n_tokens));
	if (use_tc_prefill(e, n_tokens)) INF_TRY(run_prefill(e, n_tokens, start_pos, seq_slot));
	else {
		INF_TRY(set_scalars(e, (int)seq_slot, (int)start_pos));
		INF_TRY(run_tokens(e, n_tokens));
	}
	if (logits_out) INF_TRY(copy_out(e, logits_out, e->logits, sizeof(float) * e->Vl));
	if (argmax_out) INF_TRY(copy_out(e, argmax_out, e->cur_id, 4));
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	return check_dev_err(e);
}

Error_t inf_forward_batch(Model* model, u32 n_seqs, const u32* seq_slots, const u32* ids, const u32* positions,
                          f32* logits_out, u32* argmax_out)
{
	return forward_batch(model, n_seqs, seq_slots, ids, positions, logits_out, argmax_out, false);
}

} // extern "C"

Error_t inf::forward_batch(Model* model, u32 n_seqs, const u32* seq_slots, const u32* ids, const u32* positions,
                           f32* logits_out, u32* argmax_out, bool single_batched)
{
	if (!model || !model->engine || !seq_slots || !ids || !positions || n_seqs == 0)
		return fail(ErrorInvalidValue, "inf_forward_batch: bad arguments");
	InfEngine* e = model->engine;
	const InfConfig& c = e->cfg;
	const bool host_args = !is_device_ptr(seq_slots) && !is_device_ptr(ids) && !is_device_ptr(positions);
	const bool batched = host_args && c.dtype == InfBF16 && c.tp_size <= 1 && (n_seqs > 1 || single_batched) &&
	                     n_seqs <= c.max_batch && (int)n_seqs <= e->chunk && e->logits_p;
	if (!batched) {
		for (u32 i = 0; i < n_seqs; ++i) {
			f32* lo = logits_out ? logits_out + (size_t)i * e->Vl : nullptr;
			u32* am = argmax_out ? argmax_out + i : nullptr;
			const bool samp = host_args && seq_slots[i] < c.max_batch && e->slot_samp[seq_slots[i]].temperature > 0.0f;
			if (!samp) {
				INF_TRY(inf_forward(model, ids + i, 1, positions[i], seq_slots[i], lo, am));
				continue;
			}
			u32 id = 0;
			INF_TRY(inf_forward(model, ids + i, 1, positions[i], seq_slots[i], lo, &id));
			INF_TRY(sample_slot_token(model, seq_slots[i], positions[i] + 1, &id));
			if (am) {
				if (is_device_ptr(am)) INF_CUDA_TRY(cudaMemcpy(am, &id, 4, cudaMemcpyHostToDevice));
				else *am = id;
			}
		}
		return Success;
	}
	std::vector<char> seen(c.max_batch, 0);
	for (u32 i = 0; i < n_seqs; ++i) {
		if (seq_slots[i] >= c.max_batch) return fail(ErrorInvalidValue, "slot %u >= max_batch", seq_slots[i]);
		if (seen[seq_slots[i]]++) return fail(ErrorInvalidValue, "slot %u appears twice in one batch", seq_slots[i]);
		if (positions[i] >= c.max_seq) return fail(ErrorKvOutOfRange, "position %u beyond max_seq", positions[i]);
		if (ids[i] >= c.vocab_size) return fail(ErrorTokenOutOfRange, "id %u >= vocab %u", ids[i], c.vocab_size);
	}
	for (u32 i = 0; i < n_seqs; ++i) INF_TRY(ensure_pages(e, seq_slots[i], positions[i] + 1));
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream)); // pinned staging reuse
	for (u32 i = 0; i < n_seqs; ++i) {
		e->h_pin[i] = ids[i];
		e->h_tok[i] = (int)positions[i];
		e->h_tok[e->chunk + i] = (int)seq_slots[i];
	}
	INF_CUDA_TRY(cudaMemcpyAsync(e->d_ids, e->h_pin, sizeof(u32) * n_seqs, cudaMemcpyHostToDevice, e->stream));
	INF_CUDA_TRY(cudaMemcpyAsync(e->tok_pos, e->h_tok, sizeof(int) * n_seqs, cudaMemcpyHostToDevice, e->stream));
	INF_CUDA_TRY(cudaMemcpyAsync(e->tok_slot, e->h_tok + e->chunk, sizeof(int) * n_seqs, cudaMemcpyHostToDevice, e->stream));
	e->h2d_bytes += 12ull * n_seqs;
	e->n_attn_units = 0;
	if (c.kv_block == 16 && attn_decode_mma_kernel(e->Hl / e->KVl, (int)c.head_dim)) {
		e->n_attn_units = build_attn_units(e, positions, n_seqs);
		if (e->n_attn_units > 0) {
			INF_CUDA_TRY(cudaMemcpyAsync(e->attn_units, e->h_units, (size_t)e->n_attn_units * 8, cudaMemcpyHostToDevice,
			                             e->stream));
			e->h2d_bytes += (u64)e->n_attn_units * 8;
		}
	}
	e->gemm_split = true;
	const Error_t eb = enqueue_decode_batch(e, (int)n_seqs);
	e->gemm_split = false;
	e->n_attn_units = 0;
	INF_TRY(eb);
	{
		std::vector<u32> pos_new(positions, positions + n_seqs);
		for (u32& p : pos_new) ++p;
		INF_TRY(enqueue_sample_rows(e, (int)n_seqs, e->logits_p, seq_slots, pos_new.data(), e->argmax_p));
	}
	if (logits_out) INF_TRY(copy_out(e, logits_out, e->logits_p, sizeof(float) * e->Vl * n_seqs));
	if (argmax_out) INF_TRY(copy_out(e, argmax_out, e->argmax_p, sizeof(u32) * n_seqs));
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	return check_dev_err(e);
}

Error_t inf::sample_slot_token(Model* model, u32 slot, u32 pos_new, u32* id)
{
	if (!model || !model->engine || !id) return fail(ErrorInvalidValue, "sample_slot_token: NULL argument");
	InfEngine* e = model->engine;
	if (slot >= e->cfg.max_batch || !(e->slot_samp[slot].temperature > 0.0f)) return Success;
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream)); // the pinned row staging may feed an earlier copy
	// the forward left its logits in e->logits; the drawn id replaces the chosen one in the ctl
	// block as well, so a decode that continues from here feeds it
	*reinterpret_cast<uint32_t*>(e->h_pin) = *id;
	INF_CUDA_TRY(cudaMemcpyAsync(e->cur_id, e->h_pin, 4, cudaMemcpyHostToDevice, e->stream));
	INF_TRY(enqueue_sample_rows(e, 1, e->logits, &slot, &pos_new, e->cur_id));
	INF_CUDA_TRY(cudaMemcpyAsync(e->h_pin, e->cur_id, 4, cudaMemcpyDeviceToHost, e->stream));
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	*id = *reinterpret_cast<uint32_t*>(e->h_pin);
	return check_dev_err(e);
}

extern "C" {

Error_t inf_set_slot_sampling(Model* model, u32 seq_slot, const InfSampling* s)
{
	if (!model || !model->engine || !s) return fail(ErrorInvalidValue, "inf_set_slot_sampling: NULL argument");
	InfEngine* e = model->engine;
	if (seq_slot >= e->cfg.max_batch) return fail(ErrorInvalidValue, "slot %u >= max_batch", seq_slot);
	if (!(s->temperature >= 0.0f) || !std::isfinite(s->temperature)) return fail(ErrorInvalidValue, "temperature %g", (double)s->temperature);
	const bool on = s->temperature > 0.0f; // greedy settings need no top_p
	if (on && !(s->top_p > 0.0f && s->top_p <= 1.0f)) return fail(ErrorInvalidValue, "top_p %g outside (0, 1]", (double)s->top_p);
	if (on && e->cfg.tp_size > 1) return fail(ErrorUnsupported, "sampling with the vocabulary split across ranks");
	if (on && 1.0 / (double)s->temperature > 3.0e38) return fail(ErrorInvalidValue, "temperature %g too small", (double)s->temperature);
	if (on && e->Vl % 4 != 0) return fail(ErrorUnsupported, "per-slot sampling needs vocab_size %% 4 == 0");
	e->slot_samp[seq_slot] = *s;
	return Success;
}

Error_t inf_generate(Model* model, const u32* prompt, u32 n_prompt, u32 n_new, u32* out_ids, InfStats* stats)
{
	if (!model || !model->engine || !prompt || !out_ids || n_prompt == 0 || n_new == 0)
		return fail(ErrorInvalidValue, "inf_generate: bad arguments");
	InfEngine* e = model->engine;
	if ((u64)n_prompt + n_new - 1 > e->cfg.max_seq) return fail(ErrorKvOutOfRange, "prompt + n_new beyond max_seq");
	if (n_new > (u32)e->max_out) return fail(ErrorInvalidValue, "n_new above %d", e->max_out);
	const u64 l0 = e->launches;
	INF_TRY(release_pages(e, 0));
	INF_TRY(ensure_pages(e, 0, n_prompt + n_new - 1));
	INF_TRY(copy_in_ids(e, prompt, n_prompt));
	INF_TRY(set_scalars(e, 0, 0));
	cudaEvent_t ev[3];
	for (auto& x : ev) INF_CUDA_TRY(cudaEventCreate(&x));
	INF_CUDA_TRY(cudaEventRecord(ev[0], e->stream));
	if (use_tc_prefill(e, n_prompt)) {
		INF_CUDA_TRY(cudaMemsetAsync(e->step, 0, 4, e->stream));
		INF_TRY(run_prefill(e, n_prompt, 0, 0)); // writes out_ids[0]
	} else {
		INF_TRY(run_tokens(e, n_prompt - 1));
		INF_CUDA_TRY(cudaMemsetAsync(e->step, 0, 4, e->stream));
		INF_CUDA_TRY(cudaMemcpyAsync(e->cur_id, e->d_ids + (n_prompt - 1), 4, cudaMemcpyDeviceToDevice, e->stream));
		INF_TRY(launch_decode_graph(e));
	}
	INF_CUDA_TRY(cudaEventRecord(ev[1], e->stream));
	for (u32 s = 1; s < n_new; ++s) INF_TRY(launch_decode_graph(e));
	INF_CUDA_TRY(cudaEventRecord(ev[2], e->stream));
	INF_CUDA_TRY(cudaMemcpyAsync(out_ids, e->out_ids, (size_t)n_new * 4,
	                             is_device_ptr(out_ids) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, e->stream));
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	float ms_pre = 0.f, ms_dec = 0.f;
	cudaEventElapsedTime(&ms_pre, ev[0], ev[1]);
	cudaEventElapsedTime(&ms_dec, ev[1], ev[2]);
	for (auto& x : ev) cudaEventDestroy(x);
	if (stats) {
		stats->prefill_ms = ms_pre;
		stats->decode_ms = ms_dec;
		stats->n_prompt = n_prompt;
		stats->n_new = n_new;
		stats->kernel_launches = e->launches - l0;
	}
	return check_dev_err(e);
}

Error_t inf_decode(Model* model, u32 seq_slot, u32 start_pos, u32 first_id, u32 n_steps, u32* out_ids, InfStats* stats)
{
	if (!model || !model->engine || n_steps == 0) return fail(ErrorInvalidValue, "inf_decode: bad arguments");
	InfEngine* e = model->engine;
	if (seq_slot >= e->cfg.max_batch) return fail(ErrorInvalidValue, "slot %u >= max_batch", seq_slot);
	if (first_id >= e->cfg.vocab_size) return fail(ErrorTokenOutOfRange, "id %u", first_id);
	if ((u64)start_pos + n_steps > e->cfg.max_seq) return fail(ErrorKvOutOfRange, "positions beyond max_seq");
	if (n_steps > (u32)e->max_out) return fail(ErrorInvalidValue, "n_steps above %d", e->max_out);
	const u64 l0 = e->launches;
	INF_TRY(ensure_pages(e, seq_slot, start_pos + n_steps));
	int* in = e->h_ctl;
	in[kCtlId] = (int)first_id;
	in[kCtlPos] = (int)start_pos;
	in[kCtlSlot] = (int)seq_slot;
	in[kCtlStep] = 0;
	INF_CUDA_TRY(cudaMemcpyAsync(e->ctl, in, 4 * sizeof(int), cudaMemcpyHostToDevice, e->stream));
	cudaEvent_t ev[2];
	for (auto& x : ev) INF_CUDA_TRY(cudaEventCreate(&x));
	INF_CUDA_TRY(cudaEventRecord(ev[0], e->stream));
	for (u32 s = 0; s < n_steps; ++s) INF_TRY(launch_decode_graph(e));
	INF_CUDA_TRY(cudaEventRecord(ev[1], e->stream));
	if (out_ids)
		INF_CUDA_TRY(cudaMemcpyAsync(out_ids, e->out_ids, (size_t)n_steps * 4,
		                             is_device_ptr(out_ids) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, e->stream));
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	float ms = 0.f;
	cudaEventElapsedTime(&ms, ev[0], ev[1]);
	for (auto& x : ev) cudaEventDestroy(x);
	if (stats) {
		stats->prefill_ms = 0.0;
		stats->decode_ms = ms;
		stats->n_prompt = 0;
		stats->n_new = n_steps;
		stats->kernel_launches = e->launches - l0;
	}
	return check_dev_err(e);
}

Error_t inf_synth_ids(u64 seed, u64 stream, u64 n, u32 lo, u32 hi_inclusive, u32* out)
{
	if (!out || hi_inclusive < lo) return fail(ErrorInvalidValue, "inf_synth_ids: bad arguments");
	const PhiloxKey key = stream_key(seed, stream);
	const u64 range = (u64)hi_inclusive - lo + 1u;
	for (u64 i = 0; i < n; ++i) {
		uint32_t c0 = (uint32_t)i, c1 = (uint32_t)(i >> 32), c2 = 0, c3 = 0, k0 = key.k0, k1 = key.k1;
		for (int r = 0; r < 10; ++r) {
			const u64 p0 = (u64)0xD2511F53u * c0, p1 = (u64)0xCD9E8D57u * c2;
			c0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
			c1 = (uint32_t)p1;
			c2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
			c3 = (uint32_t)p0;
			k0 += 0x9E3779B9u;
			k1 += 0xBB67AE85u;
		}
		out[i] = lo + (u32)(((u64)c0 * range) >> 32);
	}
	return Success;
}

Error_t inf_tp_export(Model* model, void* handle_out, u64 handle_bytes)
{
	if (!model || !model->engine || !handle_out) return fail(ErrorInvalidValue, "inf_tp_export: bad arguments");
	if (handle_bytes < sizeof(cudaIpcMemHandle_t)) return fail(ErrorInvalidValue, "inf_tp_export: need %zu bytes", sizeof(cudaIpcMemHandle_t));
	InfEngine* e = model->engine;
	if (e->cfg.tp_size <= 1) return fail(ErrorInvalidValue, "inf_tp_export: tp_size is 1");
	cudaIpcMemHandle_t h;
	INF_CUDA_TRY(cudaIpcGetMemHandle(&h, e->ctx->dev_arena._d_ptr));
	memcpy(handle_out, &h, sizeof h);
	return Success;
}

Error_t inf_tp_connect(Model* model, const void* handles, u32 n_ranks)
{
	if (!model || !model->engine || !handles) return fail(ErrorInvalidValue, "inf_tp_connect: bad arguments");
	InfEngine* e = model->engine;
	const InfConfig& c = e->cfg;
	if (c.tp_size <= 1 || n_ranks != c.tp_size) return fail(ErrorInvalidValue, "inf_tp_connect: %u handles for tp_size %u", n_ranks, c.tp_size);
	if (e->tpc.size > 1) return fail(ErrorAlreadyInitialized, "inf_tp_connect: already connected");
	TpComm t = e->tpc;
	const int me = (int)c.tp_rank;
	auto rebase = [&](auto* local, uint8_t* base) {
		using P = decltype(local);
		return (P)(base + ((uint8_t*)local - e->ctx->dev_arena._d_ptr));
	};
	e->peer_bases.assign(c.tp_size, nullptr);
	for (u32 k = 0; k < c.tp_size; ++k) {
		uint8_t* base = e->ctx->dev_arena._d_ptr;
		if ((int)k != me) {
			cudaIpcMemHandle_t h;
			memcpy(&h, (const uint8_t*)handles + (size_t)k * sizeof h, sizeof h);
			void* p = nullptr;
			INF_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
			e->peer_bases[k] = p;
			base = (uint8_t*)p;
		}
		t.inbox[k] = rebase(e->tpc.inbox[me], base);
		t.am_inbox[k] = rebase(e->tpc.am_inbox[me], base);
		t.am_flags[k] = rebase(e->tpc.am_flags[me], base);
		t.ready[k] = rebase(e->tpc.ready[me], base);
		t.done[k] = rebase(e->tpc.done[me], base);
		if (e->chunk > 0) {
			t.part[k] = rebase(e->tpc.part[me], base);
			t.red[k] = rebase(e->tpc.red[me], base);
		}
	}
	t.size = (int)c.tp_size;
	e->tpc = t;
	// the decode graph bakes the comm descriptor into its kernel arguments: rebuild it
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	if (e->decode_exec) {
		cudaGraphExecDestroy(e->decode_exec);
		e->decode_exec = nullptr;
	}
	return build_decode_graph(e);
}

Error_t inf_set_sampling(Model* model, const InfSampling* s)
{
	if (!model || !model->engine || !s) return fail(ErrorInvalidValue, "inf_set_sampling: NULL argument");
	InfEngine* e = model->engine;
	if (!(s->temperature >= 0.0f) || !std::isfinite(s->temperature)) return fail(ErrorInvalidValue, "temperature %g", (double)s->temperature);
	if (!(s->top_p > 0.0f && s->top_p <= 1.0f)) return fail(ErrorInvalidValue, "top_p %g outside (0, 1]", (double)s->top_p);
	const bool on = s->temperature > 0.0f;
	if (on && e->cfg.tp_size > 1) return fail(ErrorUnsupported, "sampling with the vocabulary split across ranks");
	if (on && 1.0 / (double)s->temperature > 3.0e38) return fail(ErrorInvalidValue, "temperature %g too small", (double)s->temperature);
	e->samp = *s;
	if (on == e->sampling && !on) return Success;
	e->sampling = on;
	// the decode graph holds the sampler's arguments: rebuild it
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	if (e->decode_exec) {
		cudaGraphExecDestroy(e->decode_exec);
		e->decode_exec = nullptr;
	}
	return build_decode_graph(e);
}

Error_t inf_debug_read(Model* model, u32 buffer, u32 layer, u32 seq_slot, u32 pos, f32* out, u64 n_out)
{
	if (!model || !model->engine || !out) return fail(ErrorInvalidValue, "inf_debug_read: bad arguments");
	InfEngine* e = model->engine;
	const InfConfig& c = e->cfg;
	const u64 hd = c.head_dim;
	INF_CUDA_TRY(cudaStreamSynchronize(e->stream));
	const void* src = nullptr;
	u64 n = 0;
	bool is_f32 = false;
	std::vector<uint8_t> tmp;
	switch (buffer) {
	case InfBufResid: src = e->gemma ? e->resid_final : e->resid; n = c.dim; is_f32 = true; break;
	case InfBufQ: src = e->q; n = (u64)e->Hl * hd; break;
	case InfBufAttn: src = e->attn; n = (u64)e->Hl * hd; break;
	case InfBufH: src = e->h; n = (u64)e->Fl; break;
	case InfBufLogits: src = e->logits; n = (u64)e->Vl; is_f32 = true; break;
	case InfBufSampleQ: src = e->sample_q; n = (u64)e->Vl; is_f32 = true; break; // raw u32 bits
	case InfBufSampleQRow:
		if (pos >= c.max_batch) return fail(ErrorInvalidValue, "inf_debug_read: row %u >= max_batch", pos);
		src = e->sample_q_rows + (size_t)pos * e->Vl;
		n = (u64)e->Vl;
		is_f32 = true;
		break;
	case InfBufK:
	case InfBufV: {
		if (layer >= c.n_layers || seq_slot >= c.max_batch || pos >= c.max_seq)
			return fail(ErrorInvalidValue, "inf_debug_read: layer/slot/pos");
		const int page = e->h_block_table[(size_t)seq_slot * e->pages_per_seq + pos / c.kv_block];
		if (page < 0) return fail(ErrorKvOutOfRange, "inf_debug_read: position has no page");
		n = (u64)e->KVl * hd;
		if (n_out < n) return fail(ErrorInvalidValue, "inf_debug_read: need %llu floats", (unsigned long long)n);
		tmp.resize(n * e->esz);
		const uint8_t* pool = (const uint8_t*)(buffer == InfBufK ? e->layers[layer].kpool : e->layers[layer].vpool);
		for (int kvh = 0; kvh < e->KVl; ++kvh) {
			const size_t off = ((((size_t)page * e->KVl + kvh) * c.kv_block) + pos % c.kv_block) * hd * e->esz;
			INF_CUDA_TRY(cudaMemcpy(tmp.data() + (size_t)kvh * hd * e->esz, pool + off, hd * e->esz, cudaMemcpyDeviceToHost));
		}
		break;
	}
	default: return fail(ErrorInvalidValue, "inf_debug_read: buffer %u", buffer);
	}
	if (n_out < n) return fail(ErrorInvalidValue, "inf_debug_read: need %llu floats", (unsigned long long)n);
	if (src) {
		tmp.resize(n * (is_f32 ? 4 : e->esz));
		INF_CUDA_TRY(cudaMemcpy(tmp.data(), src, tmp.size(), cudaMemcpyDeviceToHost));
	}
	if (is_f32 || e->esz == 4) {
		memcpy(out, tmp.data(), n * 4);
	} else {
		const uint16_t* h = (const uint16_t*)tmp.data();
		for (u64 i = 0; i < n; ++i) {
			const uint32_t u = (uint32_t)h[i] << 16;
			memcpy(&out[i], &u, 4);
		}
	}
	return Success;
}

Error_t inf_seq_reset(Model* model, u32 seq_slot)
{
	if (!model || !model->engine) return fail(ErrorInvalidValue, "inf_seq_reset: no model");
	if (seq_slot >= model->engine->cfg.max_batch) return fail(ErrorInvalidValue, "slot");
	return release_pages(model->engine, seq_slot);
}

void* inf_model_stream(Model* model) { return model && model->engine ? (void*)model->engine->stream : nullptr; }

u64 inf_kernel_launches(Model* model) { return model && model->engine ? model->engine->launches : 0; }
u64 inf_batch_h2d_bytes(Model* model) { return model && model->engine ? model->engine->h2d_bytes : 0; }

u64 inf_decode_bytes(const InfConfig* c, u32 ctx)
{
	if (!c) return 0;
	const u64 es = c->dtype == InfBF16 ? 2 : 4, d = c->dim, hd = c->head_dim, L = c->n_layers;
	u64 layer = ((u64)(c->n_heads + 2 * c->n_kv_heads) * hd * d + d * c->n_heads * hd + 3ull * c->ffn_dim * d + 2 * d) * es;
	u64 weights = (u64)c->vocab_size * d * es + d * es + d * es; // LM head, final norm, one embedding row
	if (c->arch == InfArchGemma) {
		const u64 P = c->ple_dim;
		layer += (2 * hd + 3 * d + 2 * P * d) * es;              // q/k/post norms, PLE gate and projection
		weights += (L * P * d + P + L * P) * es;                   // per-layer-input projection, its norm, one E_ple row
	}
	weights += L * layer;
	const u64 kv = 2ull * L * c->n_kv_heads * hd * es * ((u64)ctx + 1);       // read ctx, write 1
	return weights + kv;
}

u32 inf_profile_decode_step(Model* model, u32 seq_slot, u32 pos, u32 id, f32* ms_out, u32 max_kinds)
{
	if (!model || !model->engine || !ms_out) return 0;
	InfEngine* e = model->engine;
	if (seq_slot >= e->cfg.max_batch || pos >= e->cfg.max_seq || id >= e->cfg.vocab_size) return 0;
	if (ensure_pages(e, seq_slot, pos + 1) != Success) return 0;
	int* in = e->h_ctl;
	in[kCtlId] = (int)id;
	in[kCtlPos] = (int)pos;
	in[kCtlSlot] = (int)seq_slot;
	if (cudaMemcpyAsync(e->ctl, in, 3 * sizeof(int), cudaMemcpyHostToDevice, e->stream) != cudaSuccess) return 0;
	for (float& v : e->prof_ms) v = 0.f;
	e->profiling = true;
	const Error_t r = enqueue_step(e);
	e->profiling = false;
	if (r != Success) return 0;
	const u32 n = std::min<u32>(max_kinds, InfKNumKinds);
	for (u32 k = 0; k < n; ++k) ms_out[k] = e->prof_ms[k];
	return n;
}

// ---- stand-alone kernels --------------------------------------------------------------

Error_t inf_fetch_input_embeddings(const u32* d_ids, u64 n_tokens, u32 dim, u32 vocab_size, const void* d_table,
                                   void* d_out, u32 dtype, void* stream)
{
	if (!d_ids || !d_table || !d_out || n_tokens == 0 || dim == 0 || n_tokens > 65535u * 1024u)
		return fail(ErrorInvalidValue, "inf_fetch_input_embeddings: bad arguments");
	if (!is_device_ptr(d_ids) || !is_device_ptr(d_table) || !is_device_ptr(d_out))
		return fail(ErrorInvalidDevPtr, "inf_fetch_input_embeddings: device pointers required");
	int* d_err = nullptr;
	INF_CUDA_TRY(cudaMallocAsync((void**)&d_err, sizeof(int), (cudaStream_t)stream));
	INF_CUDA_TRY(cudaMemsetAsync(d_err, 0, sizeof(int), (cudaStream_t)stream));
	const size_t es = dtype == InfBF16 ? 2 : 4;
	const u32 units = (u32)((dim * es + 15) / 16);
	const dim3 grid((units + 255) / 256, (unsigned)n_tokens);
	if (dtype == InfBF16)
		k_embed_copy<bf16><<<grid, 256, 0, (cudaStream_t)stream>>>(d_ids, (int)n_tokens, (int)dim, vocab_size,
		                                                            (const bf16*)d_table, (bf16*)d_out, d_err);
	else if (dtype == InfF32)
		k_embed_copy<float><<<grid, 256, 0, (cudaStream_t)stream>>>(d_ids, (int)n_tokens, (int)dim, vocab_size,
		                                                             (const float*)d_table, (float*)d_out, d_err);
	else {
		cudaFreeAsync(d_err, (cudaStream_t)stream);
		return fail(ErrorInvalidValue, "dtype %u", dtype);
	}
	INF_CUDA_TRY(cudaGetLastError());
	int h_err = 0;
	INF_CUDA_TRY(cudaMemcpyAsync(&h_err, d_err, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
	INF_CUDA_TRY(cudaFreeAsync(d_err, (cudaStream_t)stream));
	INF_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
	if (h_err == kDevTokenRange) return fail(ErrorTokenOutOfRange, "token id >= vocab_size");
	return Success;
}

Error_t inf_gemm_bf16(const void* d_x, const void* d_w, void* d_y, u32 T, u32 N, u32 K, u32 out_f32, void* stream)
{
	if (!d_x || !d_w || !d_y || T == 0 || N == 0 || K == 0 || K % 8 != 0 || T > 65535u * kTcBM)
		return fail(ErrorInvalidValue, "inf_gemm_bf16: bad arguments");
	if (!is_device_ptr(d_x) || !is_device_ptr(d_w) || !is_device_ptr(d_y))
		return fail(ErrorInvalidDevPtr, "inf_gemm_bf16: device pointers required");
	if (((uintptr_t)d_x | (uintptr_t)d_w) & 15) return fail(ErrorInvalidValue, "inf_gemm_bf16: 16-byte alignment");
	InfEngine tmp;
	tmp.stream = (cudaStream_t)stream;
	int* d_err = nullptr;
	INF_CUDA_TRY(cudaMallocAsync((void**)&d_err, sizeof(int), tmp.stream));
	INF_CUDA_TRY(cudaMemsetAsync(d_err, 0, sizeof(int), tmp.stream));
	tmp.err = d_err;
	TcArgs a = tc_base(&tmp, (int)T, (int)N, (int)K, out_f32 ? kTcStoreF32 : kTcStore);
	a.out = d_y;
	Error_t r = launch_gemm_tc(&tmp, d_x, d_w, a);
	int h_err = 0;
	if (r == Success) {
		INF_CUDA_TRY(cudaMemcpyAsync(&h_err, d_err, sizeof(int), cudaMemcpyDeviceToHost, tmp.stream));
	}
	cudaFreeAsync(d_err, tmp.stream);
	INF_CUDA_TRY(cudaStreamSynchronize(tmp.stream));
	tmp.stream = nullptr;
	if (r != Success) return r;
	return map_dev_err(h_err);
}

// ---- stand-alone decode attention -------------------------------------------------------
} // extern "C"

namespace {
struct AttnPlan {
	int kernel;                   // InfAttnKernel that runs (never InfAttnAuto)
	int splits, max_pages_split;  // of that kernel
	size_t part_bytes, counter_bytes, smem;
};

// Every kernel's plan for the shape; scratch is sized for the largest, so any kernel can run in
// a buffer of inf_attn_decode_scratch_bytes.  `kernel` resolves InfAttnAuto the way the model's
// decode step does: the cluster kernel for single tokens when it fits, the tensor-core streaming
// kernel for batches (bf16, 16-token pages, head_dim 64 or 128), else the split-K kernel.
Error_t attn_plan(u32 kernel, u32 n_tokens, u32 n_heads, u32 n_kv_heads, u32 head_dim, u32 kv_block, u32 pages_per_seq,
                  u32 dtype, AttnPlan* p)
{
	if (n_tokens == 0 || n_heads == 0 || n_kv_heads == 0 || head_dim == 0 || head_dim % 2 || kv_block == 0 ||
	    pages_per_seq == 0 || n_heads % n_kv_heads || (dtype != InfBF16 && dtype != InfF32) || n_tokens > 65535)
		return fail(ErrorInvalidValue, "attention: bad shape");
	if (kernel > InfAttnClusterTc) return fail(ErrorInvalidValue, "attention: kernel %u", kernel);
	const u32 G = n_heads / n_kv_heads;
	if (!attn_decode_supported((int)G, (int)head_dim) || G * head_dim > (u32)(kAttnThreads * kAttnMaxAcc))
		return fail(ErrorUnsupported, "attention: GQA group %u x head_dim %u", G, head_dim);
	const size_t esz = dtype == InfBF16 ? 2 : 4;
	if ((kv_block * head_dim * esz) % 16) return fail(ErrorUnsupported, "attention: page block not a multiple of 16 bytes");
	int sms = 148, dev = 0;
	if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
	// split-K
	int sk_splits = 1, sk_pages = 1;
	attn_decode_plan(sms, (int)n_kv_heads, (int)n_tokens, (int)pages_per_seq, (int)kv_block, (int)head_dim, esz,
	                 &sk_splits, &sk_pages);
	// tensor-core streaming (the batched decode step's kernel)
	const bool mma_ok = dtype == InfBF16 && kv_block == 16 && attn_decode_mma_kernel((int)G, (int)head_dim) != nullptr;
	const int mma_splits = attn_stream_splits(sms, (int)n_kv_heads, (int)n_tokens, (int)pages_per_seq);
	const size_t hd2 = head_dim + 2;
	p->part_bytes = (size_t)n_tokens * n_heads * (size_t)std::max(sk_splits, mma_ok ? mma_splits : 1) * hd2 * sizeof(float);
	p->counter_bytes = (size_t)n_tokens * n_kv_heads * sizeof(unsigned) + 16; // + error word
	int k = (int)kernel;
	int cl_splits = 0, cl_pages = 0, ct_splits = 0, ct_pages = 0;
	if ((k == InfAttnAuto && n_tokens == 1) || k == InfAttnClusterTc) {
		INF_TRY(attn_cltc_plan((int)G, (int)head_dim, (int)kv_block, esz, (int)pages_per_seq, (int)n_kv_heads, &ct_splits,
		                       &ct_pages));
		if (k == InfAttnClusterTc && ct_splits == 0)
			return fail(ErrorUnsupported, "attention: the tensor-core cluster kernel needs bf16, 16-token pages, head_dim 64 "
			                              "or 128, GQA group <= 8 and at most 16 pages per CTA");
		if (ct_splits > 0) k = InfAttnClusterTc;
	}
	if (k == InfAttnAuto || k == InfAttnCluster) {
		if (n_tokens == 1 || k == InfAttnCluster)
			INF_TRY(attn_cl_plan((int)G, (int)head_dim, (int)kv_block, esz, (int)pages_per_seq, (int)n_kv_heads, &cl_splits,
			                     &cl_pages));
		if (k == InfAttnCluster && cl_splits == 0)
			return fail(ErrorUnsupported, "attention: %u pages per sequence do not fit one cluster", pages_per_seq);
	}
	if (k == InfAttnMma && !mma_ok)
		return fail(ErrorUnsupported, "attention: the tensor-core kernel needs bf16, 16-token pages and head_dim 64 or 128");
	if (k == InfAttnAuto) k = cl_splits > 0 ? InfAttnCluster : (n_tokens > 1 && mma_ok) ? InfAttnMma : InfAttnSplitK;
	p->kernel = k;
	if (k == InfAttnClusterTc) {
		p->splits = ct_splits;
		p->max_pages_split = ct_pages;
		p->smem = attn_cltc_layout((int)G, (int)head_dim, ct_pages, ct_splits).total;
	} else if (k == InfAttnCluster) {
		p->splits = cl_splits;
		p->max_pages_split = cl_pages;
		p->smem = attn_cl_layout((int)G, (int)head_dim, (int)kv_block, esz, cl_pages, cl_splits).total;
	} else if (k == InfAttnMma) {
		p->splits = mma_splits;
		p->max_pages_split = 0;
		p->smem = attn_mma_smem_bytes((int)head_dim, (int)kv_block, (int)pages_per_seq);
	} else {
		p->splits = sk_splits;
		p->max_pages_split = sk_pages;
		p->smem = attn_decode_smem_bytes((int)G, (int)head_dim, (int)kv_block, esz, sk_pages, sk_splits);
	}
	return Success;
}

template <typename T>
Error_t attn_launch_t(const AttnPlan& P, const AttnDecodeArgs& a, u32 n_tokens, u32 n_pages, cudaStream_t st)
{
	const int G = a.H / a.KV;
	if (P.kernel == InfAttnCluster) {
		const AttnKernel<T> k = attn_decode_cl_kernel<T>(G, a.hd);
		if (!k) return fail(ErrorUnsupported, "attention: GQA group %d, head_dim %d", G, a.hd);
		INF_CUDA_TRY(set_smem(k, P.smem));
		if (P.splits > 8) INF_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
		cudaLaunchConfig_t lc = {};
		lc.gridDim = dim3((unsigned)P.splits, (unsigned)a.KV, n_tokens);
		lc.blockDim = dim3(kAttnThreads);
		lc.dynamicSmemBytes = P.smem;
		lc.stream = st;
		cudaLaunchAttribute attr[1];
		attr[0].id = cudaLaunchAttributeClusterDimension;
		attr[0].val.clusterDim.x = (unsigned)P.splits;
		attr[0].val.clusterDim.y = 1;
		attr[0].val.clusterDim.z = 1;
		lc.attrs = attr;
		lc.numAttrs = 1;
		INF_CUDA_TRY(cudaLaunchKernelEx(&lc, k, a));
		return Success;
	}
	if constexpr (sizeof(T) == 2) {
		if (P.kernel == InfAttnClusterTc) {
			const AttnClTcKernel k = attn_decode_cltc_kernel(G, a.hd);
			if (!k) return fail(ErrorUnsupported, "attention: GQA group %d, head_dim %d", G, a.hd);
			if ((uintptr_t)a.q & 15) return fail(ErrorInvalidValue, "inf_attn_decode: q not 16-byte aligned");
			CUtensorMap tk, tv; // one page (16 positions x 64 head dims) per box
			INF_TRY(tensor_map_kv(&tk, a.kpool, (u32)a.hd, (u32)a.blk, (u32)a.KV, n_pages, 1));
			INF_TRY(tensor_map_kv(&tv, a.vpool, (u32)a.hd, (u32)a.blk, (u32)a.KV, n_pages, 1));
			INF_CUDA_TRY(set_smem(k, P.smem));
			if (P.splits > 8) INF_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
			cudaLaunchConfig_t lc = {};
			lc.gridDim = dim3((unsigned)P.splits, (unsigned)a.KV, n_tokens);
			lc.blockDim = dim3(kClTcThreads);
			lc.dynamicSmemBytes = P.smem;
			lc.stream = st;
			cudaLaunchAttribute attr[1];
			attr[0].id = cudaLaunchAttributeClusterDimension;
			attr[0].val.clusterDim.x = (unsigned)P.splits;
			attr[0].val.clusterDim.y = 1;
			attr[0].val.clusterDim.z = 1;
			lc.attrs = attr;
			lc.numAttrs = 1;
			INF_CUDA_TRY(cudaLaunchKernelEx(&lc, k, tk, tv, a));
			return Success;
		}
		if (P.kernel == InfAttnMma) {
			const AttnMmaKernel k = attn_decode_mma_kernel(G, a.hd);
			if (!k) return fail(ErrorUnsupported, "attention: GQA group %d, head_dim %d", G, a.hd);
			CUtensorMap tk, tv; // one page (blk positions x 64 head dims) per box
			INF_TRY(tensor_map_kv(&tk, a.kpool, (u32)a.hd, (u32)a.blk, (u32)a.KV, n_pages, 1));
			INF_TRY(tensor_map_kv(&tv, a.vpool, (u32)a.hd, (u32)a.blk, (u32)a.KV, n_pages, 1));
			INF_CUDA_TRY(set_smem(k, P.smem));
			k<<<dim3((unsigned)a.KV, (unsigned)P.splits, n_tokens), kAmThreads, P.smem, st>>>(tk, tv, a);
			INF_CUDA_TRY(cudaGetLastError());
			return Success;
		}
	}
	const AttnKernel<T> k = attn_decode_kernel<T>(G, a.hd);
	if (!k) return fail(ErrorUnsupported, "attention: GQA group %d, head_dim %d", G, a.hd);
	INF_CUDA_TRY(set_smem(k, P.smem));
	k<<<dim3((unsigned)a.KV, (unsigned)P.splits, n_tokens), kAttnThreads, P.smem, st>>>(a);
	INF_CUDA_TRY(cudaGetLastError());
	return Success;
}
} // namespace

extern "C" {

u64 inf_attn_decode_scratch_bytes(u32 n_tokens, u32 n_heads, u32 n_kv_heads, u32 head_dim, u32 kv_block,
                                  u32 pages_per_seq, u32 dtype)
{
	AttnPlan P = {};
	if (attn_plan(InfAttnSplitK, n_tokens, n_heads, n_kv_heads, head_dim, kv_block, pages_per_seq, dtype, &P) != Success)
		return 0;
	return (u64)(P.part_bytes + P.counter_bytes);
}

Error_t inf_attn_decode_with(u32 kernel, const void* d_q, const void* d_kpool, const void* d_vpool,
                             const i32* d_block_table, u32 pages_per_seq, u32 n_pages, const i32* d_tok_slot,
                             const i32* d_tok_pos, u32 n_tokens, u32 n_heads, u32 n_kv_heads, u32 head_dim, u32 kv_block,
                             u32 dtype, void* d_out, void* d_scratch, u64 scratch_bytes, void* stream)
{
	if (!d_q || !d_kpool || !d_vpool || !d_block_table || !d_tok_slot || !d_tok_pos || !d_out || !d_scratch)
		return fail(ErrorInvalidValue, "inf_attn_decode: NULL pointer");
	AttnPlan P;
	INF_TRY(attn_plan(kernel, n_tokens, n_heads, n_kv_heads, head_dim, kv_block, pages_per_seq, dtype, &P));
	if (scratch_bytes < P.part_bytes + P.counter_bytes)
		return fail(ErrorInvalidValue, "inf_attn_decode: scratch needs %zu bytes", P.part_bytes + P.counter_bytes);
	if (((uintptr_t)d_scratch & 15) || ((uintptr_t)d_kpool & 15) || ((uintptr_t)d_vpool & 15))
		return fail(ErrorInvalidValue, "inf_attn_decode: 16-byte alignment");
	if (n_pages == 0) return fail(ErrorInvalidValue, "inf_attn_decode: no pages");
	const cudaStream_t st = (cudaStream_t)stream;
	uint8_t* scr = (uint8_t*)d_scratch;
	unsigned* counters = (unsigned*)(scr + P.part_bytes);
	int* err = (int*)(scr + P.part_bytes + P.counter_bytes - 16);
	INF_CUDA_TRY(cudaMemsetAsync(counters, 0, P.counter_bytes, st)); // tickets and error word start at zero
	AttnDecodeArgs a;
	memset(&a, 0, sizeof a);
	a.q = d_q;
	a.kpool = d_kpool;
	a.vpool = d_vpool;
	a.block_table = d_block_table;
	a.pages_per_seq = (int)pages_per_seq;
	a.max_pages = (int)n_pages;
	a.tok_slot = d_tok_slot;
	a.tok_pos = d_tok_pos;
	a.H = (int)n_heads;
	a.KV = (int)n_kv_heads;
	a.hd = (int)head_dim;
	a.blk = (int)kv_block;
	a.n_splits = P.splits;
	a.max_pages_split = P.max_pages_split;
	a.scale = (float)(1.0 / std::sqrt((double)head_dim));
	a.part = (float*)scr;
	a.counters = counters;
	a.out = d_out;
	a.err = err;
	if (dtype == InfBF16) INF_TRY(attn_launch_t<bf16>(P, a, n_tokens, n_pages, st));
	else INF_TRY(attn_launch_t<float>(P, a, n_tokens, n_pages, st));
	int h_err = 0;
	INF_CUDA_TRY(cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, st));
	INF_CUDA_TRY(cudaStreamSynchronize(st));
	return map_dev_err(h_err);
}

Error_t inf_attn_decode(const void* d_q, const void* d_kpool, const void* d_vpool, const i32* d_block_table,
                        u32 pages_per_seq, u32 n_pages, const i32* d_tok_slot, const i32* d_tok_pos, u32 n_tokens,
                        u32 n_heads, u32 n_kv_heads, u32 head_dim, u32 kv_block, u32 dtype, void* d_out,
                        void* d_scratch, u64 scratch_bytes, void* stream)
{
	return inf_attn_decode_with(InfAttnAuto, d_q, d_kpool, d_vpool, d_block_table, pages_per_seq, n_pages, d_tok_slot,
	                            d_tok_pos, n_tokens, n_heads, n_kv_heads, head_dim, kv_block, dtype, d_out, d_scratch,
	                            scratch_bytes, stream);
}

Error_t inf_attn_prefill(u32 kernel, const void* d_q, const void* d_kpool, const void* d_vpool,
                         const i32* d_block_table, u32 pages_per_seq, u32 n_pages, const i32* d_tok_slot,
                         const i32* d_tok_pos, u32 n_tokens, u32 n_heads, u32 n_kv_heads, u32 head_dim, u32 kv_block,
                         void* d_out, void* stream)
{
	if (!d_q || !d_kpool || !d_vpool || !d_block_table || !d_tok_slot || !d_tok_pos || !d_out)
		return fail(ErrorInvalidValue, "inf_attn_prefill: NULL pointer");
	if (n_tokens == 0 || n_heads == 0 || n_kv_heads == 0 || n_heads % n_kv_heads || head_dim == 0 || head_dim % 2 ||
	    kv_block == 0 || pages_per_seq == 0 || n_pages == 0 || kernel > InfPrefillAttnSimt || n_tokens > 65535u * 16u)
		return fail(ErrorInvalidValue, "inf_attn_prefill: bad shape");
	if (((uintptr_t)d_kpool | (uintptr_t)d_vpool | (uintptr_t)d_q) & 15)
		return fail(ErrorInvalidValue, "inf_attn_prefill: 16-byte alignment");
	const int G = (int)(n_heads / n_kv_heads), hd = (int)head_dim, blk = (int)kv_block;
	if (G * hd * kPfTq > kPfThreads * kPfMaxAcc || (G != 1 && G != 2 && G != 4 && G != 8) || hd > 256)
		return fail(ErrorUnsupported, "inf_attn_prefill: GQA group %d x head_dim %d", G, hd);
	const bool tc = kernel == InfPrefillAttnAuto && (hd == 64 || hd == 128) && kPtRows % G == 0 && blk % 8 == 0 &&
	                kPtKeys % blk == 0;
	const cudaStream_t st = (cudaStream_t)stream;
	int* d_err = nullptr;
	INF_CUDA_TRY(cudaMallocAsync((void**)&d_err, sizeof(int), st));
	INF_CUDA_TRY(cudaMemsetAsync(d_err, 0, sizeof(int), st));
	AttnPrefillArgs a;
	memset(&a, 0, sizeof a);
	a.q = d_q;
	a.kpool = d_kpool;
	a.vpool = d_vpool;
	a.block_table = d_block_table;
	a.pages_per_seq = (int)pages_per_seq;
	a.max_pages = (int)n_pages;
	a.tok_pos = d_tok_pos;
	a.tok_slot = d_tok_slot;
	a.T = (int)n_tokens;
	a.H = (int)n_heads;
	a.KV = (int)n_kv_heads;
	a.hd = hd;
	a.blk = blk;
	a.scale = (float)(1.0 / std::sqrt((double)hd));
	a.out = d_out;
	a.err = d_err;
	Error_t r = Success;
	if (tc) {
		const size_t smem = attn_prefill_tc_smem_bytes(hd);
		const u32 bp = kPtKeys / kv_block;
		CUtensorMap tk8, tk1, tv8, tv1;
		r = tensor_map_kv(&tk8, d_kpool, head_dim, kv_block, n_kv_heads, n_pages, bp);
		if (r == Success) r = tensor_map_kv(&tk1, d_kpool, head_dim, kv_block, n_kv_heads, n_pages, 1);
		if (r == Success) r = tensor_map_kv(&tv8, d_vpool, head_dim, kv_block, n_kv_heads, n_pages, bp);
		if (r == Success) r = tensor_map_kv(&tv1, d_vpool, head_dim, kv_block, n_kv_heads, n_pages, 1);
		cudaError_t ce = cudaSuccess;
		if (r == Success) ce = set_smem(k_attn_prefill_tc, smem);
		if (r == Success && ce == cudaSuccess) {
			const int tq = kPtRows / G;
			k_attn_prefill_tc<<<dim3(n_kv_heads, (n_tokens + tq - 1) / tq), kPtThreads, smem, st>>>(tk8, tk1, tv8, tv1, a);
			ce = cudaGetLastError();
		}
		if (r == Success && ce != cudaSuccess) r = fail(ErrorCuda, "inf_attn_prefill: %s", cudaGetErrorString(ce));
	} else {
		const size_t smem = attn_prefill_smem_bytes(G, hd, blk);
		cudaError_t ce = set_smem(k_attn_prefill<bf16>, smem);
		if (ce == cudaSuccess) {
			k_attn_prefill<bf16><<<dim3(n_kv_heads, (n_tokens + kPfTq - 1) / kPfTq), kPfThreads, smem, st>>>(a);
			ce = cudaGetLastError();
		}
		if (ce != cudaSuccess) r = fail(ErrorCuda, "inf_attn_prefill: %s", cudaGetErrorString(ce));
	}
	int h_err = 0;
	if (r == Success) INF_CUDA_TRY(cudaMemcpyAsync(&h_err, d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
	cudaFreeAsync(d_err, st);
	INF_CUDA_TRY(cudaStreamSynchronize(st));
	if (r != Success) return r;
	return map_dev_err(h_err);
}

Error_t inf_rmsnorm(const void* d_x, void* d_y, u32 rows, u32 dim, const void* d_gain, f32 eps, u32 dtype, void* stream)
{
	if (!d_x || !d_y || !d_gain || rows == 0 || dim == 0 || rows > 2147483647u)
		return fail(ErrorInvalidValue, "inf_rmsnorm: bad arguments");
	if (!is_device_ptr(d_x) || !is_device_ptr(d_y) || !is_device_ptr(d_gain))
		return fail(ErrorInvalidDevPtr, "inf_rmsnorm: device pointers required");
	if (dtype == InfBF16)
		k_rmsnorm_rows<bf16, bf16, bf16><<<rows, 256, 0, (cudaStream_t)stream>>>((const bf16*)d_x, (bf16*)d_y, (int)rows,
		                                                                        (int)dim, (const bf16*)d_gain, eps);
	else if (dtype == InfF32)
		k_rmsnorm_rows<float, float, float><<<rows, 256, 0, (cudaStream_t)stream>>>(
		    (const float*)d_x, (float*)d_y, (int)rows, (int)dim, (const float*)d_gain, eps);
	else
		return fail(ErrorInvalidValue, "dtype %u", dtype);
	INF_CUDA_TRY(cudaGetLastError());
	INF_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
	return Success;
}

} // extern "C"
