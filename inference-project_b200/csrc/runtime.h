// Host-side helpers shared by the translation units of libinf.so.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/inf.h"

namespace inf {

// Records a description of the failure for inf_last_error_detail() and returns err.
Error_t fail(Error_t err, const char* fmt, ...);

#define INF_CUDA_TRY(expr)                                                                                  \
	do {                                                                                                    \
		cudaError_t inf_e_ = (expr);                                                                        \
		if (inf_e_ != cudaSuccess)                                                                          \
			return ::inf::fail(ErrorCuda, "%s:%d %s: %s", __FILE__, __LINE__, #expr, cudaGetErrorString(inf_e_)); \
	} while (0)

#define INF_TRY(expr)                          \
	do {                                       \
		Error_t inf_r_ = (expr);               \
		if (inf_r_ != Success) return inf_r_;  \
	} while (0)

bool is_device_ptr(const void* p);

// Whether inf_set_sampling turned sampling on for this model (false for NULL).
bool model_sampling_on(const Model* m);

// inf_forward_batch; single_batched runs even one sequence through the batched tensor-core
// step (inf_forward_batch gives a lone sequence the batch-1 decode kernels instead), so a
// sequence's results do not depend on how many others share the step.
Error_t forward_batch(Model* model, u32 n_seqs, const u32* seq_slots, const u32* ids, const u32* positions,
                      f32* logits_out, u32* argmax_out, bool single_batched);

// After an inf_forward of `slot` whose new token sits at pos_new: replaces *id (the token the
// forward chose) by a draw under the slot's inf_set_slot_sampling settings, when they sample.
Error_t sample_slot_token(Model* model, u32 slot, u32 pos_new, u32* id);

} // namespace inf
