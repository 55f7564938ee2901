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

} // namespace inf
