// Checkpoint loading (host side): safetensors files and Hugging Face config.json.
//
// Replaces model_build's file handling (src/main.cu:177-352) and model_parse_config
// (src/main.cu:120-157).  A checkpoint is one .safetensors file, a *.safetensors.index.json
// naming the shard of every tensor, or a directory holding either.  Every tensor the decoder
// needs is looked up by its Hugging Face Llama name ("model." or "model.language_model."
// prefix), checked for dtype, shape and offsets, and written in the device layout of the
// engine (csrc/synth.cuh RowMap: QKV rows in rotate-half pairs, gate/up rows interleaved, the
// rank's tensor-parallel shard).
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/inf.h"

namespace inf {

// ---- JSON (RFC 8259) ------------------------------------------------------------------------
struct JVal {
	enum Kind : unsigned char { Null, Bool, Num, Str, Arr, Obj } kind = Null;
	bool b = false;
	bool is_uint = false; // an integer literal without sign, fraction or exponent that fits u64
	uint64_t u = 0;
	double num = 0.0;
	std::string s;
	std::vector<JVal> arr;
	std::vector<std::pair<std::string, JVal>> obj;
	const JVal* get(const char* key) const; // first member named key, objects only
};

// Parses text[0, n) as one JSON value (surrounding whitespace allowed); ErrorInvalidValue with
// the byte offset of the first error.
Error_t json_parse(const char* text, size_t n, JVal* out);

// ---- safetensors ----------------------------------------------------------------------------
struct StTensor {
	std::string dtype;
	int esize = 0;               // bytes per element, 0 for a dtype this library does not know
	std::vector<uint64_t> shape;
	uint64_t begin = 0, end = 0; // relative to the file's byte buffer (after 8 + header bytes)
	int file = 0;
};

struct StFile {
	std::string path;
	int fd = -1;
	const unsigned char* map = nullptr;
	uint64_t size = 0;
	uint64_t data0 = 0; // 8 + header length: where the byte buffer starts
};

struct Checkpoint {
	std::vector<StFile> files;
	std::unordered_map<std::string, StTensor> tensors;
	Checkpoint() = default;
	Checkpoint(const Checkpoint&) = delete;
	Checkpoint& operator=(const Checkpoint&) = delete;
	~Checkpoint();
	const unsigned char* data(const StTensor& t) const { return files[t.file].map + files[t.file].data0 + t.begin; }
};

// Opens and maps every file of the checkpoint and indexes its tensors (checks header length,
// JSON, dtype sizes against shapes, offsets inside the buffer, no holes and no overlaps).
Error_t checkpoint_open(const char* path, Checkpoint* ck);

// Checks that every tensor the decoder of c needs is present with a supported dtype (BF16 or
// F32) and the shape c implies.  c has tp_size >= 1 and passed the engine's config checks.
Error_t checkpoint_check(const Checkpoint& ck, const InfConfig& c);

// Rows and columns of one weight (InfWeightKind) in the device layout of rank c.tp_rank.
void weight_dims(const InfConfig& c, uint32_t kind, uint64_t* rows, uint64_t* cols);

// Device rows [row0, row0 + n) of one weight of layer `layer`, converted to c.dtype, into dst.
Error_t weight_rows(const Checkpoint& ck, const InfConfig& c, int layer, uint32_t kind, uint64_t row0, uint64_t n,
                    void* dst);

// weight_rows split over up to 16 host threads (page faults of the mapping and the copies run
// in parallel; one thread assembles about 3.5 GB/s).
Error_t weight_rows_parallel(const Checkpoint& ck, const InfConfig& c, int layer, uint32_t kind, uint64_t row0, uint64_t n,
                             void* dst);

// One weight and where it goes on the device.
struct WeightDst {
	int layer;
	uint32_t kind;
	void* dst;
};

// Writes every weight of `dsts` to the device: rows are assembled in two pinned staging
// buffers and copied with cudaMemcpyAsync on `stream`, one buffer filling while the other
// copies.  Returns after the last copy has completed.
Error_t checkpoint_upload(const Checkpoint& ck, const InfConfig& c, const std::vector<WeightDst>& dsts,
                          cudaStream_t stream);

// model_parse_config (src/main.cu:120-157) for a Llama-family config.json.
Error_t config_from_json(const char* path, InfConfig* inout);

} // namespace inf
