// Checkpoint loading: JSON, safetensors files, the device layout of the weights and the
// pinned upload.  Host code only.
//
// The reference's model_build (src/main.cu:200-352) reads one safetensors file, takes the byte
// span of the "model.language_model." tensors, copies it to the device with one blocking
// cudaMemcpy and maps per-layer pointers by name.  Differences, each deliberate:
//  - offsets count from the byte buffer after the 8-byte length and the header (the reference
//    adds them to the file start, defect D7);
//  - tensors are found by name and checked one by one for dtype, shape and offsets, in any
//    order, in any number of files (the reference assumes one contiguous, offset-sorted bf16
//    span, defect D8);
//  - the weights land in the engine's device layout (csrc/synth.cuh RowMap) and the rank's
//    tensor-parallel shard, assembled row by row in pinned staging buffers that alternate with
//    asynchronous copies (the reference's cuda_mem_wrapper.cu:54-61 names that intent);
//  - nothing aborts: every failure returns an Error_t described by inf_last_error_detail().
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <unordered_set>

#include "loader.h"
#include "runtime.h"

namespace inf {

// ============================================================================ JSON
const JVal* JVal::get(const char* key) const
{
	if (kind != Obj) return nullptr;
	for (const auto& m : obj)
		if (m.first == key) return &m.second;
	return nullptr;
}

namespace {

constexpr int kJsonMaxDepth = 64;

struct JParser {
	const char* b;
	const char* p;
	const char* e;
	int depth = 0;
	const char* why = nullptr;

	bool fail(const char* w)
	{
		if (!why) why = w;
		return false;
	}
	void ws()
	{
		while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
	}
	bool lit(const char* s)
	{
		const size_t n = strlen(s);
		if ((size_t)(e - p) < n || memcmp(p, s, n) != 0) return fail("invalid literal");
		p += n;
		return true;
	}
	static void put_utf8(std::string& s, uint32_t cp)
	{
		if (cp < 0x80) {
			s += (char)cp;
		} else if (cp < 0x800) {
			s += (char)(0xC0 | (cp >> 6));
			s += (char)(0x80 | (cp & 0x3F));
		} else if (cp < 0x10000) {
			s += (char)(0xE0 | (cp >> 12));
			s += (char)(0x80 | ((cp >> 6) & 0x3F));
			s += (char)(0x80 | (cp & 0x3F));
		} else {
			s += (char)(0xF0 | (cp >> 18));
			s += (char)(0x80 | ((cp >> 12) & 0x3F));
			s += (char)(0x80 | ((cp >> 6) & 0x3F));
			s += (char)(0x80 | (cp & 0x3F));
		}
	}
	bool hex4(uint32_t* v)
	{
		if (e - p < 4) return fail("short \\u escape");
		uint32_t x = 0;
		for (int i = 0; i < 4; ++i) {
			const char c = p[i];
			x <<= 4;
			if (c >= '0' && c <= '9') x |= (uint32_t)(c - '0');
			else if (c >= 'a' && c <= 'f') x |= (uint32_t)(c - 'a' + 10);
			else if (c >= 'A' && c <= 'F') x |= (uint32_t)(c - 'A' + 10);
			else return fail("bad \\u escape");
		}
		p += 4;
		*v = x;
		return true;
	}
	bool string(std::string& s)
	{
		if (p >= e || *p != '"') return fail("expected a string");
		++p;
		s.clear();
		while (true) {
			if (p >= e) return fail("unterminated string");
			const unsigned char c = (unsigned char)*p++;
			if (c == '"') return true;
			if (c < 0x20) return fail("control character in a string");
			if (c != '\\') {
				s += (char)c;
				continue;
			}
			if (p >= e) return fail("unterminated escape");
			const char x = *p++;
			switch (x) {
			case '"': s += '"'; break;
			case '\\': s += '\\'; break;
			case '/': s += '/'; break;
			case 'b': s += '\b'; break;
			case 'f': s += '\f'; break;
			case 'n': s += '\n'; break;
			case 'r': s += '\r'; break;
			case 't': s += '\t'; break;
			case 'u': {
				uint32_t cp;
				if (!hex4(&cp)) return false;
				if (cp >= 0xD800 && cp < 0xDC00) { // high surrogate: a low one must follow
					uint32_t lo;
					if (e - p < 2 || p[0] != '\\' || p[1] != 'u') return fail("lone surrogate");
					p += 2;
					if (!hex4(&lo)) return false;
					if (lo < 0xDC00 || lo >= 0xE000) return fail("lone surrogate");
					cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
				} else if (cp >= 0xDC00 && cp < 0xE000) {
					return fail("lone surrogate");
				}
				put_utf8(s, cp);
				break;
			}
			default: return fail("bad escape");
			}
		}
	}
	bool number(JVal& v)
	{
		const char* s0 = p;
		bool plain = true; // no sign, fraction or exponent
		if (p < e && *p == '-') {
			plain = false;
			++p;
		}
		if (p >= e || !(*p >= '0' && *p <= '9')) return fail("bad number");
		if (*p == '0') ++p;
		else
			while (p < e && *p >= '0' && *p <= '9') ++p;
		if (p < e && *p == '.') {
			plain = false;
			++p;
			if (p >= e || !(*p >= '0' && *p <= '9')) return fail("bad fraction");
			while (p < e && *p >= '0' && *p <= '9') ++p;
		}
		if (p < e && (*p == 'e' || *p == 'E')) {
			plain = false;
			++p;
			if (p < e && (*p == '+' || *p == '-')) ++p;
			if (p >= e || !(*p >= '0' && *p <= '9')) return fail("bad exponent");
			while (p < e && *p >= '0' && *p <= '9') ++p;
		}
		const std::string txt(s0, (size_t)(p - s0));
		v.kind = JVal::Num;
		v.num = strtod(txt.c_str(), nullptr);
		if (plain) {
			uint64_t u = 0;
			bool fits = true;
			for (char c : txt) {
				const uint64_t d = (uint64_t)(c - '0');
				if (u > (UINT64_MAX - d) / 10) {
					fits = false;
					break;
				}
				u = u * 10 + d;
			}
			v.is_uint = fits;
			v.u = fits ? u : 0;
		}
		return true;
	}
	bool value(JVal& v)
	{
		ws();
		if (p >= e) return fail("unexpected end");
		switch (*p) {
		case '{': {
			if (++depth > kJsonMaxDepth) return fail("nesting too deep");
			++p;
			v.kind = JVal::Obj;
			ws();
			if (p < e && *p == '}') {
				++p;
				--depth;
				return true;
			}
			while (true) {
				ws();
				std::string k;
				if (!string(k)) return false;
				ws();
				if (p >= e || *p != ':') return fail("expected ':'");
				++p;
				v.obj.emplace_back(std::move(k), JVal());
				if (!value(v.obj.back().second)) return false;
				ws();
				if (p < e && *p == ',') {
					++p;
					continue;
				}
				if (p < e && *p == '}') {
					++p;
					--depth;
					return true;
				}
				return fail("expected ',' or '}'");
			}
		}
		case '[': {
			if (++depth > kJsonMaxDepth) return fail("nesting too deep");
			++p;
			v.kind = JVal::Arr;
			ws();
			if (p < e && *p == ']') {
				++p;
				--depth;
				return true;
			}
			while (true) {
				v.arr.emplace_back();
				if (!value(v.arr.back())) return false;
				ws();
				if (p < e && *p == ',') {
					++p;
					continue;
				}
				if (p < e && *p == ']') {
					++p;
					--depth;
					return true;
				}
				return fail("expected ',' or ']'");
			}
		}
		case '"': v.kind = JVal::Str; return string(v.s);
		case 't': v.kind = JVal::Bool; v.b = true; return lit("true");
		case 'f': v.kind = JVal::Bool; v.b = false; return lit("false");
		case 'n': v.kind = JVal::Null; return lit("null");
		default: return number(v);
		}
	}
};

} // namespace

Error_t json_parse(const char* text, size_t n, JVal* out)
{
	JParser P{text, text, text + n};
	*out = JVal();
	if (!P.value(*out)) return fail(ErrorInvalidValue, "JSON: %s at byte %zu", P.why, (size_t)(P.p - P.b));
	P.ws();
	if (P.p != P.e) return fail(ErrorInvalidValue, "JSON: trailing bytes at %zu", (size_t)(P.p - P.b));
	return Success;
}

// ============================================================================ files
namespace {

Error_t read_file(const std::string& path, std::string* out)
{
	const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
	if (fd < 0) return fail(ErrorIo, "cannot open %s: %s", path.c_str(), strerror(errno));
	struct stat st;
	if (fstat(fd, &st) != 0) {
		close(fd);
		return fail(ErrorIo, "cannot stat %s", path.c_str());
	}
	out->resize((size_t)st.st_size);
	size_t got = 0;
	while (got < out->size()) {
		const ssize_t r = read(fd, &(*out)[got], out->size() - got);
		if (r <= 0) {
			close(fd);
			return fail(ErrorIo, "short read of %s", path.c_str());
		}
		got += (size_t)r;
	}
	close(fd);
	return Success;
}

int dtype_size(const std::string& d)
{
	static const std::pair<const char*, int> k[] = {
	    {"BOOL", 1}, {"U8", 1}, {"I8", 1}, {"F8_E5M2", 1}, {"F8_E4M3", 1}, {"I16", 2}, {"U16", 2}, {"F16", 2},
	    {"BF16", 2}, {"I32", 4}, {"U32", 4}, {"F32", 4}, {"F64", 8}, {"I64", 8}, {"U64", 8},
	};
	for (const auto& x : k)
		if (d == x.first) return x.second;
	return 0;
}

bool ends_with(const std::string& s, const char* suf)
{
	const size_t n = strlen(suf);
	return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

std::string dir_of(const std::string& p)
{
	const size_t k = p.find_last_of('/');
	return k == std::string::npos ? std::string(".") : p.substr(0, k);
}

constexpr uint64_t kStMaxHeader = 100000000; // the format's header limit

// Maps one safetensors file and adds its tensors to ck (file index = ck->files.size()).
Error_t open_one(Checkpoint* ck, const std::string& path)
{
	StFile f;
	f.path = path;
	f.fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
	if (f.fd < 0) return fail(ErrorIo, "cannot open %s: %s", path.c_str(), strerror(errno));
	ck->files.push_back(f); // owned (closed) by ck from here on
	StFile& F = ck->files.back();
	const int fi = (int)ck->files.size() - 1;
	struct stat st;
	if (fstat(F.fd, &st) != 0) return fail(ErrorIo, "cannot stat %s", path.c_str());
	if (!S_ISREG(st.st_mode)) return fail(ErrorIo, "%s is not a regular file", path.c_str());
	F.size = (uint64_t)st.st_size;
	if (F.size < 8) return fail(ErrorInvalidValue, "%s: %llu bytes, shorter than the 8-byte header length", path.c_str(), (unsigned long long)F.size);
	void* m = mmap(nullptr, F.size, PROT_READ, MAP_PRIVATE, F.fd, 0);
	if (m == MAP_FAILED) return fail(ErrorIo, "cannot map %s: %s", path.c_str(), strerror(errno));
	F.map = (const unsigned char*)m;
	uint64_t hlen = 0;
	for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | F.map[i]; // little-endian
	if (hlen < 2 || hlen > kStMaxHeader)
		return fail(ErrorInvalidValue, "%s: header length %llu outside [2, %llu]", path.c_str(), (unsigned long long)hlen, (unsigned long long)kStMaxHeader);
	if (hlen > F.size - 8)
		return fail(ErrorInvalidValue, "%s: header of %llu bytes runs past the end of the file (%llu bytes): truncated",
		            path.c_str(), (unsigned long long)hlen, (unsigned long long)F.size);
	F.data0 = 8 + hlen;
	const uint64_t buf_len = F.size - F.data0;
	const char* h = (const char*)F.map + 8;
	if (h[0] != '{') return fail(ErrorInvalidValue, "%s: header does not start with '{'", path.c_str());
	JVal root;
	if (json_parse(h, (size_t)hlen, &root) != Success) {
		const std::string why = inf_last_error_detail();
		return fail(ErrorInvalidValue, "%s: header: %s", path.c_str(), why.c_str());
	}
	if (root.kind != JVal::Obj) return fail(ErrorInvalidValue, "%s: header is not an object", path.c_str());
	std::unordered_set<std::string> seen;
	std::vector<std::pair<uint64_t, uint64_t>> spans;
	for (const auto& m2 : root.obj) {
		const std::string& name = m2.first;
		const JVal& v = m2.second;
		if (!seen.insert(name).second) return fail(ErrorInvalidValue, "%s: duplicate key \"%s\"", path.c_str(), name.c_str());
		if (name == "__metadata__") {
			if (v.kind != JVal::Obj) return fail(ErrorInvalidValue, "%s: __metadata__ is not an object", path.c_str());
			for (const auto& kv : v.obj)
				if (kv.second.kind != JVal::Str)
					return fail(ErrorInvalidValue, "%s: __metadata__ value \"%s\" is not a string", path.c_str(), kv.first.c_str());
			continue;
		}
		if (v.kind != JVal::Obj) return fail(ErrorInvalidValue, "%s: tensor \"%s\" is not an object", path.c_str(), name.c_str());
		const JVal* dt = v.get("dtype");
		const JVal* sh = v.get("shape");
		const JVal* of = v.get("data_offsets");
		if (!dt || dt->kind != JVal::Str || !sh || sh->kind != JVal::Arr || !of || of->kind != JVal::Arr || of->arr.size() != 2)
			return fail(ErrorInvalidValue, "%s: tensor \"%s\" needs dtype, shape and data_offsets [begin, end]", path.c_str(), name.c_str());
		StTensor t;
		t.dtype = dt->s;
		t.esize = dtype_size(t.dtype);
		t.file = fi;
		uint64_t elems = 1;
		for (const JVal& d : sh->arr) {
			if (d.kind != JVal::Num || !d.is_uint)
				return fail(ErrorInvalidValue, "%s: tensor \"%s\": shape entries must be non-negative integers", path.c_str(), name.c_str());
			if (d.u != 0 && elems > UINT64_MAX / d.u)
				return fail(ErrorInvalidValue, "%s: tensor \"%s\": shape overflows", path.c_str(), name.c_str());
			elems *= d.u;
			t.shape.push_back(d.u);
		}
		if (of->arr[0].kind != JVal::Num || !of->arr[0].is_uint || of->arr[1].kind != JVal::Num || !of->arr[1].is_uint)
			return fail(ErrorInvalidValue, "%s: tensor \"%s\": data_offsets must be non-negative integers", path.c_str(), name.c_str());
		t.begin = of->arr[0].u;
		t.end = of->arr[1].u;
		if (t.begin > t.end || t.end > buf_len)
			return fail(ErrorInvalidValue, "%s: tensor \"%s\": data_offsets [%llu, %llu] outside the %llu-byte buffer%s", path.c_str(),
			            name.c_str(), (unsigned long long)t.begin, (unsigned long long)t.end, (unsigned long long)buf_len,
			            t.end > buf_len ? " (truncated file?)" : "");
		if (t.esize) {
			if (elems > UINT64_MAX / (uint64_t)t.esize || elems * (uint64_t)t.esize != t.end - t.begin)
				return fail(ErrorInvalidValue, "%s: tensor \"%s\": %llu bytes for %llu elements of %s", path.c_str(), name.c_str(),
				            (unsigned long long)(t.end - t.begin), (unsigned long long)elems, t.dtype.c_str());
		}
		spans.emplace_back(t.begin, t.end);
		if (!ck->tensors.emplace(name, std::move(t)).second)
			return fail(ErrorInvalidValue, "%s: tensor \"%s\" is also in another file", path.c_str(), name.c_str());
	}
	// the byte buffer is indexed without holes or overlaps
	std::sort(spans.begin(), spans.end());
	uint64_t at = 0;
	for (const auto& s : spans) {
		if (s.first != at)
			return fail(ErrorInvalidValue, "%s: byte buffer has a %s at offset %llu", path.c_str(), s.first > at ? "hole" : "overlap",
			            (unsigned long long)std::min(s.first, at));
		at = s.second;
	}
	if (at != buf_len)
		return fail(ErrorInvalidValue, "%s: tensors index %llu of the %llu buffer bytes", path.c_str(), (unsigned long long)at,
		            (unsigned long long)buf_len);
	return Success;
}

} // namespace

Checkpoint::~Checkpoint()
{
	for (StFile& f : files) {
		if (f.map) munmap((void*)f.map, f.size);
		if (f.fd >= 0) close(f.fd);
	}
}

Error_t checkpoint_open(const char* path_c, Checkpoint* ck)
{
	if (!path_c || !ck) return fail(ErrorInvalidValue, "checkpoint: NULL argument");
	std::string path = path_c;
	struct stat st;
	if (stat(path.c_str(), &st) != 0) return fail(ErrorIo, "cannot open %s: %s", path.c_str(), strerror(errno));
	if (S_ISDIR(st.st_mode)) {
		const std::string idx = path + "/model.safetensors.index.json";
		path = stat(idx.c_str(), &st) == 0 ? idx : path + "/model.safetensors";
	}
	if (!ends_with(path, ".json")) return open_one(ck, path);

	// sharded checkpoint: {"metadata": {...}, "weight_map": {tensor name: shard file}}
	std::string text;
	INF_TRY(read_file(path, &text));
	JVal root;
	if (json_parse(text.data(), text.size(), &root) != Success) {
		const std::string why = inf_last_error_detail();
		return fail(ErrorInvalidValue, "%s: %s", path.c_str(), why.c_str());
	}
	const JVal* wm = root.get("weight_map");
	if (!wm || wm->kind != JVal::Obj || wm->obj.empty())
		return fail(ErrorInvalidValue, "%s: no \"weight_map\" object", path.c_str());
	const std::string dir = dir_of(path);
	std::vector<std::string> shards;
	for (const auto& m : wm->obj) {
		if (m.second.kind != JVal::Str || m.second.s.empty() || m.second.s.find('/') != std::string::npos)
			return fail(ErrorInvalidValue, "%s: weight_map entry \"%s\" is not a file name", path.c_str(), m.first.c_str());
		if (std::find(shards.begin(), shards.end(), m.second.s) == shards.end()) shards.push_back(m.second.s);
	}
	for (const std::string& s : shards) INF_TRY(open_one(ck, dir + "/" + s));
	for (const auto& m : wm->obj) {
		const auto it = ck->tensors.find(m.first);
		if (it == ck->tensors.end())
			return fail(ErrorInvalidValue, "%s: tensor \"%s\" is not in %s", path.c_str(), m.first.c_str(), m.second.s.c_str());
		if (ck->files[it->second.file].path != dir + "/" + m.second.s)
			return fail(ErrorInvalidValue, "%s: tensor \"%s\" is in %s, not %s", path.c_str(), m.first.c_str(),
			            ck->files[it->second.file].path.c_str(), m.second.s.c_str());
	}
	return Success;
}

// ============================================================================ the model's tensors
namespace {

struct Need {
	const StTensor* t;
	std::string name;
};

// "model." or "model.language_model." + suffix
const StTensor* find_model(const Checkpoint& ck, const std::string& suffix, std::string* name)
{
	static const char* const pre[] = {"model.", "model.language_model."};
	for (const char* p : pre) {
		const std::string n = std::string(p) + suffix;
		const auto it = ck.tensors.find(n);
		if (it != ck.tensors.end()) {
			*name = n;
			return &it->second;
		}
	}
	*name = std::string("model.") + suffix;
	return nullptr;
}

Error_t need(const Checkpoint& ck, const std::string& suffix, uint64_t r, uint64_t c, bool vec, Need* out)
{
	out->t = find_model(ck, suffix, &out->name);
	if (!out->t) return fail(ErrorInvalidValue, "checkpoint has no tensor %s (nor model.language_model.%s)", out->name.c_str(), suffix.c_str());
	const StTensor& t = *out->t;
	if (t.dtype != "BF16" && t.dtype != "F32")
		return fail(ErrorUnsupported, "%s: dtype %s (BF16 or F32 are read)", out->name.c_str(), t.dtype.c_str());
	const bool ok = vec ? (t.shape.size() == 1 && t.shape[0] == c) : (t.shape.size() == 2 && t.shape[0] == r && t.shape[1] == c);
	if (!ok) {
		std::string got;
		for (size_t i = 0; i < t.shape.size(); ++i) got += (i ? "," : "") + std::to_string(t.shape[i]);
		if (vec) return fail(ErrorBadConfig, "%s: shape [%s], the config implies [%llu]", out->name.c_str(), got.c_str(), (unsigned long long)c);
		return fail(ErrorBadConfig, "%s: shape [%s], the config implies [%llu,%llu]", out->name.c_str(), got.c_str(),
		            (unsigned long long)r, (unsigned long long)c);
	}
	return Success;
}

std::string lyr(int l, const char* s) { return "layers." + std::to_string(l) + "." + s; }

Error_t lm_head(const Checkpoint& ck, const InfConfig& c, Need* out)
{
	const auto it = ck.tensors.find("lm_head.weight");
	if (it == ck.tensors.end()) return need(ck, "embed_tokens.weight", c.vocab_size, c.dim, false, out); // tied
	out->t = &it->second;
	out->name = "lm_head.weight";
	const StTensor& t = *out->t;
	if (t.dtype != "BF16" && t.dtype != "F32") return fail(ErrorUnsupported, "lm_head.weight: dtype %s (BF16 or F32 are read)", t.dtype.c_str());
	if (t.shape.size() != 2 || t.shape[0] != c.vocab_size || t.shape[1] != c.dim)
		return fail(ErrorBadConfig, "lm_head.weight: shape does not match [%u,%u]", c.vocab_size, c.dim);
	return Success;
}

// The source tensors of one weight kind: up to three (qkv: q, k, v; gate/up: gate, up).
Error_t sources(const Checkpoint& ck, const InfConfig& c, int l, uint32_t kind, Need s[3])
{
	const uint64_t d = c.dim, hd = c.head_dim, H = c.n_heads, KV = c.n_kv_heads, F = c.ffn_dim, P = c.ple_dim;
	const bool gemma = c.arch == InfArchGemma;
	switch (kind) {
	case InfWEmbed: return need(ck, "embed_tokens.weight", c.vocab_size, d, false, &s[0]);
	case InfWLmHead: return lm_head(ck, c, &s[0]);
	case InfWFinalNorm: return need(ck, "norm.weight", 0, d, true, &s[0]);
	case InfWQkv:
		INF_TRY(need(ck, lyr(l, "self_attn.q_proj.weight"), H * hd, d, false, &s[0]));
		INF_TRY(need(ck, lyr(l, "self_attn.k_proj.weight"), KV * hd, d, false, &s[1]));
		return need(ck, lyr(l, "self_attn.v_proj.weight"), KV * hd, d, false, &s[2]);
	case InfWO: return need(ck, lyr(l, "self_attn.o_proj.weight"), d, H * hd, false, &s[0]);
	case InfWGateUp:
		INF_TRY(need(ck, lyr(l, "mlp.gate_proj.weight"), F, d, false, &s[0]));
		return need(ck, lyr(l, "mlp.up_proj.weight"), F, d, false, &s[1]);
	case InfWDown: return need(ck, lyr(l, "mlp.down_proj.weight"), d, F, false, &s[0]);
	case InfWAttnNorm: return need(ck, lyr(l, "input_layernorm.weight"), 0, d, true, &s[0]);
	// Llama normalises the MLP input with post_attention_layernorm; Gemma uses that name for the
	// norm of the attention output and pre_feedforward_layernorm for the MLP input
	case InfWFfnNorm:
		return need(ck, lyr(l, gemma ? "pre_feedforward_layernorm.weight" : "post_attention_layernorm.weight"), 0, d, true, &s[0]);
	}
	if (!gemma) return fail(ErrorInvalidValue, "weight kind %u", kind);
	switch (kind) {
	case InfWEmbedPle: return need(ck, "embed_tokens_per_layer.weight", c.vocab_size, c.n_layers * P, false, &s[0]);
	case InfWPleModelProj: return need(ck, "per_layer_model_projection.weight", c.n_layers * P, d, false, &s[0]);
	case InfWPleProjNorm: return need(ck, "per_layer_projection_norm.weight", 0, P, true, &s[0]);
	case InfWQNorm: return need(ck, lyr(l, "self_attn.q_norm.weight"), 0, hd, true, &s[0]);
	case InfWKNorm: return need(ck, lyr(l, "self_attn.k_norm.weight"), 0, hd, true, &s[0]);
	case InfWPostAttnNorm: return need(ck, lyr(l, "post_attention_layernorm.weight"), 0, d, true, &s[0]);
	case InfWPostFfnNorm: return need(ck, lyr(l, "post_feedforward_layernorm.weight"), 0, d, true, &s[0]);
	case InfWPleGate: return need(ck, lyr(l, "per_layer_input_gate.weight"), P, d, false, &s[0]);
	case InfWPleProj: return need(ck, lyr(l, "per_layer_projection.weight"), d, P, false, &s[0]);
	case InfWPlePostNorm: return need(ck, lyr(l, "post_per_layer_input_norm.weight"), 0, d, true, &s[0]);
	default: return fail(ErrorInvalidValue, "weight kind %u", kind);
	}
}

const uint32_t kLayerKinds[] = {InfWQkv, InfWO, InfWGateUp, InfWDown, InfWAttnNorm, InfWFfnNorm};
const uint32_t kModelKinds[] = {InfWEmbed, InfWLmHead, InfWFinalNorm};
const uint32_t kGemmaLayerKinds[] = {InfWQNorm, InfWKNorm, InfWPostAttnNorm, InfWPostFfnNorm};
const uint32_t kGemmaPleLayerKinds[] = {InfWPleGate, InfWPleProj, InfWPlePostNorm};
const uint32_t kGemmaPleModelKinds[] = {InfWEmbedPle, InfWPleModelProj, InfWPleProjNorm};

inline uint16_t f32_to_bf16_rne(uint32_t u)
{
	if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x0040u); // quiet NaN
	return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// cols source elements starting at src, converted to the model dtype, to dst
void convert_row(const unsigned char* src, bool src_f32, bool dst_bf16, uint64_t cols, void* dst)
{
	if (src_f32 == !dst_bf16) {
		memcpy(dst, src, cols * (src_f32 ? 4 : 2));
	} else if (src_f32) { // F32 -> bf16
		uint16_t* o = (uint16_t*)dst;
		for (uint64_t i = 0; i < cols; ++i) {
			uint32_t u;
			memcpy(&u, src + 4 * i, 4);
			o[i] = f32_to_bf16_rne(u);
		}
	} else { // BF16 -> f32, exact
		uint32_t* o = (uint32_t*)dst;
		for (uint64_t i = 0; i < cols; ++i) {
			uint16_t h;
			memcpy(&h, src + 2 * i, 2);
			o[i] = (uint32_t)h << 16;
		}
	}
}

} // namespace

// A tensor under the decoder's prefix that this decoder does not use changes the model's
// function (q/k norms, extra norms, biases, per-layer embeddings of other families): refuse
// it rather than run a different model.  Buffers that carry no weights are allowed.
bool decoder_tensor_known(const std::string& rest, const InfConfig& c)
{
	const bool gemma = c.arch == InfArchGemma, ple = gemma && c.ple_dim > 0;
	static const char* const top[] = {"embed_tokens.weight", "norm.weight"};
	for (const char* t : top)
		if (rest == t) return true;
	static const char* const top_ple[] = {"embed_tokens_per_layer.weight", "per_layer_model_projection.weight",
	                                      "per_layer_projection_norm.weight"};
	if (ple)
		for (const char* t : top_ple)
			if (rest == t) return true;
	if (rest.compare(0, 7, "layers.") != 0) return false;
	size_t k = 7;
	while (k < rest.size() && rest[k] >= '0' && rest[k] <= '9') ++k;
	if (k == 7 || k >= rest.size() || rest[k] != '.') return false;
	const std::string leaf = rest.substr(k + 1);
	static const char* const used[] = {
	    "input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
	    "self_attn.v_proj.weight", "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
	    "mlp.down_proj.weight", "self_attn.rotary_emb.inv_freq", // a RoPE buffer some exports keep: no weights
	};
	for (const char* u : used)
		if (leaf == u) return true;
	static const char* const used_gemma[] = {"self_attn.q_norm.weight", "self_attn.k_norm.weight",
	                                         "pre_feedforward_layernorm.weight", "post_feedforward_layernorm.weight"};
	static const char* const used_ple[] = {"per_layer_input_gate.weight", "per_layer_projection.weight",
	                                       "post_per_layer_input_norm.weight"};
	if (gemma)
		for (const char* u : used_gemma)
			if (leaf == u) return true;
	if (ple)
		for (const char* u : used_ple)
			if (leaf == u) return true;
	return false;
}

Error_t checkpoint_check(const Checkpoint& ck, const InfConfig& c)
{
	const bool gemma = c.arch == InfArchGemma, ple = gemma && c.ple_dim > 0;
	Need s[3];
	for (uint32_t k : kModelKinds)
		if (!(gemma && k == InfWLmHead)) INF_TRY(sources(ck, c, 0, k, s));
	if (ple)
		for (uint32_t k : kGemmaPleModelKinds) INF_TRY(sources(ck, c, 0, k, s));
	for (uint32_t l = 0; l < c.n_layers; ++l) {
		for (uint32_t k : kLayerKinds) INF_TRY(sources(ck, c, (int)l, k, s));
		if (gemma)
			for (uint32_t k : kGemmaLayerKinds) INF_TRY(sources(ck, c, (int)l, k, s));
		if (ple)
			for (uint32_t k : kGemmaPleLayerKinds) INF_TRY(sources(ck, c, (int)l, k, s));
	}
	if (gemma && ck.tensors.count("lm_head.weight"))
		return fail(ErrorUnsupported, "lm_head.weight: a Gemma-style model's LM head is its embedding (tied)");
	// the prefix the embedding was found under is the decoder's
	std::string emb;
	find_model(ck, "embed_tokens.weight", &emb);
	const std::string prefix = emb.substr(0, emb.size() - strlen("embed_tokens.weight"));
	for (const auto& t : ck.tensors) {
		const std::string& n = t.first;
		if (n.compare(0, prefix.size(), prefix) != 0) continue; // another component (vision tower, ...)
		if (prefix == "model." && n.compare(0, 21, "model.language_model.") == 0) continue;
		if (!decoder_tensor_known(n.substr(prefix.size()), c))
			return fail(ErrorUnsupported, "%s: a tensor this %s decoder does not implement (its model would compute "
			            "something else)", n.c_str(), gemma ? "Gemma-style" : "Llama");
	}
	return Success;
}

void weight_dims(const InfConfig& c, uint32_t kind, uint64_t* rows, uint64_t* cols)
{
	const uint64_t tp = c.tp_size ? c.tp_size : 1, d = c.dim, hd = c.head_dim;
	const uint64_t Hl = c.n_heads / tp, KVl = c.n_kv_heads / tp, Fl = c.ffn_dim / tp;
	uint64_t r = 1, k = d;
	switch (kind) {
	case InfWEmbed: r = c.vocab_size; break;
	case InfWLmHead: r = c.vocab_size / tp; break;
	case InfWQkv: r = (Hl + 2 * KVl) * hd; break;
	case InfWO: r = d; k = Hl * hd; break;
	case InfWGateUp: r = 2 * Fl; break;
	case InfWDown: r = d; k = Fl; break;
	case InfWEmbedPle: r = c.vocab_size; k = (uint64_t)c.n_layers * c.ple_dim; break;
	case InfWPleModelProj: r = (uint64_t)c.n_layers * c.ple_dim; break;
	case InfWPleProjNorm: k = c.ple_dim; break;
	case InfWQNorm: case InfWKNorm: k = hd; break;
	case InfWPleGate: r = c.ple_dim; break;
	case InfWPleProj: r = d; k = c.ple_dim; break;
	default: break; // gains: one row of dim
	}
	*rows = r;
	*cols = k;
}

Error_t weight_rows(const Checkpoint& ck, const InfConfig& c, int l, uint32_t kind, uint64_t row0, uint64_t n, void* dst)
{
	Need s[3];
	INF_TRY(sources(ck, c, l, kind, s));
	uint64_t rows, cols;
	weight_dims(c, kind, &rows, &cols);
	if (row0 > rows || n > rows - row0) return fail(ErrorInvalidValue, "rows [%llu, +%llu) of %llu", (unsigned long long)row0, (unsigned long long)n, (unsigned long long)rows);
	const uint64_t tp = c.tp_size ? c.tp_size : 1, rk = c.tp_rank, hd = c.head_dim;
	const uint64_t Hl = c.n_heads / tp, KVl = c.n_kv_heads / tp, Fl = c.ffn_dim / tp;
	const bool dst_bf16 = c.dtype == InfBF16;
	const uint64_t dst_row = cols * (dst_bf16 ? 2 : 4);
	for (uint64_t i = 0; i < n; ++i) {
		const uint64_t r = row0 + i;
		const StTensor* t = s[0].t;
		uint64_t crow = r, col0 = 0;
		switch (kind) {
		case InfWLmHead: crow = rk * (c.vocab_size / tp) + r; break;
		case InfWQkv: { // head rows in (i, i + hd/2) pairs: device row 2j is dim j, 2j+1 is dim j + hd/2
			const uint64_t head = r / hd, rr = r % hd;
			const uint64_t dim = (rr & 1) ? (rr >> 1) + hd / 2 : (rr >> 1);
			if (head < Hl) {
				crow = (rk * Hl + head) * hd + dim;
			} else if (head < Hl + KVl) {
				t = s[1].t;
				crow = (rk * KVl + head - Hl) * hd + dim;
			} else {
				t = s[2].t;
				crow = (rk * KVl + head - Hl - KVl) * hd + dim;
			}
			break;
		}
		case InfWO: col0 = rk * Hl * hd; break;
		case InfWGateUp:
			t = s[r & 1].t;
			crow = rk * Fl + (r >> 1);
			break;
		case InfWDown: col0 = rk * Fl; break;
		default: break;
		}
		const bool src_f32 = t->dtype == "F32";
		const uint64_t ccols = t->shape.size() == 2 ? t->shape[1] : t->shape[0];
		const uint64_t es = src_f32 ? 4 : 2;
		convert_row(ck.data(*t) + (crow * ccols + col0) * es, src_f32, dst_bf16, cols, (unsigned char*)dst + i * dst_row);
	}
	return Success;
}

Error_t weight_rows_parallel(const Checkpoint& ck, const InfConfig& c, int l, uint32_t kind, uint64_t row0, uint64_t n,
                             void* dst)
{
	uint64_t rows, cols;
	weight_dims(c, kind, &rows, &cols);
	const uint64_t row_bytes = cols * (c.dtype == InfBF16 ? 2 : 4);
	const unsigned hw = std::thread::hardware_concurrency();
	const int threads = (int)std::min<uint64_t>(std::min(16u, hw ? hw : 1u), n * row_bytes / (1u << 20) + 1); // >= 1 MB each
	if (threads <= 1) return weight_rows(ck, c, l, kind, row0, n, dst);
	const uint64_t per = (n + threads - 1) / threads;
	std::vector<Error_t> err((size_t)threads, Success);
	std::vector<std::thread> pool;
	for (int t = 0; t < threads; ++t) {
		const uint64_t a = (uint64_t)t * per;
		if (a >= n) break;
		const uint64_t m = std::min(per, n - a);
		pool.emplace_back([&, t, a, m] { err[(size_t)t] = weight_rows(ck, c, l, kind, row0 + a, m, (unsigned char*)dst + a * row_bytes); });
	}
	for (std::thread& th : pool) th.join();
	for (int t = 0; t < (int)pool.size(); ++t)
		if (err[(size_t)t] != Success) { // again on this thread, for the error detail
			const uint64_t a = (uint64_t)t * per;
			return weight_rows(ck, c, l, kind, row0 + a, std::min(per, n - a), (unsigned char*)dst + a * row_bytes);
		}
	return Success;
}

Error_t checkpoint_upload(const Checkpoint& ck, const InfConfig& c, const std::vector<WeightDst>& dsts, cudaStream_t stream)
{
	constexpr uint64_t kStage = 64ull << 20;
	void* buf[2] = {nullptr, nullptr};
	cudaEvent_t ev[2] = {nullptr, nullptr};
	Error_t r = Success;
	auto cu = [&](cudaError_t e, const char* what) {
		if (e != cudaSuccess && r == Success) r = fail(ErrorCuda, "checkpoint upload: %s: %s", what, cudaGetErrorString(e));
		return r == Success;
	};
	bool ok = cu(cudaMallocHost(&buf[0], kStage), "cudaMallocHost") && cu(cudaMallocHost(&buf[1], kStage), "cudaMallocHost") &&
	          cu(cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming), "cudaEventCreate") &&
	          cu(cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming), "cudaEventCreate");
	bool used[2] = {false, false};
	int b = 0;
	const uint64_t es = c.dtype == InfBF16 ? 2 : 4;
	for (size_t w = 0; ok && w < dsts.size(); ++w) {
		uint64_t rows, cols;
		weight_dims(c, dsts[w].kind, &rows, &cols);
		const uint64_t row_bytes = cols * es;
		const uint64_t per = std::max<uint64_t>(1, kStage / row_bytes); // rows of one staging buffer (a row is <= 64 KB)
		for (uint64_t r0 = 0; ok && r0 < rows; r0 += per) {
			const uint64_t n = std::min(per, rows - r0);
			if (used[b]) ok = cu(cudaEventSynchronize(ev[b]), "cudaEventSynchronize"); // its previous copy is done
			if (!ok) break;
			const Error_t e = weight_rows_parallel(ck, c, dsts[w].layer, dsts[w].kind, r0, n, buf[b]);
			if (e != Success) {
				r = e;
				ok = false;
				break;
			}
			ok = cu(cudaMemcpyAsync((unsigned char*)dsts[w].dst + r0 * row_bytes, buf[b], n * row_bytes, cudaMemcpyHostToDevice, stream),
			        "cudaMemcpyAsync") &&
			     cu(cudaEventRecord(ev[b], stream), "cudaEventRecord");
			used[b] = true;
			b ^= 1;
		}
	}
	// drain before the staging buffers go away, on every path
	for (int i = 0; i < 2; ++i)
		if (used[i]) cu(cudaEventSynchronize(ev[i]), "cudaEventSynchronize");
	for (int i = 0; i < 2; ++i) {
		if (ev[i]) cudaEventDestroy(ev[i]);
		if (buf[i]) cudaFreeHost(buf[i]);
	}
	return r;
}

// ============================================================================ config.json
Error_t config_from_json(const char* path, InfConfig* c)
{
	if (!path || !c) return fail(ErrorInvalidValue, "inf_config_from_json: NULL argument");
	std::string text;
	INF_TRY(read_file(path, &text));
	JVal root;
	if (json_parse(text.data(), text.size(), &root) != Success) {
		const std::string why = inf_last_error_detail();
		return fail(ErrorInvalidValue, "%s: %s", path, why.c_str());
	}
	if (root.kind != JVal::Obj) return fail(ErrorInvalidValue, "%s: not a JSON object", path);
	const JVal* tc = root.get("text_config");
	const JVal& m = (tc && tc->kind == JVal::Obj) ? *tc : root;
	InfConfig o = *c;
	auto u32f = [&](const char* key, u32* out) -> Error_t {
		const JVal* v = m.get(key);
		if (!v || v->kind == JVal::Null) return Success;
		if (v->kind != JVal::Num || !v->is_uint || v->u == 0 || v->u > 0xFFFFFFFFull)
			return fail(ErrorInvalidValue, "%s: \"%s\" must be a positive 32-bit integer", path, key);
		*out = (u32)v->u;
		return Success;
	};
	auto f32f = [&](const char* key, f32* out) -> Error_t {
		const JVal* v = m.get(key);
		if (!v || v->kind == JVal::Null) return Success;
		if (v->kind != JVal::Num || !std::isfinite(v->num) || v->num < 0) return fail(ErrorInvalidValue, "%s: \"%s\" must be a non-negative number", path, key);
		*out = (f32)v->num;
		return Success;
	};
	INF_TRY(u32f("hidden_size", &o.dim));
	INF_TRY(u32f("intermediate_size", &o.ffn_dim));
	INF_TRY(u32f("num_hidden_layers", &o.n_layers));
	INF_TRY(u32f("num_attention_heads", &o.n_heads));
	INF_TRY(u32f("vocab_size", &o.vocab_size));
	if (m.get("num_attention_heads") && !m.get("num_key_value_heads")) o.n_kv_heads = o.n_heads; // multi-head attention
	INF_TRY(u32f("num_key_value_heads", &o.n_kv_heads));
	const JVal* hdv = m.get("head_dim");
	if (hdv && hdv->kind != JVal::Null) INF_TRY(u32f("head_dim", &o.head_dim));
	else if (m.get("hidden_size") || m.get("num_attention_heads")) {
		if (o.n_heads == 0 || o.dim % o.n_heads) return fail(ErrorInvalidValue, "%s: hidden_size is not a multiple of num_attention_heads", path);
		o.head_dim = o.dim / o.n_heads;
	}
	INF_TRY(f32f("rms_norm_eps", &o.norm_eps));
	INF_TRY(f32f("rope_theta", &o.rope_theta));
	const JVal* dt = m.get("torch_dtype");
	if (!dt) dt = m.get("dtype");
	if (dt && dt->kind != JVal::Null) {
		if (dt->kind != JVal::Str) return fail(ErrorInvalidValue, "%s: torch_dtype is not a string", path);
		if (dt->s == "bfloat16") o.dtype = InfBF16;
		else if (dt->s == "float32") o.dtype = InfF32;
		else return fail(ErrorUnsupported, "%s: torch_dtype %s (bfloat16 or float32)", path, dt->s.c_str());
	}
	// what the decoder does not implement is refused, not ignored
	const JVal* mt = m.get("model_type");
	const bool gemma = mt && mt->kind == JVal::Str && mt->s.compare(0, 5, "gemma") == 0;
	if (mt && mt->kind == JVal::Str && mt->s != "llama" && !gemma)
		return fail(ErrorUnsupported, "%s: model_type %s (the Llama and Gemma-style decoders only)", path, mt->s.c_str());
	o.arch = gemma ? InfArchGemma : InfArchLlama;
	if (gemma) {
		// the reference reads global_head_dim (src/main.cu:152); every layer uses it here
		const JVal* g = m.get("global_head_dim");
		if (g && g->kind != JVal::Null) INF_TRY(u32f("global_head_dim", &o.head_dim));
		o.ple_dim = 0;
		INF_TRY(u32f("hidden_size_per_layer_input", &o.ple_dim));
		o.final_softcap = 0.0f;
		INF_TRY(f32f("final_logit_softcapping", &o.final_softcap));
		// Gemma variants whose blocks this decoder does not compute
		for (const char* k : {"altup_num_inputs", "laurel_rank", "num_kv_shared_layers", "attn_logit_softcapping",
		                      "sliding_window"}) {
			const JVal* v = m.get(k);
			const bool set = v && v->kind != JVal::Null && !(v->kind == JVal::Num && v->num == 0) &&
			                 !(v->kind == JVal::Bool && !v->b);
			if (set) return fail(ErrorUnsupported, "%s: %s (not implemented by the Gemma-style decoder)", path, k);
		}
		const JVal* qs = m.get("query_pre_attn_scalar");
		if (qs && qs->kind == JVal::Num && qs->num != (double)o.head_dim)
			return fail(ErrorUnsupported, "%s: query_pre_attn_scalar %g (the scale is 1/sqrt(head_dim))", path, qs->num);
	}
	for (const char* key : {"hidden_act", "hidden_activation"}) {
		const JVal* act = m.get(key);
		const char* want = gemma ? "gelu_pytorch_tanh" : "silu";
		if (act && act->kind == JVal::Str && act->s != want)
			return fail(ErrorUnsupported, "%s: %s %s (%s)", path, key, act->s.c_str(), want);
	}
	for (const char* k : {"attention_bias", "mlp_bias"}) {
		const JVal* v = m.get(k);
		if (v && v->kind == JVal::Bool && v->b) return fail(ErrorUnsupported, "%s: %s (projections have no bias)", path, k);
	}
	const JVal* rs = m.get("rope_scaling");
	if (rs && rs->kind == JVal::Obj) {
		const JVal* ty = rs->get("rope_type");
		if (!ty) ty = rs->get("type");
		if (!ty || ty->kind != JVal::Str || ty->s != "default")
			return fail(ErrorUnsupported, "%s: rope_scaling %s (plain RoPE only)", path, ty && ty->kind == JVal::Str ? ty->s.c_str() : "?");
	}
	*c = o;
	return Success;
}

} // namespace inf
