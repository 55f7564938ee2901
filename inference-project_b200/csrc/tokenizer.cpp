// Host tokenizer: the BPE encoder of a Hugging Face tokenizer.json and the decoder the
// reference declares but never defines.
//
// Replaces tokenizer_build / tokenizer_encode / tokenizer_destroy (src/tokenizer.c:39-278)
// and tokenizer_decode (declared src/tokenizer.h:38).  The segmentation and the merge order
// are the reference's: words split at ' ', every word after the first prefixed with U+2581
// ("▁"), characters by the reference's UTF-8 lead-byte rule, and per round the pair of lowest
// merge rank merged at all its non-overlapping occurrences, left to right, until no adjacent
// pair has a rank.  Differences, each deliberate:
//  - a final piece outside the vocabulary becomes byte tokens (<0xXX>, when the model has
//    byte_fallback) or the unk token, else an error; the reference drops it and still counts
//    it in the returned length (defect D13);
//  - a text that starts with a space has an empty first word that yields nothing (the
//    reference indexes its piece array at [UINT32_MAX] there);
//  - a character's bytes never reach past its word (the reference copies the lead-byte count
//    even when the text ends first);
//  - merge pairs are keyed by symbol, not by the string "left right", so tokens that contain
//    spaces cannot collide, and the first of duplicate merges wins;
//  - a round costs O(log n) per merged pair (a heap of candidate pairs over a linked list of
//    pieces) instead of a rescan of the word, so long unspaced text stays linear-logarithmic.
#include <algorithm>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "loader.h"
#include "runtime.h"

using namespace inf;

namespace {
constexpr uint32_t kNoSym = 0xFFFFFFFFu;
constexpr uint32_t kNoRank = 0xFFFFFFFFu;
const char kSpaceMark[] = "\xE2\x96\x81"; // U+2581, SentencePiece's word boundary
}

struct InfTokenizer {
	std::unordered_map<std::string, uint32_t> sym_of; // interned piece strings
	std::vector<std::string> sym_str;
	std::vector<int64_t> sym_id;                      // vocabulary id of a symbol, -1 if none
	std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> merges; // (left, right) -> (rank, merged)
	std::vector<std::string> piece;                   // by id, for decoding
	std::vector<uint8_t> has_piece;
	int64_t byte_id[256];
	bool byte_fallback = false;
	int64_t unk_id = -1;
	// added tokens marked "special", by first byte, longest first (inf_tokenizer_encode_special)
	std::vector<std::pair<std::string, uint32_t>> specials;
	std::vector<std::vector<uint32_t>> special_by_byte = std::vector<std::vector<uint32_t>>(256);

	uint32_t intern(const std::string& s)
	{
		const auto it = sym_of.find(s);
		if (it != sym_of.end()) return it->second;
		const uint32_t k = (uint32_t)sym_str.size();
		sym_of.emplace(s, k);
		sym_str.push_back(s);
		sym_id.push_back(-1);
		return k;
	}
	uint32_t find(const char* p, size_t n) const
	{
		const auto it = sym_of.find(std::string(p, n));
		return it == sym_of.end() ? kNoSym : it->second;
	}
};

namespace {

// the reference's character length rule (src/tokenizer.c:24-37)
inline uint32_t utf8_len(unsigned char c) { return c < 0x80 ? 1 : c < 0xE0 ? 2 : c < 0xF0 ? 3 : 4; }

struct Node {
	uint32_t begin, end, sym;
	int32_t prev, next;
};

struct Cand {
	uint32_t rank, pos; // pos: the left piece's first byte, unique among live pieces
	int32_t left, right;
	uint32_t lsym, rsym;
	bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : pos > o.pos; }
};

// Buffers of one encode call, reused word to word.
struct Work {
	std::vector<Node> nodes, pieces;
	std::vector<Cand> heap; // min-heap by (rank, pos) through std::push_heap / pop_heap
	std::vector<char> alive;
	std::vector<int32_t> touched;
};

// BPE over one word (already prefixed); leaves the final pieces' (begin, end, sym) in W.pieces.
void bpe_word(const InfTokenizer& t, const std::string& w, Work& W)
{
	std::vector<Node>& nodes = W.nodes;
	W.pieces.clear();
	nodes.clear();
	for (uint32_t i = 0; i < w.size();) {
		const uint32_t n = std::min<uint32_t>(utf8_len((unsigned char)w[i]), (uint32_t)w.size() - i);
		nodes.push_back({i, i + n, t.find(w.data() + i, n), (int32_t)nodes.size() - 1, (int32_t)nodes.size() + 1});
		i += n;
	}
	if (nodes.empty()) return;
	nodes.back().next = -1;
	auto rank_of = [&](int32_t a, int32_t b, uint32_t* merged) {
		if (nodes[a].sym == kNoSym || nodes[b].sym == kNoSym) return kNoRank;
		const auto it = t.merges.find(((uint64_t)nodes[a].sym << 32) | nodes[b].sym);
		if (it == t.merges.end()) return kNoRank;
		*merged = it->second.second;
		return it->second.first;
	};
	std::vector<Cand>& heap = W.heap;
	heap.clear();
	const auto later = std::greater<Cand>();
	auto push = [&](int32_t a) {
		if (a < 0 || nodes[a].next < 0) return;
		const int32_t b = nodes[a].next;
		uint32_t m;
		const uint32_t r = rank_of(a, b, &m);
		if (r == kNoRank) return;
		heap.push_back({r, nodes[a].begin, a, b, nodes[a].sym, nodes[b].sym});
		std::push_heap(heap.begin(), heap.end(), later);
	};
	for (int32_t i = 0; i + 1 < (int32_t)nodes.size(); ++i) push(i);
	std::vector<char>& alive = W.alive;
	alive.assign(nodes.size(), 1);
	std::vector<int32_t>& touched = W.touched;
	while (!heap.empty()) {
		// one round: every live occurrence of the lowest-rank pair, left to right; pairs the
		// round creates join the heap after it
		const uint32_t r = heap.front().rank;
		touched.clear();
		while (!heap.empty() && heap.front().rank == r) {
			std::pop_heap(heap.begin(), heap.end(), later);
			const Cand c = heap.back();
			heap.pop_back();
			if (!alive[c.left] || !alive[c.right] || nodes[c.left].next != c.right || nodes[c.left].sym != c.lsym ||
			    nodes[c.right].sym != c.rsym)
				continue; // stale: a piece of it was merged earlier in this round or before
			uint32_t m = kNoSym;
			rank_of(c.left, c.right, &m);
			Node& L = nodes[c.left];
			const Node& R = nodes[c.right];
			L.end = R.end;
			L.sym = m;
			L.next = R.next;
			if (R.next >= 0) nodes[R.next].prev = c.left;
			alive[c.right] = 0;
			touched.push_back(c.left);
		}
		for (int32_t a : touched) {
			if (!alive[a]) continue;
			if (nodes[a].prev >= 0) push(nodes[a].prev);
			push(a);
		}
	}
	for (int32_t i = 0; i >= 0; i = nodes[i].next) W.pieces.push_back(nodes[i]);
}

// Appends the ids of one final piece; false if it has none.
bool emit(const InfTokenizer& t, const std::string& w, const Node& n, std::vector<uint32_t>& ids)
{
	if (n.sym != kNoSym && t.sym_id[n.sym] >= 0) {
		ids.push_back((uint32_t)t.sym_id[n.sym]);
		return true;
	}
	if (t.byte_fallback) {
		bool all = true;
		for (uint32_t i = n.begin; i < n.end; ++i) all = all && t.byte_id[(unsigned char)w[i]] >= 0;
		if (all) {
			for (uint32_t i = n.begin; i < n.end; ++i) ids.push_back((uint32_t)t.byte_id[(unsigned char)w[i]]);
			return true;
		}
	}
	if (t.unk_id >= 0) {
		ids.push_back((uint32_t)t.unk_id);
		return true;
	}
	return false;
}

bool parse_byte_token(const std::string& s, int* b)
{
	if (s.size() != 6 || s.compare(0, 3, "<0x") != 0 || s[5] != '>') return false;
	int v = 0;
	for (int i = 3; i < 5; ++i) {
		const char c = s[i];
		v <<= 4;
		if (c >= '0' && c <= '9') v |= c - '0';
		else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
		else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
		else return false;
	}
	*b = v;
	return true;
}

Error_t build(const char* path, InfTokenizer* t)
{
	std::string text;
	{
		FILE* f = fopen(path, "rb");
		if (!f) return fail(ErrorIo, "cannot open %s", path);
		char buf[1 << 16];
		size_t n;
		while ((n = fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, n);
		const bool err = ferror(f) != 0;
		fclose(f);
		if (err) return fail(ErrorIo, "cannot read %s", path);
	}
	JVal root;
	if (json_parse(text.data(), text.size(), &root) != Success) {
		const std::string why = inf_last_error_detail();
		return fail(ErrorInvalidValue, "%s: %s", path, why.c_str());
	}
	text.clear();
	text.shrink_to_fit();
	const JVal* model = root.get("model");
	if (!model || model->kind != JVal::Obj) return fail(ErrorInvalidValue, "%s: no \"model\" object", path);
	const JVal* type = model->get("type");
	if (type && type->kind == JVal::Str && type->s != "BPE") return fail(ErrorUnsupported, "%s: model type %s (BPE)", path, type->s.c_str());
	// byte-level BPE (GPT-2 / Llama-3 style) maps bytes to printable characters and splits text
	// with a regex first; this segmentation is the reference's SentencePiece-style one, so such
	// a tokenizer would give other ids: refuse it
	auto byte_level = [](const JVal* v) {
		if (!v || v->kind != JVal::Obj) return false;
		const JVal* t = v->get("type");
		if (t && t->kind == JVal::Str && t->s == "ByteLevel") return true;
		const JVal* seq = v->get("pretokenizers");
		if (seq && seq->kind == JVal::Arr)
			for (const JVal& x : seq->arr) {
				const JVal* tt = x.get("type");
				if (tt && tt->kind == JVal::Str && tt->s == "ByteLevel") return true;
			}
		return false;
	};
	if (byte_level(root.get("pre_tokenizer")) || byte_level(root.get("decoder")))
		return fail(ErrorUnsupported, "%s: a byte-level BPE tokenizer (its regex pre-tokenizer is not implemented)", path);
	const JVal* vocab = model->get("vocab");
	if (!vocab || vocab->kind != JVal::Obj) return fail(ErrorInvalidValue, "%s: no \"model\".\"vocab\" object", path);
	const JVal* merges = model->get("merges");
	if (!merges || merges->kind != JVal::Arr) return fail(ErrorInvalidValue, "%s: no \"model\".\"merges\" array", path);
	for (int i = 0; i < 256; ++i) t->byte_id[i] = -1;
	auto set_piece = [&](uint64_t id, const std::string& s) {
		if (id >= t->piece.size()) {
			t->piece.resize(id + 1);
			t->has_piece.resize(id + 1, 0);
		}
		if (!t->has_piece[id]) {
			t->piece[id] = s;
			t->has_piece[id] = 1;
		}
	};
	for (const auto& m : vocab->obj) {
		if (m.second.kind != JVal::Num || !m.second.is_uint || m.second.u > 0x7FFFFFFFull)
			return fail(ErrorInvalidValue, "%s: vocab id of \"%s\" is not an integer in [0, 2^31)", path, m.first.c_str());
		const uint32_t s = t->intern(m.first);
		if (t->sym_id[s] < 0) t->sym_id[s] = (int64_t)m.second.u;
		set_piece(m.second.u, m.first);
		int b;
		if (parse_byte_token(m.first, &b) && t->byte_id[b] < 0) t->byte_id[b] = (int64_t)m.second.u;
	}
	uint32_t rank = 0;
	for (const JVal& m : merges->arr) {
		std::string l, r;
		if (m.kind == JVal::Arr && m.arr.size() == 2 && m.arr[0].kind == JVal::Str && m.arr[1].kind == JVal::Str) {
			l = m.arr[0].s;
			r = m.arr[1].s;
		} else if (m.kind == JVal::Str && m.s.find(' ') != std::string::npos) { // legacy "left right"
			const size_t k = m.s.find(' ');
			l = m.s.substr(0, k);
			r = m.s.substr(k + 1);
		} else {
			return fail(ErrorInvalidValue, "%s: merge %u is neither [left, right] nor \"left right\"", path, rank);
		}
		const uint32_t a = t->intern(l), b = t->intern(r), c = t->intern(l + r);
		t->merges.emplace(((uint64_t)a << 32) | b, std::make_pair(rank, c)); // the first of duplicates wins
		++rank;
	}
	const JVal* bf = model->get("byte_fallback");
	t->byte_fallback = bf && bf->kind == JVal::Bool && bf->b;
	const JVal* unk = model->get("unk_token");
	if (unk && unk->kind == JVal::Str) {
		const auto it = t->sym_of.find(unk->s);
		if (it != t->sym_of.end()) t->unk_id = t->sym_id[it->second];
	}
	const JVal* added = root.get("added_tokens");
	if (added && added->kind == JVal::Arr)
		for (const JVal& a : added->arr) {
			const JVal* id = a.get("id");
			const JVal* content = a.get("content");
			if (id && id->kind == JVal::Num && id->is_uint && id->u <= 0x7FFFFFFFull && content && content->kind == JVal::Str) {
				set_piece(id->u, content->s);
				const JVal* sp = a.get("special");
				if (sp && sp->kind == JVal::Bool && sp->b && !content->s.empty())
					t->specials.emplace_back(content->s, (uint32_t)id->u);
			}
		}
	for (uint32_t k = 0; k < t->specials.size(); ++k)
		t->special_by_byte[(unsigned char)t->specials[k].first[0]].push_back(k);
	for (auto& v : t->special_by_byte)
		std::sort(v.begin(), v.end(), [&](uint32_t x, uint32_t y) { return t->specials[x].first.size() > t->specials[y].first.size(); });
	return Success;
}

} // namespace

extern "C" {

Error_t inf_tokenizer_build(const char* tokenizer_json_path, InfTokenizer** out)
{
	if (!tokenizer_json_path || !out) return fail(ErrorInvalidValue, "inf_tokenizer_build: NULL argument");
	*out = nullptr;
	InfTokenizer* t = new (std::nothrow) InfTokenizer();
	if (!t) return fail(ErrorMemoryAllocation, "tokenizer");
	const Error_t e = build(tokenizer_json_path, t);
	if (e != Success) {
		delete t;
		return e;
	}
	*out = t;
	return Success;
}

Error_t inf_tokenizer_destroy(InfTokenizer** tok)
{
	if (!tok || !*tok) return fail(ErrorInvalidValue, "inf_tokenizer_destroy: no tokenizer");
	delete *tok;
	*tok = nullptr;
	return Success;
}

u32 inf_tokenizer_vocab_size(const InfTokenizer* tok) { return tok ? (u32)tok->piece.size() : 0; }

} // extern "C"

namespace {

// One encode call's state: the ids so far and, because words repeat (natural text is
// Zipf-distributed), the ids of short words already encoded.
struct Encoder {
	const InfTokenizer& tok;
	std::vector<uint32_t> out;
	Work W;
	std::unordered_map<std::string, std::pair<uint32_t, uint32_t>> seen; // word -> (first id in out, count)
	std::string w;
	explicit Encoder(const InfTokenizer& t) : tok(t) {}

	// text[p, end) as a whole text: words split at ' ', "▁" before every word but the first
	Error_t text(const char* p, const char* end);
	Error_t finish(u32* ids, u64 max_ids, u64* n_ids) const
	{
		*n_ids = out.size();
		if (!ids) return Success;
		if (out.size() > max_ids) return fail(ErrorInvalidValue, "%zu ids, room for %llu", out.size(), (unsigned long long)max_ids);
		std::copy(out.begin(), out.end(), ids);
		return Success;
	}
};

Error_t Encoder::text(const char* p, const char* end)
{
	constexpr size_t kMemoWord = 48, kMemoWords = 1 << 16;
	bool first = true;
	while (p < end) {
		const char* l = p;
		while (p < end && *p != ' ') ++p;
		w.clear();
		if (!first) w = kSpaceMark;
		w.append(l, (size_t)(p - l));
		first = false;
		if (p < end && *p == ' ') ++p;
		if (w.size() <= kMemoWord) {
			const auto it = seen.find(w);
			if (it != seen.end()) {
				const uint32_t at = it->second.first, n = it->second.second;
				for (uint32_t i = 0; i < n; ++i) out.push_back(out[at + i]);
				continue;
			}
		}
		const size_t at = out.size();
		bpe_word(tok, w, W);
		for (const Node& n : W.pieces)
			if (!emit(tok, w, n, out))
				return fail(ErrorInvalidValue, "piece \"%s\" is not in the vocabulary and the model has neither byte fallback nor an unk token",
				            w.substr(n.begin, n.end - n.begin).c_str());
		if (w.size() <= kMemoWord && seen.size() < kMemoWords && at <= 0xFFFFFFFFull)
			seen.emplace(w, std::make_pair((uint32_t)at, (uint32_t)(out.size() - at)));
	}
	return Success;
}

} // namespace

extern "C" {

Error_t inf_tokenizer_encode(const InfTokenizer* tok, const char* text, u32* ids, u64 max_ids, u64* n_ids)
{
	if (!tok || !text || !n_ids) return fail(ErrorInvalidValue, "inf_tokenizer_encode: NULL argument");
	Encoder E(*tok);
	INF_TRY(E.text(text, text + strlen(text)));
	return E.finish(ids, max_ids, n_ids);
}

Error_t inf_tokenizer_encode_special(const InfTokenizer* tok, const char* text, u32* ids, u64 max_ids, u64* n_ids)
{
	if (!tok || !text || !n_ids) return fail(ErrorInvalidValue, "inf_tokenizer_encode_special: NULL argument");
	Encoder E(*tok);
	const char* end = text + strlen(text);
	const char* seg = text;
	for (const char* p = text; p < end;) {
		const std::vector<uint32_t>& cand = tok->special_by_byte[(unsigned char)*p];
		const std::pair<std::string, uint32_t>* hit = nullptr;
		for (uint32_t k : cand) { // longest first
			const std::string& c = tok->specials[k].first;
			if ((size_t)(end - p) >= c.size() && memcmp(p, c.data(), c.size()) == 0) {
				hit = &tok->specials[k];
				break;
			}
		}
		if (!hit) {
			++p;
			continue;
		}
		INF_TRY(E.text(seg, p));
		E.out.push_back(hit->second);
		p += hit->first.size();
		seg = p;
	}
	INF_TRY(E.text(seg, end));
	return E.finish(ids, max_ids, n_ids);
}

Error_t inf_tokenizer_decode(const InfTokenizer* tok, const u32* ids, u64 n_ids, char* out, u64 out_bytes, u64* out_len)
{
	if (!tok || (!ids && n_ids) || !out_len) return fail(ErrorInvalidValue, "inf_tokenizer_decode: NULL argument");
	std::string s;
	for (u64 i = 0; i < n_ids; ++i) {
		const u32 id = ids[i];
		if (id >= tok->piece.size() || !tok->has_piece[id]) return fail(ErrorTokenOutOfRange, "id %u has no piece", id);
		const std::string& pc = tok->piece[id];
		int b;
		if (tok->byte_fallback && parse_byte_token(pc, &b)) {
			s += (char)b;
			continue;
		}
		for (size_t k = 0; k < pc.size();) {
			if (pc.compare(k, 3, kSpaceMark) == 0) {
				s += ' ';
				k += 3;
			} else {
				s += pc[k++];
			}
		}
	}
	*out_len = s.size();
	if (!out) return Success;
	if (out_bytes < s.size() + 1) return fail(ErrorInvalidValue, "%zu bytes + NUL, room for %llu", s.size(), (unsigned long long)out_bytes);
	memcpy(out, s.data(), s.size());
	out[s.size()] = '\0';
	return Success;
}

} // extern "C"
