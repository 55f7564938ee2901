// Continuous batching over the paged KV cache: a request queue in front of the model's
// sequence slots.  Host code only.
//
// Every inf_server_step:
//   1. admits waiting requests, first come first served, into free slots (at most max_active
//      sequences at once): the slot's pages are released, the prompt is prefilled with
//      inf_forward and its greedy next token is the request's first output;
//   2. advances every other active sequence by one token with one batched decode step (the
//      projections of all of them in one pass over the weights on the tensor cores,
//      per-sequence attention over each one's pages) -- the batched step even for a lone
//      sequence, so that a request's ids never depend on how many others are running;
//   3. retires sequences that produced their end-of-sequence id, reached max_new tokens or
//      the end of the slot's positions, and releases their pages for the next admissions.
// KV pages are accounted for at admission: a request reserves the pages of every position it
// can write before it retires (its prompt plus max_new - 1 fed tokens, at most max_seq), and
// waits -- keeping its place in the queue -- while the pool cannot cover that, so a batched
// step never runs out of pages halfway through a sequence.
// A request admitted in step s contributes its first token in step s and joins the batched
// decode from step s + 1.  The reference has no serving loop (it stops after one RMSNorm,
// src/main.cu:396-412); this is the scheduler a caller would otherwise write around
// inf_forward_batch.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <deque>
#include <memory>
#include <unordered_map>
#include <vector>

#include "runtime.h"

using namespace inf;

namespace {

// The model calls the scheduler makes; the device model or the host stand-in below.
struct Backend {
	virtual ~Backend() = default;
	virtual u32 slots() const = 0;
	virtual u32 max_seq() const = 0;
	virtual u32 kv_block() const = 0; // positions per KV page
	virtual u32 kv_pages() const = 0; // pages in the pool, shared by all slots
	virtual Error_t release(u32 slot) = 0;
	virtual Error_t set_sampling(u32 slot, const InfSampling& s) = 0; // the slot's request's settings
	virtual Error_t prefill(const u32* ids, u32 n, u32 slot, u32* next) = 0;
	virtual Error_t decode(u32 n, const u32* slots, const u32* ids, const u32* pos, u32* next) = 0;
};

struct ModelBackend final : Backend {
	Model* m;
	explicit ModelBackend(Model* model) : m(model) {}
	u32 slots() const override { return m->config.max_batch; }
	u32 max_seq() const override { return m->config.max_seq; }
	u32 kv_block() const override { return m->config.kv_block ? m->config.kv_block : 16; }
	u32 kv_pages() const override
	{
		const InfConfig& c = m->config;
		return c.kv_pages ? c.kv_pages : c.max_batch * ((c.max_seq + kv_block() - 1) / kv_block());
	}
	Error_t release(u32 slot) override { return inf_seq_reset(m, slot); }
	Error_t set_sampling(u32 slot, const InfSampling& s) override { return inf_set_slot_sampling(m, slot, &s); }
	Error_t prefill(const u32* ids, u32 n, u32 slot, u32* next) override
	{
		// requests carry their own settings (per slot); the model-wide batch-1 setting would mix a
		// second rule into the first token
		if (model_sampling_on(m)) return fail(ErrorUnsupported, "the server samples per request; turn inf_set_sampling off");
		INF_TRY(inf_forward(m, ids, n, 0, slot, nullptr, next));
		return sample_slot_token(m, slot, n, next); // the new token sits at position n
	}
	Error_t decode(u32 n, const u32* s, const u32* ids, const u32* pos, u32* next) override
	{
		return forward_batch(m, n, s, ids, pos, nullptr, next, true);
	}
};

// Host stand-in: the next id is a hash of the sequence's previous id and position only, so a
// sequence's outputs cannot depend on what else shares its batch.  Tracks which positions each
// slot has written, to check the scheduler feeds every sequence its own positions in order, and
// holds a pool of 16-position pages that fails like the device cache when it runs out.  A prompt
// that starts with id vocab - 1 makes the first batched step its sequence is in fail with
// ErrorGeneric (to test how the scheduler handles a failing step).
struct SyntheticBackend final : Backend {
	u32 n_slots, seq, vocab, pages;
	std::vector<u32> filled;   // positions written per slot
	std::vector<char> poison;  // slot's prompt started with vocab - 1
	std::vector<u64> salt;     // per slot: 0 greedy, else derived from the request's seed and settings
	SyntheticBackend(u32 s, u32 ms, u32 v, u32 p)
	    : n_slots(s), seq(ms), vocab(v), pages(p ? p : s * ((ms + 15) / 16)), filled(s, 0), poison(s, 0), salt(s, 0)
	{
	}
	u32 slots() const override { return n_slots; }
	u32 max_seq() const override { return seq; }
	u32 kv_block() const override { return 16; }
	u32 kv_pages() const override { return pages; }
	static u32 mix(u64 x)
	{
		x ^= x >> 33;
		x *= 0xff51afd7ed558ccdull;
		x ^= x >> 33;
		x *= 0xc4ceb9fe1a85ec53ull;
		return (u32)(x ^ (x >> 33));
	}
	u32 pages_in_use(int except_slot, u32 positions_there) const
	{
		u32 n = 0;
		for (u32 k = 0; k < n_slots; ++k) n += ((int)k == except_slot ? positions_there : filled[k]) / 16 +
		                                        (((int)k == except_slot ? positions_there : filled[k]) % 16 != 0);
		return n;
	}
	Error_t release(u32 slot) override
	{
		if (slot >= n_slots) return fail(ErrorInvalidValue, "slot %u", slot);
		filled[slot] = 0;
		poison[slot] = 0;
		return Success;
	}
	// a sampling request's ids are a different hash, keyed by its seed and settings, so that a
	// test can see each request's settings reach the slot it runs in
	Error_t set_sampling(u32 slot, const InfSampling& s) override
	{
		if (slot >= n_slots) return fail(ErrorInvalidValue, "slot %u", slot);
		u32 tb = 0, pb = 0;
		memcpy(&tb, &s.temperature, 4);
		memcpy(&pb, &s.top_p, 4);
		salt[slot] = s.temperature > 0.0f ? (mix(s.seed) | 1ull) ^ ((u64)tb << 17) ^ ((u64)pb << 3) ^ s.top_k : 0;
		return Success;
	}
	Error_t prefill(const u32* ids, u32 n, u32 slot, u32* next) override
	{
		if (slot >= n_slots || n == 0 || n > seq) return fail(ErrorInvalidValue, "prefill slot %u n %u", slot, n);
		if (filled[slot] != 0) return fail(ErrorInvalidValue, "prefill into a slot that holds %u positions", filled[slot]);
		if (pages_in_use((int)slot, n) > pages) return fail(ErrorArenaOutOfMemory, "KV cache out of pages");
		u64 h = 0;
		for (u32 i = 0; i < n; ++i) h = mix(h * 31 + ids[i]);
		filled[slot] = n;
		poison[slot] = ids[0] == vocab - 1;
		*next = mix(h ^ ((u64)n << 40) ^ salt[slot]) % vocab;
		return Success;
	}
	Error_t decode(u32 n, const u32* s, const u32* ids, const u32* pos, u32* next) override
	{
		for (u32 i = 0; i < n; ++i) {
			if (s[i] >= n_slots || pos[i] >= seq) return fail(ErrorKvOutOfRange, "slot %u position %u", s[i], pos[i]);
			if (pos[i] != filled[s[i]]) return fail(ErrorInvalidValue, "slot %u fed position %u after %u", s[i], pos[i], filled[s[i]]);
			for (u32 j = 0; j < i; ++j)
				if (s[j] == s[i]) return fail(ErrorInvalidValue, "slot %u twice in one batch", s[i]);
		}
		for (u32 i = 0; i < n; ++i)
			if (poison[s[i]]) return fail(ErrorGeneric, "stand-in failure for slot %u", s[i]);
		for (u32 i = 0; i < n; ++i) filled[s[i]] = pos[i] + 1;
		if (pages_in_use(-1, 0) > pages) {
			for (u32 i = 0; i < n; ++i) filled[s[i]] = pos[i];
			return fail(ErrorArenaOutOfMemory, "KV cache out of pages");
		}
		for (u32 i = 0; i < n; ++i) next[i] = mix(((u64)ids[i] << 32) ^ pos[i] ^ salt[s[i]]) % vocab;
		return Success;
	}
};

struct Request {
	u64 id;
	std::vector<u32> prompt;
	u32 max_new, eos;
	std::vector<u32> out;
	int slot = -1;
	u32 pos = 0;      // position of the last output token (the next one fed)
	u64 admitted = 0; // the step that prefilled it
	u32 pages = 0;    // KV pages reserved while it holds a slot
	InfSampling samp{}; // temperature 0: greedy
	bool done = false;
	Error_t err = Success;
};

} // namespace

struct InfServer {
	std::unique_ptr<Backend> be;
	u32 max_active = 0;
	u64 next_id = 1;
	u64 steps = 0;
	std::unordered_map<u64, Request> reqs;
	std::deque<u64> waiting;
	std::vector<u64> active;
	std::vector<u32> free_slots;
	u32 pages_reserved = 0;
	u64 batched_steps = 0, batched_tokens = 0;
};

namespace {

// Pages of every position a request can write before it retires: the prompt, then one fed
// token per output after the first, at most max_seq positions.
u32 pages_needed(const InfServer* s, const Request& r)
{
	const u64 positions = std::min<u64>((u64)r.prompt.size() + r.max_new - 1, s->be->max_seq());
	const u32 blk = s->be->kv_block();
	return (u32)((positions + blk - 1) / blk);
}

Error_t retire(InfServer* s, Request& r)
{
	r.done = true;
	s->pages_reserved -= r.pages;
	r.pages = 0;
	if (r.slot >= 0) {
		const u32 slot = (u32)r.slot;
		r.slot = -1;
		s->free_slots.push_back(slot);
		return s->be->release(slot);
	}
	return Success;
}

bool finished(const InfServer* s, const Request& r)
{
	return r.out.size() >= r.max_new || (!r.out.empty() && r.out.back() == r.eos) || r.pos >= s->be->max_seq();
}

Error_t create(std::unique_ptr<Backend> be, u32 max_active, InfServer** out)
{
	if (!out) return fail(ErrorInvalidValue, "inf_server_create: NULL out");
	*out = nullptr;
	const u32 n = be->slots();
	if (n == 0) return fail(ErrorInvalidValue, "the model has no sequence slots");
	InfServer* s = new (std::nothrow) InfServer();
	if (!s) return fail(ErrorMemoryAllocation, "server");
	s->be = std::move(be);
	s->max_active = max_active == 0 ? n : std::min(max_active, n);
	for (u32 k = n; k-- > 0;) s->free_slots.push_back(k); // slot 0 first
	for (u32 k = 0; k < n; ++k) {
		const Error_t e = s->be->release(k);
		if (e != Success) {
			delete s;
			return e;
		}
	}
	*out = s;
	return Success;
}

} // namespace

extern "C" {

Error_t inf_server_create(Model* model, u32 max_active, InfServer** out)
{
	if (!model || !model->engine) return fail(ErrorInvalidValue, "inf_server_create: no model");
	return create(std::unique_ptr<Backend>(new ModelBackend(model)), max_active, out);
}

Error_t inf_server_create_synthetic(u32 n_slots, u32 max_seq, u32 vocab, u32 kv_pages, u32 max_active, InfServer** out)
{
	if (n_slots == 0 || max_seq < 2 || vocab == 0) return fail(ErrorInvalidValue, "inf_server_create_synthetic: sizes");
	return create(std::unique_ptr<Backend>(new SyntheticBackend(n_slots, max_seq, vocab, kv_pages)), max_active, out);
}

Error_t inf_server_destroy(InfServer** s)
{
	if (!s || !*s) return fail(ErrorInvalidValue, "inf_server_destroy: no server");
	delete *s;
	*s = nullptr;
	return Success;
}

Error_t inf_server_submit(InfServer* s, const u32* prompt, u32 n_prompt, u32 max_new, u32 eos_id, u64* request_id)
{
	return inf_server_submit_sampled(s, prompt, n_prompt, max_new, eos_id, nullptr, request_id);
}

Error_t inf_server_submit_sampled(InfServer* s, const u32* prompt, u32 n_prompt, u32 max_new, u32 eos_id,
                                  const InfSampling* sampling, u64* request_id)
{
	if (!s || !prompt || !request_id || n_prompt == 0 || max_new == 0) return fail(ErrorInvalidValue, "inf_server_submit: arguments");
	if (n_prompt >= s->be->max_seq()) return fail(ErrorKvOutOfRange, "prompt of %u tokens, %u positions per slot", n_prompt, s->be->max_seq());
	if (sampling && (!(sampling->temperature >= 0.0f) || !std::isfinite(sampling->temperature) ||
	                 (sampling->temperature > 0.0f && !(sampling->top_p > 0.0f && sampling->top_p <= 1.0f))))
		return fail(ErrorInvalidValue, "inf_server_submit: temperature %g, top_p %g", (double)sampling->temperature,
		            (double)sampling->top_p);
	Request r;
	if (sampling) r.samp = *sampling;
	r.prompt.assign(prompt, prompt + n_prompt);
	r.max_new = max_new;
	r.eos = eos_id;
	const u32 need = pages_needed(s, r);
	if (need > s->be->kv_pages())
		return fail(ErrorArenaOutOfMemory, "request needs %u KV pages, the pool holds %u", need, s->be->kv_pages());
	r.id = s->next_id++;
	s->waiting.push_back(r.id);
	*request_id = r.id;
	s->reqs.emplace(r.id, std::move(r));
	return Success;
}

Error_t inf_server_step(InfServer* s, u32* n_finished)
{
	if (!s) return fail(ErrorInvalidValue, "inf_server_step: no server");
	const u64 step = ++s->steps;
	u32 fin = 0;
	// 1. admissions: prefill and the first token
	while (!s->waiting.empty() && !s->free_slots.empty() && s->active.size() < s->max_active) {
		Request& r = s->reqs.at(s->waiting.front());
		const u32 need = pages_needed(s, r);
		if (s->pages_reserved + need > s->be->kv_pages()) break; // first come first served: it waits for pages
		s->waiting.pop_front();
		r.pages = need;
		s->pages_reserved += need;
		r.slot = (int)s->free_slots.back();
		s->free_slots.pop_back();
		r.admitted = step;
		u32 first = 0;
		Error_t e = s->be->set_sampling((u32)r.slot, r.samp);
		if (e == Success) e = s->be->prefill(r.prompt.data(), (u32)r.prompt.size(), (u32)r.slot, &first);
		if (e != Success) { // this request fails alone; the others go on
			r.err = e;
			INF_TRY(retire(s, r));
			++fin;
			continue;
		}
		r.out.push_back(first);
		r.pos = (u32)r.prompt.size();
		if (finished(s, r)) {
			INF_TRY(retire(s, r));
			++fin;
		} else {
			s->active.push_back(r.id);
		}
	}
	// 2. one batched decode step for the sequences admitted before this step
	std::vector<u32> slots, ids, pos;
	std::vector<u64> batch;
	for (u64 id : s->active) {
		const Request& r = s->reqs.at(id);
		if (r.admitted == step) continue;
		batch.push_back(id);
		slots.push_back((u32)r.slot);
		ids.push_back(r.out.back());
		pos.push_back(r.pos);
	}
	if (!batch.empty()) {
		std::vector<u32> next(batch.size());
		const Error_t e = s->be->decode((u32)batch.size(), slots.data(), ids.data(), pos.data(), next.data());
		if (e != Success) {
			// the batch's requests end with the error (their pages and slots go back to the pool),
			// so the next step does not retry the same failing batch
			std::vector<u64> keep;
			for (u64 id : s->active) {
				Request& r = s->reqs.at(id);
				if (std::find(batch.begin(), batch.end(), id) != batch.end()) {
					r.err = e;
					(void)retire(s, r);
					++fin;
				} else {
					keep.push_back(id);
				}
			}
			s->active.swap(keep);
			if (n_finished) *n_finished = fin;
			return e;
		}
		++s->batched_steps;
		s->batched_tokens += batch.size();
		for (size_t i = 0; i < batch.size(); ++i) {
			Request& r = s->reqs.at(batch[i]);
			r.out.push_back(next[i]);
			r.pos += 1;
		}
	}
	// 3. retire
	std::vector<u64> keep;
	for (u64 id : s->active) {
		Request& r = s->reqs.at(id);
		if (finished(s, r)) {
			INF_TRY(retire(s, r));
			++fin;
		} else {
			keep.push_back(id);
		}
	}
	s->active.swap(keep);
	if (n_finished) *n_finished = fin;
	return Success;
}

Error_t inf_server_result(InfServer* s, u64 request_id, u32* out_ids, u32 cap, u32* n_out, u32* done, Error_t* status)
{
	if (!s || !n_out) return fail(ErrorInvalidValue, "inf_server_result: arguments");
	const auto it = s->reqs.find(request_id);
	if (it == s->reqs.end()) return fail(ErrorInvalidValue, "no request %llu", (unsigned long long)request_id);
	const Request& r = it->second;
	*n_out = (u32)r.out.size();
	if (done) *done = r.done ? 1u : 0u;
	if (status) *status = r.err;
	if (out_ids) {
		if (cap < r.out.size()) return fail(ErrorInvalidValue, "%zu ids, room for %u", r.out.size(), cap);
		std::copy(r.out.begin(), r.out.end(), out_ids);
	}
	return Success;
}

Error_t inf_server_release(InfServer* s, u64 request_id)
{
	if (!s) return fail(ErrorInvalidValue, "inf_server_release: no server");
	const auto it = s->reqs.find(request_id);
	if (it == s->reqs.end()) return fail(ErrorInvalidValue, "no request %llu", (unsigned long long)request_id);
	if (!it->second.done) return fail(ErrorInvalidValue, "request %llu is still running", (unsigned long long)request_id);
	s->reqs.erase(it);
	return Success;
}

Error_t inf_server_stats(const InfServer* s, u32* n_waiting, u32* n_active, u64* batched_steps, u64* batched_tokens)
{
	if (!s) return fail(ErrorInvalidValue, "inf_server_stats: no server");
	if (n_waiting) *n_waiting = (u32)s->waiting.size();
	if (n_active) *n_active = (u32)s->active.size();
	if (batched_steps) *batched_steps = s->batched_steps;
	if (batched_tokens) *batched_tokens = s->batched_tokens;
	return Success;
}

} // extern "C"
