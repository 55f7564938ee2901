/*
 * Test infrastructure: C entry points around the reference's own tokenizer, compiled from its
 * sources where they lie (src/tokenizer.c, src/allocator.c, external/cJSON.c; nothing is
 * copied) into _ref/libref_tokenizer.so by `make -C oracle ref`.  Only the tests, the golden
 * fixture script and bench.py's CPU baseline load it.
 *
 * tokenizer_build / tokenizer_encode (src/tokenizer.c:39-262) take an ExecCtx whose host arena
 * holds every string; the context's device arena is never created, so the arena_dev_destroy
 * that exec_ctx_destroy references (src/allocator.c:82-86) is stubbed here.
 */
#include <string.h>

#include "allocator.h"
#include "tokenizer.h"

Error_t arena_dev_destroy(DevArena* arena)
{
	(void)arena;
	return Success;
}

typedef struct RefTok {
	ExecCtx*  ctx;
	Tokenizer tok;
} RefTok;

static RefTok g_slots[4];

/* Returns a handle in [0, 4) or -1.  The reference aborts on malformed files. */
int ref_tok_create(const char* path)
{
	for (int i = 0; i < 4; ++i) {
		if (g_slots[i].ctx) continue;
		if (exec_ctx_create(&g_slots[i].ctx) != Success) return -1;
		memset(&g_slots[i].tok, 0, sizeof g_slots[i].tok);
		tokenizer_build(g_slots[i].ctx, &g_slots[i].tok, path);
		return i;
	}
	return -1;
}

/* Encodes text with the reference; copies min(n, cap) ids and returns n, the reference's
 * length counter (input_tokens_len), or -1.  The counter also counts pieces the reference
 * drops because they are not in the vocabulary (defect D13), so the ids are only meaningful
 * for texts whose pieces are all in the vocabulary -- the only texts the tests give it. */
long ref_tok_encode(int h, const char* text, unsigned* out, long cap)
{
	if (h < 0 || h >= 4 || !g_slots[h].ctx) return -1;
	RefTok* r = &g_slots[h];
	u32* ids = NULL;
	u32  len = 0;
	u64  pop = 0;
	const u64 pos0 = r->ctx->host_arena.pos;
	tokenizer_encode(r->ctx, &r->tok, text, &ids, &len, &pop);
	const long n = (long)len;
	for (long i = 0; i < n && i < cap; ++i) out[i] = ids[i];
	arena_host_pop_at((HostArena*)r->ctx, pos0);
	return n;
}

void ref_tok_destroy(int h)
{
	if (h < 0 || h >= 4 || !g_slots[h].ctx) return;
	tokenizer_destroy(&g_slots[h].tok);
	exec_ctx_destroy(&g_slots[h].ctx);
	g_slots[h].ctx = NULL;
}
