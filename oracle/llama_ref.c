/*
 * CPU oracle for the decoder token loop -- TEST INFRASTRUCTURE ONLY (see llama_ref.h).
 * Loaded by tests/, __graft_entry__.smoke() and bench.py's CPU legs; never by the product.
 *
 * Numerics (the rounding points the device path also uses):
 *   residual stream r            fp32
 *   normalised activation x^     bf16(r * (1/sqrt(mean(r^2)+eps)) * g)    [rmsnorm.cu:11-59 + eps]
 *   q, k, v after RoPE           bf16 (k, v are what the KV cache stores)
 *   attention output             bf16
 *   SwiGLU product h             bf16(silu(gate) * up)
 *   logits                       fp32, greedy argmax with ties to the lowest index
 * In fp32 mode (bf16 == 0) every rounding point is the identity.
 *
 * Between rounding points the oracle accumulates in double (dot products, sums of squares,
 * softmax sums), so each stored value is the correctly computed one and a comparison with
 * the device measures only the device's own fp32 accumulation error.
 */
#include "llama_ref.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------- */
/* synthetic data                                                             */
/* ------------------------------------------------------------------------- */

/* SplitMix64 (Steele, Lea, Flood, OOPSLA 2014). */
uint64_t orc_splitmix64(uint64_t x)
{
	uint64_t z = x + 0x9E3779B97F4A7C15ull;
	z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
	z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
	return z ^ (z >> 31);
}

/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11): ten rounds, key bumped by the
 * Weyl constants between rounds. */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4])
{
	uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
	uint32_t k0 = key[0], k1 = key[1];
	for (int r = 0; r < 10; ++r) {
		const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
		const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
		const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
		const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
		c0 = hi1 ^ c1 ^ k0;
		c1 = lo1;
		c2 = hi0 ^ c3 ^ k1;
		c3 = lo0;
		k0 += 0x9E3779B9u;
		k1 += 0xBB67AE85u;
	}
	out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

void orc_stream_key(uint64_t seed, uint64_t stream, uint32_t key[2])
{
	const uint64_t k = orc_splitmix64(orc_splitmix64(seed) ^ stream);
	key[0] = (uint32_t)k;
	key[1] = (uint32_t)(k >> 32);
}

/* Irwin-Hall(4) approximation of N(0, std): four 22-bit uniforms summed, centred, and
 * scaled by std*sqrt(3)/2^22.  The centred sum is an exact fp32 integer and the scale is
 * one IEEE multiply, so host and device produce identical bits. */
float orc_init_scale(float std)
{
	return (float)((double)std * 1.7320508075688772 / 4194304.0);
}

static inline float normal_from_words(const uint32_t w[4], float scale)
{
	const int32_t s = (int32_t)((w[0] >> 10) + (w[1] >> 10) + (w[2] >> 10) + (w[3] >> 10)) - (1 << 23);
	return (float)s * scale;
}

float orc_normal_value(uint64_t seed, uint64_t stream, uint64_t idx, float scale)
{
	uint32_t key[2], ctr[4] = { (uint32_t)idx, (uint32_t)(idx >> 32), 0u, 0u }, w[4];
	orc_stream_key(seed, stream, key);
	orc_philox4x32_10(ctr, key, w);
	return normal_from_words(w, scale);
}

/* round-to-nearest-even on the fp32 bit pattern */
static inline uint16_t f2bf(float x)
{
	uint32_t u;
	memcpy(&u, &x, 4);
	if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)0x7FC0u;
	u += 0x7FFFu + ((u >> 16) & 1u);
	return (uint16_t)(u >> 16);
}

uint16_t orc_f32_to_bf16(float x) { return f2bf(x); }

/* the exported conversions are not inlined into the loops below under -fPIC (they could be
 * interposed); these static copies are */
static inline float bf16f(uint16_t h)
{
	const uint32_t u = (uint32_t)h << 16;
	float f;
	memcpy(&f, &u, 4);
	return f;
}

float orc_bf16_to_f32(uint16_t h) { return bf16f(h); }

static inline float round_store(float x, int bf16)
{
	return bf16 ? bf16f(f2bf(x)) : x;
}

void orc_fill_tensor(uint64_t seed, uint64_t stream, uint64_t n, float std, int bf16, void* out)
{
	uint32_t key[2];
	orc_stream_key(seed, stream, key);
	const float scale = orc_init_scale(std);
#pragma omp parallel for schedule(static)
	for (int64_t i = 0; i < (int64_t)n; ++i) {
		uint32_t ctr[4] = { (uint32_t)i, (uint32_t)((uint64_t)i >> 32), 0u, 0u }, w[4];
		orc_philox4x32_10(ctr, key, w);
		const float v = normal_from_words(w, scale);
		if (bf16) ((uint16_t*)out)[i] = f2bf(v);
		else ((float*)out)[i] = v;
	}
}

/* Lemire's multiply-shift reduction of the first Philox word into [lo, hi]. */
uint32_t orc_uniform_u32(uint64_t seed, uint64_t stream, uint64_t idx, uint32_t lo, uint32_t hi_inclusive)
{
	uint32_t key[2], ctr[4] = { (uint32_t)idx, (uint32_t)(idx >> 32), 0u, 0u }, w[4];
	orc_stream_key(seed, stream, key);
	orc_philox4x32_10(ctr, key, w);
	const uint64_t range = (uint64_t)hi_inclusive - lo + 1u;
	return lo + (uint32_t)(((uint64_t)w[0] * range) >> 32);
}

void orc_gen_ids(uint64_t seed, uint64_t stream, uint64_t n, uint32_t vocab, uint32_t* out)
{
	for (uint64_t i = 0; i < n; ++i) out[i] = orc_uniform_u32(seed, stream, i, 0u, vocab - 1u);
}

uint64_t orc_tensor_stream(int32_t layer, uint32_t kind)
{
	return ((uint64_t)(int64_t)(layer + 1) << 8) | kind;
}

void orc_rope_table(uint32_t max_seq, uint32_t head_dim, float theta, float* cos_out, float* sin_out)
{
	const uint32_t half = head_dim / 2;
	for (uint32_t p = 0; p < max_seq; ++p) {
		for (uint32_t i = 0; i < half; ++i) {
			const double inv_freq = pow((double)theta, -2.0 * (double)i / (double)head_dim);
			const double a = (double)p * inv_freq;
			cos_out[(uint64_t)p * half + i] = (float)cos(a);
			sin_out[(uint64_t)p * half + i] = (float)sin(a);
		}
	}
}

/* ------------------------------------------------------------------------- */
/* stage oracles                                                              */
/* ------------------------------------------------------------------------- */

static inline float wval(const void* W, int bf16, uint64_t i)
{
	return bf16 ? bf16f(((const uint16_t*)W)[i]) : ((const float*)W)[i];
}

void orc_embed_gather(const uint32_t* ids, uint64_t n, uint32_t dim, const void* table, int bf16, float* out)
{
	for (uint64_t t = 0; t < n; ++t)
		for (uint32_t i = 0; i < dim; ++i) out[t * dim + i] = wval(table, bf16, (uint64_t)ids[t] * dim + i);
}

/* Accumulation width between rounding points: double (default) or, for measuring how far two
 * correct fp32 implementations drift apart, float (orc_set_accum_f32(1)). */
static int g_accum_f32 = 0;
void orc_set_accum_f32(int on) { g_accum_f32 = on; }

static inline double dot_bf16_f(const uint16_t* w, const float* x, uint64_t n)
{
	float acc[16] = { 0 };
	uint64_t i = 0;
	for (; i + 16 <= n; i += 16)
		for (int j = 0; j < 16; ++j) acc[j] += bf16f(w[i + j]) * x[i + j];
	float s = 0.f;
	for (int j = 0; j < 16; ++j) s += acc[j];
	for (; i < n; ++i) s += bf16f(w[i]) * x[i];
	return s;
}

static float rms_inv(const float* x, uint32_t dim, float eps)
{
	double acc[8] = { 0 };
	uint32_t i = 0;
	for (; i + 8 <= dim; i += 8)
		for (int j = 0; j < 8; ++j) acc[j] += (double)x[i + j] * (double)x[i + j];
	double ss = 0.0;
	for (int j = 0; j < 8; ++j) ss += acc[j];
	for (; i < dim; ++i) ss += (double)x[i] * (double)x[i];
	return 1.0f / sqrtf((float)ss / (float)dim + eps);
}

void orc_rmsnorm(const float* x, uint64_t rows, uint32_t dim, const void* g, int bf16, float eps, float* y)
{
	for (uint64_t r = 0; r < rows; ++r) {
		const float inv = rms_inv(x + r * dim, dim, eps);
		for (uint32_t i = 0; i < dim; ++i)
			y[r * dim + i] = round_store((x[r * dim + i] * inv) * wval(g, bf16, i), bf16);
	}
}

/* products of two floats are exact in double; only the sum rounds */
static inline double dot_bf16_d(const uint16_t* w, const float* x, uint64_t n)
{
	double acc[8] = { 0 };
	uint64_t i = 0;
	for (; i + 8 <= n; i += 8)
		for (int j = 0; j < 8; ++j) acc[j] += (double)bf16f(w[i + j]) * (double)x[i + j];
	double s = 0.0;
	for (int j = 0; j < 8; ++j) s += acc[j];
	for (; i < n; ++i) s += (double)bf16f(w[i]) * (double)x[i];
	return s;
}

static inline double dot_f32_d(const float* w, const float* x, uint64_t n)
{
	double acc[8] = { 0 };
	uint64_t i = 0;
	for (; i + 8 <= n; i += 8)
		for (int j = 0; j < 8; ++j) acc[j] += (double)w[i + j] * (double)x[i + j];
	double s = 0.0;
	for (int j = 0; j < 8; ++j) s += acc[j];
	for (; i < n; ++i) s += (double)w[i] * (double)x[i];
	return s;
}

void orc_matvec(const void* W, int bf16, uint64_t rows, uint64_t cols, const float* x, float* y)
{
#pragma omp parallel for schedule(static)
	for (int64_t r = 0; r < (int64_t)rows; ++r) {
		y[r] = (float)(bf16 ? (g_accum_f32 ? dot_bf16_f((const uint16_t*)W + (uint64_t)r * cols, x, cols)
		                                   : dot_bf16_d((const uint16_t*)W + (uint64_t)r * cols, x, cols))
		                    : dot_f32_d((const float*)W + (uint64_t)r * cols, x, cols));
	}
}

uint32_t orc_argmax(const float* x, uint64_t n)
{
	uint64_t best = 0;
	for (uint64_t i = 1; i < n; ++i)
		if (x[i] > x[best]) best = i;
	return (uint32_t)best;
}

/* ------------------------------------------------------------------------- */
/* sampling (the library's inf_set_sampling rule; it has no reference code)   */
/* ------------------------------------------------------------------------- */

void orc_sample_weights(const float* logits, uint64_t n, float inv_temp, uint32_t* q)
{
	float m = -INFINITY;
	for (uint64_t i = 0; i < n; ++i) m = logits[i] > m ? logits[i] : m;
	for (uint64_t i = 0; i < n; ++i) {
		const float w = expf((logits[i] - m) * inv_temp);
		const float s = w * 4294967296.0f;
		q[i] = s >= 4294967295.0f ? 0xFFFFFFFFu : (uint32_t)s;
	}
}

static int cmp_u32_desc(const void* a, const void* b)
{
	const uint32_t x = *(const uint32_t*)a, y = *(const uint32_t*)b;
	return x < y ? 1 : x > y ? -1 : 0;
}

uint32_t orc_sample_select(const uint32_t* q, uint64_t n, float top_p, uint32_t top_k, uint64_t seed, uint64_t counter)
{
	uint32_t* s = (uint32_t*)malloc(n * sizeof *s);
	if (!s) return 0xFFFFFFFFu;
	memcpy(s, q, n * sizeof *s);
	qsort(s, n, sizeof *s, cmp_u32_desc);
	/* top-k: the k-th largest weight (ties kept) */
	const uint32_t tk = (top_k > 0 && top_k < n) ? s[top_k - 1] : 0u;
	uint64_t zk = 0;
	for (uint64_t i = 0; i < n; ++i)
		if (q[i] >= tk) zk += q[i];
	/* top-p: walking down the distinct weights, the first whose running sum (all its ties
	 * included) reaches ceil(top_p * zk) */
	uint32_t tp = tk;
	if (top_p < 1.0f && zk > 0) {
		double tgt = ceil((double)top_p * (double)zk);
		if (tgt < 1.0) tgt = 1.0;
		if (tgt > (double)zk) tgt = (double)zk;
		uint64_t c = 0;
		for (uint64_t i = 0; i < n && s[i] >= tk;) {
			const uint32_t v = s[i];
			while (i < n && s[i] == v) c += s[i++];
			if ((double)c >= tgt) {
				tp = v;
				break;
			}
		}
	}
	free(s);
	uint64_t total = 0;
	for (uint64_t i = 0; i < n; ++i)
		if (q[i] >= tp) total += q[i];
	uint32_t key[2], w[4];
	const uint32_t ctr[4] = { (uint32_t)counter, (uint32_t)(counter >> 32), 0u, 0u };
	orc_stream_key(seed, 0x3000000u, key);
	orc_philox4x32_10(ctr, key, w);
	const uint64_t r = ((uint64_t)w[1] << 32) | w[0];
	const uint64_t target = (uint64_t)(((unsigned __int128)r * total) >> 64);
	uint64_t c = 0;
	for (uint64_t i = 0; i < n; ++i) {
		if (q[i] < tp) continue;
		c += q[i];
		if (c > target) return (uint32_t)i;
	}
	return 0xFFFFFFFFu;
}

/* ------------------------------------------------------------------------- */
/* model                                                                      */
/* ------------------------------------------------------------------------- */

enum {
	K_EMBED = 0, K_LM_HEAD = 1, K_FINAL_NORM = 2,
	K_EMBED_PLE = 3, K_PLE_MODEL_PROJ = 4, K_PLE_PROJ_NORM = 5, /* Gemma, global */
	K_WQ = 8, K_WK = 9, K_WV = 10, K_WO = 11, K_WGATE = 12, K_WUP = 13, K_WDOWN = 14,
	K_ATTN_NORM = 15, K_FFN_NORM = 16,
	K_Q_NORM = 17, K_K_NORM = 18, K_POST_ATTN_NORM = 19, K_POST_FFN_NORM = 20, /* Gemma, per layer */
	K_PLE_GATE = 21, K_PLE_PROJ = 22, K_PLE_POST_NORM = 23,
};

typedef struct OrcLayer {
	void *wq, *wk, *wv, *wo, *wg, *wu, *wd, *attn_norm, *ffn_norm;
	/* Gemma */
	void *q_norm, *k_norm, *post_attn_norm, *post_ffn_norm, *ple_gate, *ple_proj, *ple_post_norm;
} OrcLayer;

struct OrcModel {
	OrcConfig cfg;
	int       n_threads;
	void*     embed;
	void*     lm_head;   /* the embedding itself for Gemma (tied) */
	void*     final_norm;
	void*     embed_ple;      /* Gemma: [vocab][n_layers * ple_dim] */
	void*     ple_model_proj; /* Gemma: [n_layers * ple_dim][dim] */
	void*     ple_proj_norm;  /* Gemma: [ple_dim] */
	OrcLayer* layers;
	float*    rope_cos;
	float*    rope_sin;
	float*    kcache; /* [slot][layer][pos][kv][hd] */
	float*    vcache;
	float*    logits; /* last token's logits */
	/* layer-0 stage outputs of the last token, for stage tests */
	float *dbg_q, *dbg_k, *dbg_v, *dbg_att, *dbg_h, *dbg_r;
};

static void* alloc_tensor(const OrcModel* m, uint64_t n)
{
	return calloc(n, m->cfg.bf16 ? 2 : 4);
}

static void* gen_tensor(const OrcModel* m, uint64_t seed, int32_t layer, uint32_t kind, uint64_t n)
{
	void* t = alloc_tensor(m, n);
	if (t) orc_fill_tensor(seed, orc_tensor_stream(layer, kind), n, m->cfg.init_std, (int)m->cfg.bf16, t);
	return t;
}

static void* ones_tensor(const OrcModel* m, uint64_t n)
{
	void* t = alloc_tensor(m, n);
	if (!t) return NULL;
	for (uint64_t i = 0; i < n; ++i) {
		if (m->cfg.bf16) ((uint16_t*)t)[i] = 0x3F80u;
		else ((float*)t)[i] = 1.0f;
	}
	return t;
}

const void* orc_model_weight(const OrcModel* m, int32_t layer, uint32_t kind)
{
	if (layer < 0) {
		switch (kind) {
		case K_EMBED: return m->embed;
		case K_LM_HEAD: return m->lm_head;
		case K_FINAL_NORM: return m->final_norm;
		case K_EMBED_PLE: return m->embed_ple;
		case K_PLE_MODEL_PROJ: return m->ple_model_proj;
		case K_PLE_PROJ_NORM: return m->ple_proj_norm;
		default: return NULL;
		}
	}
	if ((uint32_t)layer >= m->cfg.n_layers) return NULL;
	const OrcLayer* L = &m->layers[layer];
	switch (kind) {
	case K_WQ: return L->wq;
	case K_WK: return L->wk;
	case K_WV: return L->wv;
	case K_WO: return L->wo;
	case K_WGATE: return L->wg;
	case K_WUP: return L->wu;
	case K_WDOWN: return L->wd;
	case K_ATTN_NORM: return L->attn_norm;
	case K_FFN_NORM: return L->ffn_norm;
	case K_Q_NORM: return L->q_norm;
	case K_K_NORM: return L->k_norm;
	case K_POST_ATTN_NORM: return L->post_attn_norm;
	case K_POST_FFN_NORM: return L->post_ffn_norm;
	case K_PLE_GATE: return L->ple_gate;
	case K_PLE_PROJ: return L->ple_proj;
	case K_PLE_POST_NORM: return L->ple_post_norm;
	default: return NULL;
	}
}

OrcModel* orc_model_create(const OrcConfig* cfg, uint64_t seed, int n_threads)
{
	if (!cfg || cfg->n_heads == 0 || cfg->n_kv_heads == 0 || cfg->n_heads % cfg->n_kv_heads || cfg->head_dim % 2 ||
	    cfg->head_dim > 512 || cfg->arch > 1 || (cfg->arch == 0 && (cfg->ple_dim || cfg->final_softcap != 0.0f)) ||
	    cfg->n_slots == 0 || cfg->max_seq == 0)
		return NULL;
#ifdef _OPENMP
	if (n_threads > 0) omp_set_num_threads(n_threads);
#endif
	OrcModel* m = (OrcModel*)calloc(1, sizeof *m);
	if (!m) return NULL;
	m->cfg = *cfg;
	m->n_threads = n_threads;
	const uint64_t V = cfg->vocab, d = cfg->dim, H = cfg->n_heads, KV = cfg->n_kv_heads, hd = cfg->head_dim,
	               F = cfg->ffn, L = cfg->n_layers;
	const int gemma = cfg->arch == 1;
	const uint64_t P = cfg->ple_dim;
	/* norm gains: 1.0 for Llama; Gemma scales by (1 + w), so its w are drawn like the weights */
#define NORM(layer, kind, n) (gemma ? gen_tensor(m, seed, (layer), (kind), (n)) : ones_tensor(m, (n)))
	m->embed = gen_tensor(m, seed, -1, K_EMBED, V * d);
	m->lm_head = gemma ? m->embed : gen_tensor(m, seed, -1, K_LM_HEAD, V * d);
	m->final_norm = NORM(-1, K_FINAL_NORM, d);
	if (gemma && P) {
		m->embed_ple = gen_tensor(m, seed, -1, K_EMBED_PLE, V * L * P);
		m->ple_model_proj = gen_tensor(m, seed, -1, K_PLE_MODEL_PROJ, L * P * d);
		m->ple_proj_norm = gen_tensor(m, seed, -1, K_PLE_PROJ_NORM, P);
	}
	m->layers = (OrcLayer*)calloc(L, sizeof(OrcLayer));
	for (uint32_t l = 0; l < L; ++l) {
		OrcLayer* Ly = &m->layers[l];
		Ly->wq = gen_tensor(m, seed, (int32_t)l, K_WQ, H * hd * d);
		Ly->wk = gen_tensor(m, seed, (int32_t)l, K_WK, KV * hd * d);
		Ly->wv = gen_tensor(m, seed, (int32_t)l, K_WV, KV * hd * d);
		Ly->wo = gen_tensor(m, seed, (int32_t)l, K_WO, d * H * hd);
		Ly->wg = gen_tensor(m, seed, (int32_t)l, K_WGATE, F * d);
		Ly->wu = gen_tensor(m, seed, (int32_t)l, K_WUP, F * d);
		Ly->wd = gen_tensor(m, seed, (int32_t)l, K_WDOWN, d * F);
		Ly->attn_norm = NORM((int32_t)l, K_ATTN_NORM, d);
		Ly->ffn_norm = NORM((int32_t)l, K_FFN_NORM, d);
		if (gemma) {
			Ly->q_norm = gen_tensor(m, seed, (int32_t)l, K_Q_NORM, hd);
			Ly->k_norm = gen_tensor(m, seed, (int32_t)l, K_K_NORM, hd);
			Ly->post_attn_norm = gen_tensor(m, seed, (int32_t)l, K_POST_ATTN_NORM, d);
			Ly->post_ffn_norm = gen_tensor(m, seed, (int32_t)l, K_POST_FFN_NORM, d);
			if (P) {
				Ly->ple_gate = gen_tensor(m, seed, (int32_t)l, K_PLE_GATE, P * d);
				Ly->ple_proj = gen_tensor(m, seed, (int32_t)l, K_PLE_PROJ, d * P);
				Ly->ple_post_norm = gen_tensor(m, seed, (int32_t)l, K_PLE_POST_NORM, d);
			}
		}
	}
#undef NORM
	m->rope_cos = (float*)malloc(sizeof(float) * cfg->max_seq * (hd / 2));
	m->rope_sin = (float*)malloc(sizeof(float) * cfg->max_seq * (hd / 2));
	orc_rope_table(cfg->max_seq, (uint32_t)hd, cfg->rope_theta, m->rope_cos, m->rope_sin);
	const uint64_t kv_elems = (uint64_t)cfg->n_slots * L * cfg->max_seq * KV * hd;
	m->kcache = (float*)calloc(kv_elems, sizeof(float));
	m->vcache = (float*)calloc(kv_elems, sizeof(float));
	m->logits = (float*)calloc(V, 4);
	m->dbg_q = (float*)calloc(H * hd, 4);
	m->dbg_k = (float*)calloc(KV * hd, 4);
	m->dbg_v = (float*)calloc(KV * hd, 4);
	m->dbg_att = (float*)calloc(H * hd, 4);
	m->dbg_h = (float*)calloc(F, 4);
	m->dbg_r = (float*)calloc(d, 4);
	if (!m->embed || !m->lm_head || !m->kcache || !m->vcache || !m->logits ||
	    (cfg->arch == 1 && cfg->ple_dim && (!m->embed_ple || !m->ple_model_proj || !m->ple_proj_norm))) {
		orc_model_destroy(m);
		return NULL;
	}
	for (uint32_t l = 0; l < L; ++l)
		if (!m->layers[l].wq || !m->layers[l].wd || !m->layers[l].wg || !m->layers[l].wu) {
			orc_model_destroy(m);
			return NULL;
		}
	return m;
}

void orc_model_destroy(OrcModel* m)
{
	if (!m) return;
	if (m->lm_head != m->embed) free(m->lm_head);
	free(m->embed); free(m->final_norm);
	free(m->embed_ple); free(m->ple_model_proj); free(m->ple_proj_norm);
	if (m->layers) {
		for (uint32_t l = 0; l < m->cfg.n_layers; ++l) {
			OrcLayer* Ly = &m->layers[l];
			free(Ly->wq); free(Ly->wk); free(Ly->wv); free(Ly->wo);
			free(Ly->wg); free(Ly->wu); free(Ly->wd); free(Ly->attn_norm); free(Ly->ffn_norm);
			free(Ly->q_norm); free(Ly->k_norm); free(Ly->post_attn_norm); free(Ly->post_ffn_norm);
			free(Ly->ple_gate); free(Ly->ple_proj); free(Ly->ple_post_norm);
		}
		free(m->layers);
	}
	free(m->rope_cos); free(m->rope_sin); free(m->kcache); free(m->vcache);
	free(m->logits);
	free(m->dbg_q); free(m->dbg_k); free(m->dbg_v); free(m->dbg_att); free(m->dbg_h); free(m->dbg_r);
	free(m);
}

static inline float* kv_at(const OrcModel* m, float* cache, uint32_t slot, uint32_t layer, uint32_t pos)
{
	const OrcConfig* c = &m->cfg;
	const uint64_t per_pos = (uint64_t)c->n_kv_heads * c->head_dim;
	return cache + (((uint64_t)slot * c->n_layers + layer) * c->max_seq + pos) * per_pos;
}

static void rope_inplace(float* x, uint32_t n_heads, uint32_t hd, const float* cs, const float* sn)
{
	const uint32_t half = hd / 2;
	for (uint32_t h = 0; h < n_heads; ++h) {
		float* v = x + (uint64_t)h * hd;
		for (uint32_t i = 0; i < half; ++i) {
			const float a = v[i], b = v[i + half];
			v[i] = a * cs[i] - b * sn[i];
			v[i + half] = b * cs[i] + a * sn[i];
		}
	}
}

/* Y[t][r] = W[r,:] . X[t,:] for T rows of X: each weight row is read once per block and every
 * (row, token) dot product is the same computation orc_matvec does, so a block gives the
 * per-token results bit for bit. */
/* dot_bf16_d of one weight row with four vectors at once (each sum in the same order as
 * dot_bf16_d, so the results are identical; the row is converted once for all four) */
static inline void dot4_bf16_d(const uint16_t* w, const float* x0, const float* x1, const float* x2, const float* x3,
                               uint64_t n, double out[4])
{
	double a0[8] = { 0 }, a1[8] = { 0 }, a2[8] = { 0 }, a3[8] = { 0 };
	uint64_t i = 0;
	for (; i + 8 <= n; i += 8)
		for (int j = 0; j < 8; ++j) {
			const double wv = (double)bf16f(w[i + j]);
			a0[j] += wv * (double)x0[i + j];
			a1[j] += wv * (double)x1[i + j];
			a2[j] += wv * (double)x2[i + j];
			a3[j] += wv * (double)x3[i + j];
		}
	double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
	for (int j = 0; j < 8; ++j) {
		s0 += a0[j];
		s1 += a1[j];
		s2 += a2[j];
		s3 += a3[j];
	}
	for (; i < n; ++i) {
		const double wv = (double)bf16f(w[i]);
		s0 += wv * (double)x0[i];
		s1 += wv * (double)x1[i];
		s2 += wv * (double)x2[i];
		s3 += wv * (double)x3[i];
	}
	out[0] = s0;
	out[1] = s1;
	out[2] = s2;
	out[3] = s3;
}

/* Y[t][r] = W[r,:] . X[t,:] for T rows of X: each weight row is read once per block and every
 * (row, token) dot product is the same computation orc_matvec does, so a block gives the
 * per-token results bit for bit. */
static void matmat(const void* W, int bf16, uint64_t rows, uint64_t cols, const float* X, uint32_t T, float* Y)
{
#pragma omp parallel for schedule(static)
	for (int64_t r = 0; r < (int64_t)rows; ++r) {
		uint32_t t = 0;
		if (bf16 && !g_accum_f32)
			for (; t + 4 <= T; t += 4) {
				double v[4];
				const float* x = X + (uint64_t)t * cols;
				dot4_bf16_d((const uint16_t*)W + (uint64_t)r * cols, x, x + cols, x + 2 * cols, x + 3 * cols, cols, v);
				for (int u = 0; u < 4; ++u) Y[(uint64_t)(t + u) * rows + r] = (float)v[u];
			}
		for (; t < T; ++t) {
			const float* x = X + (uint64_t)t * cols;
			const double v = bf16 ? (g_accum_f32 ? dot_bf16_f((const uint16_t*)W + (uint64_t)r * cols, x, cols)
			                                     : dot_bf16_d((const uint16_t*)W + (uint64_t)r * cols, x, cols))
			                      : dot_f32_d((const float*)W + (uint64_t)r * cols, x, cols);
			Y[(uint64_t)t * rows + r] = (float)v;
		}
	}
}

enum { kOrcBlock = 64 }; /* tokens per block of a multi-token forward */

typedef struct OrcBlockBufs {
	uint32_t cap;
	float *r, *xh, *q, *k, *v, *att, *o, *gate, *up, *h, *scores;
	int n_scores;
} OrcBlockBufs;

static void block_free(OrcBlockBufs* b)
{
	free(b->r); free(b->xh); free(b->q); free(b->k); free(b->v); free(b->att); free(b->o);
	free(b->gate); free(b->up); free(b->h); free(b->scores);
	memset(b, 0, sizeof *b);
}

static int block_alloc(const OrcConfig* c, uint32_t T, OrcBlockBufs* b)
{
	memset(b, 0, sizeof *b);
	const uint64_t d = c->dim, Hh = (uint64_t)c->n_heads * c->head_dim, KVh = (uint64_t)c->n_kv_heads * c->head_dim,
	               F = c->ffn;
	b->cap = T;
	b->r = (float*)malloc(4 * T * d);
	b->xh = (float*)malloc(4 * T * d);
	b->q = (float*)malloc(4 * T * Hh);
	b->k = (float*)malloc(4 * T * KVh);
	b->v = (float*)malloc(4 * T * KVh);
	b->att = (float*)malloc(4 * T * Hh);
	b->o = (float*)malloc(4 * T * d);
	b->gate = (float*)malloc(4 * T * F);
	b->up = (float*)malloc(4 * T * F);
	b->h = (float*)malloc(4 * T * F);
	b->n_scores = omp_get_max_threads();
	b->scores = (float*)malloc(4 * (uint64_t)b->n_scores * c->max_seq);
	if (!b->r || !b->xh || !b->q || !b->k || !b->v || !b->att || !b->o || !b->gate || !b->up || !b->h || !b->scores) {
		block_free(b);
		return -5;
	}
	return 0;
}

/* Tokens ids[0..T) at positions pos0.. through the model (KV of every position written), one
 * layer at a time for the whole block; token t attends positions 0..pos0+t.  logits_all
 * [T][vocab] (may be NULL) receives every token's logits, logits_last (may be NULL) the last
 * token's.  Per token this is the decode step's arithmetic exactly. */
static int forward_block(OrcModel* m, uint32_t slot, const uint32_t* ids, uint32_t T, uint32_t pos0, float* logits_all,
                         float* logits_last)
{
	const OrcConfig* c = &m->cfg;
	const int bf = (int)c->bf16;
	const uint32_t d = c->dim, H = c->n_heads, KV = c->n_kv_heads, hd = c->head_dim, F = c->ffn;
	const uint32_t group = H / KV, half = hd / 2;
	const float attn_scale = (float)(1.0 / sqrt((double)hd));
	OrcBlockBufs B;
	const int rc = block_alloc(c, T, &B);
	if (rc) return rc;

	orc_embed_gather(ids, T, d, m->embed, bf, B.r);
	for (uint32_t l = 0; l < c->n_layers; ++l) {
		const OrcLayer* Ly = &m->layers[l];
		orc_rmsnorm(B.r, T, d, Ly->attn_norm, bf, c->eps, B.xh);
		matmat(Ly->wq, bf, (uint64_t)H * hd, d, B.xh, T, B.q);
		matmat(Ly->wk, bf, (uint64_t)KV * hd, d, B.xh, T, B.k);
		matmat(Ly->wv, bf, (uint64_t)KV * hd, d, B.xh, T, B.v);
		for (uint32_t t = 0; t < T; ++t) {
			const uint32_t pos = pos0 + t;
			const float* cs = m->rope_cos + (uint64_t)pos * half;
			const float* sn = m->rope_sin + (uint64_t)pos * half;
			float* q = B.q + (uint64_t)t * H * hd;
			float* k = B.k + (uint64_t)t * KV * hd;
			float* v = B.v + (uint64_t)t * KV * hd;
			rope_inplace(q, H, hd, cs, sn);
			rope_inplace(k, KV, hd, cs, sn);
			for (uint32_t i = 0; i < H * hd; ++i) q[i] = round_store(q[i], bf);
			for (uint32_t i = 0; i < KV * hd; ++i) {
				k[i] = round_store(k[i], bf);
				v[i] = round_store(v[i], bf);
			}
			memcpy(kv_at(m, m->kcache, slot, l, pos), k, sizeof(float) * KV * hd);
			memcpy(kv_at(m, m->vcache, slot, l, pos), v, sizeof(float) * KV * hd);
		}
#pragma omp parallel for schedule(dynamic, 1)
		for (int64_t th = 0; th < (int64_t)T * H; ++th) {
			const uint32_t t = (uint32_t)(th / H), h = (uint32_t)(th % H);
			const uint32_t g = h / group, ctx = pos0 + t + 1;
			const float* qh = B.q + (uint64_t)t * H * hd + (uint64_t)h * hd;
			float* sc = B.scores + (uint64_t)omp_get_thread_num() * c->max_seq;
			double mx = -INFINITY;
			for (uint32_t p = 0; p < ctx; ++p) {
				const float* kt = kv_at(m, m->kcache, slot, l, p) + (uint64_t)g * hd;
				const float s = (float)dot_f32_d(kt, qh, hd) * attn_scale;
				sc[p] = s;
				if (s > mx) mx = s;
			}
			double den = 0.0;
			for (uint32_t p = 0; p < ctx; ++p) {
				sc[p] = (float)exp((double)sc[p] - mx);
				den += sc[p];
			}
			double acc[512];
			for (uint32_t i = 0; i < hd; ++i) acc[i] = 0.0;
			for (uint32_t p = 0; p < ctx; ++p) {
				const float* vt = kv_at(m, m->vcache, slot, l, p) + (uint64_t)g * hd;
				for (uint32_t i = 0; i < hd; ++i) acc[i] += (double)sc[p] * (double)vt[i];
			}
			float* oh = B.att + (uint64_t)t * H * hd + (uint64_t)h * hd;
			for (uint32_t i = 0; i < hd; ++i) oh[i] = round_store((float)(acc[i] / den), bf);
		}
		if (l == 0) {
			const uint32_t t = T - 1;
			memcpy(m->dbg_q, B.q + (uint64_t)t * H * hd, sizeof(float) * H * hd);
			memcpy(m->dbg_k, B.k + (uint64_t)t * KV * hd, sizeof(float) * KV * hd);
			memcpy(m->dbg_v, B.v + (uint64_t)t * KV * hd, sizeof(float) * KV * hd);
			memcpy(m->dbg_att, B.att + (uint64_t)t * H * hd, sizeof(float) * H * hd);
		}
		matmat(Ly->wo, bf, d, (uint64_t)H * hd, B.att, T, B.o);
		for (uint64_t i = 0; i < (uint64_t)T * d; ++i) B.r[i] += B.o[i];

		orc_rmsnorm(B.r, T, d, Ly->ffn_norm, bf, c->eps, B.xh);
		matmat(Ly->wg, bf, F, d, B.xh, T, B.gate);
		matmat(Ly->wu, bf, F, d, B.xh, T, B.up);
		for (uint64_t j = 0; j < (uint64_t)T * F; ++j) {
			const double gt = B.gate[j];
			const double s = gt / (1.0 + exp(-gt));
			B.h[j] = round_store((float)(s * (double)B.up[j]), bf);
		}
		matmat(Ly->wd, bf, d, F, B.h, T, B.o);
		for (uint64_t i = 0; i < (uint64_t)T * d; ++i) B.r[i] += B.o[i];
		if (l == 0) {
			memcpy(m->dbg_h, B.h + (uint64_t)(T - 1) * F, sizeof(float) * F);
			memcpy(m->dbg_r, B.r + (uint64_t)(T - 1) * d, sizeof(float) * d);
		}
	}
	if (logits_all) {
		orc_rmsnorm(B.r, T, d, m->final_norm, bf, c->eps, B.xh);
		matmat(m->lm_head, bf, c->vocab, d, B.xh, T, logits_all);
		if (logits_last) memcpy(logits_last, logits_all + (uint64_t)(T - 1) * c->vocab, sizeof(float) * c->vocab);
	} else if (logits_last) {
		orc_rmsnorm(B.r + (uint64_t)(T - 1) * d, 1, d, m->final_norm, bf, c->eps, B.xh);
		orc_matvec(m->lm_head, bf, c->vocab, d, B.xh, logits_last);
	}
	block_free(&B);
	return 0;
}

/* ---- Gemma-style decoder (arch 1; see OrcConfig) ------------------------------------ */

/* the model's constants (embedding and per-layer-input scales) are rounded to bf16 (RNE) from
 * double, for fp32 models too */
static inline float bf16_const(double v) { return bf16f(f2bf((float)v)); }

static inline double gelu_tanh(double x)
{
	return 0.5 * x * (1.0 + tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)));
}

/* y = (x * (1/sqrt(mean(x^2) + eps))) * (1 + w), fp32 products in that order, not rounded */
static void rms1p(const float* x, uint32_t dim, const void* g, int gbf, float eps, float* y)
{
	const float inv = rms_inv(x, dim, eps);
	for (uint32_t i = 0; i < dim; ++i) y[i] = (x[i] * inv) * (1.0f + wval(g, gbf, i));
}

/* r += rms1p(x) */
static void add_rms1p(float* r, const float* x, uint32_t dim, const void* g, int gbf, float eps)
{
	const float inv = rms_inv(x, dim, eps);
	for (uint32_t i = 0; i < dim; ++i) r[i] = r[i] + (x[i] * inv) * (1.0f + wval(g, gbf, i));
}

static int forward_block_gemma(OrcModel* m, uint32_t slot, const uint32_t* ids, uint32_t T, uint32_t pos0,
                               float* logits_all, float* logits_last)
{
	const OrcConfig* c = &m->cfg;
	const int bf = (int)c->bf16;
	const uint32_t d = c->dim, H = c->n_heads, KV = c->n_kv_heads, hd = c->head_dim, F = c->ffn, L = c->n_layers;
	const uint32_t P = c->ple_dim, group = H / KV, half = hd / 2;
	const float attn_scale = (float)(1.0 / sqrt((double)hd));
	const float eps = c->eps;
	const float es = bf16_const(sqrt((double)d));
	OrcBlockBufs B;
	int rc = block_alloc(c, T, &B);
	if (rc) return rc;
	float* ple = NULL;  /* [T][L][P] bf16 values */
	float* ptmp = NULL; /* [T][max(L*P, d)] */
	if (P) {
		ple = (float*)malloc(4 * (uint64_t)T * L * P);
		ptmp = (float*)malloc(4 * (uint64_t)T * ((uint64_t)L * P > d ? (uint64_t)L * P : d));
		if (!ple || !ptmp) {
			free(ple);
			free(ptmp);
			block_free(&B);
			return -5;
		}
	}
	for (uint32_t t = 0; t < T; ++t)
		for (uint32_t i = 0; i < d; ++i) B.r[(uint64_t)t * d + i] = wval(m->embed, bf, (uint64_t)ids[t] * d + i) * es;
	if (P) {
		/* per-layer inputs: (E_ple[id] * sqrt(P) + rms1p(W_pmp . bf16(r) * dim^-1/2)) * 2^-1/2 */
		const float s_ple = bf16_const(sqrt((double)P)), s_proj = bf16_const(1.0 / sqrt((double)d)),
		            s_sum = bf16_const(1.0 / sqrt(2.0));
		for (uint64_t i = 0; i < (uint64_t)T * d; ++i) B.xh[i] = round_store(B.r[i], bf);
		matmat(m->ple_model_proj, bf, (uint64_t)L * P, d, B.xh, T, ptmp);
		float* nb = (float*)malloc(4 * (uint64_t)P);
		if (!nb) {
			free(ple);
			free(ptmp);
			block_free(&B);
			return -5;
		}
		for (uint32_t t = 0; t < T; ++t)
			for (uint32_t l = 0; l < L; ++l) {
				float* v = ptmp + ((uint64_t)t * L + l) * P;
				for (uint32_t j = 0; j < P; ++j) v[j] = v[j] * s_proj;
				rms1p(v, P, m->ple_proj_norm, bf, eps, nb);
				for (uint32_t j = 0; j < P; ++j) {
					const float a = wval(m->embed_ple, bf, (uint64_t)ids[t] * L * P + (uint64_t)l * P + j) * s_ple;
					ple[((uint64_t)t * L + l) * P + j] = round_store((a + nb[j]) * s_sum, bf);
				}
			}
		free(nb);
	}
	for (uint32_t l = 0; l < L; ++l) {
		const OrcLayer* Ly = &m->layers[l];
		for (uint32_t t = 0; t < T; ++t) {
			rms1p(B.r + (uint64_t)t * d, d, Ly->attn_norm, bf, eps, B.xh + (uint64_t)t * d);
			for (uint32_t i = 0; i < d; ++i) B.xh[(uint64_t)t * d + i] = round_store(B.xh[(uint64_t)t * d + i], bf);
		}
		matmat(Ly->wq, bf, (uint64_t)H * hd, d, B.xh, T, B.q);
		matmat(Ly->wk, bf, (uint64_t)KV * hd, d, B.xh, T, B.k);
		matmat(Ly->wv, bf, (uint64_t)KV * hd, d, B.xh, T, B.v);
		for (uint32_t t = 0; t < T; ++t) {
			const uint32_t pos = pos0 + t;
			const float* cs = m->rope_cos + (uint64_t)pos * half;
			const float* sn = m->rope_sin + (uint64_t)pos * half;
			float* q = B.q + (uint64_t)t * H * hd;
			float* k = B.k + (uint64_t)t * KV * hd;
			float* v = B.v + (uint64_t)t * KV * hd;
			float tmp[512];
			for (uint32_t h = 0; h < H; ++h) {
				rms1p(q + (uint64_t)h * hd, hd, Ly->q_norm, bf, eps, tmp);
				memcpy(q + (uint64_t)h * hd, tmp, 4 * hd);
			}
			for (uint32_t h = 0; h < KV; ++h) {
				rms1p(k + (uint64_t)h * hd, hd, Ly->k_norm, bf, eps, tmp);
				memcpy(k + (uint64_t)h * hd, tmp, 4 * hd);
			}
			rope_inplace(q, H, hd, cs, sn);
			rope_inplace(k, KV, hd, cs, sn);
			for (uint32_t i = 0; i < H * hd; ++i) q[i] = round_store(q[i], bf);
			for (uint32_t i = 0; i < KV * hd; ++i) {
				k[i] = round_store(k[i], bf);
				v[i] = round_store(v[i], bf);
			}
			memcpy(kv_at(m, m->kcache, slot, l, pos), k, sizeof(float) * KV * hd);
			memcpy(kv_at(m, m->vcache, slot, l, pos), v, sizeof(float) * KV * hd);
		}
#pragma omp parallel for schedule(dynamic, 1)
		for (int64_t th = 0; th < (int64_t)T * H; ++th) {
			const uint32_t t = (uint32_t)(th / H), h = (uint32_t)(th % H);
			const uint32_t g = h / group, ctx = pos0 + t + 1;
			const float* qh = B.q + (uint64_t)t * H * hd + (uint64_t)h * hd;
			float* sc = B.scores + (uint64_t)omp_get_thread_num() * c->max_seq;
			double mx = -INFINITY;
			for (uint32_t p = 0; p < ctx; ++p) {
				const float s = (float)dot_f32_d(kv_at(m, m->kcache, slot, l, p) + (uint64_t)g * hd, qh, hd) * attn_scale;
				sc[p] = s;
				if (s > mx) mx = s;
			}
			double den = 0.0;
			for (uint32_t p = 0; p < ctx; ++p) {
				sc[p] = (float)exp((double)sc[p] - mx);
				den += sc[p];
			}
			double acc[512];
			for (uint32_t i = 0; i < hd; ++i) acc[i] = 0.0;
			for (uint32_t p = 0; p < ctx; ++p) {
				const float* vt = kv_at(m, m->vcache, slot, l, p) + (uint64_t)g * hd;
				for (uint32_t i = 0; i < hd; ++i) acc[i] += (double)sc[p] * (double)vt[i];
			}
			float* oh = B.att + (uint64_t)t * H * hd + (uint64_t)h * hd;
			for (uint32_t i = 0; i < hd; ++i) oh[i] = round_store((float)(acc[i] / den), bf);
		}
		if (l == 0) {
			const uint32_t t = T - 1;
			memcpy(m->dbg_q, B.q + (uint64_t)t * H * hd, sizeof(float) * H * hd);
			memcpy(m->dbg_k, B.k + (uint64_t)t * KV * hd, sizeof(float) * KV * hd);
			memcpy(m->dbg_v, B.v + (uint64_t)t * KV * hd, sizeof(float) * KV * hd);
			memcpy(m->dbg_att, B.att + (uint64_t)t * H * hd, sizeof(float) * H * hd);
		}
		matmat(Ly->wo, bf, d, (uint64_t)H * hd, B.att, T, B.o);
		for (uint32_t t = 0; t < T; ++t) add_rms1p(B.r + (uint64_t)t * d, B.o + (uint64_t)t * d, d, Ly->post_attn_norm, bf, eps);
		for (uint32_t t = 0; t < T; ++t) {
			rms1p(B.r + (uint64_t)t * d, d, Ly->ffn_norm, bf, eps, B.xh + (uint64_t)t * d);
			for (uint32_t i = 0; i < d; ++i) B.xh[(uint64_t)t * d + i] = round_store(B.xh[(uint64_t)t * d + i], bf);
		}
		matmat(Ly->wg, bf, F, d, B.xh, T, B.gate);
		matmat(Ly->wu, bf, F, d, B.xh, T, B.up);
		for (uint64_t j = 0; j < (uint64_t)T * F; ++j)
			B.h[j] = round_store((float)(gelu_tanh((double)B.gate[j]) * (double)B.up[j]), bf);
		if (l == 0) memcpy(m->dbg_h, B.h + (uint64_t)(T - 1) * F, sizeof(float) * F);
		matmat(Ly->wd, bf, d, F, B.h, T, B.o);
		for (uint32_t t = 0; t < T; ++t) add_rms1p(B.r + (uint64_t)t * d, B.o + (uint64_t)t * d, d, Ly->post_ffn_norm, bf, eps);
		if (P) {
			/* per-layer-embedding block: r += rms1p(W_proj . bf16(gelu_tanh(W_gate . bf16(r)) * ple_l)) */
			for (uint64_t i = 0; i < (uint64_t)T * d; ++i) B.xh[i] = round_store(B.r[i], bf);
			matmat(Ly->ple_gate, bf, P, d, B.xh, T, ptmp);
			for (uint32_t t = 0; t < T; ++t)
				for (uint32_t j = 0; j < P; ++j) {
					const uint64_t i = (uint64_t)t * P + j;
					B.h[i] = round_store((float)(gelu_tanh((double)ptmp[i]) * (double)ple[((uint64_t)t * L + l) * P + j]), bf);
				}
			matmat(Ly->ple_proj, bf, d, P, B.h, T, B.o);
			for (uint32_t t = 0; t < T; ++t) add_rms1p(B.r + (uint64_t)t * d, B.o + (uint64_t)t * d, d, Ly->ple_post_norm, bf, eps);
		}
		if (l == 0) memcpy(m->dbg_r, B.r + (uint64_t)(T - 1) * d, sizeof(float) * d);
	}
	const uint32_t t0 = logits_all ? 0 : T - 1;
	for (uint32_t t = t0; t < T; ++t) {
		rms1p(B.r + (uint64_t)t * d, d, m->final_norm, bf, eps, B.xh + (uint64_t)(t - t0) * d);
		for (uint32_t i = 0; i < d; ++i) B.xh[(uint64_t)(t - t0) * d + i] = round_store(B.xh[(uint64_t)(t - t0) * d + i], bf);
	}
	float* lo = logits_all ? logits_all : logits_last;
	if (lo) {
		matmat(m->lm_head, bf, c->vocab, d, B.xh, T - t0, lo);
		if (c->final_softcap > 0.0f) {
			const double cap = c->final_softcap;
			for (uint64_t i = 0; i < (uint64_t)(T - t0) * c->vocab; ++i) lo[i] = (float)(cap * tanh((double)lo[i] / cap));
		}
		if (logits_all && logits_last)
			memcpy(logits_last, logits_all + (uint64_t)(T - 1) * c->vocab, sizeof(float) * c->vocab);
	}
	free(ple);
	free(ptmp);
	block_free(&B);
	return 0;
}

int orc_forward(OrcModel* m, uint32_t slot, const uint32_t* ids, uint32_t n, uint32_t start_pos,
                float* logits_all, float* logits_last, uint32_t* argmax_last)
{
	const OrcConfig* c = &m->cfg;
	if (slot >= c->n_slots) return -1;
	if ((uint64_t)start_pos + n > c->max_seq) return -2;
	for (uint32_t t = 0; t < n; ++t)
		if (ids[t] >= c->vocab) return -3;
	for (uint32_t t0 = 0; t0 < n; t0 += kOrcBlock) {
		const uint32_t T = (n - t0 < (uint32_t)kOrcBlock) ? n - t0 : (uint32_t)kOrcBlock;
		const int last = (t0 + T == n);
		float* la = logits_all ? logits_all + (uint64_t)t0 * c->vocab : NULL;
		const int rc = c->arch == 1 ? forward_block_gemma(m, slot, ids + t0, T, start_pos + t0, la, last ? m->logits : NULL)
		                            : forward_block(m, slot, ids + t0, T, start_pos + t0, la, last ? m->logits : NULL);
		if (rc) return rc;
	}
	if (n > 0) {
		if (logits_last) memcpy(logits_last, m->logits, sizeof(float) * c->vocab);
		if (argmax_last) *argmax_last = orc_argmax(m->logits, c->vocab);
	}
	return 0;
}

int orc_generate(OrcModel* m, uint32_t slot, const uint32_t* prompt, uint32_t n_prompt, uint32_t n_new,
                 uint32_t* out_ids, float* logits_steps)
{
	const OrcConfig* c = &m->cfg;
	if (n_prompt == 0 || n_new == 0) return -4;
	if ((uint64_t)n_prompt + n_new - 1 > c->max_seq) return -2;
	uint32_t next = 0;
	int rc = orc_forward(m, slot, prompt, n_prompt, 0, NULL, logits_steps, &next);
	if (rc) return rc;
	out_ids[0] = next;
	for (uint32_t s = 1; s < n_new; ++s) {
		float* lo = logits_steps ? logits_steps + (uint64_t)s * c->vocab : NULL;
		rc = orc_forward(m, slot, &out_ids[s - 1], 1, n_prompt + s - 1, NULL, lo, &next);
		if (rc) return rc;
		out_ids[s] = next;
	}
	return 0;
}

int orc_fill_kv_synthetic(OrcModel* m, uint32_t slot, uint32_t ctx, uint64_t seed)
{
	const OrcConfig* c = &m->cfg;
	if (slot >= c->n_slots || ctx > c->max_seq) return -1;
	const uint64_t per_pos = (uint64_t)c->n_kv_heads * c->head_dim;
	for (uint32_t l = 0; l < c->n_layers; ++l) {
		float* kb = kv_at(m, m->kcache, slot, l, 0);
		float* vb = kv_at(m, m->vcache, slot, l, 0);
		orc_fill_tensor(seed, 0x3000000ull | ((uint64_t)l << 1), (uint64_t)ctx * per_pos, 1.0f, 0, kb);
		orc_fill_tensor(seed, 0x3000000ull | ((uint64_t)l << 1) | 1u, (uint64_t)ctx * per_pos, 1.0f, 0, vb);
		if (c->bf16)
			for (uint64_t i = 0; i < (uint64_t)ctx * per_pos; ++i) {
				kb[i] = round_store(kb[i], 1);
				vb[i] = round_store(vb[i], 1);
			}
	}
	return 0;
}

int orc_last_layer0_mlp(const OrcModel* m, float* h, float* resid)
{
	if (h) memcpy(h, m->dbg_h, sizeof(float) * m->cfg.ffn);
	if (resid) memcpy(resid, m->dbg_r, sizeof(float) * m->cfg.dim);
	return 0;
}

int orc_kv_read(const OrcModel* m, uint32_t slot, uint32_t layer, uint32_t pos, float* k, float* v)
{
	const OrcConfig* c = &m->cfg;
	if (slot >= c->n_slots || layer >= c->n_layers || pos >= c->max_seq) return -1;
	const uint64_t n = (uint64_t)c->n_kv_heads * c->head_dim;
	if (k) memcpy(k, kv_at(m, m->kcache, slot, layer, pos), sizeof(float) * n);
	if (v) memcpy(v, kv_at(m, m->vcache, slot, layer, pos), sizeof(float) * n);
	return 0;
}

int orc_last_layer0(const OrcModel* m, float* q, float* k, float* v, float* attn)
{
	const OrcConfig* c = &m->cfg;
	if (q) memcpy(q, m->dbg_q, sizeof(float) * c->n_heads * c->head_dim);
	if (k) memcpy(k, m->dbg_k, sizeof(float) * c->n_kv_heads * c->head_dim);
	if (v) memcpy(v, m->dbg_v, sizeof(float) * c->n_kv_heads * c->head_dim);
	if (attn) memcpy(attn, m->dbg_att, sizeof(float) * c->n_heads * c->head_dim);
	return 0;
}
