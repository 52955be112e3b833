/*
 * mlf2_synth.c — seeded synthetic Qwen2-shaped models in the MLF2 container,
 * and random k-quant blocks for the GEMV sweeps.
 *
 * The benchmark configurations name random-init models ("fp32 N(0, 0.02) from
 * seed 0, round-to-nearest quantized into Q4_K / Q6_K"); no checkpoints exist
 * here, so this file writes them. The container follows the MLF2 v2 layout the
 * reference loader reads (include/mlf2.h:55-102 of mithraeums/hako): a 128-byte
 * header, 104-byte directory entries, a tokenizer blob, 32-byte aligned data.
 *
 * Determinism: every tensor row draws from its own splitmix64 stream keyed by
 * (seed, tensor index, row), so the bytes do not depend on the thread count.
 * Normals are Box-Muller in double precision.
 */
#define _GNU_SOURCE
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <unistd.h>

/* ------------------------------------------------------------------ RNG */

static inline uint64_t sm64(uint64_t *s) {
	uint64_t z = (*s += 0x9E3779B97F4A7C15ULL);
	z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
	z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
	return z ^ (z >> 31);
}
static uint64_t key3(uint64_t a, uint64_t b, uint64_t c) {
	uint64_t s = a ^ 0x6A09E667F3BCC909ULL;
	uint64_t x = sm64(&s) ^ (b * 0xD1B54A32D192ED03ULL);
	s = x; x = sm64(&s) ^ (c * 0x8CB92BA72F3D8DD7ULL);
	s = x; return sm64(&s);
}
typedef struct { uint64_t s; int have; double spare; } rng_t;
static void rng_init(rng_t *r, uint64_t key) { r->s = key; r->have = 0; }
static inline double rng_u01(rng_t *r) {            /* (0, 1] */
	return ((double)(sm64(&r->s) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
}
static inline double rng_normal(rng_t *r) {
	if (r->have) { r->have = 0; return r->spare; }
	double u1 = rng_u01(r), u2 = rng_u01(r);
	double rad = sqrt(-2.0 * log(u1)), th = 6.283185307179586 * u2;
	r->spare = rad * sin(th); r->have = 1;
	return rad * cos(th);
}
static inline uint32_t rng_u32(rng_t *r) { return (uint32_t)(sm64(&r->s) >> 32); }

/* ---------------------------------------------------------------- fp16 */

static uint16_t to_f16(float f) {
	uint32_t x; memcpy(&x, &f, 4);
	uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7FFFFFFFu;
	if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0));
	if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
	if (ax < 0x33000001u) return (uint16_t)sign;
	int e = (int)(ax >> 23) - 127;
	uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u, base = 0;
	int shift;
	if (e < -14) { shift = -e - 1; }
	else { shift = 13; base = (uint32_t)(e + 15) << 10; mant &= 0x7FFFFFu; }
	uint32_t q = mant >> shift, rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
	if (rem > half || (rem == half && (q & 1u))) q++;
	return (uint16_t)(sign | (base + q));
}
static float from_f16(uint16_t h) {
	int s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
	float v = e == 0 ? ldexpf((float)m, -24) : ldexpf((float)(1024 + m), e - 25);
	return s ? -v : v;
}
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* ------------------------------------------------------- RTN quantizers */

/* One Q4_K super-block (144 B: d, dmin, scales[12], qs[128]) from 256 floats.
 * Round-to-nearest: per 32 sub-block an affine [min<=0, max] range over 16
 * levels, the 8 scales and 8 offsets quantized to 6 bits against fp16 d and
 * dmin. Decoding is y = d*s*q - dmin*m. */
void synth_quantize_q4k_block(const float *x, uint8_t *blk) {
	float sc[8], mo[8], msc = 0.f, mmo = 0.f;
	for (int j = 0; j < 8; j++) {
		float lo = x[32 * j], hi = x[32 * j];
		for (int l = 1; l < 32; l++) { float v = x[32 * j + l]; lo = v < lo ? v : lo; hi = v > hi ? v : hi; }
		if (lo > 0.f) lo = 0.f;
		sc[j] = (hi - lo) / 15.f; mo[j] = -lo;
		msc = sc[j] > msc ? sc[j] : msc; mmo = mo[j] > mmo ? mo[j] : mmo;
	}
	uint16_t dh = to_f16(msc / 63.f), mh = to_f16(mmo / 63.f);
	float df = from_f16(dh), mf = from_f16(mh);
	int ls[8], lm[8];
	for (int j = 0; j < 8; j++) {
		ls[j] = df > 0.f ? clampi((int)lrintf(sc[j] / df), 0, 63) : 0;
		lm[j] = mf > 0.f ? clampi((int)lrintf(mo[j] / mf), 0, 63) : 0;
	}
	blk[0] = (uint8_t)(dh & 0xFF); blk[1] = (uint8_t)(dh >> 8);
	blk[2] = (uint8_t)(mh & 0xFF); blk[3] = (uint8_t)(mh >> 8);
	uint8_t *s12 = blk + 4, *qs = blk + 16;
	for (int j = 0; j < 4; j++) {
		s12[j]     = (uint8_t)((ls[j] & 63) | ((ls[j + 4] >> 4) << 6));
		s12[j + 4] = (uint8_t)((lm[j] & 63) | ((lm[j + 4] >> 4) << 6));
		s12[j + 8] = (uint8_t)((ls[j + 4] & 15) | ((lm[j + 4] & 15) << 4));
	}
	memset(qs, 0, 128);
	for (int j = 0; j < 8; j++) {
		float ed = df * (float)ls[j], em = mf * (float)lm[j];
		for (int l = 0; l < 32; l++) {
			int q = ed > 0.f ? clampi((int)lrintf((x[32 * j + l] + em) / ed), 0, 15) : 0;
			qs[32 * (j >> 1) + l] |= (uint8_t)((j & 1) ? (q << 4) : q);
		}
	}
}

/* One Q6_K super-block (210 B: ql[128], qh[64], int8 scales[16], d) from
 * 256 floats: symmetric per-16 scales quantized to int8 against fp16 d,
 * values to 6 bits stored as q + 32. Decoding is y = d*sc*(q6 - 32). */
void synth_quantize_q6k_block(const float *x, uint8_t *blk) {
	float gs[16], mx = 0.f;
	for (int g = 0; g < 16; g++) {
		float a = 0.f;
		for (int l = 0; l < 16; l++) { float v = fabsf(x[16 * g + l]); a = v > a ? v : a; }
		gs[g] = a / 31.f;
		mx = gs[g] > mx ? gs[g] : mx;
	}
	uint16_t dh = to_f16(mx / 127.f);
	float df = from_f16(dh);
	int8_t *sc = (int8_t *)(blk + 192);
	uint8_t *ql = blk, *qh = blk + 128;
	memset(blk, 0, 192);
	for (int g = 0; g < 16; g++) sc[g] = (int8_t)(df > 0.f ? clampi((int)lrintf(gs[g] / df), -128, 127) : 0);
	for (int e = 0; e < 256; e++) {
		float ed = df * (float)sc[e >> 4];
		int q = ed != 0.f ? clampi((int)lrintf(x[e] / ed), -32, 31) : 0;
		int u = q + 32, n = e >> 7, k = (e >> 5) & 3, l = e & 31;
		ql[64 * n + 32 * (k & 1) + l] |= (uint8_t)((k < 2) ? (u & 15) : ((u & 15) << 4));
		qh[32 * n + l] |= (uint8_t)((u >> 4) << (2 * k));
	}
	blk[208] = (uint8_t)(dh & 0xFF); blk[209] = (uint8_t)(dh >> 8);
}

/* ------------------------------------------------------ random blocks */

/* Random Q4_K blocks: nibbles and 6-bit scales/mins uniform, d and dmin
 * |N(0, 1e-3)| as fp16. */
void synth_random_q4k(uint8_t *dst, long rows, long k, uint64_t seed) {
	long nb = k / 256;
	for (long r = 0; r < rows; r++) {
		rng_t g; rng_init(&g, key3(seed, 0x51, (uint64_t)r));
		for (long b = 0; b < nb; b++) {
			uint8_t *blk = dst + (r * nb + b) * 144;
			uint16_t d = to_f16((float)fabs(rng_normal(&g) * 1e-3));
			uint16_t dm = to_f16((float)fabs(rng_normal(&g) * 1e-3));
			blk[0] = d & 0xFF; blk[1] = d >> 8; blk[2] = dm & 0xFF; blk[3] = dm >> 8;
			for (int i = 4; i < 144; i += 4) { uint32_t u = rng_u32(&g); memcpy(blk + i, &u, 4); }
		}
	}
}

/* Random Q6_K blocks: ql/qh bits uniform, int8 sub-scales U[-32, 31],
 * d |N(0, 1e-3)| as fp16. */
void synth_random_q6k(uint8_t *dst, long rows, long k, uint64_t seed) {
	long nb = k / 256;
	for (long r = 0; r < rows; r++) {
		rng_t g; rng_init(&g, key3(seed, 0x61, (uint64_t)r));
		for (long b = 0; b < nb; b++) {
			uint8_t *blk = dst + (r * nb + b) * 210;
			for (int i = 0; i < 192; i += 4) { uint32_t u = rng_u32(&g); memcpy(blk + i, &u, 4); }
			for (int i = 0; i < 16; i++) blk[192 + i] = (uint8_t)(int8_t)((int)(rng_u32(&g) % 64) - 32);
			uint16_t d = to_f16((float)fabs(rng_normal(&g) * 1e-3));
			blk[208] = d & 0xFF; blk[209] = d >> 8;
		}
	}
}

void synth_normal(float *dst, long n, uint64_t seed, float stdv) {
	rng_t g; rng_init(&g, key3(seed, 0x71, 0));
	for (long i = 0; i < n; i++) dst[i] = (float)(rng_normal(&g) * stdv);
}

/* ------------------------------------------------------------- model */

typedef struct {
	int n_layers, d_model, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, ctx;
	float rope_theta, rms_eps;
	int tied;           /* lm_head == token_embd */
	int qkv_bias;
	uint64_t seed;
	float wstd;         /* weight std (0.02) */
} synth_cfg;

enum { T_F32 = 0, T_Q4K = 12, T_Q6K = 14 };
enum { K_ONES = 0, K_NORMAL = 1 };

typedef struct {
	char name[48];
	int type, kind, n_dims;
	long cols, rows;      /* dims[0] = cols, dims[1] = rows */
	uint64_t rel, nbytes;
} tdesc;

static uint64_t tbytes(int type, long cols, long rows) {
	if (type == T_Q4K) return (uint64_t)(cols / 256) * 144 * rows;
	if (type == T_Q6K) return (uint64_t)(cols / 256) * 210 * rows;
	return (uint64_t)cols * rows * 4;
}

static int build_dir(const synth_cfg *c, tdesc *t) {
	int n = 0, D = c->d_model, KV = c->n_kv_heads * c->head_dim, F = c->ffn_dim;
#define ADD(nm_, ty_, kd_, nd_, co_, ro_) do { \
		snprintf(t[n].name, 48, "%s", nm_); t[n].type = ty_; t[n].kind = kd_; \
		t[n].n_dims = nd_; t[n].cols = co_; t[n].rows = ro_; \
		t[n].nbytes = tbytes(ty_, co_, ro_); n++; } while (0)
	char nm[64];
	ADD("token_embd.weight", T_Q6K, K_NORMAL, 2, D, c->vocab);
	for (int l = 0; l < c->n_layers; l++) {
#define L_(s, ty, kd, nd, co, ro) snprintf(nm, 64, "blk.%d.%s", l, s); ADD(nm, ty, kd, nd, co, ro);
		L_("attn_norm.weight", T_F32, K_ONES, 1, D, 1)
		L_("attn_q.weight", T_Q4K, K_NORMAL, 2, D, D)
		L_("attn_k.weight", T_Q4K, K_NORMAL, 2, D, KV)
		L_("attn_v.weight", T_Q6K, K_NORMAL, 2, D, KV)
		if (c->qkv_bias) {
			L_("attn_q.bias", T_F32, K_NORMAL, 1, D, 1)
			L_("attn_k.bias", T_F32, K_NORMAL, 1, KV, 1)
			L_("attn_v.bias", T_F32, K_NORMAL, 1, KV, 1)
		}
		L_("attn_output.weight", T_Q4K, K_NORMAL, 2, D, D)
		L_("ffn_norm.weight", T_F32, K_ONES, 1, D, 1)
		L_("ffn_gate.weight", T_Q4K, K_NORMAL, 2, D, F)
		L_("ffn_up.weight", T_Q4K, K_NORMAL, 2, D, F)
		L_("ffn_down.weight", T_Q6K, K_NORMAL, 2, F, D)
#undef L_
	}
	ADD("output_norm.weight", T_F32, K_ONES, 1, D, 1);
	if (!c->tied) ADD("output.weight", T_Q6K, K_NORMAL, 2, D, c->vocab);
#undef ADD
	return n;
}

/* Tokenizer blob (include/mlf2.h:89-102): byte tokens 0..255 under the GPT-2
 * byte map, four merged tokens, placeholders, then three control tokens
 * <|endoftext|>, <|im_start|>, <|im_end|> (at 151643.. when the vocab is
 * Qwen-sized, else the last three ids). */
static int gpt2_cp(int b) {
	int n = 0;
	for (int x = 0; x < 256; x++) {
		int pr = (x >= 33 && x <= 126) || (x >= 0xA1 && x <= 0xAC) || (x >= 0xAE && x <= 0xFF);
		if (x == b) return pr ? x : 256 + n;
		if (!pr) n++;
	}
	return -1;
}
static int put_utf8(int cp, char *o) {
	if (cp < 0x80) { o[0] = (char)cp; return 1; }
	o[0] = (char)(0xC0 | (cp >> 6)); o[1] = (char)(0x80 | (cp & 0x3F)); return 2;
}
static int special_base(int V) { return V >= 151646 ? 151643 : V - 3; }

static size_t tok_blob(const synth_cfg *c, uint8_t *o) {
	size_t p = 0;
	int V = c->vocab, sb = special_base(V);
	static const char *merged[4][2] = { { "Ġt", "Ġ t" }, { "he", "h e" }, { "in", "i n" }, { "Ġthe", "Ġt he" } };
	uint32_t nt = (uint32_t)V, nm = 4;
	if (o) { memcpy(o, &nt, 4); memcpy(o + 4, &nm, 4); }
	p = 8;
	for (int id = 0; id < V; id++) {
		char s[64]; int len; uint8_t type = 1;
		if (id < 256) len = put_utf8(gpt2_cp(id), s);
		else if (id < 260) len = (int)strlen(strcpy(s, merged[id - 256][0]));
		else if (id == sb) { len = (int)strlen(strcpy(s, "<|endoftext|>")); type = 3; }
		else if (id == sb + 1) { len = (int)strlen(strcpy(s, "<|im_start|>")); type = 3; }
		else if (id == sb + 2) { len = (int)strlen(strcpy(s, "<|im_end|>")); type = 3; }
		else len = snprintf(s, sizeof s, "<t%d>", id);
		if (o) { o[p] = type; uint32_t l = (uint32_t)len; memcpy(o + p + 1, &l, 4); memcpy(o + p + 5, s, (size_t)len); }
		p += 5 + (size_t)len;
	}
	for (int i = 0; i < 4; i++) {
		uint32_t l = (uint32_t)strlen(merged[i][1]);
		if (o) { memcpy(o + p, &l, 4); memcpy(o + p + 4, merged[i][1], l); }
		p += 4 + l;
	}
	return p;
}

typedef struct {
	const synth_cfg *c; tdesc *t; int nt; uint8_t *data;
	long *work_t, *work_r0, *work_r1; long n_work; long next;
	pthread_mutex_t mu;
} job_t;

static void gen_rows(const synth_cfg *c, const tdesc *t, int ti, long r0, long r1, uint8_t *dst) {
	long cols = t->cols;
	float *buf = malloc(sizeof(float) * (size_t)cols);
	for (long r = r0; r < r1; r++) {
		if (t->kind == K_ONES) { for (long i = 0; i < cols; i++) buf[i] = 1.0f; }
		else {
			rng_t g; rng_init(&g, key3(c->seed, (uint64_t)ti, (uint64_t)r));
			for (long i = 0; i < cols; i++) buf[i] = (float)(rng_normal(&g) * c->wstd);
		}
		if (t->type == T_F32) memcpy(dst + (size_t)r * cols * 4, buf, (size_t)cols * 4);
		else if (t->type == T_Q4K)
			for (long b = 0; b < cols / 256; b++)
				synth_quantize_q4k_block(buf + 256 * b, dst + ((size_t)r * (cols / 256) + b) * 144);
		else
			for (long b = 0; b < cols / 256; b++)
				synth_quantize_q6k_block(buf + 256 * b, dst + ((size_t)r * (cols / 256) + b) * 210);
	}
	free(buf);
}

static void *worker(void *arg) {
	job_t *j = (job_t *)arg;
	for (;;) {
		pthread_mutex_lock(&j->mu);
		long w = j->next++;
		pthread_mutex_unlock(&j->mu);
		if (w >= j->n_work) return NULL;
		int ti = (int)j->work_t[w];
		gen_rows(j->c, &j->t[ti], ti, j->work_r0[w], j->work_r1[w], j->data + j->t[ti].rel);
	}
}

/* Size in bytes of the MLF2 file synth_write_model would produce. */
uint64_t synth_model_size(const synth_cfg *c) {
	tdesc *t = calloc(16 + 16 * (size_t)c->n_layers, sizeof(tdesc));
	int n = build_dir(c, t);
	uint64_t data_off = (128 + 104 * (uint64_t)n + tok_blob(c, NULL) + 31) / 32 * 32, cur = 0;
	for (int i = 0; i < n; i++) cur += (t[i].nbytes + 31) / 32 * 32;
	free(t);
	return data_off + cur;
}

/* Write a synthetic MLF2 model to `path`. Returns 0 on success. */
int synth_write_model(const char *path, const synth_cfg *c, int n_threads) {
	if (c->d_model % 256 || c->ffn_dim % 256 || c->n_heads % c->n_kv_heads ||
	    c->head_dim % 2 || c->n_heads * c->head_dim != c->d_model) return -2;
	tdesc *t = calloc(16 + 16 * (size_t)c->n_layers, sizeof(tdesc));
	int n = build_dir(c, t);
	size_t tb = tok_blob(c, NULL);
	uint64_t tensors_off = 128, tok_off = tensors_off + 104 * (uint64_t)n;
	uint64_t data_off = (tok_off + tb + 31) / 32 * 32, cur = 0;
	for (int i = 0; i < n; i++) { t[i].rel = cur; cur += (t[i].nbytes + 31) / 32 * 32; }
	uint64_t total = data_off + cur;

	int fd = open(path, O_RDWR | O_CREAT | O_TRUNC, 0644);
	if (fd < 0) { free(t); return -1; }
	if (ftruncate(fd, (off_t)total) != 0) { close(fd); free(t); return -1; }
	uint8_t *m = mmap(NULL, total, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
	close(fd);
	if (m == MAP_FAILED) { free(t); return -1; }

	uint8_t *h = m;
	memcpy(h, "MLF2", 4);
	uint32_t u[14] = { 2, 0, (uint32_t)c->n_layers, (uint32_t)c->d_model, (uint32_t)c->n_heads,
	                   (uint32_t)c->n_kv_heads, (uint32_t)c->head_dim, (uint32_t)c->ffn_dim,
	                   (uint32_t)c->ctx, (uint32_t)c->vocab, 0, 0, 0, (uint32_t)n };
	memcpy(u + 10, &c->rope_theta, 4); memcpy(u + 11, &c->rms_eps, 4);
	u[12] = (c->qkv_bias ? 1u : 0u) | (c->tied ? 2u : 0u);
	memcpy(h + 4, u, sizeof u);                           /* 4 .. 60 */
	memcpy(h + 60, &tensors_off, 8); memcpy(h + 68, &tok_off, 8); memcpy(h + 76, &data_off, 8);
	uint32_t bos = (uint32_t)special_base(c->vocab), eos = bos + 2;
	memcpy(h + 84, &bos, 4); memcpy(h + 88, &eos, 4);     /* reserved[36] stays zero */
	for (int i = 0; i < n; i++) {
		uint8_t *e = m + tensors_off + 104 * (uint64_t)i;
		memcpy(e, t[i].name, 48);
		uint32_t ty = (uint32_t)t[i].type, nd = (uint32_t)t[i].n_dims;
		uint64_t dims[4] = { (uint64_t)t[i].cols, t[i].n_dims > 1 ? (uint64_t)t[i].rows : 0, 0, 0 };
		memcpy(e + 48, &ty, 4); memcpy(e + 52, &nd, 4); memcpy(e + 56, dims, 32);
		memcpy(e + 88, &t[i].rel, 8); memcpy(e + 96, &t[i].nbytes, 8);
	}
	tok_blob(c, m + tok_off);

	job_t j;
	memset(&j, 0, sizeof j);
	j.c = c; j.t = t; j.nt = n; j.data = m + data_off;
	long cap = 0;
	for (int i = 0; i < n; i++) cap += (t[i].rows + 63) / 64;
	j.work_t = malloc(sizeof(long) * cap); j.work_r0 = malloc(sizeof(long) * cap); j.work_r1 = malloc(sizeof(long) * cap);
	for (int i = 0; i < n; i++)
		for (long r = 0; r < t[i].rows; r += 64) {
			j.work_t[j.n_work] = i; j.work_r0[j.n_work] = r;
			j.work_r1[j.n_work] = r + 64 < t[i].rows ? r + 64 : t[i].rows; j.n_work++;
		}
	pthread_mutex_init(&j.mu, NULL);
	if (n_threads < 1) n_threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
	if (n_threads > 256) n_threads = 256;
	pthread_t th[256];
	for (int i = 0; i < n_threads; i++) pthread_create(&th[i], NULL, worker, &j);
	for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
	free(j.work_t); free(j.work_r0); free(j.work_r1); free(t);
	msync(m, total, MS_SYNC);
	munmap(m, total);
	return 0;
}

#ifdef SYNTH_MAIN
/* Stand-alone writer (hako_b200/_lib/hakm_synth): lets a process that must
 * not map this library (the benchmark's reference arm) still produce the
 * seeded model file.
 *   hakm_synth size  L D H KVH HD F V CTX THETA EPS TIED BIAS SEED WSTD
 *   hakm_synth write PATH L D H KVH HD F V CTX THETA EPS TIED BIAS SEED WSTD */
#include <stdio.h>
int main(int argc, char **argv) {
	int write = argc == 17 && strcmp(argv[1], "write") == 0;
	if (!write && !(argc == 16 && strcmp(argv[1], "size") == 0)) {
		fprintf(stderr, "usage: %s size|write [PATH] L D H KVH HD F V CTX THETA EPS TIED BIAS SEED WSTD\n", argv[0]);
		return 2;
	}
	char **a = argv + (write ? 3 : 2);
	synth_cfg c;
	c.n_layers = atoi(a[0]); c.d_model = atoi(a[1]); c.n_heads = atoi(a[2]); c.n_kv_heads = atoi(a[3]);
	c.head_dim = atoi(a[4]); c.ffn_dim = atoi(a[5]); c.vocab = atoi(a[6]); c.ctx = atoi(a[7]);
	c.rope_theta = strtof(a[8], NULL); c.rms_eps = strtof(a[9], NULL); c.tied = atoi(a[10]);
	c.qkv_bias = atoi(a[11]); c.seed = strtoull(a[12], NULL, 10); c.wstd = strtof(a[13], NULL);
	if (!write) {
		printf("%llu\n", (unsigned long long)synth_model_size(&c));
		return 0;
	}
	return synth_write_model(argv[2], &c, 0) == 0 ? 0 : 1;
}
#endif
