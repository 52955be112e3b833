/* hakm_bpe.c — Qwen2 byte-level BPE over the MLF2 tokenizer blob, with the
 * full Qwen2 pretokenizer (hakm_pretok.c). C11, no dependencies.
 *
 * Behaviour follows the reference's tokenizer (src/bpe.c of mithraeums/hako)
 * except for the pretokenizer, which there splits at spaces only
 * (bpe.c:167-172):
 *  - bytes map to symbols by the GPT-2 byte table (bpe.c:57-68): printable
 *    bytes '!'..'~', 0xA1..0xAC and 0xAE..0xFF are their own code point, the
 *    other 68 bytes take 256, 257, ... in byte order;
 *  - inside a piece, the adjacent pair with the lowest merge rank merges
 *    first, the leftmost among equal ranks (bpe.c:133-151); a merge record
 *    that appears twice keeps its later rank (bpe.c:28-35 overwrites);
 *  - a string that appears twice in the vocabulary resolves to its later id.
 * The merge loop here keys merges by token-id pairs. Pieces of up to 48
 * bytes keep their pairs' ranks in an array; longer ones take them from a
 * heap ordered by (rank, left position), discarding entries whose pair has
 * changed since they were pushed. Both give the same sequence of merges as
 * rescanning every pair after each merge; the heap in O(n log n).
 */
#include "hakm_tok.h"

#include <limits.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

struct hakm_bpe {
	int n_tokens, n_merges, eos;
	const unsigned char **tok;   /* token strings, into a private copy of the blob */
	int32_t *tok_len;
	unsigned char *blob;         /* the copy */
	int32_t *vslot;              /* vocabulary hash: slot -> token id, -1 empty */
	uint32_t vmask;
	uint64_t *mkey;              /* merge hash: (a << 32 | b) + 1, 0 empty */
	int32_t *mrank, *mres;       /* rank and result token (-1: not a token) */
	uint32_t mmask;
	int32_t byte_tok[256];       /* the one-byte symbol's token, -1 if absent */
	int16_t cp_byte[324];        /* mapped code point -> byte */
};

static uint64_t mix64(uint64_t x) {
	x ^= x >> 30; x *= 0xbf58476d1ce4e5b9ULL;
	x ^= x >> 27; x *= 0x94d049bb133111ebULL;
	return x ^ (x >> 31);
}

static uint64_t str_hash(const unsigned char *p, size_t n) {
	uint64_t h = n;
	size_t i = 0;
	for (; i + 8 <= n; i += 8) {
		uint64_t w;
		memcpy(&w, p + i, 8);
		h = mix64(h ^ w);
	}
	uint64_t w = 0;
	for (int k = 0; i < n; i++, k++) w |= (uint64_t)p[i] << (8 * k);
	return mix64(h ^ w ^ 0x9e3779b97f4a7c15ULL);
}

static uint32_t pow2_above(uint64_t n) {
	uint32_t c = 16;
	while (c < 2 * n && c < (1u << 31)) c <<= 1;
	return c;
}

static int vocab_find(const hakm_bpe *t, const unsigned char *s, size_t n) {
	for (uint32_t i = (uint32_t)str_hash(s, n) & t->vmask;; i = (i + 1) & t->vmask) {
		const int32_t id = t->vslot[i];
		if (id < 0) return -1;
		if ((size_t)t->tok_len[id] == n && !memcmp(t->tok[id], s, n)) return id;
	}
}

static void vocab_put(hakm_bpe *t, int id) {
	const unsigned char *s = t->tok[id];
	const size_t n = (size_t)t->tok_len[id];
	for (uint32_t i = (uint32_t)str_hash(s, n) & t->vmask;; i = (i + 1) & t->vmask) {
		const int32_t o = t->vslot[i];
		if (o < 0 || ((size_t)t->tok_len[o] == n && !memcmp(t->tok[o], s, n))) { t->vslot[i] = id; return; }
	}
}

static uint32_t merge_slot(const hakm_bpe *t, uint64_t key) {
	uint32_t i = (uint32_t)mix64(key) & t->mmask;
	while (t->mkey[i] && t->mkey[i] != key) i = (i + 1) & t->mmask;
	return i;
}

/* Rank of merging tokens a, b (INT32_MAX: no merge) and its result token. */
static int32_t merge_rank(const hakm_bpe *t, int32_t a, int32_t b, int32_t *res) {
	const uint32_t i = merge_slot(t, (((uint64_t)(uint32_t)a << 32) | (uint32_t)b) + 1);
	if (!t->mkey[i]) return INT32_MAX;
	*res = t->mres[i];
	return t->mrank[i];
}

static int utf8_put(uint32_t cp, unsigned char *o) {
	if (cp < 0x80) { o[0] = (unsigned char)cp; return 1; }
	o[0] = (unsigned char)(0xC0 | (cp >> 6));
	o[1] = (unsigned char)(0x80 | (cp & 0x3F));
	return 2;
}

static hakm_bpe *fail(hakm_bpe *t, void *scratch, const char *what) {
	fprintf(stderr, "hakm_bpe: malformed tokenizer blob: %s\n", what);
	free(scratch);
	hakm_bpe_free(t);
	return NULL;
}

hakm_bpe *hakm_bpe_new(const void *blob_in, size_t size, int eos_id)
{
	hakm_bpe *t = calloc(1, sizeof *t);
	if (!t || !blob_in || size < 8) return fail(t, NULL, "shorter than its counts");
	t->blob = malloc(size);
	if (!t->blob) return fail(t, NULL, "out of memory");
	memcpy(t->blob, blob_in, size);
	const unsigned char *p = t->blob, *end = t->blob + size;
	uint32_t nt, nm;
	memcpy(&nt, p, 4);
	memcpy(&nm, p + 4, 4);
	p += 8;
	if (nt == 0 || nt > (uint32_t)INT_MAX / 2 || nm > (uint32_t)INT_MAX / 2 || nt > size / 5)
		return fail(t, NULL, "token or merge count out of range");
	t->n_tokens = (int)nt;
	t->n_merges = (int)nm;
	t->eos = eos_id;
	t->tok = malloc(nt * sizeof *t->tok);
	t->tok_len = malloc(nt * sizeof *t->tok_len);
	t->vmask = pow2_above(nt) - 1;
	t->vslot = malloc(((size_t)t->vmask + 1) * sizeof *t->vslot);
	if (!t->tok || !t->tok_len || !t->vslot) return fail(t, NULL, "out of memory");
	memset(t->vslot, 0xff, ((size_t)t->vmask + 1) * sizeof *t->vslot);
	for (uint32_t i = 0; i < nt; i++) {
		uint32_t len;
		if (end - p < 5) return fail(t, NULL, "token records run past the end");
		memcpy(&len, p + 1, 4);   /* record: u8 type, u32 len, bytes */
		p += 5;
		if ((size_t)(end - p) < len || len > (uint32_t)INT_MAX) return fail(t, NULL, "token string runs past the end");
		t->tok[i] = p;
		t->tok_len[i] = (int32_t)len;
		vocab_put(t, (int)i);
		p += len;
	}
	t->mmask = pow2_above(nm) - 1;
	t->mkey = calloc((size_t)t->mmask + 1, sizeof *t->mkey);
	t->mrank = malloc(((size_t)t->mmask + 1) * sizeof *t->mrank);
	t->mres = malloc(((size_t)t->mmask + 1) * sizeof *t->mres);
	if (!t->mkey || !t->mrank || !t->mres) return fail(t, NULL, "out of memory");
	unsigned char *cat = NULL;
	size_t cat_cap = 0;
	for (uint32_t r = 0; r < nm; r++) {
		uint32_t len;
		if (end - p < 4) return fail(t, cat, "merge records run past the end");
		memcpy(&len, p, 4);
		p += 4;
		if ((size_t)(end - p) < len) return fail(t, cat, "merge string runs past the end");
		/* "A B": the first space at which both halves are tokens */
		int32_t a = -1, b = -1;
		for (uint32_t k = 1; k + 1 < len && b < 0; k++) {
			if (p[k] != ' ') continue;
			a = vocab_find(t, p, k);
			b = a < 0 ? -1 : vocab_find(t, p + k + 1, len - k - 1);
		}
		if (b >= 0) {
			if (cat_cap < len) {
				unsigned char *nc = realloc(cat, len);
				if (!nc) return fail(t, cat, "out of memory");
				cat = nc;
				cat_cap = len;
			}
			const size_t la = (size_t)t->tok_len[a], lb = (size_t)t->tok_len[b];
			memcpy(cat, t->tok[a], la);
			memcpy(cat + la, t->tok[b], lb);
			const uint32_t i = merge_slot(t, (((uint64_t)(uint32_t)a << 32) | (uint32_t)b) + 1);
			t->mkey[i] = (((uint64_t)(uint32_t)a << 32) | (uint32_t)b) + 1;
			t->mrank[i] = (int32_t)r;
			t->mres[i] = vocab_find(t, cat, la + lb);
		}
		p += len;
	}
	free(cat);
	/* the GPT-2 byte table */
	for (int i = 0; i < 324; i++) t->cp_byte[i] = -1;
	int extra = 0;
	for (int c = 0; c < 256; c++) {
		const int printable = (c >= '!' && c <= '~') || (c >= 0xA1 && c <= 0xAC) || (c >= 0xAE && c <= 0xFF);
		const uint32_t cp = printable ? (uint32_t)c : 256u + (uint32_t)extra++;
		unsigned char u[2];
		t->byte_tok[c] = vocab_find(t, u, (size_t)utf8_put(cp, u));
		t->cp_byte[cp] = (int16_t)c;
	}
	return t;
}

void hakm_bpe_free(hakm_bpe *t)
{
	if (!t) return;
	free(t->tok); free(t->tok_len); free(t->blob); free(t->vslot);
	free(t->mkey); free(t->mrank); free(t->mres);
	free(t);
}

int hakm_bpe_vocab(const hakm_bpe *t) { return t ? t->n_tokens : 0; }
int hakm_bpe_eos(const hakm_bpe *t) { return t ? t->eos : -1; }

int hakm_bpe_token_id(const hakm_bpe *t, const char *literal, size_t n)
{
	return t && literal ? vocab_find(t, (const unsigned char *)literal, n) : -1;
}

/* Per-call scratch for the merge loop of one piece. */
typedef struct {
	int32_t *sym, *next, *prev;
	uint64_t *heap;   /* rank << 32 | left symbol's position */
	size_t cap, nheap;
} work_t;

static int work_reserve(work_t *w, size_t n) {
	if (n <= w->cap) return 0;
	size_t c = w->cap ? w->cap : 64;
	while (c < n) c *= 2;
	int32_t *s = realloc(w->sym, c * sizeof *s);
	if (s) w->sym = s;
	int32_t *nx = realloc(w->next, c * sizeof *nx);
	if (nx) w->next = nx;
	int32_t *pv = realloc(w->prev, c * sizeof *pv);
	if (pv) w->prev = pv;
	uint64_t *h = realloc(w->heap, 3 * c * sizeof *h);
	if (h) w->heap = h;
	if (!s || !nx || !pv || !h) return -1;
	w->cap = c;
	return 0;
}

static void heap_push(work_t *w, uint64_t v) {
	size_t i = w->nheap++;
	while (i) {
		const size_t up = (i - 1) / 2;
		if (w->heap[up] <= v) break;
		w->heap[i] = w->heap[up];
		i = up;
	}
	w->heap[i] = v;
}

static uint64_t heap_pop(work_t *w) {
	const uint64_t top = w->heap[0], v = w->heap[--w->nheap];
	size_t i = 0;
	for (;;) {
		size_t c = 2 * i + 1;
		if (c >= w->nheap) break;
		if (c + 1 < w->nheap && w->heap[c + 1] < w->heap[c]) c++;
		if (w->heap[c] >= v) break;
		w->heap[i] = w->heap[c];
		i = c;
	}
	if (w->nheap) w->heap[i] = v;
	return top;
}

static void push_pair(const hakm_bpe *t, work_t *w, int32_t left) {
	const int32_t right = w->next[left];
	if (right < 0) return;
	int32_t res = -1;
	const int32_t rank = merge_rank(t, w->sym[left], w->sym[right], &res);
	if (rank != INT32_MAX) heap_push(w, ((uint64_t)(uint32_t)rank << 32) | (uint32_t)left);
}

/* Short pieces (most of them): the pairs' ranks in an array, the lowest
 * (leftmost on ties) merged, the array closed up and the two pairs next to
 * the merge looked up again. Same merges as the heap path. */
enum { SMALL_PIECE = 48 };

static int bpe_small(const hakm_bpe *t, const unsigned char *s, int n, int *out, int oi, int max) {
	int32_t sym[SMALL_PIECE], rk[SMALL_PIECE], res[SMALL_PIECE];
	for (int i = 0; i < n; i++) sym[i] = t->byte_tok[s[i]];
	for (int i = 0; i + 1 < n; i++)
		rk[i] = sym[i] < 0 || sym[i + 1] < 0 ? INT32_MAX : merge_rank(t, sym[i], sym[i + 1], &res[i]);
	while (n > 1) {
		int b = 0;
		for (int i = 1; i + 1 < n; i++)
			if (rk[i] < rk[b]) b = i;
		if (rk[b] == INT32_MAX) break;
		sym[b] = res[b];
		for (int i = b + 1; i + 1 < n; i++) { sym[i] = sym[i + 1]; rk[i] = rk[i + 1]; res[i] = res[i + 1]; }
		n--;
		if (b > 0)
			rk[b - 1] = sym[b - 1] < 0 || sym[b] < 0 ? INT32_MAX : merge_rank(t, sym[b - 1], sym[b], &res[b - 1]);
		if (b + 1 < n)
			rk[b] = sym[b] < 0 || sym[b + 1] < 0 ? INT32_MAX : merge_rank(t, sym[b], sym[b + 1], &res[b]);
	}
	for (int i = 0; i < n; i++) {
		if (sym[i] < 0 || oi >= max) return -1;
		out[oi++] = sym[i];
	}
	return oi;
}

/* Merge the n-byte piece s and append its tokens to out[oi..max). Returns the
 * new count, or -1 on overflow / a symbol that is not a token. */
static int bpe_piece(const hakm_bpe *t, work_t *w, const unsigned char *s, size_t n, int *out, int oi, int max) {
	if (n <= SMALL_PIECE) return bpe_small(t, s, (int)n, out, oi, max);
	if (work_reserve(w, n)) return -1;
	for (size_t i = 0; i < n; i++) {
		w->sym[i] = t->byte_tok[s[i]];
		w->next[i] = i + 1 < n ? (int32_t)(i + 1) : -1;
		w->prev[i] = (int32_t)i - 1;
	}
	w->nheap = 0;
	for (size_t i = 0; i + 1 < n; i++)
		if (w->sym[i] >= 0 && w->sym[i + 1] >= 0) push_pair(t, w, (int32_t)i);
	while (w->nheap) {
		const uint64_t e = heap_pop(w);
		const int32_t left = (int32_t)(uint32_t)e, rank = (int32_t)(e >> 32);
		const int32_t right = w->next[left];
		if (right < 0 || w->sym[left] < 0 || w->sym[right] < 0) continue;   /* dead or not a token */
		int32_t res = -1;
		if (merge_rank(t, w->sym[left], w->sym[right], &res) != rank) continue;   /* stale */
		w->sym[left] = res;                 /* -1 if the result is not a token */
		w->sym[right] = INT32_MIN;          /* dead */
		w->next[left] = w->next[right];
		if (w->next[right] >= 0) w->prev[w->next[right]] = left;
		if (res < 0) continue;
		if (w->prev[left] >= 0 && w->sym[w->prev[left]] >= 0) push_pair(t, w, w->prev[left]);
		push_pair(t, w, left);
	}
	for (int32_t i = 0; i >= 0; i = w->next[i]) {
		if (w->sym[i] < 0 || oi >= max) return -1;
		out[oi++] = w->sym[i];
	}
	return oi;
}

int hakm_bpe_encode(const hakm_bpe *t, const char *text, size_t n, int *out, int max)
{
	if (!t || (!text && n)) return -1;
	if (n == 0) return 0;
	if (n > (size_t)INT_MAX) return -1;
	size_t *ends = malloc(n * sizeof *ends);
	if (!ends) return -1;
	const int np = hakm_pretok_split(text, n, ends, (int)n);
	work_t w = {0};
	int oi = np < 0 ? -1 : 0;
	for (int k = 0, start = 0; k < np && oi >= 0; start = (int)ends[k++])
		oi = bpe_piece(t, &w, (const unsigned char *)text + start, ends[k] - (size_t)start, out, oi, max);
	free(w.sym); free(w.next); free(w.prev); free(w.heap);
	free(ends);
	return oi;
}

int hakm_bpe_decode_id(const hakm_bpe *t, int id, char *out, int max)
{
	if (!t || id < 0 || id >= t->n_tokens) return 0;
	const unsigned char *p = t->tok[id];
	const int32_t n = t->tok_len[id];
	int o = 0;
	for (int32_t k = 0; k < n;) {
		/* the token's code points; those outside the byte table are dropped */
		const unsigned char c = p[k];
		uint32_t cp;
		int len;
		if (c < 0x80) { cp = c; len = 1; }
		else if ((c & 0xE0) == 0xC0 && k + 1 < n) { cp = ((uint32_t)(c & 0x1F) << 6) | (p[k + 1] & 0x3F); len = 2; }
		else { cp = UINT32_MAX; len = (c & 0xF0) == 0xE0 ? 3 : (c & 0xF8) == 0xF0 ? 4 : 1; }
		k += len;
		if (cp < 324 && t->cp_byte[cp] >= 0 && o < max) out[o++] = (char)t->cp_byte[cp];
	}
	return o;
}
