/* hakm_pretok.c — the Qwen2 pretokenizer: splits UTF-8 text into the pieces
 * that byte-level BPE then merges one at a time. The reference's tokenizer
 * splits at spaces only (src/bpe.h:10-13, src/bpe.c:167-170); Qwen2's own
 * tokenizer splits by the pattern
 *
 *   (?i:'s|'t|'re|'ve|'m|'ll|'d) | [^\r\n\p{L}\p{N}]?\p{L}+ | \p{N}
 *   | ?[^\s\p{L}\p{N}]+[\r\n]* | \s*[\r\n]+ | \s+(?!\S) | \s+
 *
 * taking at each position the first alternative that matches, each with
 * the regex engine's greedy-then-backtrack reading. This file restates that
 * as a hand-written matcher over code points (no regex engine), with the
 * Unicode classes from hakm_unicode_tables.h. Bytes that are not valid
 * UTF-8 count as single code points of no class (neither letter, number
 * nor space). C11, no dependencies.
 */
#include "hakm_tok.h"

#include "hakm_unicode_tables.h"

static int in_table(const uint32_t (*t)[2], int n, uint32_t cp) {
	int lo = 0, hi = n - 1;
	while (lo <= hi) {
		const int mid = (lo + hi) / 2;
		if (cp < t[mid][0]) hi = mid - 1;
		else if (cp > t[mid][1]) lo = mid + 1;
		else return 1;
	}
	return 0;
}

enum { C_OTHER = 0, C_LETTER = 1, C_NUMBER = 2, C_SPACE = 4, C_NEWLINE = 8 };

static int class_of(uint32_t cp) {
	if (cp == '\r' || cp == '\n') return C_SPACE | C_NEWLINE;
	if (cp < 0x80) {
		if ((cp | 0x20) >= 'a' && (cp | 0x20) <= 'z') return C_LETTER;
		if (cp >= '0' && cp <= '9') return C_NUMBER;
		if (cp == ' ' || (cp >= 0x09 && cp <= 0x0D)) return C_SPACE;
		return C_OTHER;
	}
	if (in_table(HAKM_UC_LETTER, (int)(sizeof HAKM_UC_LETTER / sizeof HAKM_UC_LETTER[0]), cp)) return C_LETTER;
	if (in_table(HAKM_UC_NUMBER, (int)(sizeof HAKM_UC_NUMBER / sizeof HAKM_UC_NUMBER[0]), cp)) return C_NUMBER;
	if (in_table(HAKM_UC_SPACE, (int)(sizeof HAKM_UC_SPACE / sizeof HAKM_UC_SPACE[0]), cp)) return C_SPACE;
	return C_OTHER;
}

/* The code point at s[i] (n bytes in all) and its byte length; an invalid or
 * truncated sequence is one byte of no class (cp 0xFFFFFFFF). */
static uint32_t decode(const unsigned char *s, size_t n, size_t i, int *len) {
	const unsigned char c = s[i];
	int need;
	uint32_t cp;
	if (c < 0x80) { *len = 1; return c; }
	if (c >= 0xC2 && c <= 0xDF) { need = 1; cp = c & 0x1F; }
	else if (c >= 0xE0 && c <= 0xEF) { need = 2; cp = c & 0x0F; }
	else if (c >= 0xF0 && c <= 0xF4) { need = 3; cp = c & 0x07; }
	else { *len = 1; return 0xFFFFFFFFu; }
	if (i + (size_t)need >= n) { *len = 1; return 0xFFFFFFFFu; }  /* truncated */
	for (int k = 1; k <= need; k++) {
		const unsigned char b = s[i + (size_t)k];
		if ((b & 0xC0) != 0x80) { *len = 1; return 0xFFFFFFFFu; }
		cp = (cp << 6) | (b & 0x3F);
	}
	/* overlong forms, surrogates and values past U+10FFFF are invalid */
	if ((need == 2 && (cp < 0x800 || (cp >= 0xD800 && cp <= 0xDFFF))) || (need == 3 && (cp < 0x10000 || cp > 0x10FFFF))) {
		*len = 1;
		return 0xFFFFFFFFu;
	}
	*len = need + 1;
	return cp;
}

/* Decoded text: code point classes and byte offsets. */
typedef struct {
	const unsigned char *s;
	size_t n;
} text_t;

static int cls_at(const text_t *t, size_t i, int *len) {
	const uint32_t cp = decode(t->s, t->n, i, len);
	return cp == 0xFFFFFFFFu ? C_OTHER : class_of(cp);
}

/* Length in bytes of the piece that starts at byte i. */
static size_t piece_at(const text_t *t, size_t i) {
	const unsigned char *s = t->s;
	const size_t n = t->n;
	int l0;
	const int c0 = cls_at(t, i, &l0);

	/* (?i:'s|'t|'re|'ve|'m|'ll|'d) */
	if (s[i] == '\'' && i + 1 < n) {
		const int a = s[i + 1] | 0x20, b = i + 2 < n ? (s[i + 2] | 0x20) : 0;
		if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
		if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
		/* U+017F LATIN SMALL LETTER LONG S case-folds to 's' */
		if (s[i + 1] == 0xC5 && i + 2 < n && s[i + 2] == 0xBF) return 3;
	}
	/* [^\r\n\p{L}\p{N}]?\p{L}+ */
	{
		size_t j = i;
		if (!(c0 & (C_NEWLINE | C_LETTER | C_NUMBER)) && i + (size_t)l0 < n) {
			int l1;
			if (cls_at(t, i + (size_t)l0, &l1) & C_LETTER) j = i + (size_t)l0;
		}
		int lj;
		if (j < n && (cls_at(t, j, &lj) & C_LETTER)) {
			j += (size_t)lj;
			while (j < n && (cls_at(t, j, &lj) & C_LETTER)) j += (size_t)lj;
			return j - i;
		}
	}
	/* \p{N} */
	if (c0 & C_NUMBER) return (size_t)l0;
	/* ' '?[^\s\p{L}\p{N}]+[\r\n]* */
	{
		size_t j = i;
		int lj;
		if (s[i] == ' ' && i + 1 < n && !(cls_at(t, i + 1, &lj) & (C_SPACE | C_LETTER | C_NUMBER))) j = i + 1;
		if (j < n && !(cls_at(t, j, &lj) & (C_SPACE | C_LETTER | C_NUMBER))) {
			j += (size_t)lj;
			while (j < n && !(cls_at(t, j, &lj) & (C_SPACE | C_LETTER | C_NUMBER))) j += (size_t)lj;
			while (j < n && (s[j] == '\r' || s[j] == '\n')) j++;
			return j - i;
		}
	}
	/* the whitespace alternatives: w = the whitespace run from i */
	if (c0 & C_SPACE) {
		size_t w = i, last_nl = 0, prev = i;
		int have_nl = 0, lw;
		while (w < n && (cls_at(t, w, &lw) & C_SPACE)) {
			if (s[w] == '\r' || s[w] == '\n') { have_nl = 1; last_nl = w; }
			prev = w;
			w += (size_t)lw;
		}
		/* \s*[\r\n]+ : up to the run's last newline */
		if (have_nl) return last_nl + 1 - i;
		/* \s+(?!\S) : the whole run at the end of the text, else all but its
		 * last code point when that leaves one */
		if (w >= n) return w - i;
		if (prev > i) return prev - i;
		/* \s+ */
		return w - i;
	}
	/* not reached for valid classes: one code point */
	return (size_t)l0;
}

int hakm_pretok_split(const char *text, size_t n, size_t *ends, int max)
{
	text_t t = { (const unsigned char *)text, n };
	int k = 0;
	for (size_t i = 0; i < n;) {
		const size_t len = piece_at(&t, i);
		i += len ? len : 1;
		if (k >= max) return -1;
		ends[k++] = i;
	}
	return k;
}
