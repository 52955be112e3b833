/* hakm_tok.h — C ABI of libhakm_tok: Qwen2 byte-level BPE with the full
 * Qwen2 pretokenizer, over the MLF2 tokenizer blob (include/mlf2.h:89-102 of
 * mithraeums/hako). Host code only (C11, no CUDA); the library is
 * hako_b200/_lib/libhakm_tok.so.
 *
 * It replaces the reference's tokenizer, src/bpe.h:8-23 / src/bpe.c, whose
 * pretokenizer splits at spaces only (bpe.h:10-13, bpe.c:167-172, listed as
 * a known gap in its README). hako_b200/host/hakm_tok_dropin.c implements
 * src/bpe.h itself over these calls, so the reference's callers (cli/main.c,
 * src/hakm_api.c) link it unchanged.
 *
 * Errors: constructors return NULL with a message on stderr; counts are -1
 * on overflow or on a symbol that is not in the vocabulary. All functions are
 * safe to call from several threads on the same tokenizer (it is read-only
 * after hakm_bpe_new).
 */
#pragma once
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct hakm_bpe hakm_bpe;

/* Parse an MLF2 tokenizer blob (at most blob_size bytes read): n_tokens,
 * n_merges, token records, merge records in rank order. eos_id comes from the
 * MLF2 header. Replaces tok_new (src/bpe.c:84-112). NULL on a malformed blob. */
hakm_bpe *hakm_bpe_new(const void *blob, size_t blob_size, int eos_id);
void      hakm_bpe_free(hakm_bpe *t);                 /* tok_free, bpe.c:114-119 */

int hakm_bpe_vocab(const hakm_bpe *t);                /* token count */
int hakm_bpe_eos(const hakm_bpe *t);                  /* tok_eos, bpe.c:121 */

/* Token id of a literal token string (e.g. "<|im_start|>"), -1 if absent.
 * tok_id, bpe.c:123-125, with an explicit length. */
int hakm_bpe_token_id(const hakm_bpe *t, const char *literal, size_t n);

/* Encode n bytes of UTF-8 text: the Qwen2 pretokenizer (hakm_pretok_split),
 * then rank-greedy BPE merges inside each piece (lowest merge rank first,
 * leftmost among equal ranks, as bpe.c:133-159). Writes at most max ids.
 * Returns the count, or -1 on overflow. Replaces tok_encode, bpe.c:161-188.
 * The text is taken as given: no Unicode normalisation, and control-token
 * strings are BPE-encoded like any other text (the reference's callers
 * inject those ids with tok_id). */
int hakm_bpe_encode(const hakm_bpe *t, const char *text, size_t n, int *out, int max);

/* Append the bytes of token id to out (at most max); returns bytes written,
 * 0 for an id out of range. Replaces tok_decode_id, bpe.c:190-200. */
int hakm_bpe_decode_id(const hakm_bpe *t, int id, char *out, int max);

/* The Qwen2 pretokenizer alone: split n bytes of UTF-8 into the pieces of
 *   (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}
 *   | ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
 * writing each piece's end offset (exclusive) to ends. Bytes that are not
 * valid UTF-8 are single code points of no class. Returns the piece count,
 * or -1 if more than max pieces. */
int hakm_pretok_split(const char *text, size_t n, size_t *ends, int max);

#ifdef __cplusplus
}
#endif
