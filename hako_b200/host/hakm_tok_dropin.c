/* hakm_tok_dropin.c — the reference's tokenizer interface (src/bpe.h of
 * mithraeums/hako: tok_new, tok_free, tok_encode, tok_decode_id, tok_id,
 * tok_eos) over libhakm_tok (include/hakm_tok.h), so that cli/main.c and
 * src/hakm_api.c get the full Qwen2 pretokenizer without a change. Linked in
 * place of src/bpe.c; compiled with the reference's src/ on the include path
 * (for bpe.h and loader.h).
 *
 * Differences from src/bpe.c that a caller can see: tok_encode splits text by
 * the Qwen2 pattern instead of at spaces (bpe.h:10-13), so digit runs,
 * punctuation runs, contractions and whitespace runs tokenize as Qwen2's own
 * tokenizer does; pieces have no length limit (bpe.c:176 caps a piece at 2048
 * bytes); tok_new returns NULL, with a message on stderr, for a tokenizer
 * blob that runs past the end of the mapped file.
 */
#include "bpe.h"
#include "hakm_tok.h"

#include <stdlib.h>
#include <string.h>

struct hakm_tok {
	hakm_bpe *bpe;
};

hakm_tok *tok_new(const hakm_model *m)
{
	const unsigned char *base = (const unsigned char *)m->map;
	const size_t avail = m->tok >= base && m->tok < base + m->map_size ? (size_t)(base + m->map_size - m->tok) : 0;
	hakm_bpe *b = hakm_bpe_new(m->tok, avail, (int)m->h.eos_id);
	if (!b) return NULL;
	hakm_tok *t = malloc(sizeof *t);
	if (!t) { hakm_bpe_free(b); return NULL; }
	t->bpe = b;
	return t;
}

void tok_free(hakm_tok *t)
{
	if (!t) return;
	hakm_bpe_free(t->bpe);
	free(t);
}

int tok_encode(const hakm_tok *t, const char *text, int *out, int max)
{
	return hakm_bpe_encode(t->bpe, text, strlen(text), out, max);
}

int tok_decode_id(const hakm_tok *t, int id, char *out, int max)
{
	return hakm_bpe_decode_id(t->bpe, id, out, max);
}

int tok_id(const hakm_tok *t, const char *literal)
{
	return hakm_bpe_token_id(t->bpe, literal, strlen(literal));
}

int tok_eos(const hakm_tok *t)
{
	return hakm_bpe_eos(t->bpe);
}
