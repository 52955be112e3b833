/* ref_tok.c — TEST INFRASTRUCTURE ONLY. Lets the tests call the reference's
 * own tokenizer (src/bpe.c of mithraeums/hako, compiled where it lies) on a
 * bare tokenizer blob: tok_new (bpe.c:84-112) reads only the blob pointer and
 * the header's eos_id from its hakm_model argument, so a model struct with
 * those two fields set stands in for a mapped MLF2 file. Built by
 * `make -C oracle reftok` into oracle/_ref/libref_bpe.so, with bpe.c.
 */
#include <string.h>

#include "bpe.h"

hakm_tok *ref_tok_from_blob(const void *blob, int eos_id)
{
	hakm_model m;
	memset(&m, 0, sizeof m);
	m.tok = (const unsigned char *)blob;
	m.h.eos_id = (unsigned)eos_id;
	return tok_new(&m);
}
