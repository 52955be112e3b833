/* hakm_model_cuda.c — drop-in replacement for the reference engine's
 * src/model.c on a B200: the same four entry points of src/model.h
 * (hakm_ctx_new, hakm_ctx_free, hakm_forward, hakm_reset) over libhakm_cuda.
 *
 * Link this file instead of src/model.c. The callers keep working unchanged:
 * cli/main.c, src/hakm_api.c and src/sample.c only read c->model (tokenizer,
 * tensor directory), c->logits, c->vocab, c->pos, c->max_seq and the shape
 * fields, all of which are maintained here. C11, no CUDA headers: the device
 * side is reached only through include/hakm_cuda.h.
 *
 * Differences a caller can see:
 *   - k_cache / v_cache and the scratch pointers are NULL: the KV cache and
 *     the activations live in device memory.
 *   - hakm_forward copies the logits of the step into c->logits (the
 *     reference returns its own scratch buffer; the pointer is equally valid
 *     until the next call).
 *   - HAKMC_DEVICE (environment) picks the GPU, default 0.
 *   - HAKMC_TOKEN_LOG (environment), if set, names a file that receives
 *     every id hakm_forward is given, one per line (stream comparisons).
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "hakm_cuda.h"
#include "model.h"

/* hakm_ctx first, so the pointer callers hold is also the wrapper's */
typedef struct {
	hakm_ctx   c;
	hakmc_ctx *dev;
	FILE      *token_log;
} cuda_ctx;

static cuda_ctx *wrapper(hakm_ctx *c) { return (cuda_ctx *)c; }

hakm_ctx *hakm_ctx_new(const char *mlf2_path, int max_seq)
{
	cuda_ctx *w = calloc(1, sizeof *w);
	if (!w) { fprintf(stderr, "hakm: out of memory\n"); return NULL; }
	hakm_ctx *c = &w->c;
	if (mlf2_open(mlf2_path, &c->model)) { free(w); return NULL; }

	const mlf2_header *h = &c->model.h;
	c->n_layers   = (int)h->n_layers;
	c->d_model    = (int)h->d_model;
	c->n_heads    = (int)h->n_heads;
	c->n_kv_heads = (int)h->n_kv_heads;
	c->head_dim   = (int)h->head_dim;
	c->kv_dim     = c->n_kv_heads * c->head_dim;
	c->ffn_dim    = (int)h->ffn_dim;
	c->vocab      = (int)h->vocab;
	c->rope_theta = h->rope_theta;
	c->rms_eps    = h->rms_eps;
	c->max_seq    = max_seq;
	c->pos        = 0;
	c->tok_embd   = mlf2_find(&c->model, "token_embd.weight");
	c->out_norm   = mlf2_find(&c->model, "output_norm.weight");
	c->out_weight = (h->flags & MLF2_FLAG_TIED_EMBED) ? c->tok_embd
	                                                  : mlf2_find(&c->model, "output.weight");

	c->logits = malloc((size_t)c->vocab * sizeof(float));
	const char *dev_env = getenv("HAKMC_DEVICE");
	const int dev = dev_env ? atoi(dev_env) : 0;
	if (c->logits)
		w->dev = hakmc_create(c->model.map, c->model.map_size, max_seq, 1, dev);
	if (!w->dev) {
		fprintf(stderr, "hakm: %s\n", c->logits ? hakmc_last_error() : "out of memory");
		free(c->logits);
		mlf2_close(&c->model);
		free(w);
		return NULL;
	}
	const char *log_path = getenv("HAKMC_TOKEN_LOG");
	if (log_path && log_path[0]) w->token_log = fopen(log_path, "w");
	return c;
}

void hakm_ctx_free(hakm_ctx *c)
{
	if (!c) return;
	cuda_ctx *w = wrapper(c);
	if (w->token_log) fclose(w->token_log);
	hakmc_destroy(w->dev);
	free(c->logits);
	mlf2_close(&c->model);
	free(w);
}

const float *hakm_forward(hakm_ctx *c, int token)
{
	cuda_ctx *w = wrapper(c);
	if (w->token_log) fprintf(w->token_log, "%d\n", token);
	if (hakmc_forward(w->dev, token, c->logits, NULL) != 0) {
		fprintf(stderr, "hakm: forward at position %d: %s\n", c->pos, hakmc_last_error());
		return c->logits;
	}
	c->pos++;
	return c->logits;
}

void hakm_reset(hakm_ctx *c)
{
	hakmc_reset(wrapper(c)->dev);
	c->pos = 0;
}
