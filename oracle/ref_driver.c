/*
 * ref_driver.c — thin C entry points over the reference engine's OWN compiled
 * sources (src/{loader,quant,nn,model,sample}.c of mithraeums/hako), so the
 * tests and the CPU baseline can call them with token ids and raw buffers.
 *
 * TEST INFRASTRUCTURE ONLY: linked into oracle/_ref/libhakm_ref.so by
 * oracle/Makefile, never into the shipped library. The reference CLI cannot
 * take token ids (cli/main.c:150-156), hence this driver.
 */
#include "model.h"
#include "nn.h"
#include "quant.h"
#include "sample.h"

#include <stdlib.h>
#include <string.h>

/* hakm_ctx_new (src/model.c:17-76) */
void *refd_open(const char *path, int max_seq) { return hakm_ctx_new(path, max_seq); }
void refd_close(void *c) { hakm_ctx_free((hakm_ctx *)c); }
void refd_reset(void *c) { hakm_reset((hakm_ctx *)c); }
int refd_vocab(void *c) { return ((hakm_ctx *)c)->vocab; }
int refd_dim(void *c) { return ((hakm_ctx *)c)->d_model; }
int refd_pos(void *c) { return ((hakm_ctx *)c)->pos; }
int refd_n_layers(void *c) { return ((hakm_ctx *)c)->n_layers; }

/* Run only the first n layers (hakm_forward loops over c->n_layers,
 * src/model.c:102); the residual stream is then left in c->xb. */
void refd_set_layers(void *c, int n) { ((hakm_ctx *)c)->n_layers = n; }
const float *refd_hidden(void *c) { return ((hakm_ctx *)c)->xb; }

/* One hakm_forward step (src/model.c:93-165); optional logits copy and the
 * greedy pick of sample_token (src/sample.c:27-32, temperature 0). */
int refd_forward(void *cv, int token, float *logits_out, int *argmax_out) {
	hakm_ctx *c = (hakm_ctx *)cv;
	if (c->pos >= c->max_seq) return -1;
	const float *lg = hakm_forward(c, token);
	if (logits_out) memcpy(logits_out, lg, sizeof(float) * (size_t)c->vocab);
	if (argmax_out) {
		sampler s;
		sampler_init(&s, 0.0f, 0.0f, 0, 1);
		*argmax_out = sample_token(&s, c->logits, c->vocab);
	}
	return 0;
}

/* Greedy decode: feed `n_prompt` ids, then generate `n_gen` ids (each sampled
 * from the logits left by the previous forward, src/hakm_api.c:157-166).
 * gaps[i] = top1 - top2 logit at generated step i (NULL to skip). */
int refd_greedy(void *cv, const int *prompt, int n_prompt, int n_gen,
                int *out_tokens, float *gaps) {
	hakm_ctx *c = (hakm_ctx *)cv;
	sampler s;
	sampler_init(&s, 0.0f, 0.0f, 0, 1);
	for (int i = 0; i < n_prompt; i++) {
		if (c->pos >= c->max_seq) return -1;
		hakm_forward(c, prompt[i]);
	}
	for (int g = 0; g < n_gen; g++) {
		int id = sample_token(&s, c->logits, c->vocab);
		out_tokens[g] = id;
		if (gaps) {
			float b1 = c->logits[id], b2 = -3.0e38f;
			for (int i = 0; i < c->vocab; i++)
				if (i != id && c->logits[i] > b2) b2 = c->logits[i];
			gaps[g] = b1 - b2;
		}
		if (g + 1 < n_gen) {
			if (c->pos >= c->max_seq) return -1;
			hakm_forward(c, id);
		}
	}
	return 0;
}

/* The reference matmul (src/nn.c:179-210) on a raw weight buffer: wraps the
 * buffer in a one-tensor model so the pool/worker code runs unchanged. */
int refd_matmul_raw(float *out, const float *x, int type, const void *w,
                    const float *bias, int n_out, int n_in) {
	hakm_model m;
	memset(&m, 0, sizeof m);
	m.data = (const unsigned char *)w;
	mlf2_tensor t;
	memset(&t, 0, sizeof t);
	t.type = (uint32_t)type;
	t.n_dims = 2;
	t.dims[0] = (uint64_t)n_in;
	t.dims[1] = (uint64_t)n_out;
	t.data_off = 0;
	matmul(out, x, &m, &t, bias, n_out, n_in);
	return 0;
}

/* Copy the KV cache of the first n_pos positions of every layer out of
 * hakm_ctx.k_cache / v_cache ([layer][max_seq][kv_dim], src/model.c:72-73)
 * into k / v laid out [layer][n_pos][kv_dim]. */
int refd_read_kv(void *cv, float *k, float *v, int n_pos) {
	hakm_ctx *c = (hakm_ctx *)cv;
	if (n_pos > c->max_seq) return -1;
	size_t row = (size_t)c->kv_dim * n_pos;
	for (int l = 0; l < c->n_layers; l++) {
		memcpy(k + (size_t)l * row, c->k_cache + (size_t)l * c->max_seq * c->kv_dim, row * sizeof(float));
		memcpy(v + (size_t)l * row, c->v_cache + (size_t)l * c->max_seq * c->kv_dim, row * sizeof(float));
	}
	return 0;
}

/* Set the decode position (hakm_ctx.pos, src/model.h:20) over a cache the
 * caller filled. */
void refd_set_pos(void *cv, int pos) { ((hakm_ctx *)cv)->pos = pos; }

/* Write k / v laid out [layer][n_pos][kv_dim] into the first n_pos
 * positions of every layer of hakm_ctx.k_cache / v_cache (src/model.h:21-22)
 * and set pos = n_pos: a pre-filled cache, as a caller of the reference can
 * make it. */
int refd_write_kv(void *cv, const float *k, const float *v, int n_pos) {
	hakm_ctx *c = (hakm_ctx *)cv;
	if (n_pos > c->max_seq) return -1;
	size_t row = (size_t)c->kv_dim * n_pos;
	for (int l = 0; l < c->n_layers; l++) {
		memcpy(c->k_cache + (size_t)l * c->max_seq * c->kv_dim, k + (size_t)l * row, row * sizeof(float));
		memcpy(c->v_cache + (size_t)l * c->max_seq * c->kv_dim, v + (size_t)l * row, row * sizeof(float));
	}
	c->pos = n_pos;
	return 0;
}
