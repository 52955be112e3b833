/* hakm_model_cuda.c — drop-in replacement for the reference engine's
 * src/model.c on a B200: the same four entry points of src/model.h
 * (hakm_ctx_new, hakm_ctx_free, hakm_forward, hakm_reset) over libhakm_cuda,
 * plus sample_token (src/sample.h) so that the pick is made on the device.
 *
 * Link this file instead of src/model.c, and compile the reference's
 * src/sample.c with -Dsample_token=hakm_ref_sample_token (its own sampler
 * stays available under that name for logits that are not a context's).
 * The callers keep working unchanged: cli/main.c, src/hakm_api.c read
 * c->model (tokenizer, tensor directory), c->pos, c->max_seq, c->vocab and
 * the shape fields, all maintained here, and they read the logits only
 * through sample_token(sp, c->logits, c->vocab).
 *
 * Deferred feed. hakm_forward records the id and returns at once; the ids
 * run on the GPU when their logits are first needed, that is when
 * sample_token is called on c->logits. A prompt fed id by id therefore runs
 * as one batched pass (hakmc_prefill_batched: every position through each
 * layer together, each weight read once per chunk) or, for a few ids, one
 * step-kernel launch (hakmc_prefill); a generated id runs as one decode
 * step. The pick is then made on the device (hakmc_sample_last: greedy or
 * temperature / top-k / top-p, bit-identical to the reference's
 * sample_token), so the logits never cross to the host. Results are the
 * reference's, bit for bit, whichever way the ids are grouped.
 *
 * Differences a caller can see:
 *   - k_cache / v_cache and the scratch pointers are NULL: the KV cache and
 *     the activations live in device memory.
 *   - c->logits holds the step's logits only with HAKMC_EAGER=1 (every
 *     hakm_forward then runs at once and copies its logits, as the
 *     reference's returns its scratch buffer). Without it, code that reads
 *     c->logits other than through sample_token sees stale values.
 *   - sample_token on c->logits does not turn the array into probabilities
 *     (the reference's does, in place); no caller reads them afterwards.
 *   - HAKMC_DEVICE (environment) picks the GPU, default 0.
 *   - HAKMC_GPUS=N (environment, 2..8) runs the context tensor parallel over
 *     GPUs HAKMC_DEVICE .. HAKMC_DEVICE+N-1 (hakmc_tp_*: every phase's rows
 *     split over all GPUs, outputs all-gathered by peer stores), one thread
 *     per GPU making the same calls; the results are the one-GPU results,
 *     bit for bit.
 *   - HAKMC_TOKEN_LOG (environment), if set, names a file that receives
 *     every id hakm_forward is given, one per line (stream comparisons).
 */
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "hakm_cuda.h"
#include "model.h"
#include "sample.h"

/* the reference's own sampler (src/sample.c compiled with
 * -Dsample_token=hakm_ref_sample_token) */
int hakm_ref_sample_token(sampler *s, float *logits, int n);

enum { BATCHED_MIN = 16 };  /* pending ids from which the batched prompt pass runs */
enum { MAX_GPUS = 8 };

/* hakm_ctx first, so the pointer callers hold is also the wrapper's */
typedef struct cuda_ctx {
	hakm_ctx         c;
	hakmc_ctx       *dev;         /* rank 0 (the pick and the logits are read here) */
	hakmc_ctx       *devs[MAX_GPUS];
	int              n_dev;
	FILE            *token_log;
	int              eager;
	int             *pending;     /* ids recorded, not yet run */
	int              n_pending, cap_pending;
	struct cuda_ctx *next;        /* live contexts (sample_token finds c->logits) */
} cuda_ctx;

static cuda_ctx *live;
static pthread_mutex_t live_mu = PTHREAD_MUTEX_INITIALIZER;

static cuda_ctx *wrapper(hakm_ctx *c) { return (cuda_ctx *)c; }

/* One call made on every GPU of the context at once (tensor parallelism
 * needs all ranks in the same call): rank 0 in the calling thread, the
 * others on threads of their own. */
enum { OP_FORWARD, OP_PREFILL, OP_PREFILL_BATCHED, OP_RESET };
typedef struct {
	hakmc_ctx *h;
	int        op, n, rc;
	const int *ids;
	float     *logits;   /* rank 0 of OP_FORWARD only (may be NULL) */
} job;

static void *job_run(void *p)
{
	job *j = p;
	switch (j->op) {
	case OP_FORWARD:         j->rc = hakmc_forward(j->h, j->ids[0], j->logits, NULL); break;
	case OP_PREFILL:         j->rc = hakmc_prefill(j->h, j->ids, j->n, NULL, NULL); break;
	case OP_PREFILL_BATCHED: j->rc = hakmc_prefill_batched(j->h, j->ids, j->n, 0, NULL, NULL); break;
	default:                 hakmc_reset(j->h); j->rc = 0; break;
	}
	return NULL;
}

static int run_all(struct cuda_ctx *w, int op, const int *ids, int n, float *logits)
{
	job jobs[MAX_GPUS];
	pthread_t th[MAX_GPUS];
	int started[MAX_GPUS] = {0};
	for (int r = 0; r < w->n_dev; r++)
		jobs[r] = (job){ w->devs[r], op, n, 0, ids, r == 0 ? logits : NULL };
	for (int r = 1; r < w->n_dev; r++)
		started[r] = pthread_create(&th[r], NULL, job_run, &jobs[r]) == 0;
	job_run(&jobs[0]);
	int rc = jobs[0].rc;
	for (int r = 1; r < w->n_dev; r++) {
		if (!started[r]) { rc = rc ? rc : -1; continue; }
		pthread_join(th[r], NULL);
		if (!rc) rc = jobs[r].rc;
	}
	return rc;
}

/* The device contexts: one, or n tensor-parallel ranks joined in this
 * process. 0, or -1 after reporting on stderr (every context created is
 * destroyed again). */
static int open_devices(struct cuda_ctx *w, int max_seq, int dev0, int n)
{
	const hakm_model *m = &w->c.model;
	for (int r = 0; r < n; r++) {
		w->devs[r] = hakmc_create(m->map, m->map_size, max_seq, 1, dev0 + r);
		if (!w->devs[r]) goto fail;
		w->n_dev = r + 1;
	}
	if (n > 1) {
		const size_t hb = hakmc_tp_handle_bytes();
		unsigned char *handles = calloc((size_t)n, hb);
		if (!handles) goto fail;
		int rc = 0;
		for (int r = 0; r < n && !rc; r++) rc = hakmc_tp_export(w->devs[r], handles + (size_t)r * hb);
		for (int r = 0; r < n && !rc; r++) rc = hakmc_tp_connect(w->devs[r], r, n, handles);
		free(handles);
		if (rc) goto fail;
	}
	w->dev = w->devs[0];
	return 0;
fail:
	fprintf(stderr, "hakm: %s\n", hakmc_last_error());
	for (int r = 0; r < w->n_dev; r++) hakmc_destroy(w->devs[r]);
	w->n_dev = 0;
	return -1;
}

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
	w->cap_pending = max_seq > 0 ? max_seq : 1;
	w->pending = malloc((size_t)w->cap_pending * sizeof(int));
	const char *dev_env = getenv("HAKMC_DEVICE"), *gpus_env = getenv("HAKMC_GPUS");
	const int dev = dev_env ? atoi(dev_env) : 0;
	int n_gpus = gpus_env ? atoi(gpus_env) : 1;
	if (n_gpus < 1) n_gpus = 1;
	if (n_gpus > MAX_GPUS) n_gpus = MAX_GPUS;
	if (!c->logits || !w->pending) fprintf(stderr, "hakm: out of memory\n");
	if (!c->logits || !w->pending || open_devices(w, max_seq, dev, n_gpus) != 0) {
		free(w->pending);
		free(c->logits);
		mlf2_close(&c->model);
		free(w);
		return NULL;
	}
	const char *eager = getenv("HAKMC_EAGER");
	w->eager = eager && eager[0] && strcmp(eager, "0") != 0;
	const char *log_path = getenv("HAKMC_TOKEN_LOG");
	if (log_path && log_path[0]) w->token_log = fopen(log_path, "w");
	pthread_mutex_lock(&live_mu);
	w->next = live;
	live = w;
	pthread_mutex_unlock(&live_mu);
	return c;
}

void hakm_ctx_free(hakm_ctx *c)
{
	if (!c) return;
	cuda_ctx *w = wrapper(c);
	pthread_mutex_lock(&live_mu);
	for (cuda_ctx **p = &live; *p; p = &(*p)->next)
		if (*p == w) { *p = w->next; break; }
	pthread_mutex_unlock(&live_mu);
	if (w->token_log) fclose(w->token_log);
	for (int r = 0; r < w->n_dev; r++) hakmc_destroy(w->devs[r]);
	free(w->pending);
	free(c->logits);
	mlf2_close(&c->model);
	free(w);
}

/* Run the recorded ids; their last position's logits stay on the device.
 * 0, or -1 after reporting on stderr. */
static int flush(cuda_ctx *w)
{
	const int n = w->n_pending;
	if (n == 0) return 0;
	w->n_pending = 0;
	const int op = n >= BATCHED_MIN ? OP_PREFILL_BATCHED : n > 1 ? OP_PREFILL : OP_FORWARD;
	const int rc = run_all(w, op, w->pending, n, NULL);
	if (rc != 0) {
		fprintf(stderr, "hakm: forward of %d id(s): %s\n", n, hakmc_last_error());
		return -1;
	}
	return 0;
}

const float *hakm_forward(hakm_ctx *c, int token)
{
	cuda_ctx *w = wrapper(c);
	if (w->token_log) fprintf(w->token_log, "%d\n", token);
	if (c->pos >= c->max_seq || token < 0 || token >= c->vocab) {
		fprintf(stderr, "hakm: forward of id %d at position %d: out of range\n", token, c->pos);
		return c->logits;
	}
	if (w->eager) {
		if (run_all(w, OP_FORWARD, &token, 1, c->logits) != 0) {
			fprintf(stderr, "hakm: forward at position %d: %s\n", c->pos, hakmc_last_error());
			return c->logits;
		}
	} else {
		w->pending[w->n_pending++] = token;
	}
	c->pos++;
	return c->logits;
}

void hakm_reset(hakm_ctx *c)
{
	cuda_ctx *w = wrapper(c);
	w->n_pending = 0;
	run_all(w, OP_RESET, NULL, 0, NULL);
	c->pos = 0;
}

int sample_token(sampler *s, float *logits, int n)
{
	cuda_ctx *w = NULL;
	pthread_mutex_lock(&live_mu);
	for (cuda_ctx *p = live; p; p = p->next)
		if (p->c.logits == logits && p->c.vocab == n) { w = p; break; }
	pthread_mutex_unlock(&live_mu);
	if (!w) return hakm_ref_sample_token(s, logits, n);
	if (flush(w) != 0) return 0;
	unsigned long long rng = s->rng;
	int tok = 0;
	if (hakmc_sample_last(w->dev, s->temp, s->top_p, s->top_k, &rng, &tok) != 0) {
		fprintf(stderr, "hakm: sample: %s\n", hakmc_last_error());
		return hakm_ref_sample_token(s, logits, n);
	}
	s->rng = rng;
	return tok;
}
