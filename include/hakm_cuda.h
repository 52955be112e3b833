/*
 * hakm_cuda.h — C ABI of libhakm_cuda, the B200 (sm_100a) decode path for the
 * hako engine (mithraeums/hako).
 *
 * Plain pointers, sizes and ints only. Every entry point names the reference
 * interface it replaces (path:line inside mithraeums/hako). Errors follow the
 * reference's convention of a negative return (or NULL) plus a message; the
 * message is available from hakmc_last_error() instead of stderr.
 *
 * Device pointers are marked [dev]; host pointers [host]. `stream` is a
 * cudaStream_t passed as void* (NULL = the legacy default stream).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HAKMC_OK          0
#define HAKMC_EINVAL    (-22)   /* bad argument / shape                     */
#define HAKMC_ENOMEM    (-12)   /* device allocation failed                 */
#define HAKMC_EFORMAT   (-74)   /* malformed MLF2 image / missing tensor    */
#define HAKMC_ECUDA     (-5)    /* CUDA runtime or kernel launch error      */
#define HAKMC_ERANGE    (-34)   /* position beyond the KV-cache capacity    */
#define HAKMC_ETIMEOUT  (-62)   /* a bounded device-side wait gave up       */
#define HAKMC_ENCCL     (-71)   /* NCCL error                               */

typedef struct hakmc_ctx hakmc_ctx;

/* Last error message of the calling thread ("" if none). */
const char *hakmc_last_error(void);
/* ABI version: 100*major + minor. */
int hakmc_version(void);

/* ==================================================================
 * Model context — replaces the decode engine of src/model.h:29-37.
 * ================================================================== */

/* Build a device context from an MLF2 image already in host memory (for
 * example the read-only mmap that mlf2_open makes: hakm_model.map and
 * .map_size, src/loader.h:6-13). Replaces hakm_ctx_new (src/model.c:17-76):
 * binds the same tensors by name, uploads them once to `device`, and sizes
 * the KV cache for max_seq positions of max_batch sequences.
 * Returns NULL on failure (see hakmc_last_error). */
hakmc_ctx *hakmc_create(const void *mlf2_image, size_t image_size,
                        int max_seq, int max_batch, int device);
/* Replaces hakm_ctx_free (src/model.c:78-86). */
void hakmc_destroy(hakmc_ctx *c);
/* The same as hakmc_destroy, under the name of the boundary's free call. */
void hakmc_free(hakmc_ctx *c);
/* Replaces hakm_reset (src/model.c:88): every sequence back to position 0. */
void hakmc_reset(hakmc_ctx *c);
int  hakmc_pos(const hakmc_ctx *c);          /* hakm_ctx.pos (model.h:20)     */
int  hakmc_set_pos(hakmc_ctx *c, int pos);   /* rewind within filled cache    */
int  hakmc_vocab(const hakmc_ctx *c);        /* hakm_ctx.vocab (model.h:17)   */
int  hakmc_dim(const hakmc_ctx *c);          /* hakm_ctx.d_model              */
int  hakmc_n_layers(const hakmc_ctx *c);

/* One decode step at the current position. Replaces hakm_forward
 * (src/model.c:93-165). [host] logits (vocab floats, may be NULL) receives
 * the logits the reference returns; [host] argmax (may be NULL) receives the
 * greedy token of sample_token at temperature 0 (src/sample.c:28-32: first
 * maximum wins). Advances the position by one. 0 or a negative code. */
int hakmc_forward(hakmc_ctx *c, int token, float *logits, int *argmax);

/* Greedy decode loop of the CLI and the embed API (cli/main.c:56-75,
 * src/hakm_api.c:148-166) kept on the device: feeds n_prompt [host] ids one
 * position at a time (as hakm_forward does), then emits n_gen greedy ids
 * into [host] out_tokens. No host round trip between tokens. */
int hakmc_generate(hakmc_ctx *c, const int *prompt, int n_prompt, int n_gen,
                   int *out_tokens);

/* Prompt processing: feeds n [host] ids at consecutive positions (as the
 * reference's feed loop calls hakm_forward per id, cli/main.c:56-60) in one
 * device launch; only the last id's lm_head runs. [host] logits (vocab
 * floats, may be NULL) and argmax (may be NULL) receive the last step's.
 * Advances the position by n. 0 or a negative code. */
int hakmc_prefill(hakmc_ctx *c, const int *tokens, int n, float *logits, int *argmax);

/* Prompt processing with the positions batched: the same state and outputs
 * as hakmc_prefill, bit for bit, but the n [host] ids go through each layer
 * together in chunks of chunk_rows positions (<= 0: 1024), so every weight
 * byte read serves a whole chunk: Q4_K matmuls on the tensor cores over each
 * row's q8_32 codes, Q6_K matmuls as fp32 lane chains over dequantized
 * tiles, each row's attention over the cache (which each chunk's own K/V
 * rows enter first). Every kernel keeps the per-position arithmetic of
 * hakm_forward (src/model.c:93-165) with the reference build's roundings
 * and summation orders. No counterpart in the reference, whose feed loop
 * calls hakm_forward per id (cli/main.c:56-60). Under tensor parallelism,
 * or when a row's attention scores would not fit in shared memory
 * (positions beyond about 51,000), this runs hakmc_prefill. 0 or a
 * negative code. */
int hakmc_prefill_batched(hakmc_ctx *c, const int *tokens, int n, int chunk_rows, float *logits,
                          int *argmax);

/* Continue the greedy stream of the current sequence for n_steps positions
 * without returning to the host between steps (the decode half of
 * cli/main.c:63-75): each step's input is the previous step's argmax. The
 * first input is the argmax of the last hakmc_forward / hakmc_generate step.
 * [host] out_tokens (may be NULL) receives the n_steps inputs consumed. */
int hakmc_decode(hakmc_ctx *c, int n_steps, int *out_tokens);

/* Batched decode: one step for n_seq independent sequences (n_seq <=
 * max_batch), sequence i at position pos[i] with input tokens[i] ([host]),
 * using KV-cache slot i (slot 0 is also the single-sequence calls' cache;
 * their position and last pick are left as they were). The reference
 * decodes one sequence at a time; each row of this call is hakm_forward on
 * a context holding that sequence's cache. Eight or more sequences on one GPU
 * go through each layer together as the rows of one pass (the kernels of
 * hakmc_prefill_batched; attention reads each row's own cache slot up to its
 * position), so each weight byte is read once per call. Fewer sequences
 * (or tensor parallelism, or max_seq beyond about 51,000) run the step
 * kernel per sequence. Either way every row equals hakm_forward's logits
 * and pick bit for bit. argmax [host] gets n_seq ids;
 * logits [host] (may be NULL) n_seq*vocab floats. 0, HAKMC_ERANGE for a
 * position beyond max_seq, or another negative code. */
int hakmc_forward_batch(hakmc_ctx *c, const int *tokens, const int *pos,
                        int n_seq, float *logits, int *argmax);

/* Tensor parallelism over `world` GPUs of one node (no counterpart in the
 * reference, whose engine runs on one CPU). Every rank creates its own
 * context with hakmc_create on its own device (same model, max_seq and
 * max_batch), exports a handle, and hands all ranks' handles (rank order,
 * world * hakmc_tp_handle_bytes() bytes, e.g. all-gathered over the job's
 * own transport) to hakmc_tp_connect. From then on every GEMV phase's rows
 * are split over all GPUs' CTAs and each output vector is written into
 * every GPU's memory by peer stores over NVLink inside the step kernel (the
 * float sums are those of one GPU, so results do not change with world).
 * All ranks must then make the same calls (forward / prefill / generate /
 * decode / reset with the same arguments) concurrently; every rank gets the
 * same tokens and logits. Ranks may be threads of one process or separate
 * processes (CUDA IPC). On connecting, every rank keeps only its own rows
 * of each split matrix (about 1/world of the weights; the embedding, and a
 * tied lm_head, stay whole), so the per-phase entry points (hakmc_time_phase,
 * hakmc_trace_phase) refuse a connected context. 0 or a negative code. */
size_t hakmc_tp_handle_bytes(void);
int hakmc_tp_export(hakmc_ctx *c, void *handle);
int hakmc_tp_connect(hakmc_ctx *c, int rank, int world, const void *handles);
int hakmc_tp_rank(const hakmc_ctx *c);
int hakmc_tp_world(const hakmc_ctx *c);

/* Test hooks. Run only the first n layers of each forward (the residual
 * stream is then what the reference holds in hakm_ctx.xb after that many
 * layers, src/model.c:102-157); n < 0 restores all layers. */
int hakmc_set_layers(hakmc_ctx *c, int n_layers);
/* Copy the residual stream of sequence `seq` after the last forward into
 * [host] out (d_model floats). */
int hakmc_hidden(hakmc_ctx *c, int seq, float *out);
/* Copy a device activation of sequence 0 after the last forward into [host]
 * out: which = 0 residual stream (d_model), 1 q after RoPE (d_model), 2 k
 * after RoPE (kv_dim), 3 v (kv_dim), 4 attention output (d_model), 5 SwiGLU
 * output (ffn_dim), 6 logits (vocab). Test hook; the buffers hold the values
 * of the last layer that ran (hakm_ctx scratch, src/model.h:24). */
int hakmc_debug_read(hakmc_ctx *c, int which, float *out);

/* Fill the KV cache of sequence `seq` for positions [0, n_pos) of every
 * layer from [host] k and v ([n_layers][n_pos][n_kv_heads*head_dim] fp32),
 * and set that sequence's position to n_pos. Mirrors pre-filling
 * hakm_ctx.k_cache / v_cache / pos (src/model.h:20-21). */
int hakmc_fill_kv(hakmc_ctx *c, int seq, const float *k, const float *v, int n_pos);

/* Fill the KV cache of sequence `seq` for positions [0, n_pos) of every
 * layer with seeded N(0, 1) fp32 values on the device (the synthetic cache
 * of a long-context measurement workload), and for seq 0 set the position
 * to n_pos. Measurement hook; no counterpart in the reference. */
int hakmc_fill_kv_normal(hakmc_ctx *c, int seq, int n_pos, unsigned long long seed);

/* Average device time in ms of one launch of decode-step phase `phase`
 * (0 qkv, 1 attention, 2 attn-output, 3 ffn gate/up, 4 ffn down, 5 lm_head),
 * over `iters` launches rotating through the layers so each launch streams
 * its weights from HBM, timed with CUDA events on the context stream.
 * No counterpart in the reference (measurement hook). */
int hakmc_time_phase(hakmc_ctx *c, int phase, int iters, float *avg_ms);

/* Measurement hook: run one launch of phase `phase` of layer `layer` (see
 * hakmc_time_phase) with per-CTA %globaltimer stamps written to [host]
 * stamps (n_ctas * 8 u64: start, prologue done, first stage ready, last unit
 * done, epilogue done, producer done). Returns the CTA count or a negative
 * code. No counterpart in the reference. */
int hakmc_trace_phase(hakmc_ctx *c, int phase, int layer, unsigned long long *stamps, int max_ctas);

/* Measurement hook: one decode step (input token in the context, as for
 * hakmc_decode) through the persistent step kernel with %globaltimer stamps
 * written to [host] stamps, laid out [cta][phase][4] for the first
 * max_phases grid phases of the step (embedding, then per layer qkv,
 * attention, attn-output, ffn gate/up, ffn down, then lm_head): barrier
 * passed, activation built, stages consumed, arrived. Advances the position
 * by one. Returns the CTA count or a negative code. No counterpart in the
 * reference. */
int hakmc_trace_step(hakmc_ctx *c, unsigned long long *stamps, int max_phases);

/* Time of the last hakmc_forward / hakmc_generate / hakmc_forward_batch
 * call's device work in milliseconds (CUDA events on the context stream). */
float hakmc_last_device_ms(const hakmc_ctx *c);

/* ==================================================================
 * Kernel-level entry points (device buffers). For unit parity tests and
 * callers that keep their own weights. Return 0 or a negative code; they
 * launch on `stream` and do not synchronize.
 * ================================================================== */

/* Replaces quantize_row_q8_32 (src/quant.c:127-144), bit-exact with the
 * reference as built (-ffast-math: xs = amax * fl(1/127)). [dev] x[n] fp32 ->
 * xq[n] int8, xs[n/32] fp32. n % 32 == 0. */
int hakmc_quantize_q8_32(const float *x, int n, int8_t *xq, float *xs, void *stream);

/* Q4_K matmul with int8 activations: out[r] = q4k_vec_dot(w row r, xq, xs)
 * (+ bias[r]) for r < n_out. Replaces the Q4_K branch of matmul / mm_worker
 * (src/nn.c:76-82, src/quant.c:150-232). [dev] w: n_out rows of n_in/256
 * verbatim 144-byte block_q4_K (src/quant.h:12-17). bias may be NULL.
 * n_in % 256 == 0. */
int hakmc_gemv_q4k_q8(float *out, const void *w, const int8_t *xq, const float *xs,
                      const float *bias, int n_out, int n_in, void *stream);

/* Batched Q4_K matmul: out[n*n_out + r] = q4k_vec_dot(w row r, xq + n*n_in,
 * xs + n*(n_in/32)) (+ bias[r]) for n < n_batch, r < n_out — the reference's
 * Q4_K matmul (src/nn.c:76-82, src/quant.c:150-232) applied to n_batch
 * activations; the reference has no batched call (it runs one vector per
 * hakm_forward). Small batches: dp4a, each weight byte read once per 16
 * activations, per-chunk partials summed in a fixed order (fp32-close to
 * the reference, rel-L2 <= 1e-5, deterministic); batches above 16 (above 8
 * for matrices of 16M weights or more in at least 64 row tiles of 128) run
 * on the tensor cores as hakmc_gemm_q4k_q8 does, bit for bit (when xs is
 * 16-byte aligned; else dp4a in launches of 16). [dev]
 * buffers; w and xq 16-byte aligned; n_in % 256 == 0.
 * scratch: [dev] hakmc_gemv_q4k_q8_batch_scratch(n_out, n_in, n_batch)
 * bytes, 16-byte aligned, zeroed before its first use (a call leaves it
 * reusable; zero it again after a failed call); one call at a time per
 * scratch. NULL takes a scratch from the stream-ordered allocator.
 * The kernel is launched as a programmatic dependent of the preceding
 * kernel in the stream and may read w before that kernel has finished, so
 * w must not be written by the immediately preceding kernel. */
size_t hakmc_gemv_q4k_q8_batch_scratch(int n_out, int n_in, int n_batch);
int hakmc_gemv_q4k_q8_batch(float *out, const void *w, const int8_t *xq, const float *xs,
                            const float *bias, int n_out, int n_in, int n_batch,
                            void *scratch, size_t scratch_bytes, void *stream);

/* The same product on the tensor cores (tcgen05 kind::i8), bit-identical
 * to q4k_vec_dot as built: the per-32 integer sums q*xq are exact int32 MMA
 * results, combined in fp32 with the reference's steps and order
 * (src/quant.c:224-227 under -O3 -ffast-math with FMA). For batches
 * (batched decode, prompt processing); any n_batch >= 1, tiles of 16 or 32
 * activations; a row is never split along K. [dev] w, xq and xs 16-byte
 * aligned; n_in % 256 == 0. scratch: unused (hakmc_gemm_q4k_q8_scratch
 * returns 0; kept for callers written against a splitting kernel).
 * Launched as a programmatic dependent of the preceding kernel (it waits
 * for that kernel before reading). */
size_t hakmc_gemm_q4k_q8_scratch(int n_out, int n_in, int n_batch);
int hakmc_gemm_q4k_q8(float *out, const void *w, const int8_t *xq, const float *xs,
                      const float *bias, int n_out, int n_in, int n_batch,
                      void *scratch, size_t scratch_bytes, void *stream);

/* The whole Q4_K matmul of src/nn.c:179-210: quantizes the fp32 [dev] x once
 * (quantize_row_q8_32), then the int8 row dots. Same layout rules. */
int hakmc_gemv_q4k(float *out, const void *w, const float *x, const float *bias,
                   int n_out, int n_in, void *stream);

/* Exact per-32 sub-block integer sums of q4k_vec_dot (src/quant.c:163-267):
 * iqx[r*(n_in/32)+j] = sum(q*xq), ix[..] = sum(xq) for row r, sub-block j. */
int hakmc_q4k_subsums(int32_t *iqx, int32_t *ix, const void *w, const int8_t *xq,
                      int n_out, int n_in, void *stream);

/* Re-lay n_rows rows of verbatim 210-byte block_q6_K (src/quant.h:19-24)
 * into this library's device layout (same byte count): per chunk of 8
 * blocks the 208-byte {ql, qh, scales} parts (the ql/qh bytes regrouped by
 * the element's index mod 8, the lane of the reference's vectorized dot that
 * adds it), then the chunk's fp16 d values. [dev] src and dst must not
 * overlap. */
int hakmc_q6k_pack(void *dst, const void *src, int n_rows, int n_in, void *stream);
size_t hakmc_q6k_packed_bytes(int n_rows, int n_in);

/* Q6_K matmul with fp32 activations (the generic dequant-and-dot path the
 * reference takes for Q6_K, src/nn.c:84-95, src/quant.c:94-123). [dev] w in
 * the packed layout of hakmc_q6k_pack. bias may be NULL. */
int hakmc_gemv_q6k(float *out, const void *w_packed, const float *x, const float *bias,
                   int n_out, int n_in, void *stream);

/* lm_head + greedy pick fused: logits (may be NULL) = W . rmsnorm(x) and
 * argmax[0] = first index of the maximum (src/model.c:160-161 then
 * src/sample.c:28-32). [dev] norm_w may be NULL for no norm. */
int hakmc_lmhead_argmax(float *logits, int *argmax, const void *w_packed,
                        const float *x, const float *norm_w, float eps,
                        int n_vocab, int n_in, void *stream);

/* Dequantize n_rows rows (verbatim Q4_K or Q6_K blocks, `type` 12 or 14 as
 * in include/mlf2.h:44-49) to fp32 (src/quant.c:68-123, 234-248). */
int hakmc_dequant(float *out, const void *w, int type, int n_rows, int n_in, void *stream);

/* y = x / rms(x) * w (src/nn.c:13-18), one vector of n (a multiple of 8),
 * with the roundings of the reference's own build (8-lane sum of squares,
 * rsqrtss plus one Newton step): bit-identical results. */
int hakmc_rmsnorm(float *y, const float *x, const float *w, int n, float eps, void *stream);

/* GQA decode attention for one layer and one sequence over an fp32 cache in
 * the reference layout [max_seq][n_kv*hd] (src/model.c:124-142, softmax
 * src/nn.c:20-27): out[h] = softmax(q_h . K[0..pos] / sqrt(hd)) V[0..pos]
 * for h < n_heads, kv head h / (n_heads/n_kv), with the reference build's
 * roundings (bit-identical results). [dev] all buffers. One CTA per (query
 * head, 32 dimensions); the score rows, n_heads * (head_dim/32) * (pos+1)
 * floats, live in a scratch area the library allocates per device (and
 * regrows). Returns after the kernel has finished. */
int hakmc_attention(float *out, const float *q, const float *k_cache, const float *v_cache,
                    int pos, int n_heads, int n_kv, int head_dim, void *stream);

/* hakmc_attention without any device allocation, for callers that cannot
 * allocate GPU memory once they are running: a host that has handed the
 * whole device budget to another framework's memory pool, or a latency-bound
 * loop that must not take cudaMalloc's implicit device synchronisation. It
 * launches the same kernel as hakmc_attention, but its scratch (the score
 * rows and the position word) lives in one fixed array of about 1 MiB
 * inside this library, which every GPU that loads the library holds until
 * the process exits. Limit: n_heads * (head_dim / 32) * (pos + 1) <= 262144
 * floats (for example 16 heads of 128 up to 4096 positions, 28 heads up to
 * 2340); larger calls return HAKMC_ERANGE. Unlike hakmc_attention it does
 * not wait: it returns once the kernels are enqueued on `stream`, so q, the
 * caches and out must stay valid until the stream has reached that point,
 * and a kernel fault shows at the caller's next synchronisation. The first
 * call on a device looks the array up (cudaGetSymbolAddress), so make it
 * before any stream capture. All calls share the array and it keeps the
 * last call's contents: calls that overlap on the GPU (other streams, other
 * threads) race, so serialise them. No counterpart in the reference. */
int hakmc_attention_noalloc(float *out, const float *q, const float *k_cache, const float *v_cache,
                            int pos, int n_heads, int n_kv, int head_dim, void *stream);

/* Attention of many rows at once (prompt chunks, batched decode), each row
 * bit-identical to hakmc_attention at its position: row r attends over
 * positions 0 .. row_pos[r] of its own cache, k_cache + r * slot_stride
 * (decode rows: one sequence per row), or, when row_pos is NULL, over
 * positions 0 .. pos0 + r of one cache (the rows of a prompt chunk, whose
 * own K/V rows are already in it). q, out: [dev] rows x n_heads*head_dim;
 * row_pos: [dev] int[rows] or NULL; max_pos >= every row's position (it
 * sizes the shared-memory score row: (max_pos + 1) * 4 bytes plus
 * (head_dim + 64) * 4 must stay within 200 KB, else HAKMC_ERANGE). The
 * reference has no batched call; its per-row arithmetic is
 * src/model.c:124-142. Asynchronous on `stream`. */
int hakmc_attention_rows(float *out, const float *q, const float *k_cache, const float *v_cache,
                         int rows, int pos0, const int *row_pos, int max_pos, size_t slot_stride,
                         int n_heads, int n_kv, int head_dim, void *stream);

/* Q6_K matmul of many fp32 activation rows: out[n*n_out + r] (+)=
 * dot(dequant(w row r), x + n*n_in) (+ bias[r]) for n < n_batch, each
 * output bit-identical to the reference's generic matmul (src/nn.c:84-95
 * as built: 8 lane chains of rounded products, folded), accumulate != 0
 * adding it to out as the residual add does (src/model.c:146,156). [dev]
 * w in the packed layout of hakmc_q6k_pack; n_in % 256 == 0. Asynchronous
 * on `stream`. */
int hakmc_gemm_q6k(float *out, const void *w, const float *x, const float *bias, int n_out, int n_in,
                   int n_batch, int accumulate, void *stream);

/* NeoX RoPE in place on n_heads heads of head_dim at position pos
 * (src/nn.c:32-42), (cos, sin) from a table built on the host through the
 * same glibc vector routines the reference's build calls (bit-identical). */
int hakmc_rope_neox(float *x, int n_heads, int head_dim, int pos, float theta, void *stream);

/* Sampling for temperature > 0 (src/sample.c:27-58) on the device, with
 * the reference build's roundings, so token and generator state equal its
 * own sample_token's bit for bit: logits / temp (as vectorized: one
 * division, multiplies by 1/temp, one rcpss-Newton group of four, divisions
 * for the rest), the softmax of src/nn.c:20-27, a stable sort by
 * probability (glibc's qsort of the candidate list keeps ties in index
 * order), top_k (0: off), the top_p nucleus (0 or >= 1: off), the
 * vectorized sum of the kept probabilities, and the xorshift64 draw.
 * temp <= 0 is the greedy argmax (first index of the maximum); it leaves
 * logits and *rng alone. [dev] logits (n >= 9 floats) are turned into
 * probabilities in place, as the reference's are; [host] *rng is the
 * sampler state (sample.h), advanced by one draw; [host] *token receives
 * the pick. Synchronous on `stream`; the scratch (4n words) is allocated
 * once per device and regrown. hakmc_sample_last samples the logits of the
 * context's last step on the device, so no logits cross to the host. */
int hakmc_sample(float *logits, int n, float temp, float top_p, int top_k, unsigned long long *rng,
                 int *token, void *stream);
int hakmc_sample_last(hakmc_ctx *c, float temp, float top_p, int top_k, unsigned long long *rng, int *token);

/* Host-only planning, for tests and tools (no GPU needed). The rows of a
 * step-kernel phase that CTA `cta` of a `grid`-CTA group computes (with
 * tensor parallelism the grid spans every rank's CTAs, rank r owning CTAs
 * r * n_sms ..): seg_rows[s] rows in each of n_seg (<= 3) segments give
 * ranges[2s] .. ranges[2s+1] (half open; 4-row groups, so row pairs of the
 * RoPE and SwiGLU epilogues are never split, and rows are whole, so every
 * row's q8_32 activation blocks stay on one GPU). The attention units
 * (query head, 32 dimensions) rank `rank` of `world` runs: returns their
 * count, the first `cap` written to units. No counterpart in the reference
 * (it has no multi-GPU path). */
int hakmc_plan_rows(const int *seg_rows, int n_seg, int grid, int cta, int *ranges);
int hakmc_plan_attn_units(int n_heads, int head_dim, int rank, int world, int *units, int cap);

/* Test hook: out[i] = the device's restatement of one of the reference
 * build's exp routines applied to in[i]: variant 0 glibc's scalar expf
 * (silu_f, the softmax tail), 1 libmvec's 8-wide expf, 2 its 4-wide expf
 * (the vectorized softmax, src/nn.c:24). [dev] buffers of n floats. No
 * counterpart in the reference (it pins the device against the host's own
 * libm / libmvec). */
int hakmc_test_expf(float *out, const float *in, int n, int variant, void *stream);

#ifdef __cplusplus
}
#endif
