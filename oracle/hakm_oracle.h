/*
 * hakm_oracle.h — CPU restatement of hako's quantized decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker that the CUDA path is compared
 * against; nothing in the shipped library links, loads or calls it. Only the
 * test suite, the smoke check and the benchmark's CPU-baseline leg use it.
 *
 * Every function restates one piece of the reference engine (mithraeums/hako)
 * and cites the reference file:line it follows. Parity of this restatement is
 * pinned against the reference's own compiled sources (oracle/Makefile builds
 * them into oracle/_ref/) and against golden vectors that build produced
 * (tests/golden/).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK 256

/* IEEE binary16 -> binary32 (src/quant.c:31-54). */
float orc_f16_to_f32(uint16_t h);
/* binary32 -> binary16, round to nearest even (used by the synthetic
 * quantizers; the reference only ever widens). */
uint16_t orc_f32_to_f16(float f);

/* 6-bit scale/min unpack for sub-block j of a Q4_K block (src/quant.c:57-66). */
void orc_scale_min_k4(int j, const uint8_t *q, int *s, int *m);

/* Dequantize nelem values (multiple of 256) (src/quant.c:68-92, 94-123). */
void orc_dequant_q4k(const void *blocks, float *out, int nelem);
void orc_dequant_q6k(const void *blocks, float *out, int nelem);

/* Per-32 absmax int8 activation quantizer, as the reference builds it with
 * -ffast-math: xs = amax * (1/127) (src/quant.c:127-144). */
void orc_quantize_q8_32(const float *x, int n, int8_t *xq, float *xs);

/* Exact per-32 sub-block integer sums of one Q4_K row against xq:
 * iqx[sb] = sum(q * xq), ix[sb] = sum(xq) (src/quant.c:163-229). */
void orc_q4k_subsums(const void *row, int n_in, const int8_t *xq,
                     int32_t *iqx, int32_t *ix);
/* One Q4_K row . q8 activation (src/quant.c:150-232), in the as-built
 * rounding order (one rounded add per pair of sub-blocks). */
float orc_q4k_dot(const void *row, int n_in, const int8_t *xq, const float *xs);
/* One Q6_K row . fp32 activation: dequantize then float dot (src/nn.c:84-95). */
float orc_q6k_dot(const void *row, int n_in, const float *x);

/* The as-built fp32 building blocks (-O3 -ffast-math -march=x86-64-v3):
 *  orc_dot_f32      the vectorized `acc += a[i]*b[i]` (src/nn.c:15,92, src/model.c:130)
 *  orc_rsqrt_table  rsqrtss on [1,4): 2 x 1024 results of this host's instruction
 *  orc_rsqrt_approx rsqrtss from that table; orc_rsqrt_nr: 1.0f/sqrtf as built
 *  orc_expf         glibc's scalar expf; orc_exp_table its 32 table words
 *  orc_expf_v8/_v4  libmvec's 8-wide (AVX2) and 4-wide (SSE4) vector expf
 *  orc_rope_table   (cos, sin) of one position's RoPE pairs, as rope_neox computes them */
float orc_dot_f32(const float *a, const float *b, int n);
void  orc_rsqrt_table(uint32_t *out);
float orc_rsqrt_approx(float v);
float orc_rsqrt_nr(float v);
float orc_expf(float x);
void  orc_exp_table(uint64_t *out);
float orc_expf_v8(float x);
float orc_expf_v4(float x);
void  orc_rope_table(float *cs, int head_dim, int pos, float theta);
/* Mismatch counts of the restated expf / vector expf / rsqrtss against the
 * host libraries over [lo, hi] by step (out[4]); a test-side pin. */
void  orc_check_libm(uint32_t lo, uint32_t hi, uint32_t step, long long *out);

/* src/nn.c:13-18, 20-27, 29, 32-42 */
void  orc_rmsnorm(float *y, const float *x, const float *w, int n, float eps);
void  orc_softmax(float *x, int n);
float orc_silu(float x);
void  orc_rope_neox(float *vec, int head_dim, int pos, float theta);

/* GQA decode attention (src/model.c:124-142) over [pos + 1][KVH * hd] caches. */
void  orc_attention(float *out, const float *q, const float *kc, const float *vc, int pos, int H, int KVH,
                    int hd);

/* Row-major out[n_out] = W . x (+bias) for an MLF2 tensor of type `type`
 * (src/nn.c:179-210 and the per-row worker src/nn.c:70-97). */
int orc_matmul(float *out, const float *x, int type, const void *w,
               const float *bias, int n_out, int n_in);

/* ---- whole-model decode over an MLF2 image (src/model.c:17-165) ---- */
typedef struct orc_model orc_model;

/* Parse an MLF2 image already in memory. Returns NULL on a malformed image. */
orc_model *orc_model_new(const void *image, size_t size, int max_seq);
void       orc_model_free(orc_model *m);
void       orc_model_reset(orc_model *m);
int        orc_model_vocab(const orc_model *m);
int        orc_model_dim(const orc_model *m);
/* Number of layers the forward runs (default: all). Used to read per-layer
 * hidden states. */
void       orc_model_set_layers(orc_model *m, int n_layers);
/* One decode step at the current position; returns logits[vocab] (borrowed). */
const float *orc_forward(orc_model *m, int token);
/* Residual stream after the last forward (borrowed, d_model floats). */
const float *orc_hidden(const orc_model *m);
/* Greedy argmax, first max wins (src/sample.c:28-32). */
int orc_argmax(const float *logits, int n);

#ifdef __cplusplus
}
#endif
