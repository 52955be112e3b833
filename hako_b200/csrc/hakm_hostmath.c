/*
 * hakm_hostmath.c — host-side tables of libhakm_cuda that must carry the
 * reference's own libm roundings (compiled by gcc with AVX2 + FMA so it can
 * call glibc's vector math entry points, and linked into the library).
 *
 *  - NeoX RoPE (cos, sin) pairs as rope_neox (src/nn.c:32-42) computes them
 *    when built with -O3 -ffast-math for x86-64-v3: the loop over pairs is
 *    vectorized 8 wide, so freq = powf(theta, 2i * (-1/hd)) and cos/sin of
 *    pos * freq go through libmvec's vector powf/cosf/sinf (the 4-wide ones
 *    for a 4-pair remainder, scalar libm for the last 0..3 pairs and for
 *    heads of fewer than 8 pairs, where gcc's alias check sends the whole
 *    loop down the scalar path).
 *  - The rsqrtss estimate behind 1.0f/sqrtf under -ffast-math (src/nn.c:16,
 *    src/model.c:97): its result depends only on the input's exponent parity
 *    and top 10 mantissa bits, so the 2048 results for [1, 4) describe it;
 *    they are measured from this host's instruction.
 */
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

__m256 _ZGVdN8vv_powf(__m256, __m256);
__m256 _ZGVdN8v_cosf(__m256);
__m256 _ZGVdN8v_sinf(__m256);
__m128 _ZGVbN4vv_powf(__m128, __m128);
__m128 _ZGVbN4v_cosf(__m128);
__m128 _ZGVbN4v_sinf(__m128);

/* (cos, sin) of the head_dim/2 pairs of one position into cs[2 * i + {0,1}]. */
void hakm_host_rope_row(float *cs, int head_dim, int pos, float theta) {
	int half = head_dim / 2, i = 0;
	float nhd = -1.0f / (float)head_dim, fp = (float)pos;
	if (half >= 8) {
		for (; i + 8 <= half; i += 8) {
			float e[8], c[8], s[8];
			for (int l = 0; l < 8; l++) e[l] = (float)(2 * (i + l)) * nhd;
			__m256 fr = _ZGVdN8vv_powf(_mm256_set1_ps(theta), _mm256_loadu_ps(e));
			__m256 ang = _mm256_mul_ps(fr, _mm256_set1_ps(fp));
			_mm256_storeu_ps(c, _ZGVdN8v_cosf(ang));
			_mm256_storeu_ps(s, _ZGVdN8v_sinf(ang));
			for (int l = 0; l < 8; l++) { cs[2 * (i + l)] = c[l]; cs[2 * (i + l) + 1] = s[l]; }
		}
		if (half - i >= 4) {
			float e[4], c[4], s[4];
			for (int l = 0; l < 4; l++) e[l] = (float)(2 * (i + l)) * nhd;
			__m128 fr = _ZGVbN4vv_powf(_mm_set1_ps(theta), _mm_loadu_ps(e));
			__m128 ang = _mm_mul_ps(fr, _mm_set1_ps(fp));
			_mm_storeu_ps(c, _ZGVbN4v_cosf(ang));
			_mm_storeu_ps(s, _ZGVbN4v_sinf(ang));
			for (int l = 0; l < 4; l++) { cs[2 * (i + l)] = c[l]; cs[2 * (i + l) + 1] = s[l]; }
			i += 4;
		}
	}
	for (; i < half; i++) {
		float ang = fp * powf(theta, (float)(2 * i) * nhd);
		cs[2 * i] = cosf(ang);
		cs[2 * i + 1] = sinf(ang);
	}
}

static float bitsf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t fbits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* out[par * 1024 + m] = rsqrtss(2^par * (1 + m/1024)), par in {0, 1}. */
void hakm_host_rsqrt_table(uint32_t *out) {
	for (int par = 0; par < 2; par++)
		for (int m = 0; m < 1024; m++) {
			float x = bitsf(((uint32_t)(127 + par) << 23) | ((uint32_t)m << 13));
			out[par * 1024 + m] = fbits(_mm_cvtss_f32(_mm_rsqrt_ss(_mm_set_ss(x))));
		}
}

/* 1 if the rsqrtss results of this host depend only on the exponent parity
 * and the top 10 mantissa bits (checked on every 97th mantissa of [1, 4)),
 * which is what the table form assumes; 0 otherwise. */
int hakm_host_rsqrt_table_ok(const uint32_t *tab) {
	for (int par = 0; par < 2; par++)
		for (uint32_t m = 0; m < (1u << 23); m += 97) {
			float x = bitsf(((uint32_t)(127 + par) << 23) | m);
			if (fbits(_mm_cvtss_f32(_mm_rsqrt_ss(_mm_set_ss(x)))) != tab[par * 1024 + (m >> 13)]) return 0;
		}
	return 1;
}

/* 1.0f / sqrtf(v) as the reference's build computes it (rsqrtss + Newton). */
float hakm_host_rsqrt_nr(float v) {
	float r = _mm_cvtss_f32(_mm_rsqrt_ss(_mm_set_ss(v)));
	float t = fmaf(r, v * r, -3.0f);
	return (r * -0.5f) * t;
}

/* The rcpss estimate (the reciprocal gcc's vectorized loop of
 * `logits[i] /= temp` uses for its 4-wide remainder step, src/sample.c:36,
 * with one Newton step): a function of the top 11 mantissa bits, the
 * exponent scaling the result. out[m] = rcpss(1 + m/2048). */
void hakm_host_rcp_table(uint32_t *out) {
	for (int m = 0; m < 2048; m++) {
		float x = bitsf((127u << 23) | ((uint32_t)m << 12));
		out[m] = fbits(_mm_cvtss_f32(_mm_rcp_ss(_mm_set_ss(x))));
	}
}

/* 1 if the table form holds on this host (every 97th mantissa, exponents
 * -64..64), 0 otherwise. */
int hakm_host_rcp_table_ok(const uint32_t *tab) {
	for (int e = -64; e <= 64; e += 8)
		for (uint32_t m = 0; m < (1u << 23); m += 97) {
			float x = bitsf(((uint32_t)(127 + e) << 23) | m);
			uint32_t want = tab[m >> 12] - ((uint32_t)e << 23);
			if (fbits(_mm_cvtss_f32(_mm_rcp_ss(_mm_set_ss(x)))) != want) return 0;
		}
	return 1;
}
