/*
 * hakm_oracle.c — CPU restatement of hako's quantized decode path.
 *
 * TEST INFRASTRUCTURE ONLY (see hakm_oracle.h). Written for clarity, not
 * speed: plain scalar C, single thread, built without -ffast-math and with
 * -ffp-contract=off, so every rounding below is the one written: fused
 * multiply-adds appear as fmaf() exactly where the reference's own build
 * fuses them. Each function cites the reference file:line it restates.
 */
#include "hakm_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ fp16 */

/* src/quant.c:31-54: sign | exponent rebias | mantissa, subnormals
 * normalised, inf/nan kept. Restated arithmetically: a binary16 value is
 * (-1)^s * 2^(e-15) * (1 + m/1024) for e in 1..30, 2^-14 * m/1024 for e = 0. */
float orc_f16_to_f32(uint16_t h) {
	int s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
	float v;
	if (e == 31) {
		uint32_t bits = ((uint32_t)s << 31) | 0x7F800000u | ((uint32_t)m << 13);
		memcpy(&v, &bits, 4);
		return v;
	}
	if (e == 0) v = ldexpf((float)m, -24);                 /* exact */
	else        v = ldexpf((float)(1024 + m), e - 25);      /* exact */
	return s ? -v : v;
}

uint16_t orc_f32_to_f16(float f) {
	uint32_t x; memcpy(&x, &f, 4);
	uint32_t sign = (x >> 16) & 0x8000u;
	uint32_t ax = x & 0x7FFFFFFFu;
	if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0));
	if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);     /* rounds to inf */
	if (ax < 0x33000001u) return (uint16_t)sign;                  /* < half min subnormal */
	int e = (int)(ax >> 23) - 127;
	uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;
	int shift;
	uint32_t base;
	if (e < -14) {            /* subnormal half: value = mant * 2^(e-23) = q * 2^-24 */
		shift = -e - 1;   /* q = mant >> (shift) where 2^(e-23)/2^-24 = 2^(e+1) */
		base = 0;
	} else {
		shift = 13;
		base = (uint32_t)(e + 15) << 10;
		mant &= 0x7FFFFFu;
	}
	uint32_t q = mant >> shift;
	uint32_t rem = mant & ((1u << shift) - 1u);
	uint32_t half = 1u << (shift - 1);
	if (rem > half || (rem == half && (q & 1u))) q++;
	return (uint16_t)(sign | (base + q));   /* carry into exponent is correct */
}

/* ------------------------------------------------------------ Q4_K / Q6_K */

/* src/quant.c:57-66. Sub-blocks 0..3 keep scale/min in the low 6 bits of
 * bytes j and j+4; sub-blocks 4..7 split them into a nibble in byte j+4 and
 * the top two bits of bytes j-4 (scale) and j (min). */
void orc_scale_min_k4(int j, const uint8_t *q, int *s, int *m) {
	if (j < 4) {
		*s = q[j] & 0x3F;
		*m = q[j + 4] & 0x3F;
	} else {
		*s = (q[j + 4] & 0x0F) | ((q[j - 4] & 0xC0) >> 2);
		*m = (q[j + 4] >> 4)   | ((q[j] & 0xC0) >> 2);
	}
}

/* block_q4_K (src/quant.h:12-17): d u16 @0, dmin u16 @2, scales[12] @4,
 * qs[128] @16; 144 bytes. */
static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* src/quant.c:68-92. Element 64g + l (l < 32) is the low nibble of qs[32g+l]
 * with sub-block 2g; element 64g + 32 + l the high nibble, sub-block 2g+1. */
void orc_dequant_q4k(const void *blocks, float *out, int nelem) {
	const uint8_t *b = (const uint8_t *)blocks;
	for (int i = 0; i < nelem / ORC_QK; i++, b += 144) {
		float d = orc_f16_to_f32(rd16(b)), dmin = orc_f16_to_f32(rd16(b + 2));
		const uint8_t *sc = b + 4, *qs = b + 16;
		for (int sb = 0; sb < 8; sb++) {
			int s, m;
			orc_scale_min_k4(sb, sc, &s, &m);
			float ds = d * (float)s, dm = dmin * (float)m;
			int g = sb >> 1, hi = sb & 1;
			for (int l = 0; l < 32; l++) {
				int q = hi ? (qs[32 * g + l] >> 4) : (qs[32 * g + l] & 0x0F);
				out[i * ORC_QK + 32 * sb + l] = ds * (float)q - dm;
			}
		}
	}
}

/* block_q6_K (src/quant.h:19-24): ql[128] @0, qh[64] @128, scales[16] int8
 * @192, d u16 @208; 210 bytes. src/quant.c:94-123: element e = 128n + 32k + l
 * (n half, k quarter, l < 32) takes the low (k even) or high (k odd... see
 * below) nibble of ql and bits 2k..2k+1 of qh[32n + l]; scale group e/16. */
void orc_dequant_q6k(const void *blocks, float *out, int nelem) {
	const uint8_t *b = (const uint8_t *)blocks;
	for (int i = 0; i < nelem / ORC_QK; i++, b += 210) {
		const uint8_t *ql = b, *qh = b + 128;
		const int8_t *sc = (const int8_t *)(b + 192);
		float d = orc_f16_to_f32(rd16(b + 208));
		for (int e = 0; e < ORC_QK; e++) {
			int n = e >> 7, k = (e >> 5) & 3, l = e & 31;
			/* quarters 0,1 use the low nibble of ql[64n + 32(k&1) + l],
			 * quarters 2,3 the high nibble of the same bytes */
			int lo_byte = ql[64 * n + 32 * (k & 1) + l];
			int nib = (k < 2) ? (lo_byte & 0x0F) : (lo_byte >> 4);
			int hb = (qh[32 * n + l] >> (2 * k)) & 3;
			int q = (nib | (hb << 4)) - 32;
			out[i * ORC_QK + e] = d * (float)sc[e >> 4] * (float)q;
		}
	}
}

/* ------------------------------------------------------------- q8_32 */

/* src/quant.c:127-144, as the reference's own flags compile it (Makefile:8,
 * -O3 -ffast-math; pinned against that build by tests/golden/q8.npz):
 *  - xs = amax * fl(1/127)   (amax/127.0f becomes a multiply by the reciprocal)
 *  - inv = 127.0f / amax     (gcc folds 1/(amax*(1/127)) into one division)
 *  - q = (int32)(int64)rint(x * inv), clamped to +-127: the conversion is a
 *    64-bit cvtss2si whose out-of-range / NaN result INT64_MIN truncates to 0.
 */
static int orc_q8_round(float r) {
	if (!(fabsf(r) < 9223372036854775808.0f)) return 0;
	long long v = llrintf(r);
	int32_t v32 = (int32_t)(uint32_t)((unsigned long long)v & 0xFFFFFFFFull);
	return v32 > 127 ? 127 : (v32 < -127 ? -127 : v32);
}

void orc_quantize_q8_32(const float *x, int n, int8_t *xq, float *xs) {
	const float inv127 = 1.0f / 127.0f;
	for (int b = 0; b < n / 32; b++) {
		float amax = 0.0f;
		for (int l = 0; l < 32; l++) {
			float a = fabsf(x[32 * b + l]);
			if (a > amax) amax = a;
		}
		float scale = amax * inv127;
		float inv = scale > 0.0f ? 127.0f / amax : 0.0f;
		xs[b] = scale;
		for (int l = 0; l < 32; l++) xq[32 * b + l] = (int8_t)orc_q8_round(x[32 * b + l] * inv);
	}
}

/* src/quant.c:163-229 (the scalar branch, quant.c:214-221, is the plain statement). */
void orc_q4k_subsums(const void *row, int n_in, const int8_t *xq,
                     int32_t *iqx, int32_t *ix) {
	const uint8_t *b = (const uint8_t *)row;
	for (int i = 0; i < n_in / ORC_QK; i++, b += 144) {
		const uint8_t *qs = b + 16;
		for (int sb = 0; sb < 8; sb++) {
			int g = sb >> 1, hi = sb & 1;
			int32_t a = 0, c = 0;
			for (int l = 0; l < 32; l++) {
				int q = hi ? (qs[32 * g + l] >> 4) : (qs[32 * g + l] & 0x0F);
				int xv = xq[i * ORC_QK + 32 * sb + l];
				a += q * xv;
				c += xv;
			}
			iqx[8 * i + sb] = a;
			ix[8 * i + sb] = c;
		}
	}
}

/* ------------------------------------------------- as-built fp32 orders
 *
 * The reference is built with -O3 -ffast-math -march=x86-64-v3 (its
 * Makefile:8 flags, ARCH pinned by oracle/Makefile). gcc then fixes every
 * floating-point rounding of the path: which products are fused (FMA), how
 * the reductions are split over the 8 lanes of a 256-bit vector and folded,
 * which libm / libmvec variant each exp/pow/cos/sin goes through, and that
 * 1/sqrtf becomes rsqrtss plus one Newton step. The functions below restate
 * those roundings one by one; tests/test_oracle.py pins each against the
 * reference's own build (bit for bit), and the CUDA kernels follow the same
 * steps. */

static inline uint32_t fbits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bitsf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline double bitsd(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
static inline uint64_t dbits(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }

/* 8-lane reduction fold of a 256-bit accumulator (the vextractf128 / movhlps
 * / shufps sequence gcc emits): ((a1+a5)+(a3+a7)) + ((a0+a4)+(a2+a6)). */
static float fold8(const float a[8]) {
	float s0 = a[0] + a[4], s1 = a[1] + a[5], s2 = a[2] + a[6], s3 = a[3] + a[7];
	return (s0 + s2) + (s1 + s3);
}
static float fold4(const float u[4]) { return (u[0] + u[2]) + (u[1] + u[3]); }

/* Σ a[i]·b[i] as gcc vectorizes `acc += a[i] * b[i]` under -ffast-math
 * (src/nn.c:15 with a == b, src/nn.c:92, src/model.c:130): lane i%8 of the
 * main loop accumulates the ROUNDED products (vmulps then vaddps, no FMA);
 * the lanes fold to 4 (lo + hi); a remainder of 4..7 takes one 4-wide FMA
 * step on those 4 lanes before they fold; the last 0..3 elements are scalar
 * FMAs. n < 8 starts from the 4-wide step with zero lanes. */
float orc_dot_f32(const float *a, const float *b, int n) {
	float acc8[8] = {0, 0, 0, 0, 0, 0, 0, 0}, c4[4] = {0, 0, 0, 0}, sum = 0.0f;
	int i = 0;
	if (n >= 8) {
		for (; i + 8 <= n; i += 8)
			for (int l = 0; l < 8; l++) acc8[l] = acc8[l] + a[i + l] * b[i + l];
		for (int l = 0; l < 4; l++) c4[l] = acc8[l] + acc8[l + 4];
		sum = fold8(acc8);
	}
	if (n - i >= 4) {
		for (int l = 0; l < 4; l++) c4[l] = fmaf(a[i + l], b[i + l], c4[l]);
		sum = fold4(c4);
		i += 4;
	}
	for (; i < n; i++) sum = fmaf(a[i], b[i], sum);
	return sum;
}

/* rsqrtss, the approximate reciprocal square root gcc emits for 1/sqrtf under
 * -ffast-math. Its result is fixed by the exponent's parity and the top 10
 * mantissa bits; the 2048 results for [1, 4) are measured once from this
 * host's instruction (orc_rsqrt_table) and the exponent is scaled by two per
 * step of four. Positive normal inputs only (the reference's arguments). */
static uint32_t RSQ[2048];
static int rsq_ready;
void orc_rsqrt_table(uint32_t *out) {
	for (int par = 0; par < 2; par++)
		for (int m = 0; m < 1024; m++) {
			float x = bitsf(((uint32_t)(127 + par) << 23) | ((uint32_t)m << 13));
			out[par * 1024 + m] = fbits(_mm_cvtss_f32(_mm_rsqrt_ss(_mm_set_ss(x))));
		}
}
float orc_rsqrt_approx(float v) {
	if (!rsq_ready) { orc_rsqrt_table(RSQ); rsq_ready = 1; }
	uint32_t u = fbits(v);
	int E = (int)(u >> 23) - 127, par = E & 1, k = (E - par) / 2;
	uint32_t r = RSQ[par * 1024 + ((u >> 13) & 1023)];
	return bitsf(r - ((uint32_t)k << 23));
}
/* 1/sqrtf(v) as built: r = rsqrtss(v); (-0.5 r) * fma(r, v r, -3). */
float orc_rsqrt_nr(float v) {
	float r = orc_rsqrt_approx(v);
	float t = fmaf(r, v * r, -3.0f);
	return (r * -0.5f) * t;
}

/* glibc's scalar expf (the FMA-built variant the host selects): the
 * published exp2f table method, 2^(k/32) from a 32-entry table of doubles,
 * a cubic in double, one rounding to float at the end. The table entries are
 * 2^(i/32) rounded to double, stored minus i << 47 (the exponent bits that
 * the index adds back). */
static const double EXP_INVLN2N = 0x1.71547652b82fep+0 * 32, EXP_SHIFT = 0x1.8p+52;
static const double EXP_C0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, EXP_C1 = 0x1.ebfce50fac4f3p-3 / 32 / 32,
                    EXP_C2 = 0x1.62e42ff0c52d6p-1 / 32;
static uint64_t EXP_T[32];
static int exp_ready;
static void exp_table(void) {
	/* 2^(i/32) correctly rounded: long double (64-bit mantissa) exp2l,
	 * rounded once more to double, agrees with the exact value here. */
	for (int i = 0; i < 32; i++) EXP_T[i] = dbits((double)exp2l((long double)i / 32.0L)) - ((uint64_t)i << 47);
	exp_ready = 1;
}
void orc_exp_table(uint64_t *out) {
	if (!exp_ready) exp_table();
	memcpy(out, EXP_T, sizeof EXP_T);
}
float orc_expf(float x) {
	if (!exp_ready) exp_table();
	uint32_t ax = fbits(x) & 0x7FFFFFFFu;
	if (ax >= 0x42B00000u) {                  /* |x| >= 88, inf, nan */
		if (fbits(x) == 0xFF800000u) return 0.0f;
		if (ax >= 0x7F800000u) return x + x;
		if (x > 0x1.62e42ep6f) return bitsf(0x7F800000u);
		if (x < -0x1.9fe368p6f) return 0.0f;
	}
	double xd = (double)x, z = EXP_INVLN2N * xd;
	double kd = z + EXP_SHIFT;
	uint64_t ki = dbits(kd);
	kd -= EXP_SHIFT;
	double r = fma(EXP_INVLN2N, xd, -kd);
	uint64_t t = EXP_T[ki % 32] + (ki << 47);
	double s = bitsd(t);
	double zz = fma(EXP_C0, r, EXP_C1), r2 = r * r, y = fma(EXP_C2, r, 1.0);
	y = fma(zz, r2, y);
	return (float)(y * s);
}

/* libmvec's vector expf (the 8-wide AVX2 and the 4-wide SSE4 entry points
 * that -ffast-math vectorization calls): n = rint(x/ln2) by the 1.5*2^23
 * shifter, r = x - n*ln2 in two parts, a degree-5 polynomial for e^r, times
 * 2^n built in the exponent field. The AVX2 form fuses each step (FMA); the
 * SSE4 form rounds every product and sum. Lanes with |x| > 87.3365 go to
 * the scalar expf. */
#define VX_INVLN2 0x3fb8aa3bu
#define VX_SHIFT 0x4b400000u
#define VX_LN2HI 0x3f317200u
#define VX_LN2LO 0x35bfbe8eu
#define VX_DOM 0x42aeac4fu
static const uint32_t VX_P[6] = {0x3f800000u, 0x3f7ffffeu, 0x3effff34u, 0x3e2aacacu, 0x3d2b8392u, 0x3c07d9feu};
float orc_expf_v8(float x) {
	if ((fbits(x) & 0x7FFFFFFFu) > VX_DOM) return orc_expf(x);
	float m = fmaf(x, bitsf(VX_INVLN2), bitsf(VX_SHIFT));
	float n = m - bitsf(VX_SHIFT);
	float r = fmaf(-n, bitsf(VX_LN2HI), x);
	r = fmaf(-n, bitsf(VX_LN2LO), r);
	float p = fmaf(bitsf(VX_P[5]), r, bitsf(VX_P[4]));
	for (int k = 3; k >= 0; k--) p = fmaf(p, r, bitsf(VX_P[k]));
	return p * bitsf((fbits(m) + 127u) << 23);
}
float orc_expf_v4(float x) {
	if ((fbits(x) & 0x7FFFFFFFu) > VX_DOM) return orc_expf(x);
	float m = x * bitsf(VX_INVLN2);
	m = m + bitsf(VX_SHIFT);
	float n = m - bitsf(VX_SHIFT);
	float t = n * bitsf(VX_LN2HI);
	float r = x - t;
	t = n * bitsf(VX_LN2LO);
	r = r - t;
	float p = bitsf(VX_P[5]) * r;
	for (int k = 4; k >= 0; k--) { p = p + bitsf(VX_P[k]); if (k) p = p * r; }
	return p * bitsf((fbits(m) + 127u) << 23);
}

/* src/quant.c:150-232 (AVX2 branch, quant.c:193-213), as built: per pair of
 * sub-blocks (A = 2g, B = 2g+1) of a super-block
 *   tA = fma(sA, d*iqxA, -(mA*(dmin*ixA)))       (gcc reassociates d*s*iqx)
 *   uA = tA * xsA
 *   acc = acc + fma(tB, xsB, uA)                 (tB likewise)
 * i.e. one rounded add into the running sum per 64 weights, in order. */
float orc_q4k_dot(const void *row, int n_in, const int8_t *xq, const float *xs) {
	const uint8_t *b = (const uint8_t *)row;
	int nsb = n_in / 32;
	int32_t *iqx = malloc(sizeof(int32_t) * nsb), *ix = malloc(sizeof(int32_t) * nsb);
	orc_q4k_subsums(row, n_in, xq, iqx, ix);
	float acc = 0.0f;
	for (int i = 0; i < n_in / ORC_QK; i++, b += 144) {
		float d = orc_f16_to_f32(rd16(b)), dmin = orc_f16_to_f32(rd16(b + 2));
		for (int g = 0; g < 4; g++) {
			int sa, ma, sb_, mb, ka = 8 * i + 2 * g, kb = ka + 1;
			orc_scale_min_k4(2 * g, b + 4, &sa, &ma);
			orc_scale_min_k4(2 * g + 1, b + 4, &sb_, &mb);
			float tA = fmaf((float)sa, d * (float)iqx[ka], -((float)ma * (dmin * (float)ix[ka])));
			float tB = fmaf((float)sb_, d * (float)iqx[kb], -((float)mb * (dmin * (float)ix[kb])));
			float uA = tA * xs[ka];
			acc = acc + fmaf(tB, xs[kb], uA);
		}
	}
	free(iqx); free(ix);
	return acc;
}

/* src/nn.c:84-95: dequantize the row (exact: d*sc*q has at most 24
 * significant bits), then the vectorized float dot. */
float orc_q6k_dot(const void *row, int n_in, const float *x) {
	float *w = malloc(sizeof(float) * (size_t)n_in);
	orc_dequant_q6k(row, w, n_in);
	float acc = orc_dot_f32(w, x, n_in);
	free(w);
	return acc;
}

/* ------------------------------------------------------------- nn ops */

/* src/nn.c:13-18 as built: Σx² by orc_dot_f32; v = ss/n + eps (one IEEE
 * division, one add); scale = the rsqrtss Newton step; y = (x*w)*scale. */
void orc_rmsnorm(float *y, const float *x, const float *w, int n, float eps) {
	float ss = orc_dot_f32(x, x, n);
	float v = ss / (float)n + eps;
	float scale = orc_rsqrt_nr(v);
	for (int i = 0; i < n; i++) y[i] = (x[i] * w[i]) * scale;
}

/* src/nn.c:20-27 as built. exp(x - max) of element i goes through the 8-wide
 * libmvec expf for the first 8*floor(n/8) elements, the 4-wide one for the
 * next 4 when at least 4 remain, the scalar expf for the last 0..3; the sum
 * follows the same split (8 lanes, folded to 4, one 4-lane step, folded,
 * then scalar adds); then one reciprocal and a multiply. */
void orc_softmax(float *x, int n) {
	float mx = x[0];
	for (int i = 1; i < n; i++) mx = x[i] > mx ? x[i] : mx;
	float acc8[8] = {0, 0, 0, 0, 0, 0, 0, 0}, c4[4] = {0, 0, 0, 0}, sum = 0.0f;
	int i = 0;
	if (n >= 8) {
		for (; i + 8 <= n; i += 8)
			for (int l = 0; l < 8; l++) {
				x[i + l] = orc_expf_v8(x[i + l] - mx);
				acc8[l] = acc8[l] + x[i + l];
			}
		for (int l = 0; l < 4; l++) c4[l] = acc8[l] + acc8[l + 4];
		sum = fold8(acc8);
	}
	if (n - i >= 4) {
		for (int l = 0; l < 4; l++) {
			x[i + l] = orc_expf_v4(x[i + l] - mx);
			c4[l] = x[i + l] + c4[l];
		}
		sum = fold4(c4);
		i += 4;
	}
	for (; i < n; i++) {
		x[i] = orc_expf(x[i] - mx);
		sum = sum + x[i];
	}
	float inv = 1.0f / sum;
	for (int k = 0; k < n; k++) x[k] *= inv;
}

/* src/nn.c:29: x / (1 + expf(-x)) with the scalar expf (silu_f is called
 * per element from src/model.c:154, not vectorized). */
float orc_silu(float x) { return x / (1.0f + orc_expf(-x)); }

/* src/nn.c:32-42 as built. The loop over pairs is vectorized 8 wide:
 * freq = powf(theta, 2i * (-1/hd)) and cos/sin of pos*freq through the
 * libmvec vector functions (4-wide ones for a 4-pair remainder, scalar libm
 * for the last 0..3 pairs, and for all pairs when there are fewer than 8);
 * then a' = fma(a, c, -(b*s)), b' = fma(a, s, b*c).
 * orc_rope_table gives the (cos, sin) pairs of one position; both are test
 * helpers that call the host's libm/libmvec, as the reference does. */
__m256 _ZGVdN8vv_powf(__m256, __m256);
__m256 _ZGVdN8v_cosf(__m256);
__m256 _ZGVdN8v_sinf(__m256);
__m128 _ZGVbN4vv_powf(__m128, __m128);
__m128 _ZGVbN4v_cosf(__m128);
__m128 _ZGVbN4v_sinf(__m128);
void orc_rope_table(float *cs, int head_dim, int pos, float theta) {
	int half = head_dim / 2, i = 0;
	float nhd = -1.0f / (float)head_dim, fp = (float)pos;
	/* below 8 pairs the two halves of vec overlap within one vector, and
	 * gcc's alias check sends the whole loop down the scalar path */
	if (half < 8) goto scalar;
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
scalar:
	for (; i < half; i++) {
		float ang = fp * powf(theta, (float)(2 * i) * nhd);
		cs[2 * i] = cosf(ang);
		cs[2 * i + 1] = sinf(ang);
	}
}
void orc_rope_neox(float *vec, int head_dim, int pos, float theta) {
	int half = head_dim / 2;
	float *cs = malloc(sizeof(float) * 2 * (size_t)half);
	orc_rope_table(cs, head_dim, pos, theta);
	for (int i = 0; i < half; i++) {
		float c = cs[2 * i], s = cs[2 * i + 1], a = vec[i], b = vec[i + half];
		vec[i] = fmaf(a, c, -(b * s));
		vec[i + half] = fmaf(a, s, b * c);
	}
	free(cs);
}

/* GQA decode attention at position pos over caches kc / vc laid out
 * [pos + 1][KVH * hd] (src/model.c:124-142 as built): scores by the
 * vectorized dot times the rsqrtss scale, the softmax above, then
 * out[d] = fma(p_s, v_s[d], out[d]) for s = 0..pos from +0. */
void orc_attention(float *out, const float *q, const float *kc, const float *vc, int pos, int H, int KVH,
                   int hd) {
	int KV = KVH * hd, group = H / KVH;
	float scale = orc_rsqrt_nr((float)hd);
	float *sc = malloc(sizeof(float) * (size_t)(pos + 1));
	for (int h = 0; h < H; h++) {
		int kh = h / group;
		for (int s = 0; s <= pos; s++) sc[s] = orc_dot_f32(q + h * hd, kc + (size_t)s * KV + kh * hd, hd) * scale;
		orc_softmax(sc, pos + 1);
		float *o = out + h * hd;
		for (int d = 0; d < hd; d++) o[d] = 0.0f;
		for (int s = 0; s <= pos; s++)
			for (int d = 0; d < hd; d++) o[d] = fmaf(sc[s], vc[(size_t)s * KV + kh * hd + d], o[d]);
	}
	free(sc);
}

/* MLF2 tensor types (include/mlf2.h:44-49). */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4K = 12, ORC_Q6K = 14 };

static size_t orc_row_bytes(int type, int n_in) {   /* src/nn.c:45-53 */
	switch (type) {
	case ORC_F32: return (size_t)n_in * 4;
	case ORC_F16: return (size_t)n_in * 2;
	case ORC_Q4K: return (size_t)(n_in / ORC_QK) * 144;
	case ORC_Q6K: return (size_t)(n_in / ORC_QK) * 210;
	default: return 0;
	}
}

static void orc_dequant_row(int type, const uint8_t *src, float *out, int n) {
	switch (type) {     /* src/quant.c:234-248 */
	case ORC_F32: memcpy(out, src, (size_t)n * 4); break;
	case ORC_F16: for (int i = 0; i < n; i++) out[i] = orc_f16_to_f32(rd16(src + 2 * i)); break;
	case ORC_Q4K: orc_dequant_q4k(src, out, n); break;
	case ORC_Q6K: orc_dequant_q6k(src, out, n); break;
	}
}

/* src/nn.c:179-210 with mm_worker src/nn.c:70-97: Q4_K rows take the int8
 * path against one shared quantized copy of x; every other type dequantizes
 * the row and dots it with the fp32 x. Bias is added after the dot. */
int orc_matmul(float *out, const float *x, int type, const void *w,
               const float *bias, int n_out, int n_in) {
	size_t rb = orc_row_bytes(type, n_in);
	if (!rb) return -1;
	const uint8_t *base = (const uint8_t *)w;
	if (type == ORC_Q4K) {
		int8_t *xq = malloc((size_t)n_in);
		float *xs = malloc(sizeof(float) * (size_t)(n_in / 32));
		orc_quantize_q8_32(x, n_in, xq, xs);
		for (int r = 0; r < n_out; r++) {
			float acc = orc_q4k_dot(base + (size_t)r * rb, n_in, xq, xs);
			out[r] = bias ? acc + bias[r] : acc;
		}
		free(xq); free(xs);
		return 0;
	}
	float *tmp = malloc(sizeof(float) * (size_t)n_in);
	for (int r = 0; r < n_out; r++) {
		orc_dequant_row(type, base + (size_t)r * rb, tmp, n_in);
		float acc = orc_dot_f32(tmp, x, n_in);
		out[r] = bias ? acc + bias[r] : acc;
	}
	free(tmp);
	return 0;
}

/* ------------------------------------------------------------- model */

/* MLF2 header / directory field offsets (include/mlf2.h:55-87). */
#define H_NLAYERS 12
#define H_DMODEL 16
#define H_NHEADS 20
#define H_NKV 24
#define H_HEADDIM 28
#define H_FFN 32
#define H_VOCAB 40
#define H_THETA 44
#define H_EPS 48
#define H_FLAGS 52
#define H_NTENS 56
#define H_TENSOFF 60
#define H_DATAOFF 76
#define T_SIZE 104

typedef struct { int type; const uint8_t *data; } orc_t;

typedef struct {
	orc_t attn_norm, ffn_norm, wq, wk, wv, wo, bq, bk, bv, gate, up, down;
} orc_layer;

struct orc_model {
	int L, D, H, KVH, hd, F, V, max_seq, pos, run_layers;
	float theta, eps;
	orc_layer *layers;
	orc_t tok_embd, out_norm, out_w;
	float *xb, *xn, *q, *k, *v, *att, *hbuf, *ubuf, *logits, *kc, *vc, *scores;
};

static uint32_t g32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }
static uint64_t g64(const uint8_t *p) { uint64_t v; memcpy(&v, p, 8); return v; }
static float gf(const uint8_t *p) { float v; memcpy(&v, p, 4); return v; }

static orc_t orc_find(const uint8_t *img, size_t size, const char *name) {
	orc_t t = { -1, NULL };
	uint32_t n = g32(img + H_NTENS);
	uint64_t toff = g64(img + H_TENSOFF), doff = g64(img + H_DATAOFF);
	for (uint32_t i = 0; i < n; i++) {
		const uint8_t *e = img + toff + (size_t)i * T_SIZE;
		if (strncmp((const char *)e, name, 48) == 0) {
			uint64_t rel = g64(e + 88), nb = g64(e + 96);
			if (doff + rel + nb > size) return t;
			t.type = (int)g32(e + 48);
			t.data = img + doff + rel;
			return t;
		}
	}
	return t;
}

orc_model *orc_model_new(const void *image, size_t size, int max_seq) {
	const uint8_t *img = (const uint8_t *)image;
	if (size < 128 || memcmp(img, "MLF2", 4) != 0 || g32(img + 4) != 2) return NULL;
	if (g64(img + H_TENSOFF) + (uint64_t)g32(img + H_NTENS) * T_SIZE > size) return NULL;
	orc_model *m = calloc(1, sizeof(*m));
	m->L = (int)g32(img + H_NLAYERS); m->D = (int)g32(img + H_DMODEL);
	m->H = (int)g32(img + H_NHEADS); m->KVH = (int)g32(img + H_NKV);
	m->hd = (int)g32(img + H_HEADDIM); m->F = (int)g32(img + H_FFN);
	m->V = (int)g32(img + H_VOCAB); m->theta = gf(img + H_THETA); m->eps = gf(img + H_EPS);
	m->max_seq = max_seq; m->run_layers = m->L;
	uint32_t flags = g32(img + H_FLAGS);
	int ok = 1;
	m->tok_embd = orc_find(img, size, "token_embd.weight");
	m->out_norm = orc_find(img, size, "output_norm.weight");
	m->out_w = (flags & 2u) ? m->tok_embd : orc_find(img, size, "output.weight");
	ok &= m->tok_embd.data && m->out_norm.data && m->out_w.data;
	m->layers = calloc((size_t)m->L, sizeof(orc_layer));
	char nm[64];
	for (int l = 0; l < m->L && ok; l++) {
		orc_layer *y = &m->layers[l];
#define F_(fld, s) snprintf(nm, sizeof nm, "blk.%d." s, l); y->fld = orc_find(img, size, nm);
		F_(attn_norm, "attn_norm.weight") F_(ffn_norm, "ffn_norm.weight")
		F_(wq, "attn_q.weight") F_(wk, "attn_k.weight") F_(wv, "attn_v.weight")
		F_(wo, "attn_output.weight") F_(gate, "ffn_gate.weight") F_(up, "ffn_up.weight")
		F_(down, "ffn_down.weight") F_(bq, "attn_q.bias") F_(bk, "attn_k.bias") F_(bv, "attn_v.bias")
#undef F_
		ok &= y->attn_norm.data && y->ffn_norm.data && y->wq.data && y->wk.data &&
		      y->wv.data && y->wo.data && y->gate.data && y->up.data && y->down.data;
	}
	if (!ok) { orc_model_free(m); return NULL; }
	int KV = m->KVH * m->hd;
	m->xb = calloc((size_t)m->D, 4); m->xn = calloc((size_t)m->D, 4);
	m->q = calloc((size_t)m->D, 4); m->k = calloc((size_t)KV, 4); m->v = calloc((size_t)KV, 4);
	m->att = calloc((size_t)m->D, 4); m->hbuf = calloc((size_t)m->F, 4);
	m->ubuf = calloc((size_t)m->F, 4); m->logits = calloc((size_t)m->V, 4);
	m->scores = calloc((size_t)max_seq, 4);
	m->kc = calloc((size_t)m->L * max_seq * KV, 4);
	m->vc = calloc((size_t)m->L * max_seq * KV, 4);
	return m;
}

void orc_model_free(orc_model *m) {
	if (!m) return;
	free(m->layers); free(m->xb); free(m->xn); free(m->q); free(m->k); free(m->v);
	free(m->att); free(m->hbuf); free(m->ubuf); free(m->logits); free(m->scores);
	free(m->kc); free(m->vc); free(m);
}

void orc_model_reset(orc_model *m) { m->pos = 0; }
int orc_model_vocab(const orc_model *m) { return m->V; }
int orc_model_dim(const orc_model *m) { return m->D; }
void orc_model_set_layers(orc_model *m, int n) { m->run_layers = (n < 0 || n > m->L) ? m->L : n; }
const float *orc_hidden(const orc_model *m) { return m->xb; }

static const float *fp(orc_t t) { return (const float *)t.data; }

/* src/model.c:93-165, step for step. */
const float *orc_forward(orc_model *m, int token) {
	int D = m->D, H = m->H, KVH = m->KVH, hd = m->hd, KV = KVH * hd, F = m->F, pos = m->pos;
	if (pos >= m->max_seq || token < 0 || token >= m->V) return NULL;
	orc_dequant_row(m->tok_embd.type,
	                m->tok_embd.data + (size_t)token * orc_row_bytes(m->tok_embd.type, D), m->xb, D);
	for (int l = 0; l < m->run_layers; l++) {
		orc_layer *y = &m->layers[l];
		orc_rmsnorm(m->xn, m->xb, fp(y->attn_norm), D, m->eps);
		orc_matmul(m->q, m->xn, y->wq.type, y->wq.data, y->bq.data ? fp(y->bq) : NULL, D, D);
		orc_matmul(m->k, m->xn, y->wk.type, y->wk.data, y->bk.data ? fp(y->bk) : NULL, KV, D);
		orc_matmul(m->v, m->xn, y->wv.type, y->wv.data, y->bv.data ? fp(y->bv) : NULL, KV, D);
		for (int h = 0; h < H; h++) orc_rope_neox(m->q + h * hd, hd, pos, m->theta);
		for (int h = 0; h < KVH; h++) orc_rope_neox(m->k + h * hd, hd, pos, m->theta);
		float *kc = m->kc + ((size_t)l * m->max_seq) * KV, *vc = m->vc + ((size_t)l * m->max_seq) * KV;
		memcpy(kc + (size_t)pos * KV, m->k, sizeof(float) * KV);
		memcpy(vc + (size_t)pos * KV, m->v, sizeof(float) * KV);
		orc_attention(m->att, m->q, kc, vc, pos, H, KVH, hd);
		orc_matmul(m->xn, m->att, y->wo.type, y->wo.data, NULL, D, D);
		for (int i = 0; i < D; i++) m->xb[i] += m->xn[i];
		orc_rmsnorm(m->xn, m->xb, fp(y->ffn_norm), D, m->eps);
		orc_matmul(m->hbuf, m->xn, y->gate.type, y->gate.data, NULL, F, D);
		orc_matmul(m->ubuf, m->xn, y->up.type, y->up.data, NULL, F, D);
		for (int i = 0; i < F; i++) m->hbuf[i] = orc_silu(m->hbuf[i]) * m->ubuf[i];
		orc_matmul(m->xn, m->hbuf, y->down.type, y->down.data, NULL, D, F);
		for (int i = 0; i < D; i++) m->xb[i] += m->xn[i];
	}
	float *fin = malloc(sizeof(float) * D);
	orc_rmsnorm(fin, m->xb, fp(m->out_norm), D, m->eps);
	orc_matmul(m->logits, fin, m->out_w.type, m->out_w.data, NULL, m->V, D);
	free(fin);
	m->pos++;
	return m->logits;
}

/* src/sample.c:28-32: strict '>' so the lowest index wins ties. */
int orc_argmax(const float *logits, int n) {
	int best = 0;
	for (int i = 1; i < n; i++) if (logits[i] > logits[best]) best = i;
	return best;
}

/* ------------------------------------------------- pins of the libm steps */

/* Counts inputs in [lo, hi] (float bit patterns, every step-th) where the
 * restatements above differ from what the host's libm / libmvec / rsqrtss
 * return: out[0] scalar expf, out[1] 8-wide expf, out[2] 4-wide expf,
 * out[3] rsqrtss (positive normal inputs only). */
__m256 _ZGVdN8v_expf(__m256);
__m128 _ZGVbN4v_expf(__m128);
void orc_check_libm(uint32_t lo, uint32_t hi, uint32_t step, long long *out) {
	out[0] = out[1] = out[2] = out[3] = 0;
	for (uint64_t u = lo; u <= hi; u += step) {
		float x = bitsf((uint32_t)u);
		float e8[8], e4[4];
		_mm256_storeu_ps(e8, _ZGVdN8v_expf(_mm256_set1_ps(x)));
		_mm_storeu_ps(e4, _ZGVbN4v_expf(_mm_set1_ps(x)));
		if (!isnan(x)) {
			out[0] += fbits(expf(x)) != fbits(orc_expf(x));
			out[1] += fbits(e8[0]) != fbits(orc_expf_v8(x));
			out[2] += fbits(e4[0]) != fbits(orc_expf_v4(x));
		}
		uint32_t a = (uint32_t)u;
		if (a >= 0x00800000u && a < 0x7F800000u)
			out[3] += fbits(_mm_cvtss_f32(_mm_rsqrt_ss(_mm_set_ss(x)))) != fbits(orc_rsqrt_approx(x));
	}
}
