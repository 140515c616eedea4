/*
 * ceb_oracle.c -- CPU restatement of CrispEmbed's NomicBERT-MoE encoder path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA path
 * in crispembed_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load it; the shipped
 * library never links, loads or falls back to it.
 *
 * Parity status: the reference's arithmetic lives in ggml, an un-vendored git
 * submodule of the reference (.gitmodules:1-4, fork CrispStrobe/ggml, branch
 * sync/upstream-v0.17, no commit pinned, directory empty), so the reference
 * cannot be built or run here.  The block formats below are pinned against
 * gguf-py (the converter's own quantizer/dequantizer); the graph semantics
 * (router, softmax, top-k, mul_mat_id, GELU, combine, norms, attention,
 * pooling) are restated from the reference call sites and ggml's published
 * CPU algorithms and are NOT pinned by any reference-produced vector:
 * "parity unpinned" for the graph part.
 *
 * Three arithmetic modes for every matrix product:
 *   CEO_EXACT : f32 activations x exactly-dequantized weights, double accumulation.
 *   CEO_GGML  : what ggml's x86 CPU backend computes: activations re-quantized to
 *               the weight's vec_dot type (Q8_0 for Q8_0, Q8_K for Q4_K), integer
 *               block dots, float accumulation in ggml's lane order.
 *   CEO_F16   : operands rounded to fp16 (weights as fp16(dequant), activations as
 *               fp16), double accumulation, MoE expert outputs stored as fp16 --
 *               the precision of the device kernels, used to check them tightly.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#if defined(__AVX2__) || defined(__F16C__)
#include <immintrin.h>
#endif

#ifdef _OPENMP
#include <omp.h>
#endif

/* exp / erf shared bit for bit with the device kernels (see the header).  The
 * build that times the CPU path (CEO_LIBM_MATH) calls the C library's expf / erff
 * instead, as ggml does: the shared routines compute in double precision and cost
 * several times more on the CPU; the two differ by at most one ulp. */
#include "ceb_portable_math.h"
#ifdef CEO_LIBM_MATH
#define ceo_expf_ expf
#define ceo_erff_ erff
#else
#define ceo_expf_ ceb_expf
#define ceo_erff_ ceb_erff
#endif

enum { CEO_EXACT = 0, CEO_GGML = 1, CEO_F16 = 2 };
enum {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13,
    T_Q6_K = 14, T_IQ4_NL = 20, T_IQ4_XS = 23, T_BF16 = 30
};

#define QK8_0 32
#define QK_K 256
#define Q8_0_BYTES 34
#define Q4_K_BYTES 144
#define Q8_K_BYTES 292 /* float d, int8 qs[256], int16 bsums[16] */

/* ---------------------------------------------------------------- fp16 --- */
/* IEEE binary16 <-> binary32, round-to-nearest-even (what F16C's
 * _cvtss_sh(x, 0) and numpy's astype(float16) do). */
float ceo_f16_to_f32(uint16_t h) {
#if defined(__F16C__)
    return _cvtsh_ss(h); /* the hardware conversion: exact, the same value as below */
#endif
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t man = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { e++; man <<= 1; } while ((man & 0x400) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t ceo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000;
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) return (uint16_t)(sign | 0x7C00 | (absx > 0x7F800000u ? 0x200 : 0));
    if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00); /* rounds to >= 65520 -> inf */
    if (absx < 0x38800000u) { /* result is subnormal or zero */
        if (absx < 0x33000000u) return (uint16_t)sign;     /* < 2^-25: rounds to 0 */
        uint32_t e = absx >> 23;
        uint32_t m = (absx & 0x7FFFFF) | 0x800000;
        uint32_t shift = 126 - e; /* 14..24 */
        uint32_t half = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half & 1))) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t e = (absx >> 23) - 127 + 15;
    uint32_t m = absx & 0x7FFFFF;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFF;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return (uint16_t)(sign | h);
}

static inline float round_f16(float x) { return ceo_f16_to_f32(ceo_f32_to_f16(x)); }

static inline uint16_t rd_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ------------------------------------------------------------- dequant --- */
/* ggml's published block formats.  IQ4_NL / IQ4_XS index ggml's non-linear
 * 16-value codebook (kvalues_iq4nl). */
static const int8_t IQ4NL_VALUES[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
int64_t ceo_row_bytes(int type, int64_t k);
/* Q4_K 6-bit scale/min unpacking: sub-block j < 4 keeps its 6 bits in bytes
 * j / j+4; j >= 4 splits 4 low bits in byte j+4 and 2 high bits in the top of
 * bytes j-4 / j (the published Q4_K block layout). */
static inline void q4k_scale_min(int j, const uint8_t *s, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

void ceo_dequant_row(int type, const uint8_t *src, int64_t k, float *dst) {
    if (type == T_F32) {
        memcpy(dst, src, (size_t)k * 4);
    } else if (type == T_F16) {
        for (int64_t i = 0; i < k; i++) dst[i] = ceo_f16_to_f32(rd_u16(src + 2 * i));
    } else if (type == T_Q8_0) {
        for (int64_t b = 0; b < k / QK8_0; b++) {
            const uint8_t *blk = src + b * Q8_0_BYTES;
            float d = ceo_f16_to_f32(rd_u16(blk));
            const int8_t *q = (const int8_t *)(blk + 2);
            for (int j = 0; j < QK8_0; j++) dst[b * QK8_0 + j] = (float)q[j] * d;
        }
    } else if (type == T_BF16) {
        for (int64_t i = 0; i < k; i++) {
            uint32_t u = (uint32_t)rd_u16(src + 2 * i) << 16;
            memcpy(dst + i, &u, 4);
        }
    } else if (type == T_Q4_0 || type == T_Q4_1 || type == T_Q5_0 || type == T_Q5_1 || type == T_IQ4_NL) {
        /* 32-value blocks: fp16 d (+ fp16 m for _1), (+ uint32 fifth bits for Q5), 16 nibble bytes
           (value j in the low nibble of byte j, value j+16 in its high nibble) */
        const int64_t bytes = ceo_row_bytes(type, 32);
        for (int64_t b = 0; b < k / 32; b++) {
            const uint8_t *blk = src + b * bytes;
            float d = ceo_f16_to_f32(rd_u16(blk)), m = 0.0f;
            const uint8_t *qs = blk + 2;
            uint32_t qh = 0;
            if (type == T_Q4_1 || type == T_Q5_1) { m = ceo_f16_to_f32(rd_u16(blk + 2)); qs += 2; }
            if (type == T_Q5_0 || type == T_Q5_1) { memcpy(&qh, qs, 4); qs += 4; }
            for (int j = 0; j < 32; j++) {
                int q = j < 16 ? (qs[j] & 0xF) : (qs[j - 16] >> 4);
                float v;
                if (type == T_Q4_0) v = d * (float)(q - 8);
                else if (type == T_Q4_1) v = d * (float)q + m;
                else if (type == T_Q5_0) v = d * (float)((q | (int)(((qh >> j) & 1) << 4)) - 16);
                else if (type == T_Q5_1) v = d * (float)(q | (int)(((qh >> j) & 1) << 4)) + m;
                else v = d * (float)IQ4NL_VALUES[q];
                dst[b * 32 + j] = v;
            }
        }
    } else if (type == T_IQ4_XS) {
        for (int64_t b = 0; b < k / QK_K; b++) {
            const uint8_t *blk = src + b * 136;
            float d = ceo_f16_to_f32(rd_u16(blk));
            uint16_t sh = rd_u16(blk + 2);
            for (int ib = 0; ib < 8; ib++) {
                int ls = ((blk[4 + ib / 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
                float dl = d * (float)(ls - 32);
                const uint8_t *qs = blk + 8 + 16 * ib;
                for (int j = 0; j < 16; j++) {
                    dst[b * QK_K + 32 * ib + j] = dl * (float)IQ4NL_VALUES[qs[j] & 0xF];
                    dst[b * QK_K + 32 * ib + j + 16] = dl * (float)IQ4NL_VALUES[qs[j] >> 4];
                }
            }
        }
    } else if (type == T_Q5_K) {
        for (int64_t b = 0; b < k / QK_K; b++) {
            const uint8_t *blk = src + b * 176;
            float d = ceo_f16_to_f32(rd_u16(blk)), dmin = ceo_f16_to_f32(rd_u16(blk + 2));
            const uint8_t *sc = blk + 4, *qh = blk + 16, *qs = blk + 48;
            for (int c = 0; c < 4; c++) {
                int s0, m0, s1, m1;
                q4k_scale_min(2 * c, sc, &s0, &m0);
                q4k_scale_min(2 * c + 1, sc, &s1, &m1);
                for (int l = 0; l < 32; l++) {
                    int lo = (qs[32 * c + l] & 0xF) | (((qh[l] >> (2 * c)) & 1) << 4);
                    int hi = (qs[32 * c + l] >> 4) | (((qh[l] >> (2 * c + 1)) & 1) << 4);
                    dst[b * QK_K + 64 * c + l] = d * (float)s0 * (float)lo - dmin * (float)m0;
                    dst[b * QK_K + 64 * c + 32 + l] = d * (float)s1 * (float)hi - dmin * (float)m1;
                }
            }
        }
    } else if (type == T_Q6_K) {
        for (int64_t b = 0; b < k / QK_K; b++) {
            const uint8_t *blk = src + b * 210;
            float d = ceo_f16_to_f32(rd_u16(blk + 208));
            for (int n = 0; n < 2; n++) {
                const uint8_t *ql = blk + 64 * n, *qh = blk + 128 + 32 * n;
                const int8_t *sc = (const int8_t *)(blk + 192 + 8 * n);
                float *y = dst + b * QK_K + 128 * n;
                for (int l = 0; l < 32; l++) {
                    int is = l / 16;
                    int q1 = (int)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
                    int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    y[l] = d * (float)sc[is] * (float)q1;
                    y[l + 32] = d * (float)sc[is + 2] * (float)q2;
                    y[l + 64] = d * (float)sc[is + 4] * (float)q3;
                    y[l + 96] = d * (float)sc[is + 6] * (float)q4;
                }
            }
        }
    } else if (type == T_Q4_K) {
        for (int64_t b = 0; b < k / QK_K; b++) {
            const uint8_t *blk = src + b * Q4_K_BYTES;
            float d = ceo_f16_to_f32(rd_u16(blk));
            float dmin = ceo_f16_to_f32(rd_u16(blk + 2));
            const uint8_t *sc = blk + 4, *qs = blk + 16;
            float *y = dst + b * QK_K;
            for (int c = 0; c < 4; c++) {
                int s0, m0, s1, m1;
                q4k_scale_min(2 * c, sc, &s0, &m0);
                q4k_scale_min(2 * c + 1, sc, &s1, &m1);
                float d1 = d * (float)s0, mm1 = dmin * (float)m0;
                float d2 = d * (float)s1, mm2 = dmin * (float)m1;
                for (int l = 0; l < 32; l++) y[64 * c + l] = d1 * (float)(qs[32 * c + l] & 0xF) - mm1;
                for (int l = 0; l < 32; l++) y[64 * c + 32 + l] = d2 * (float)(qs[32 * c + l] >> 4) - mm2;
            }
        }
    }
}

int64_t ceo_row_bytes(int type, int64_t k) {
    switch (type) {
        case T_F32: return k * 4;
        case T_F16: return k * 2;
        case T_BF16: return k * 2;
        case T_Q4_0: return k / 32 * 18;
        case T_Q4_1: return k / 32 * 20;
        case T_Q5_0: return k / 32 * 22;
        case T_Q5_1: return k / 32 * 24;
        case T_Q8_0: return k / QK8_0 * Q8_0_BYTES;
        case T_Q4_K: return k / QK_K * Q4_K_BYTES;
        case T_Q5_K: return k / QK_K * 176;
        case T_Q6_K: return k / QK_K * 210;
        case T_IQ4_NL: return k / 32 * 18;
        case T_IQ4_XS: return k / QK_K * 136;
    }
    return -1;
}

/* ----------------------------------------------- activation quantizers --- */
/* Q8_0 activation quantization as ggml's x86 AVX2 quantize_row_q8_0 does it:
 * d = amax/127 (stored fp16), multiplier 127/amax, round half to even. */
void ceo_quant_act_q8_0(const float *x, int64_t k, uint8_t *out) {
    for (int64_t b = 0; b < k / QK8_0; b++) {
        const float *xb = x + b * QK8_0;
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        uint16_t dh = ceo_f32_to_f16(d);
        float id = amax != 0.0f ? 127.0f / amax : 0.0f;
        uint8_t *blk = out + b * Q8_0_BYTES;
        blk[0] = (uint8_t)(dh & 0xFF);
        blk[1] = (uint8_t)(dh >> 8);
        int8_t *q = (int8_t *)(blk + 2);
        for (int j = 0; j < QK8_0; j++) q[j] = (int8_t)(int)nearbyintf(xb[j] * id);
    }
}

/* Q8_K (ggml quantize_row_q8_K_ref): per 256 values, scale from the signed
 * value of largest magnitude, iscale = -127/max, nearest-even rounding capped at
 * 127, d = 1/iscale, bsums over 16-value groups. */
void ceo_quant_act_q8_k(const float *x, int64_t k, uint8_t *out) {
    for (int64_t b = 0; b < k / QK_K; b++) {
        const float *xb = x + b * QK_K;
        uint8_t *blk = out + b * Q8_K_BYTES;
        float maxv = 0.0f, amax = 0.0f;
        for (int j = 0; j < QK_K; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) { amax = a; maxv = xb[j]; }
        }
        int8_t *q = (int8_t *)(blk + 4);
        int16_t bs[16];
        float d;
        if (amax == 0.0f) {
            d = 0.0f;
            memset(q, 0, QK_K);
            memset(bs, 0, sizeof bs);
        } else {
            float iscale = -127.0f / maxv;
            for (int j = 0; j < QK_K; j++) {
                int v = (int)nearbyintf(iscale * xb[j]);
                q[j] = (int8_t)(v > 127 ? 127 : v);
            }
            for (int g = 0; g < 16; g++) {
                int s = 0;
                for (int j = 0; j < 16; j++) s += q[16 * g + j];
                bs[g] = (int16_t)s;
            }
            d = 1.0f / iscale;
        }
        memcpy(blk, &d, 4);
        memcpy(blk + 4 + QK_K, bs, sizeof bs);
    }
}

/* ------------------------------------------------------------ dot products */
/* ggml x86 AVX2 ggml_vec_dot_q8_0_q8_0 (and llamafile tinyBLAS_Q0_AVX, which has
 * the same structure): eight float lanes, lane l holds the int sum of products
 * 4l..4l+3 of each block, scaled by d_w*d_a with an FMA per block; horizontal
 * sum ((a0+a4)+(a2+a6))+((a1+a5)+(a3+a7)). */
#if defined(__AVX2__) && defined(__FMA__)
/* The same lanes with AVX2 integer arithmetic, as ggml's x86 kernel forms them:
 * |w| times sign(w)*a byte pairs summed to int16 (no saturation: |q| <= 127), pairs of
 * those summed to the eight int32 lane sums, converted exactly to float and FMA'd
 * with the block's d.  Bit-identical to the scalar form below (same integer lanes,
 * same float operations in the same order); used where the host has AVX2. */
static float dot_q8_0_avx2(int64_t k, const uint8_t *w, const uint8_t *a) {
    __m256 acc = _mm256_setzero_ps();
    const __m256i ones = _mm256_set1_epi16(1);
    for (int64_t b = 0; b < k / QK8_0; b++) {
        const uint8_t *wb = w + b * Q8_0_BYTES, *ab = a + b * Q8_0_BYTES;
        const __m256 d = _mm256_set1_ps(ceo_f16_to_f32(rd_u16(wb)) * ceo_f16_to_f32(rd_u16(ab)));
        const __m256i qw = _mm256_loadu_si256((const __m256i *)(wb + 2));
        const __m256i qa = _mm256_loadu_si256((const __m256i *)(ab + 2));
        const __m256i pairs = _mm256_maddubs_epi16(_mm256_sign_epi8(qw, qw), _mm256_sign_epi8(qa, qw));
        const __m256i lanes = _mm256_madd_epi16(pairs, ones);
        acc = _mm256_fmadd_ps(d, _mm256_cvtepi32_ps(lanes), acc);
    }
    float l[8];
    _mm256_storeu_ps(l, acc);
    return ((l[0] + l[4]) + (l[2] + l[6])) + ((l[1] + l[5]) + (l[3] + l[7]));
}
#endif

float ceo_dot_q8_0_scalar(int64_t k, const uint8_t *w, const uint8_t *a);

#if defined(__AVX2__) && defined(__FMA__)
/* Four dots at once (weight rows w0, w1 x activation rows a0, a1), each with exactly the
 * lanes and float operations of dot_q8_0_avx2: the blocking only shares the loads and the
 * per-row block scales (wd, ad: the fp16 scales already widened, d = wd * ad as before). */
static void dot_q8_0_2x2_avx2(int64_t nb, const uint8_t *w0, const uint8_t *w1, const float *wd0, const float *wd1,
                              const uint8_t *a0, const uint8_t *a1, const float *ad0, const float *ad1,
                              float out[4]) {
    __m256 c00 = _mm256_setzero_ps(), c01 = _mm256_setzero_ps(), c10 = _mm256_setzero_ps(),
           c11 = _mm256_setzero_ps();
    const __m256i ones = _mm256_set1_epi16(1);
    for (int64_t b = 0; b < nb; b++) {
        const __m256i qw0 = _mm256_loadu_si256((const __m256i *)(w0 + b * Q8_0_BYTES + 2));
        const __m256i qw1 = _mm256_loadu_si256((const __m256i *)(w1 + b * Q8_0_BYTES + 2));
        const __m256i qa0 = _mm256_loadu_si256((const __m256i *)(a0 + b * Q8_0_BYTES + 2));
        const __m256i qa1 = _mm256_loadu_si256((const __m256i *)(a1 + b * Q8_0_BYTES + 2));
        const __m256i u0 = _mm256_sign_epi8(qw0, qw0), u1 = _mm256_sign_epi8(qw1, qw1);
        const __m256i l00 = _mm256_madd_epi16(_mm256_maddubs_epi16(u0, _mm256_sign_epi8(qa0, qw0)), ones);
        const __m256i l01 = _mm256_madd_epi16(_mm256_maddubs_epi16(u1, _mm256_sign_epi8(qa0, qw1)), ones);
        const __m256i l10 = _mm256_madd_epi16(_mm256_maddubs_epi16(u0, _mm256_sign_epi8(qa1, qw0)), ones);
        const __m256i l11 = _mm256_madd_epi16(_mm256_maddubs_epi16(u1, _mm256_sign_epi8(qa1, qw1)), ones);
        c00 = _mm256_fmadd_ps(_mm256_set1_ps(wd0[b] * ad0[b]), _mm256_cvtepi32_ps(l00), c00);
        c01 = _mm256_fmadd_ps(_mm256_set1_ps(wd1[b] * ad0[b]), _mm256_cvtepi32_ps(l01), c01);
        c10 = _mm256_fmadd_ps(_mm256_set1_ps(wd0[b] * ad1[b]), _mm256_cvtepi32_ps(l10), c10);
        c11 = _mm256_fmadd_ps(_mm256_set1_ps(wd1[b] * ad1[b]), _mm256_cvtepi32_ps(l11), c11);
    }
    const __m256 c[4] = {c00, c01, c10, c11};
    for (int i = 0; i < 4; i++) {
        float l[8];
        _mm256_storeu_ps(l, c[i]);
        out[i] = ((l[0] + l[4]) + (l[2] + l[6])) + ((l[1] + l[5]) + (l[3] + l[7]));
    }
}
#endif

float ceo_dot_q8_0(int64_t k, const uint8_t *w, const uint8_t *a) {
#if defined(__AVX2__) && defined(__FMA__)
    return dot_q8_0_avx2(k, w, a);
#else
    return ceo_dot_q8_0_scalar(k, w, a);
#endif
}

/* the lanes one product at a time (also the reference form the AVX2 one is tested against) */
float ceo_dot_q8_0_scalar(int64_t k, const uint8_t *w, const uint8_t *a) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t b = 0; b < k / QK8_0; b++) {
        const uint8_t *wb = w + b * Q8_0_BYTES, *ab = a + b * Q8_0_BYTES;
        float d = ceo_f16_to_f32(rd_u16(wb)) * ceo_f16_to_f32(rd_u16(ab));
        const int8_t *qw = (const int8_t *)(wb + 2), *qa = (const int8_t *)(ab + 2);
        for (int l = 0; l < 8; l++) {
            int s = qw[4 * l] * qa[4 * l] + qw[4 * l + 1] * qa[4 * l + 1] + qw[4 * l + 2] * qa[4 * l + 2] +
                    qw[4 * l + 3] * qa[4 * l + 3];
            acc[l] = fmaf(d, (float)s, acc[l]);
        }
    }
    return ((acc[0] + acc[4]) + (acc[2] + acc[6])) + ((acc[1] + acc[5]) + (acc[3] + acc[7]));
}

/* ggml generic ggml_vec_dot_q4_K_q8_K: per super-block, integer sub-block dots
 * scaled by the 6-bit scales into eight int lanes, d*lane accumulated into eight
 * float sums; the min term dmin*d_a*sum(m_j*bsum) subtracted once per block. */
#if defined(__AVX2__)
/* The eight int32 lanes of one Q4_K super-block with AVX2: per 32-value sub-block j,
 * int16 products of the 4-bit quants and the Q8_K values, folded so that element i
 * lands in lane i % 8 (the two 16-element halves, then the two 8-element halves),
 * widened and scaled by the sub-block's 6-bit scale.  Integer sums only: the lanes
 * equal the scalar loop's exactly (|products| <= 15 * 127, four per lane and
 * sub-block, no int16 overflow). */
static void q4k_lanes_avx2(const uint8_t *qs, const int8_t *q8, const int *scs, int32_t aux[8]) {
    __m256i acc = _mm256_setzero_si256();
    const __m128i m4 = _mm_set1_epi8(0x0F);
    for (int j = 0; j < 8; j++) {
        const uint8_t *src = qs + 32 * (j >> 1);
        __m128i b0 = _mm_loadu_si128((const __m128i *)src), b1 = _mm_loadu_si128((const __m128i *)(src + 16));
        if (j & 1) {
            b0 = _mm_srli_epi16(b0, 4);
            b1 = _mm_srli_epi16(b1, 4);
        }
        b0 = _mm_and_si128(b0, m4);
        b1 = _mm_and_si128(b1, m4);
        const __m256i a0 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(q8 + 32 * j)));
        const __m256i a1 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(q8 + 32 * j + 16)));
        const __m256i t = _mm256_add_epi16(_mm256_mullo_epi16(_mm256_cvtepu8_epi16(b0), a0),
                                           _mm256_mullo_epi16(_mm256_cvtepu8_epi16(b1), a1));
        const __m128i u = _mm_add_epi16(_mm256_castsi256_si128(t), _mm256_extracti128_si256(t, 1));
        acc = _mm256_add_epi32(acc, _mm256_mullo_epi32(_mm256_cvtepi16_epi32(u), _mm256_set1_epi32(scs[j])));
    }
    _mm256_storeu_si256((__m256i *)aux, acc);
}
#endif

static float dot_q4_k(int64_t k, const uint8_t *w, const uint8_t *a, int use_simd);

float ceo_dot_q4_k(int64_t k, const uint8_t *w, const uint8_t *a) { return dot_q4_k(k, w, a, 1); }
float ceo_dot_q4_k_scalar(int64_t k, const uint8_t *w, const uint8_t *a) { return dot_q4_k(k, w, a, 0); }

static float dot_q4_k(int64_t k, const uint8_t *w, const uint8_t *a, int use_simd) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float sumf = 0.0f;
    for (int64_t b = 0; b < k / QK_K; b++) {
        const uint8_t *wb = w + b * Q4_K_BYTES, *ab = a + b * Q8_K_BYTES;
        float ad;
        memcpy(&ad, ab, 4);
        const int8_t *q8 = (const int8_t *)(ab + 4);
        int16_t bs[16];
        memcpy(bs, ab + 4 + QK_K, sizeof bs);
        const uint8_t *sc = wb + 4, *qs = wb + 16;
        int scs[8], mns[8];
        for (int j = 0; j < 8; j++) q4k_scale_min(j, sc, &scs[j], &mns[j]);
        int sumi = 0;
        for (int j = 0; j < 16; j++) sumi += bs[j] * mns[j / 2];
        int32_t aux32[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#if defined(__AVX2__)
        if (use_simd) {
            q4k_lanes_avx2(qs, q8, scs, aux32);
        } else
#endif
        {
            (void)use_simd;
            int8_t q4[QK_K];
            for (int c = 0; c < 4; c++)
                for (int l = 0; l < 32; l++) {
                    q4[64 * c + l] = (int8_t)(qs[32 * c + l] & 0xF);
                    q4[64 * c + 32 + l] = (int8_t)(qs[32 * c + l] >> 4);
                }
            for (int j = 0; j < 8; j++) {
                for (int g = 0; g < 4; g++)
                    for (int l = 0; l < 8; l++) {
                        int idx = 32 * j + 8 * g + l;
                        aux32[l] += scs[j] * (int)(q8[idx] * q4[idx]);
                    }
            }
        }
        float d = ceo_f16_to_f32(rd_u16(wb)) * ad;
        for (int l = 0; l < 8; l++) sums[l] += d * (float)aux32[l];
        float dmin = ceo_f16_to_f32(rd_u16(wb + 2)) * ad;
        sumf -= dmin * (float)sumi;
    }
    for (int l = 0; l < 8; l++) sumf += sums[l];
    return sumf;
}

#if defined(__AVX2__)
/* Four Q4_K x Q8_K dots of one weight row against activation rows a[0..3]: per super-block
 * the weight's scales, mins and 4-bit values are unpacked once and reused; each dot keeps
 * exactly dot_q4_k's integer lanes and float operations in the same order. */
static void dot_q4_k_1x4_avx2(int64_t nsb, const uint8_t *w, const uint8_t *const a[4], float out[4]) {
    float sums[4][8] = {{0}}, sumf[4] = {0, 0, 0, 0};
    const __m128i m4 = _mm_set1_epi8(0x0F);
    for (int64_t b = 0; b < nsb; b++) {
        const uint8_t *wb = w + b * Q4_K_BYTES, *sc = wb + 4, *qs = wb + 16;
        int scs[8], mns[8];
        for (int j = 0; j < 8; j++) q4k_scale_min(j, sc, &scs[j], &mns[j]);
        __m256i acc[4] = {_mm256_setzero_si256(), _mm256_setzero_si256(), _mm256_setzero_si256(),
                          _mm256_setzero_si256()};
        for (int j = 0; j < 8; j++) {
            const uint8_t *src = qs + 32 * (j >> 1);
            __m128i b0 = _mm_loadu_si128((const __m128i *)src), b1 = _mm_loadu_si128((const __m128i *)(src + 16));
            if (j & 1) {
                b0 = _mm_srli_epi16(b0, 4);
                b1 = _mm_srli_epi16(b1, 4);
            }
            const __m256i w0 = _mm256_cvtepu8_epi16(_mm_and_si128(b0, m4));
            const __m256i w1 = _mm256_cvtepu8_epi16(_mm_and_si128(b1, m4));
            const __m256i scj = _mm256_set1_epi32(scs[j]);
            for (int r = 0; r < 4; r++) {
                const int8_t *q8 = (const int8_t *)(a[r] + b * Q8_K_BYTES + 4);
                const __m256i a0 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(q8 + 32 * j)));
                const __m256i a1 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(q8 + 32 * j + 16)));
                const __m256i t = _mm256_add_epi16(_mm256_mullo_epi16(w0, a0), _mm256_mullo_epi16(w1, a1));
                const __m128i u = _mm_add_epi16(_mm256_castsi256_si128(t), _mm256_extracti128_si256(t, 1));
                acc[r] = _mm256_add_epi32(acc[r], _mm256_mullo_epi32(_mm256_cvtepi16_epi32(u), scj));
            }
        }
        const float dw = ceo_f16_to_f32(rd_u16(wb)), dminw = ceo_f16_to_f32(rd_u16(wb + 2));
        for (int r = 0; r < 4; r++) {
            const uint8_t *ab = a[r] + b * Q8_K_BYTES;
            float ad;
            memcpy(&ad, ab, 4);
            int16_t bs[16];
            memcpy(bs, ab + 4 + QK_K, sizeof bs);
            int sumi = 0;
            for (int j = 0; j < 16; j++) sumi += bs[j] * mns[j / 2];
            int32_t aux32[8];
            _mm256_storeu_si256((__m256i *)aux32, acc[r]);
            const float d = dw * ad;
            for (int l = 0; l < 8; l++) sums[r][l] += d * (float)aux32[l];
            const float dmin = dminw * ad;
            sumf[r] -= dmin * (float)sumi;
        }
    }
    for (int r = 0; r < 4; r++) {
        for (int l = 0; l < 8; l++) sumf[r] += sums[r][l];
        out[r] = sumf[r];
    }
}
#endif

/* ---------------------------------------------------------- matrix product */
/* out[m, n] = sum_k W[n, k] * x[m, k] (+ bias[n]).  W is N rows of `type`. */
void ceo_matmul(int type, const uint8_t *w, int64_t n_out, int64_t k, const float *x, int64_t m_rows,
                const float *bias, float *out, int mode) {
    const int64_t rb = ceo_row_bytes(type, k);
    if (mode == CEO_GGML && (type == T_Q8_0 || type == T_Q4_K)) {
        const int64_t qb = type == T_Q8_0 ? k / QK8_0 * Q8_0_BYTES : k / QK_K * Q8_K_BYTES;
        uint8_t *xq = (uint8_t *)malloc((size_t)(qb * m_rows));
#pragma omp parallel for schedule(static)
        for (int64_t m = 0; m < m_rows; m++) {
            if (type == T_Q8_0) ceo_quant_act_q8_0(x + m * k, k, xq + m * qb);
            else ceo_quant_act_q8_k(x + m * k, k, xq + m * qb);
        }
        /* 32 x 32 tiles of (activation row, weight row): a tile's rows stay in the core's
         * cache while every dot of the tile is formed (each dot is computed on its own, so
         * the tiling changes no result) */
        const int64_t TM = 32, TN = 32, mt = (m_rows + TM - 1) / TM, nt = (n_out + TN - 1) / TN;
#if defined(__AVX2__) && defined(__FMA__)
        if (type == T_Q8_0) {
            /* Q8_0: dots two weight rows x two activation rows at a time (dot_q8_0_2x2_avx2,
             * the same value for every dot as ceo_dot_q8_0), block scales widened once */
            const int64_t nb = k / QK8_0;
            float *wd = (float *)malloc((size_t)(n_out * nb) * sizeof(float));
            float *ad = (float *)malloc((size_t)(m_rows * nb) * sizeof(float));
#pragma omp parallel for schedule(static)
            for (int64_t n = 0; n < n_out; n++)
                for (int64_t b = 0; b < nb; b++) wd[n * nb + b] = ceo_f16_to_f32(rd_u16(w + n * rb + b * Q8_0_BYTES));
#pragma omp parallel for schedule(static)
            for (int64_t m = 0; m < m_rows; m++)
                for (int64_t b = 0; b < nb; b++) ad[m * nb + b] = ceo_f16_to_f32(rd_u16(xq + m * qb + b * Q8_0_BYTES));
#pragma omp parallel for schedule(static) collapse(2)
            for (int64_t bm = 0; bm < mt; bm++)
                for (int64_t bn = 0; bn < nt; bn++) {
                    const int64_t m1 = m_rows < (bm + 1) * TM ? m_rows : (bm + 1) * TM;
                    const int64_t n1 = n_out < (bn + 1) * TN ? n_out : (bn + 1) * TN;
                    for (int64_t m = bm * TM; m < m1; m += 2)
                        for (int64_t n = bn * TN; n < n1; n += 2) {
                            if (m + 1 < m1 && n + 1 < n1) {
                                float r[4];
                                dot_q8_0_2x2_avx2(nb, w + n * rb, w + (n + 1) * rb, wd + n * nb, wd + (n + 1) * nb,
                                                  xq + m * qb, xq + (m + 1) * qb, ad + m * nb, ad + (m + 1) * nb, r);
                                out[m * n_out + n] = bias ? r[0] + bias[n] : r[0];
                                out[m * n_out + n + 1] = bias ? r[1] + bias[n + 1] : r[1];
                                out[(m + 1) * n_out + n] = bias ? r[2] + bias[n] : r[2];
                                out[(m + 1) * n_out + n + 1] = bias ? r[3] + bias[n + 1] : r[3];
                            } else {
                                for (int64_t mm = m; mm < m + 2 && mm < m1; mm++)
                                    for (int64_t nn = n; nn < n + 2 && nn < n1; nn++) {
                                        const float s = ceo_dot_q8_0(k, w + nn * rb, xq + mm * qb);
                                        out[mm * n_out + nn] = bias ? s + bias[nn] : s;
                                    }
                            }
                        }
                }
            free(wd);
            free(ad);
            free(xq);
            return;
        }
#endif
#if defined(__AVX2__)
        if (type == T_Q4_K) {
            /* Q4_K: one weight row against four activation rows per pass (dot_q4_k_1x4_avx2,
             * the same value for every dot as ceo_dot_q4_k) */
#pragma omp parallel for schedule(static) collapse(2)
            for (int64_t bm = 0; bm < mt; bm++)
                for (int64_t bn = 0; bn < nt; bn++) {
                    const int64_t m1 = m_rows < (bm + 1) * TM ? m_rows : (bm + 1) * TM;
                    const int64_t n1 = n_out < (bn + 1) * TN ? n_out : (bn + 1) * TN;
                    int64_t m = bm * TM;
                    for (; m + 4 <= m1; m += 4)
                        for (int64_t n = bn * TN; n < n1; n++) {
                            const uint8_t *a4[4] = {xq + m * qb, xq + (m + 1) * qb, xq + (m + 2) * qb,
                                                    xq + (m + 3) * qb};
                            float r[4];
                            dot_q4_k_1x4_avx2(k / QK_K, w + n * rb, a4, r);
                            for (int i = 0; i < 4; i++) out[(m + i) * n_out + n] = bias ? r[i] + bias[n] : r[i];
                        }
                    for (; m < m1; m++)
                        for (int64_t n = bn * TN; n < n1; n++) {
                            const float s = ceo_dot_q4_k(k, w + n * rb, xq + m * qb);
                            out[m * n_out + n] = bias ? s + bias[n] : s;
                        }
                }
            free(xq);
            return;
        }
#endif
#pragma omp parallel for schedule(static) collapse(2)
        for (int64_t bm = 0; bm < mt; bm++)
            for (int64_t bn = 0; bn < nt; bn++)
                for (int64_t m = bm * TM; m < m_rows && m < (bm + 1) * TM; m++)
                    for (int64_t n = bn * TN; n < n_out && n < (bn + 1) * TN; n++) {
                        float s = type == T_Q8_0 ? ceo_dot_q8_0(k, w + n * rb, xq + m * qb)
                                                 : ceo_dot_q4_k(k, w + n * rb, xq + m * qb);
                        out[m * n_out + n] = bias ? s + bias[n] : s;
                    }
        free(xq);
        return;
    }
    float *xa = NULL;
    if (mode == CEO_GGML && type != T_F32 && type != T_F16 && type != T_BF16) {
        /* other block formats: the activations are re-quantized to the format's ggml
         * vec_dot type (Q8_0-valued for the 32-value formats, Q8_K for the 256-value
         * ones) and dotted in float with the decoded weights.  The activation
         * rounding is ggml's; the accumulation order of its integer dots is not
         * reproduced (float rounding differences only). */
        const int kq = (type == T_Q5_K || type == T_Q6_K || type == T_IQ4_XS) ? 1 : 0;
        const int64_t qb = kq ? k / QK_K * Q8_K_BYTES : k / QK8_0 * Q8_0_BYTES;
        xa = (float *)malloc((size_t)(m_rows * k) * sizeof(float));
#pragma omp parallel for schedule(static)
        for (int64_t m = 0; m < m_rows; m++) {
            uint8_t *tmp = (uint8_t *)malloc((size_t)qb);
            float *xr = xa + m * k;
            if (kq) {
                ceo_quant_act_q8_k(x + m * k, k, tmp);
                for (int64_t b = 0; b < k / QK_K; b++) {
                    float d;
                    memcpy(&d, tmp + b * Q8_K_BYTES, 4);
                    const int8_t *q = (const int8_t *)(tmp + b * Q8_K_BYTES + 4);
                    for (int j = 0; j < QK_K; j++) xr[b * QK_K + j] = d * (float)q[j];
                }
            } else {
                ceo_quant_act_q8_0(x + m * k, k, tmp);
                ceo_dequant_row(T_Q8_0, tmp, k, xr);
            }
            free(tmp);
        }
        x = xa;
    }
    /* exact / f16 / (ggml with float weights): dequantize weights once */
    float *wf = (float *)malloc((size_t)(n_out * k) * sizeof(float));
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < n_out; n++) {
        ceo_dequant_row(type, w + n * rb, k, wf + n * k);
        if (mode == CEO_F16)
            for (int64_t i = 0; i < k; i++) wf[n * k + i] = round_f16(wf[n * k + i]);
    }
    float *xf = NULL;
    if (mode == CEO_F16) {
        xf = (float *)malloc((size_t)(m_rows * k) * sizeof(float));
        for (int64_t i = 0; i < m_rows * k; i++) xf[i] = round_f16(x[i]);
        x = xf;
    }
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t m = 0; m < m_rows; m++)
        for (int64_t n = 0; n < n_out; n++) {
            const float *xr = x + m * k, *wr = wf + n * k;
            float s;
            if (mode == CEO_GGML) { /* f32 weights: float accumulation */
                float acc = 0.0f;
                for (int64_t i = 0; i < k; i++) acc = fmaf(xr[i], wr[i], acc);
                s = acc;
            } else {
                double acc = 0.0;
                for (int64_t i = 0; i < k; i++) acc += (double)xr[i] * (double)wr[i];
                s = (float)acc;
            }
            out[m * n_out + n] = bias ? s + bias[n] : s;
        }
    free(xf);
    free(xa);
    free(wf);
}

/* the shared exp / erf, exported for their accuracy test */
float ceo_expf(float x) { return ceb_expf(x); }
float ceo_erff(float x) { return ceb_erff(x); }

/* ------------------------------------------------------------ elementwise */
/* exact erf GELU, as ggml_vec_gelu_erf_f32 computes it: 0.5x(1+erf(x/sqrt2)) */
void ceo_gelu_erf(float *x, int64_t n) {
    const float s2 = 0.70710678118654752440f;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) x[i] = 0.5f * x[i] * (1.0f + ceo_erff_(x[i] * s2));
}

/* ggml_norm_f32 then ggml_mul(gamma) and ggml_add(beta): mean and variance
 * accumulated in double, centred values kept in float, scale 1/sqrtf(var+eps). */
void ceo_layernorm(const float *x, int64_t rows, int64_t d, const float *gamma, const float *beta, float eps,
                   float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * d;
        float *y = out + r * d;
        double sum = 0.0;
        for (int64_t i = 0; i < d; i++) sum += (double)xr[i];
        float mean = (float)(sum / (double)d);
        double sum2 = 0.0;
        for (int64_t i = 0; i < d; i++) {
            float v = xr[i] - mean;
            y[i] = v;
            sum2 += (double)(v * v);
        }
        float variance = (float)(sum2 / (double)d);
        float scale = 1.0f / sqrtf(variance + eps);
        for (int64_t i = 0; i < d; i++) {
            float v = y[i] * scale;
            if (gamma) v = v * gamma[i];
            if (beta) v = v + beta[i];
            y[i] = v;
        }
    }
}

/* ------------------------------------------------------------- attention */
/* Per-sequence multi-head attention over packed rows, as ggml's CPU
 * flash_attn_ext runs it for f32 K/V: one pass over keys with an online
 * softmax (running max M, running sum S, V accumulator rescaled by expf(Mold-M)).
 * q/k/v rows have stride ld (elements); head h uses columns h*hd..h*hd+hd-1. */
/* q . k of one head.  The parity build sums in index order (one fmaf chain); the
 * timing build (CEO_LIBM_MATH) uses eight-lane AVX2 partial sums, as ggml's SIMD
 * vector dot does, so the CPU baseline pays ggml's cost, not a serial chain's. */
static inline float attn_dot(const float *a, const float *b, int n) {
#if defined(CEO_LIBM_MATH) && defined(__AVX2__) && defined(__FMA__)
    if (n % 8 == 0) {
        __m256 acc = _mm256_setzero_ps();
        for (int c = 0; c < n; c += 8) acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + c), _mm256_loadu_ps(b + c), acc);
        float l[8];
        _mm256_storeu_ps(l, acc);
        return ((l[0] + l[4]) + (l[2] + l[6])) + ((l[1] + l[5]) + (l[3] + l[7]));
    }
#endif
    float s = 0.0f;
    for (int c = 0; c < n; c++) s = fmaf(a[c], b[c], s);
    return s;
}

void ceo_attention(const float *q, const float *k, const float *v, int64_t ld, const int32_t *cu_seqlens,
                   int n_seqs, int n_head, int hd, float scale, float *out, int64_t ldo) {
    for (int s = 0; s < n_seqs; s++) {
        const int t0 = cu_seqlens[s], len = cu_seqlens[s + 1] - cu_seqlens[s];
#pragma omp parallel for schedule(static) collapse(2)
        for (int h = 0; h < n_head; h++)
            for (int i = 0; i < len; i++) {
                const float *qi = q + (int64_t)(t0 + i) * ld + h * hd;
                float acc[256];
                for (int c = 0; c < hd; c++) acc[c] = 0.0f;
                float M = -INFINITY, S = 0.0f;
                for (int j = 0; j < len; j++) {
                    const float *kj = k + (int64_t)(t0 + j) * ld + h * hd;
                    const float *vj = v + (int64_t)(t0 + j) * ld + h * hd;
                    const float sdot = attn_dot(qi, kj, hd);
                    float sc = sdot * scale;
                    float ms = 1.0f, vs = 1.0f;
                    if (sc > M) {
                        float Mold = M;
                        M = sc;
                        ms = ceo_expf_(Mold - M);
                        for (int c = 0; c < hd; c++) acc[c] *= ms;
                    } else {
                        vs = ceo_expf_(sc - M);
                    }
                    for (int c = 0; c < hd; c++) acc[c] = fmaf(vj[c], vs, acc[c]);
                    S = S * ms + vs;
                }
                float inv = S == 0.0f ? 0.0f : 1.0f / S;
                float *o = out + (int64_t)(t0 + i) * ldo + h * hd;
                for (int c = 0; c < hd; c++) o[c] = acc[c] * inv;
            }
    }
}

/* --------------------------------------------------------------- routing */
/* Router for one token block: logits = W_r x (ggml_mul_mat), probs = softmax
 * (max-subtracted expf, double sum, scaled by 1/sum), ids = indices of the k
 * largest probs in descending order (ties to the lower index), weights =
 * probs[ids] without renormalisation (src/crispembed.cpp:1333-1345). */
void ceo_route(const float *logits, int64_t T, int E, int k, int32_t *ids, float *wts, float *probs_out) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; t++) {
        const float *lg = logits + t * E;
        float mx = -INFINITY;
        for (int e = 0; e < E; e++) mx = lg[e] > mx ? lg[e] : mx;
        float p[256];
        double sum = 0.0;
        for (int e = 0; e < E; e++) {
            p[e] = ceo_expf_(lg[e] - mx);
            sum += (double)p[e];
        }
        float inv = (float)(1.0 / sum);
        for (int e = 0; e < E; e++) p[e] *= inv;
        if (probs_out)
            for (int e = 0; e < E; e++) probs_out[t * E + e] = p[e];
        unsigned char used[256];
        memset(used, 0, sizeof used);
        for (int j = 0; j < k; j++) {
            int best = -1;
            for (int e = 0; e < E; e++)
                if (!used[e] && (best < 0 || p[e] > p[best])) best = e;
            used[best] = 1;
            ids[t * k + j] = best;
            wts[t * k + j] = p[best];
        }
    }
}

/* ------------------------------------------------------------ MoE FFN --- */
/* The (token, slot) rows routed to expert e, in token order then slot order: the
 * grouping ggml_mul_mat_id builds for each expert (src/crispembed.cpp:1365,1371).
 * rows[i] = t*k + j; returns the count. */
static int64_t expert_rows(const int32_t *ids, int64_t T, int k, int e, int64_t *rows) {
    int64_t n = 0;
    for (int64_t t = 0; t < T; t++)
        for (int j = 0; j < k; j++)
            if (ids[t * k + j] == e) rows[n++] = t * k + j;
    return n;
}

/* The permutation of all experts' rows stacked in expert order: offsets[e] = first
 * permuted row of expert e (offsets[E] = T*k), slot_pos[t*k + j] = permuted row of
 * (token t, slot j). */
void ceo_moe_permutation(const int32_t *ids, int64_t T, int k, int E, int32_t *slot_pos, int32_t *offsets) {
    int64_t *rows = (int64_t *)malloc((size_t)(T * k + 1) * sizeof(int64_t));
    int64_t base = 0;
    for (int e = 0; e < E; e++) {
        offsets[e] = (int32_t)base;
        const int64_t n = expert_rows(ids, T, k, e, rows);
        for (int64_t i = 0; i < n; i++) slot_pos[rows[i]] = (int32_t)(base + i);
        base += n;
    }
    offsets[E] = (int32_t)base;
    free(rows);
}

/* The MoE branch of build_encoder_graph (src/crispembed.cpp:1327-1381):
 * router -> softmax -> top-k -> per-slot fc1 (ggml_mul_mat_id) -> erf-GELU
 * -> fc2 -> y[t] = sum_j w[t,j]*down[t,j] (+ bias).  Expert rows are
 * processed grouped by expert in token order, the grouping ggml_mul_mat_id
 * builds; within a token the combine runs j = 0..k-1.
 * fc1 is [E][F][d], fc2 is [E][d][F] (rows of `wtype`); router is [E][d].
 * If ids_in is non-NULL the routing is taken from it (and wts_in) instead of
 * being computed, so the expert math can be checked on a given routing. */
/* fc1 and fc2 may use different block formats (wtype2: fc2's; llama.cpp K-quant
 * mixes keep the down projection at a wider type) */
void ceo_moe_ffn2(const float *x, int64_t T, int d, int E, int k, int F, int router_type, const uint8_t *router,
                  int wtype, const uint8_t *fc1, int wtype2, const uint8_t *fc2, const float *bias, int mode,
                  const int32_t *ids_in, const float *wts_in, float *y, int32_t *ids_out, float *wts_out,
                  float *logits_out) {
    float *logits = (float *)malloc((size_t)(T * E) * sizeof(float));
    int rmode = mode == CEO_F16 ? CEO_GGML : mode; /* the device router reproduces the ggml router */
    ceo_matmul(router_type, router, E, d, x, T, NULL, logits, rmode);
    if (logits_out) memcpy(logits_out, logits, (size_t)(T * E) * sizeof(float));
    int32_t *ids = ids_out;
    float *wts = wts_out;
    if (ids_in) {
        memcpy(ids, ids_in, (size_t)(T * k) * sizeof(int32_t));
        memcpy(wts, wts_in, (size_t)(T * k) * sizeof(float));
    } else {
        ceo_route(logits, T, E, k, ids, wts, NULL);
    }
    free(logits);

    const int64_t rb1 = ceo_row_bytes(wtype, d), rb2 = ceo_row_bytes(wtype2, F);
    float *down = (float *)calloc((size_t)(T * k) * d, sizeof(float));
    /* gather rows per expert (stable in token order) */
    int64_t *rows = (int64_t *)malloc((size_t)(T * k) * sizeof(int64_t));
    for (int e = 0; e < E; e++) {
        int64_t n = expert_rows(ids, T, k, e, rows);
        if (!n) continue;
        float *xe = (float *)malloc((size_t)(n * d) * sizeof(float));
        float *he = (float *)malloc((size_t)(n * F) * sizeof(float));
        float *oe = (float *)malloc((size_t)(n * d) * sizeof(float));
        for (int64_t i = 0; i < n; i++) memcpy(xe + i * d, x + (rows[i] / k) * d, (size_t)d * sizeof(float));
        ceo_matmul(wtype, fc1 + (int64_t)e * F * rb1, F, d, xe, n, NULL, he, mode);
        ceo_gelu_erf(he, n * F);
        ceo_matmul(wtype2, fc2 + (int64_t)e * d * rb2, d, F, he, n, NULL, oe, mode);
        if (mode == CEO_F16) /* the device stores the expert outputs as fp16 */
            for (int64_t i = 0; i < n * d; i++) oe[i] = round_f16(oe[i]);
        for (int64_t i = 0; i < n; i++) memcpy(down + rows[i] * d, oe + i * d, (size_t)d * sizeof(float));
        free(xe);
        free(he);
        free(oe);
    }
    free(rows);
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; t++)
        for (int c = 0; c < d; c++) {
            float s = 0.0f;
            for (int j = 0; j < k; j++) s = fmaf(wts[t * k + j], down[(t * k + j) * d + c], s);
            y[t * d + c] = bias ? s + bias[c] : s;
        }
    free(down);
}

/* --------------------------------------------------------------- pooling */
/* Mean pool + L2 normalise per sequence (src/crispembed.cpp:1822-1846):
 * sequential float accumulation t-outer / h-inner, divide by the count, then
 * p /= sqrtf(max(sum p^2, 1e-12)). */
void ceo_moe_ffn(const float *x, int64_t T, int d, int E, int k, int F, int router_type, const uint8_t *router,
                 int wtype, const uint8_t *fc1, const uint8_t *fc2, const float *bias, int mode,
                 const int32_t *ids_in, const float *wts_in, float *y, int32_t *ids_out, float *wts_out,
                 float *logits_out) {
    ceo_moe_ffn2(x, T, d, E, k, F, router_type, router, wtype, fc1, wtype, fc2, bias, mode, ids_in, wts_in, y,
                 ids_out, wts_out, logits_out);
}

void ceo_pool_l2(const float *hidden, const int32_t *cu_seqlens, int n_seqs, int d, float *out) {
    for (int s = 0; s < n_seqs; s++) {
        float *p = out + (int64_t)s * d;
        for (int h = 0; h < d; h++) p[h] = 0.0f;
        int n = cu_seqlens[s + 1] - cu_seqlens[s];
        if (n > 0) {
            for (int t = cu_seqlens[s]; t < cu_seqlens[s + 1]; t++)
                for (int h = 0; h < d; h++) p[h] += hidden[(int64_t)t * d + h];
            for (int h = 0; h < d; h++) p[h] /= (float)n;
        }
        float norm = 0.0f;
        for (int h = 0; h < d; h++) norm += p[h] * p[h];
        norm = sqrtf(norm > 1e-12f ? norm : 1e-12f);
        for (int h = 0; h < d; h++) p[h] /= norm;
    }
}

/* Matryoshka truncation (src/crispembed.cpp:2786-2793): keep `dim` values and
 * renormalise with the same epsilon rule. */
void ceo_truncate_renorm(const float *in, int n, int d, int dim, float *out) {
    for (int s = 0; s < n; s++) {
        float norm = 0.0f;
        for (int i = 0; i < dim; i++) norm += in[(int64_t)s * d + i] * in[(int64_t)s * d + i];
        norm = sqrtf(norm > 1e-12f ? norm : 1e-12f);
        for (int i = 0; i < dim; i++) out[(int64_t)s * dim + i] = in[(int64_t)s * d + i] / norm;
    }
}

int ceo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}
