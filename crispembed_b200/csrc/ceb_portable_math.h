/*
 * ceb_portable_math.h -- exp and erf for float arguments that give the same bits
 * on the host (C99) and on the device (CUDA).
 *
 * The reference's graph evaluates expf (softmax, flash attention) and erff (the
 * erf-GELU) through the C library.  Library implementations differ from each
 * other by an ulp here and there, and with activations re-quantized to Q8_0 an
 * ulp upstream can change which expert a token is sent to, so a bit-for-bit
 * comparison of two arithmetics needs one shared definition.  These functions
 * compute in double precision and round once to float, which gives the
 * correctly rounded result except within ~1e-16 of a rounding midpoint:
 *
 *  - exp: Cody & Waite argument reduction x = k ln2 + r, |r| <= ln2/2, with ln2
 *    split into a double and its remainder; e^r by its Taylor series to r^13
 *    (remainder below 4e-18); scaling by 2^k built exactly.
 *  - erf: |x| < 2 by the Maclaurin series 2/sqrt(pi) sum (-1)^n x^(2n+1) /
 *    (n! (2n+1)) (Abramowitz & Stegun 7.1.5), 48 terms; |x| >= 2 as
 *    1 - erfc(x) with erfc from the Laplace continued fraction
 *    erfc(x) = e^(-x^2)/sqrt(pi) / (x + (1/2)/(x + 1/(x + (3/2)/(x + ...))))
 *    (A&S 7.1.14), evaluated backwards from depth 60.
 *
 * Constants are hexadecimal literals (exact).  Only correctly rounded IEEE
 * operations are used (+, -, *, /, fma, rint), in a fixed order with explicit
 * fma calls: compile the host side with -ffp-contract=off and the device side
 * with -fmad=false so nothing else is fused.
 */
#ifndef CEB_PORTABLE_MATH_H
#define CEB_PORTABLE_MATH_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define CEB_PM_FN static __host__ __device__ __forceinline__
#else
#define CEB_PM_FN static inline
#endif

/* 2^k as a double for -1022 <= k <= 1023 (exact) */
CEB_PM_FN double ceb_pm_pow2(int k) {
    const uint64_t bits = (uint64_t)(k + 1023) << 52;
    double r;
#if defined(__CUDA_ARCH__)
    r = __longlong_as_double((long long)bits);
#else
    memcpy(&r, &bits, sizeof r);
#endif
    return r;
}

CEB_PM_FN double ceb_exp_d(double x) {
    if (x != x) return x;
    if (x > 89.0) return INFINITY; /* above float's overflow threshold */
    if (x < -104.0) return 0.0;    /* below half of float's smallest subnormal */
    const double k = rint(x * 0x1.71547652b82fep+0);        /* x / ln2 */
    double r = fma(-k, 0x1.62e42fefa39efp-1, x);            /* ln2, leading double */
    r = fma(-k, 0x1.abc9e3b39803fp-56, r);                  /* ln2 - leading double */
    double p = 0x1.6124613a86d09p-33;                       /* 1/13! */
    p = fma(p, r, 0x1.1eed8eff8d898p-29); /* 1/12! */
    p = fma(p, r, 0x1.ae64567f544e4p-26); /* 1/11! */
    p = fma(p, r, 0x1.27e4fb7789f5cp-22); /* 1/10! */
    p = fma(p, r, 0x1.71de3a556c734p-19); /* 1/9! */
    p = fma(p, r, 0x1.a01a01a01a01ap-16); /* 1/8! */
    p = fma(p, r, 0x1.a01a01a01a01ap-13); /* 1/7! */
    p = fma(p, r, 0x1.6c16c16c16c17p-10); /* 1/6! */
    p = fma(p, r, 0x1.1111111111111p-7);  /* 1/5! */
    p = fma(p, r, 0x1.5555555555555p-5);  /* 1/4! */
    p = fma(p, r, 0x1.5555555555555p-3);  /* 1/3! */
    p = fma(p, r, 0.5);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    return p * ceb_pm_pow2((int)k);
}

CEB_PM_FN double ceb_erf_d(double x) {
    const double a = fabs(x);
    double r;
    if (a < 2.0) {
        const double x2 = a * a;
        double term = a, s = a;
        for (int n = 1; n < 48; ++n) {
            term = term * (-x2) / (double)n;
            s = s + term / (double)(2 * n + 1);
        }
        r = s * 0x1.20dd750429b6dp+0; /* 2/sqrt(pi) */
    } else {
        double f = a;
        for (int n = 60; n >= 1; --n) f = a + ((double)n * 0.5) / f;
        r = 1.0 - ceb_exp_d(-(a * a)) * 0x1.20dd750429b6dp-1 / f; /* 1/sqrt(pi) */
    }
    return x < 0 ? -r : r;
}

/* float exp / erf through the double routines, rounded once to nearest */
CEB_PM_FN float ceb_expf(float x) { return (float)ceb_exp_d((double)x); }
CEB_PM_FN float ceb_erff(float x) { return (float)ceb_erf_d((double)x); }

#endif /* CEB_PORTABLE_MATH_H */
