/*
 * cubf_oracle.c -- CPU restatement of cuButterfly's reference algorithms.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels of cubutterfly_b200; it is never linked into the product library and
 * the product path never calls it.  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg load it.
 *
 * Parity is pinned: tests/test_oracle.py checks every function here against
 * (a) the known answers in the reference's own tests and (b) the reference's
 * own CPU oracles (src/butterfly_reference.cpp, src/reference.cpp), compiled
 * unchanged from the reference tree into oracle/_ref by oracle/Makefile, on
 * seeded inputs (fixtures in tests/golden/, made by tests/golden/make_golden.py).
 *
 * Each function names the reference lines it restates.  Arithmetic order is
 * kept identical to the reference so that results are bit-identical when both
 * are compiled with -ffp-contract=off.
 */
#include <math.h>
#include <stdlib.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

typedef unsigned __int128 u128;

#define ORACLE_API __attribute__((visibility("default")))

static int is_pow2(size_t n) { return n != 0 && (n & (n - 1)) == 0; }

static unsigned log2_exact(size_t n) {
    unsigned l = 0;
    while (((size_t)1 << l) < n) ++l;
    return l;
}

static size_t reverse_bits(size_t index, unsigned bits) {
    size_t r = 0;
    for (unsigned j = 0; j < bits; ++j, index >>= 1) r = (r << 1) | (index & 1u);
    return r;
}

/* In-place bit-reversal permutation of n elements of `width` bytes, visiting
 * indices in the same order as butterfly_reference.cpp:396-407. */
static void bitrev_permute(void* data, size_t n, size_t width) {
    unsigned char* p = (unsigned char*)data;
    unsigned char tmp[16];
    size_t reversed = 0;
    for (size_t index = 1; index < n; ++index) {
        size_t bit = n >> 1;
        while ((reversed & bit) != 0) {
            reversed ^= bit;
            bit >>= 1;
        }
        reversed ^= bit;
        if (index < reversed) {
            memcpy(tmp, p + index * width, width);
            memcpy(p + index * width, p + reversed * width, width);
            memcpy(p + reversed * width, tmp, width);
        }
    }
}

/* ---------------------------------------------------------------- FFT ---- */

/* Radix-2 DIT FFT over interleaved complex fp32, twiddles evaluated in double
 * per butterfly and the product rounded to float, exactly as
 * cuntt::reference_fft(std::vector<Complex32>&) in
 * src/butterfly_reference.cpp:392-433.  `data` holds `batch` transforms of n
 * complex values each (2n floats per transform). */
ORACLE_API int cubf_oracle_fft_c32(float* data, size_t n, size_t batch, int inverse, int normalize) {
    if (!is_pow2(n)) return 1;
    const double kPi = 3.141592653589793238462643383279502884;
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t b = 0; b < batch; ++b) {
        float* v = data + 2 * n * b;
        bitrev_permute(v, n, 2 * sizeof(float));
        for (size_t half = 1; half < n; half <<= 1) {
            for (size_t base = 0; base < n; base += 2 * half) {
                for (size_t offset = 0; offset < half; ++offset) {
                    const double direction = inverse ? 1.0 : -1.0;
                    const double angle = direction * kPi * (double)offset / (double)half;
                    const double wr = cos(angle);
                    const double wi = sin(angle);
                    float* a = v + 2 * (base + offset);
                    float* c = v + 2 * (base + half + offset);
                    const float ar = a[0], ai = a[1];
                    const float br = c[0], bi = c[1];
                    const float vr = (float)(br * wr - bi * wi);
                    const float vi = (float)(br * wi + bi * wr);
                    a[0] = ar + vr;
                    a[1] = ai + vi;
                    c[0] = ar - vr;
                    c[1] = ai - vi;
                }
            }
        }
        if (inverse && normalize) {
            const float scale = 1.0f / (float)n;
            for (size_t i = 0; i < 2 * n; ++i) v[i] *= scale;
        }
    }
    return 0;
}

/* Double-precision variant: cuntt::reference_fft(std::vector<Complex64>&),
 * src/butterfly_reference.cpp:435-473.  Used as the truth for large-N checks. */
ORACLE_API int cubf_oracle_fft_c64(double* data, size_t n, size_t batch, int inverse, int normalize) {
    if (!is_pow2(n)) return 1;
    const double kPi = 3.141592653589793238462643383279502884;
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t b = 0; b < batch; ++b) {
        double* v = data + 2 * n * b;
        bitrev_permute(v, n, 2 * sizeof(double));
        for (size_t half = 1; half < n; half <<= 1) {
            for (size_t base = 0; base < n; base += 2 * half) {
                for (size_t offset = 0; offset < half; ++offset) {
                    const double angle = (inverse ? 1.0 : -1.0) * kPi * (double)offset / (double)half;
                    const double wr = cos(angle);
                    const double wi = sin(angle);
                    double* a = v + 2 * (base + offset);
                    double* c = v + 2 * (base + half + offset);
                    const double ar = a[0], ai = a[1];
                    const double br = c[0], bi = c[1];
                    const double vr = br * wr - bi * wi;
                    const double vi = br * wi + bi * wr;
                    a[0] = ar + vr;
                    a[1] = ai + vi;
                    c[0] = ar - vr;
                    c[1] = ai - vi;
                }
            }
        }
        if (inverse && normalize) {
            const double scale = 1.0 / (double)n;
            for (size_t i = 0; i < 2 * n; ++i) v[i] *= scale;
        }
    }
    return 0;
}

/* Selected bins of the DFT of one complex fp32 vector, in long double:
 * X[k] = sum_j x[j] W^(j k), W = exp(-+2 pi i / n), the definition every FFT
 * here is held to (the reference's reference_fft, src/butterfly_reference.cpp:
 * 392-433, computes the same sums by radix-2 stages).  j k is reduced mod n
 * exactly (incrementally: m += k mod n per term), and W^m is formed from a
 * two-level table of long-double unit roots, W^m = W^(hi 2^s) W^lo with
 * m = hi 2^s + lo, so a bin of a 2^30-point vector costs table loads and one
 * long-double complex product per term (relative error ~1e-19 per term).  Each
 * bin is summed in fixed chunks on all threads, then the chunk sums in order. */
ORACLE_API void cubf_oracle_dft_bins(const float* data, size_t n, const size_t* bins, size_t count,
                                     int inverse, double* out) {
    const long double kPi = 3.141592653589793238462643383279502884L;
    unsigned s = 0;
    while (((size_t)1 << (2 * s)) < n) ++s; /* 2^s >= sqrt(n) */
    const size_t lo_n = (size_t)1 << s, hi_n = (n + lo_n - 1) / lo_n;
    long double* lo = (long double*)malloc(2 * lo_n * sizeof(long double));
    long double* hi = (long double*)malloc(2 * hi_n * sizeof(long double));
    enum { kChunks = 256 };
    long double* part = (long double*)malloc(2 * kChunks * (count ? count : 1) * sizeof(long double));
    if (!lo || !hi || !part) {
        free(lo);
        free(hi);
        free(part);
        for (size_t i = 0; i < 2 * count; ++i) out[i] = NAN;
        return;
    }
    const long double sign = inverse ? 2.0L : -2.0L;
    for (size_t m = 0; m < lo_n; ++m) {
        const long double a = sign * kPi * (long double)(m % n) / (long double)n;
        lo[2 * m] = cosl(a);
        lo[2 * m + 1] = sinl(a);
    }
    for (size_t h = 0; h < hi_n; ++h) {
        const long double a = sign * kPi * (long double)((h * lo_n) % n) / (long double)n;
        hi[2 * h] = cosl(a);
        hi[2 * h + 1] = sinl(a);
    }
    const size_t chunk = (n + kChunks - 1) / kChunks;
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t t = 0; t < count * kChunks; ++t) {
        const size_t i = t / kChunks, c = t % kChunks;
        const size_t k = bins[i] % n;
        const size_t j0 = c * chunk, j1 = j0 + chunk < n ? j0 + chunk : n;
        size_t m = (size_t)(((u128)j0 * k) % n);
        long double sr = 0, si = 0;
        for (size_t j = j0; j < j1; ++j) {
            const long double* a = hi + 2 * (m >> s);
            const long double* b = lo + 2 * (m & (lo_n - 1));
            const long double c_ = a[0] * b[0] - a[1] * b[1], s_ = a[0] * b[1] + a[1] * b[0];
            const long double xr = data[2 * j], xi = data[2 * j + 1];
            sr += xr * c_ - xi * s_;
            si += xr * s_ + xi * c_;
            m += k;
            if (m >= n) m -= n;
        }
        part[2 * t] = sr;
        part[2 * t + 1] = si;
    }
    for (size_t i = 0; i < count; ++i) {
        long double sr = 0, si = 0;
        for (size_t c = 0; c < kChunks; ++c) {
            sr += part[2 * (i * kChunks + c)];
            si += part[2 * (i * kChunks + c) + 1];
        }
        out[2 * i] = (double)sr;
        out[2 * i + 1] = (double)si;
    }
    free(lo);
    free(hi);
    free(part);
}

/* Direct DFT of any length in long double, rows of n complex doubles:
 * X[k] = sum_j x[j] exp(-+2 pi i j k / n) (1/n on a normalised inverse), the
 * definition the reference's arbitrary-length FFT plans (src/bluestein_fft.cu)
 * are held to by tests/test_c_api.c:49-108.  j k is reduced mod n exactly
 * before the angle is formed; one table of n unit roots serves every term. */
ORACLE_API int cubf_oracle_dft_c128(const double* in, double* out, size_t n, size_t batch, int inverse,
                                    int normalize) {
    if (n == 0) return 1;
    const long double kPi = 3.141592653589793238462643383279502884L;
    long double* tw = (long double*)malloc(2 * n * sizeof(long double));
    if (!tw) return 1;
    for (size_t m = 0; m < n; ++m) {
        const long double ang = (inverse ? 2.0L : -2.0L) * kPi * (long double)m / (long double)n;
        tw[2 * m] = cosl(ang);
        tw[2 * m + 1] = sinl(ang);
    }
    const long double scale = (inverse && normalize) ? 1.0L / (long double)n : 1.0L;
    for (size_t b = 0; b < batch; ++b) {
        const double* x = in + 2 * b * n;
        double* y = out + 2 * b * n;
        for (size_t k = 0; k < n; ++k) {
            long double sr = 0, si = 0;
            size_t m = 0; /* j k mod n */
            for (size_t j = 0; j < n; ++j) {
                const long double c = tw[2 * m], s = tw[2 * m + 1];
                sr += x[2 * j] * c - x[2 * j + 1] * s;
                si += x[2 * j] * s + x[2 * j + 1] * c;
                m += k;
                if (m >= n) m -= n;
            }
            y[2 * k] = (double)(sr * scale);
            y[2 * k + 1] = (double)(si * scale);
        }
    }
    free(tw);
    return 0;
}

/* --------------------------------------------------------------- FWHT ---- */

/* cuntt::reference_fwht(std::vector<double>&), src/butterfly_reference.cpp:371-390. */
static void fwht_f64_one(double* v, size_t n, int inverse, int normalize) {
    for (size_t half = 1; half < n; half <<= 1) {
        for (size_t base = 0; base < n; base += 2 * half) {
            for (size_t offset = 0; offset < half; ++offset) {
                const double left = v[base + offset];
                const double right = v[base + half + offset];
                v[base + offset] = left + right;
                v[base + half + offset] = left - right;
            }
        }
    }
    if (inverse && normalize) {
        const double scale = 1.0 / (double)n;
        for (size_t i = 0; i < n; ++i) v[i] *= scale;
    }
}

ORACLE_API int cubf_oracle_fwht_f64(double* data, size_t n, size_t batch, int inverse, int normalize) {
    if (!is_pow2(n)) return 1;
#pragma omp parallel for schedule(static)
    for (size_t b = 0; b < batch; ++b) fwht_f64_one(data + n * b, n, inverse, normalize);
    return 0;
}

/* cuntt::reference_fwht(std::vector<float>&), src/butterfly_reference.cpp:349-369. */
ORACLE_API int cubf_oracle_fwht_f32(float* data, size_t n, size_t batch, int inverse, int normalize) {
    if (!is_pow2(n)) return 1;
#pragma omp parallel for schedule(static)
    for (size_t b = 0; b < batch; ++b) {
        float* v = data + n * b;
        for (size_t half = 1; half < n; half <<= 1)
            for (size_t base = 0; base < n; base += 2 * half)
                for (size_t offset = 0; offset < half; ++offset) {
                    const float left = v[base + offset];
                    const float right = v[base + half + offset];
                    v[base + offset] = left + right;
                    v[base + half + offset] = left - right;
                }
        if (inverse && normalize) {
            const float scale = 1.0f / (float)n;
            for (size_t i = 0; i < n; ++i) v[i] *= scale;
        }
    }
    return 0;
}

static double bf16_to_double(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return (double)f;
}

/* Round a double to bfloat16, nearest-even (one rounding, no double rounding
 * through float: the tie test is made on the exact double value). */
static uint16_t double_to_bf16(double x) {
    if (isnan(x)) return 0x7fc0;
    float f = (float)x; /* exact when |x| has <= 24 significant bits */
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((double)f != x && isfinite(f)) {
        /* Resolve directly from the double: truncate to bf16 then compare. */
        uint32_t trunc = u & 0xffff0000u;
        float lo_f, hi_f;
        memcpy(&lo_f, &trunc, 4);
        uint32_t next = trunc + 0x10000u;
        memcpy(&hi_f, &next, 4);
        /* lo_f and hi_f bracket x in magnitude order of the sign */
        double dlo = fabs(x - (double)lo_f), dhi = fabs(x - (double)hi_f);
        if (dlo < dhi) return (uint16_t)(trunc >> 16);
        if (dhi < dlo) return (uint16_t)(next >> 16);
        return (uint16_t)(((trunc >> 16) & 1u) ? (next >> 16) : (trunc >> 16));
    }
    /* f == x exactly (or overflow to inf): round the float's bits. */
    uint32_t lsb = (u >> 16) & 1u;
    uint32_t rounded = u + 0x7fffu + lsb;
    return (uint16_t)(rounded >> 16);
}

/* FWHT with bf16 storage, wide compute and one final rounding:
 * widen -> reference_fwht<double> -> x output_scale -> round to bf16.
 * This is the final-storage contract of the reference's FP16 path
 * (src/butterfly.cu:1451-1470, :1882-1897; tests/test_fwht_final_storage.py:25-38)
 * applied to bf16 storage. */
ORACLE_API int cubf_oracle_fwht_bf16_final(const uint16_t* in, uint16_t* out, size_t n, size_t batch,
                                           int inverse, int normalize, double scale) {
    if (!is_pow2(n)) return 1;
    int failed = 0;
#pragma omp parallel reduction(| : failed)
    {
        double* v = (double*)malloc(n * sizeof(double));
        if (!v) failed = 1;
#pragma omp for schedule(static)
        for (size_t b = 0; b < batch; ++b) {
            if (!v) continue;
            for (size_t i = 0; i < n; ++i) v[i] = bf16_to_double(in[n * b + i]);
            fwht_f64_one(v, n, inverse, normalize);
            for (size_t i = 0; i < n; ++i) out[n * b + i] = double_to_bf16(v[i] * scale);
        }
        free(v);
    }
    return failed;
}

/* --------------------------------------------------------------- zeta ---- */

/* cuntt::reference_subset_zeta(std::vector<uint32_t>&), butterfly_reference.cpp:475-490,
 * and reference_superset_zeta :492-507.  Wrap-around mod 2^32. */
ORACLE_API int cubf_oracle_zeta_u32(uint32_t* data, size_t n, size_t batch, int superset, int inverse) {
    if (!is_pow2(n)) return 1;
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t b = 0; b < batch; ++b) {
        uint32_t* v = data + n * b;
        for (size_t half = 1; half < n; half <<= 1)
            for (size_t base = 0; base < n; base += 2 * half)
                for (size_t offset = 0; offset < half; ++offset) {
                    uint32_t* target = &v[base + offset + (superset ? 0 : half)];
                    const uint32_t source = v[base + offset + (superset ? half : 0)];
                    *target = inverse ? *target - source : *target + source;
                }
    }
    return 0;
}

/* cuntt::reference_structured_2x2 (butterfly_reference.cpp:541-591): stage s
 * (s = 0 .. log n - 1, in that order) maps each pair (left, right) at index
 * bit s clear / set to (m00 left + m01 right, m10 left + m11 right) with the
 * stage's matrix (one shared matrix, or one per stage) cast to the storage
 * precision; the inverse uses each matrix's inverse computed in double.
 * mats: 4 doubles (m00, m01, m10, m11) per matrix.  Products and sums are
 * rounded separately (the oracle is compiled with -ffp-contract=off). */
static int structured_mats(const double* mats, size_t count, unsigned log_n, int inverse, double* out) {
    if (count != 1 && count != log_n) return 1;
    for (unsigned s = 0; s < log_n; ++s) {
        const double* m = mats + 4 * (count == 1 ? 0 : s);
        double m00 = m[0], m01 = m[1], m10 = m[2], m11 = m[3];
        if (!isfinite(m00) || !isfinite(m01) || !isfinite(m10) || !isfinite(m11)) return 1;
        if (inverse) {
            const double det = m00 * m11 - m01 * m10;
            if (!isfinite(det) || det == 0.0) return 1;
            const double a = m[3] / det, b = -m[1] / det, c = -m[2] / det, d = m[0] / det;
            m00 = a; m01 = b; m10 = c; m11 = d;
        }
        out[4 * s] = m00; out[4 * s + 1] = m01; out[4 * s + 2] = m10; out[4 * s + 3] = m11;
    }
    return 0;
}

ORACLE_API int cubf_oracle_structured_f32(float* data, size_t n, size_t batch, const double* mats, size_t count,
                                          int inverse) {
    if (!is_pow2(n)) return 1;
    const unsigned log_n = log2_exact(n);
    double m[4 * 64];
    if (log_n > 64 || structured_mats(mats, count, log_n, inverse, m)) return 1;
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t b = 0; b < batch; ++b) {
        float* v = data + b * n;
        for (unsigned s = 0; s < log_n; ++s) {
            const float m00 = (float)m[4 * s], m01 = (float)m[4 * s + 1], m10 = (float)m[4 * s + 2],
                        m11 = (float)m[4 * s + 3];
            const size_t half = (size_t)1 << s;
            for (size_t base = 0; base < n; base += 2 * half)
                for (size_t o = 0; o < half; ++o) {
                    const float l = v[base + o], r = v[base + half + o];
                    v[base + o] = m00 * l + m01 * r;
                    v[base + half + o] = m10 * l + m11 * r;
                }
        }
    }
    return 0;
}

ORACLE_API int cubf_oracle_structured_f64(double* data, size_t n, size_t batch, const double* mats, size_t count,
                                          int inverse) {
    if (!is_pow2(n)) return 1;
    const unsigned log_n = log2_exact(n);
    double m[4 * 64];
    if (log_n > 64 || structured_mats(mats, count, log_n, inverse, m)) return 1;
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t b = 0; b < batch; ++b) {
        double* v = data + b * n;
        for (unsigned s = 0; s < log_n; ++s) {
            const size_t half = (size_t)1 << s;
            for (size_t base = 0; base < n; base += 2 * half)
                for (size_t o = 0; o < half; ++o) {
                    const double l = v[base + o], r = v[base + half + o];
                    v[base + o] = m[4 * s] * l + m[4 * s + 1] * r;
                    v[base + half + o] = m[4 * s + 2] * l + m[4 * s + 3] * r;
                }
        }
    }
    return 0;
}

/* FWHT with native bf16 / fp16 stage storage: the semantics of the reference's
 * LowFwhtOperator<Storage, Native = true> (src/operator_traits.cuh:114-154)
 * applied in stage order 0 .. log n - 1: every add / sub / halving is the
 * correctly rounded storage-precision result (computed exactly in double,
 * then rounded to nearest even, subnormals included); a normalised inverse
 * halves after the butterfly when both operands' magnitude bits are within
 * 0x7e7f (bf16) / 0x73ff (fp16), before it otherwise.  The reference has no
 * CPU function for this path, so this restatement is checked against the
 * FP32 final-storage oracle within the bf16 / fp16 tolerance. */
static double low_decode(uint16_t b, int bf16) {
    if (bf16) {
        const uint32_t u = (uint32_t)b << 16;
        float f;
        memcpy(&f, &u, 4);
        return (double)f;
    }
    const int sign = b >> 15, exp = (b >> 10) & 31, mant = b & 1023;
    double v;
    if (exp == 0) v = ldexp((double)mant, -24);
    else if (exp == 31) v = mant ? NAN : INFINITY;
    else v = ldexp((double)(1024 + mant), exp - 25);
    return sign ? -v : v;
}
static uint16_t low_encode(double x, int bf16) {
    const uint16_t sign = signbit(x) ? 0x8000 : 0;
    if (isnan(x)) return bf16 ? 0x7fc0 : 0x7e00;
    double a = fabs(x);
    const int digits = bf16 ? 8 : 11, min_q = bf16 ? -133 : -24;
    const double max = bf16 ? ldexp(255.0, 120) : 65504.0;
    if (a != 0.0 && !isinf(a)) {
        int e;
        frexp(a, &e);
        const int q = e - digits > min_q ? e - digits : min_q;
        a = ldexp(nearbyint(ldexp(a, -q)), q);  /* round to nearest even at quantum 2^q */
        if (a > max) a = INFINITY;
    }
    if (bf16) {
        const float f = (float)a;  /* exact: a is a bf16 value */
        uint32_t u;
        memcpy(&u, &f, 4);
        return sign | (uint16_t)(u >> 16);
    }
    if (isinf(a)) return sign | 0x7c00;
    if (a == 0.0) return sign;
    if (a < ldexp(1.0, -14)) return sign | (uint16_t)ldexp(a, 24);
    int e;
    const double m = frexp(a, &e); /* a = m 2^e, m in [0.5, 1) */
    return sign | (uint16_t)((e - 1 + 15) << 10) | (uint16_t)(ldexp(m, 11) - 1024.0);
}

ORACLE_API int cubf_oracle_fwht_native(uint16_t* data, size_t n, size_t batch, int bf16, int normalize) {
    if (!is_pow2(n)) return 1;
    const uint16_t limit = bf16 ? 0x7e7f : 0x73ff;
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t b = 0; b < batch; ++b) {
        uint16_t* v = data + b * n;
        for (size_t half = 1; half < n; half <<= 1)
            for (size_t base = 0; base < n; base += 2 * half)
                for (size_t o = 0; o < half; ++o) {
                    uint16_t l = v[base + o], r = v[base + half + o];
                    const int after = normalize && (l & 0x7fff) <= limit && (r & 0x7fff) <= limit;
                    if (normalize && !after) {
                        l = low_encode(low_decode(l, bf16) * 0.5, bf16);
                        r = low_encode(low_decode(r, bf16) * 0.5, bf16);
                    }
                    const double a = low_decode(l, bf16), c = low_decode(r, bf16);
                    l = low_encode(a + c, bf16);
                    r = low_encode(a - c, bf16);
                    if (after) {
                        l = low_encode(low_decode(l, bf16) * 0.5, bf16);
                        r = low_encode(low_decode(r, bf16) * 0.5, bf16);
                    }
                    v[base + o] = l;
                    v[base + half + o] = r;
                }
    }
    return 0;
}

/* uint64 variants, butterfly_reference.cpp:513-538. */
ORACLE_API int cubf_oracle_zeta_u64(uint64_t* data, size_t n, size_t batch, int superset, int inverse) {
    if (!is_pow2(n)) return 1;
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t b = 0; b < batch; ++b) {
        uint64_t* v = data + n * b;
        for (size_t half = 1; half < n; half <<= 1)
            for (size_t base = 0; base < n; base += 2 * half)
                for (size_t offset = 0; offset < half; ++offset) {
                    uint64_t* target = &v[base + offset + (superset ? 0 : half)];
                    const uint64_t source = v[base + offset + (superset ? half : 0)];
                    *target = inverse ? *target - source : *target + source;
                }
    }
    return 0;
}

/* ---------------------------------------------------------------- NTT ---- */

static uint64_t mod_mul(uint64_t a, uint64_t b, uint64_t q) { return (uint64_t)(((u128)a * b) % q); }

/* src/reference.cpp:506-520 */
ORACLE_API uint64_t cubf_oracle_mod_pow(uint64_t base, uint64_t exponent, uint64_t q) {
    uint64_t result = 1;
    base %= q;
    while (exponent) {
        if (exponent & 1u) result = mod_mul(result, base, q);
        base = mod_mul(base, base, q);
        exponent >>= 1;
    }
    return result;
}

/* Deterministic Miller-Rabin with the 7-witness set valid for all 64-bit
 * integers, as src/reference.cpp:522-562. */
ORACLE_API int cubf_oracle_is_prime(uint64_t value) {
    static const uint64_t small[12] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
    static const uint64_t witnesses[7] = {2, 325, 9375, 28178, 450775, 9780504, 1795265022};
    if (value < 2) return 0;
    for (int i = 0; i < 12; ++i)
        if (value % small[i] == 0) return value == small[i];
    uint64_t d = value - 1;
    unsigned s = 0;
    while ((d & 1u) == 0) {
        d >>= 1;
        ++s;
    }
    for (int w = 0; w < 7; ++w) {
        if (witnesses[w] % value == 0) continue;
        uint64_t x = cubf_oracle_mod_pow(witnesses[w], d, value);
        if (x == 1 || x == value - 1) continue;
        int ok = 0;
        for (unsigned r = 1; r < s; ++r) {
            x = mod_mul(x, x, value);
            if (x == value - 1) {
                ok = 1;
                break;
            }
        }
        if (!ok) return 0;
    }
    return 1;
}

/* Smallest-candidate primitive 2^log_n-th root, src/reference.cpp:564-582.
 * Returns 0 when the modulus is not prime or has no such root. */
ORACLE_API uint64_t cubf_oracle_find_root(unsigned log_n, uint64_t q) {
    if (log_n == 0 || log_n >= 63 || !cubf_oracle_is_prime(q)) return 0;
    const uint64_t n = 1ull << log_n;
    if ((q - 1) % n != 0) return 0;
    for (uint64_t c = 2; c < (1ull << 20); ++c) {
        const uint64_t root = cubf_oracle_mod_pow(c, (q - 1) / n, q);
        if (cubf_oracle_mod_pow(root, n, q) == 1 && cubf_oracle_mod_pow(root, n >> 1, q) != 1) return root;
    }
    return 0;
}

/* The largest `count` primes q < 2^60 with q == 1 (mod 2^root_log), found by
 * descending q = k * 2^root_log + 1 (the RNS limb generator of the benchmark). */
ORACLE_API size_t cubf_oracle_rns_primes(unsigned root_log, size_t count, uint64_t* out) {
    const uint64_t step = 1ull << root_log;
    uint64_t k = ((1ull << 60) - 2) / step;
    size_t found = 0;
    while (found < count && k > 0) {
        const uint64_t q = k * step + 1;
        if (q < (1ull << 60) && cubf_oracle_is_prime(q)) out[found++] = q;
        --k;
    }
    return found;
}

/* Cyclic radix-2 DIT NTT, src/reference.cpp:584-630: natural in, natural out,
 * root = find_primitive_power_of_two_root(log n, q). */
ORACLE_API int cubf_oracle_ntt_cyclic(uint64_t* values, size_t n, uint64_t q, int inverse) {
    if (n < 2 || !is_pow2(n) || q >= (1ull << 63)) return 1;
    const unsigned log_n = log2_exact(n);
    uint64_t root = cubf_oracle_find_root(log_n, q);
    if (!root) return 1;
    if (inverse) root = cubf_oracle_mod_pow(root, q - 2, q);
    for (size_t i = 0; i < n; ++i) values[i] %= q;
    bitrev_permute(values, n, sizeof(uint64_t));
    for (size_t length = 2; length <= n; length <<= 1) {
        const size_t half = length >> 1;
        const uint64_t step_root = cubf_oracle_mod_pow(root, n / length, q);
        for (size_t start = 0; start < n; start += length) {
            uint64_t omega = 1;
            for (size_t offset = 0; offset < half; ++offset) {
                const size_t left = start + offset;
                const uint64_t u = values[left];
                const uint64_t v = mod_mul(values[left + half], omega, q);
                const uint64_t sum = u + v;
                values[left] = sum >= q ? sum - q : sum;
                values[left + half] = u >= v ? u - v : q + u - v;
                omega = mod_mul(omega, step_root, q);
            }
        }
    }
    if (inverse) {
        const uint64_t inv_n = cubf_oracle_mod_pow((uint64_t)n, q - 2, q);
        for (size_t i = 0; i < n; ++i) values[i] = mod_mul(values[i], inv_n, q);
    }
    return 0;
}

/* RNS NTT of one polynomial, restating the independent CPU reference of the
 * reference's RNS tests (tests/test_rns_ntt.cu:61-110): optional input
 * bit-reversal, negacyclic twist by root^j (forward), cyclic DIT with
 * omega = root^2 (negacyclic) or root (cyclic), inverse scaling by n^-1 and
 * untwist by root^-j, optional output bit-reversal.  `root` is the FORWARD
 * primitive 2n-th (negacyclic) or n-th (cyclic) root. */
ORACLE_API int cubf_oracle_rns_ntt(const uint64_t* physical, uint64_t* result, unsigned log_n, uint64_t q,
                                   uint64_t root, int negacyclic, int inverse, int input_bitrev,
                                   int output_bitrev) {
    const size_t n = (size_t)1 << log_n;
    uint64_t* values = result;
    if (physical == result) return 1;
    for (size_t j = 0; j < n; ++j) values[j] = physical[input_bitrev ? reverse_bits(j, log_n) : j];
    if (negacyclic && !inverse) {
        uint64_t twist = 1;
        for (size_t j = 0; j < n; ++j) {
            values[j] = mod_mul(values[j], twist, q);
            twist = mod_mul(twist, root, q);
        }
    }
    uint64_t omega = negacyclic ? mod_mul(root, root, q) : root;
    if (inverse) omega = cubf_oracle_mod_pow(omega, q - 2, q);
    bitrev_permute(values, n, sizeof(uint64_t));
    for (size_t length = 2; length <= n; length *= 2) {
        const uint64_t step = cubf_oracle_mod_pow(omega, n / length, q);
        for (size_t base = 0; base < n; base += length) {
            uint64_t tw = 1;
            for (size_t j = 0; j < length / 2; ++j) {
                const uint64_t a = values[base + j];
                const uint64_t b = mod_mul(values[base + j + length / 2], tw, q);
                values[base + j] = (uint64_t)(((u128)a + b) % q);
                values[base + j + length / 2] = (uint64_t)(((u128)a + q - b) % q);
                tw = mod_mul(tw, step, q);
            }
        }
    }
    if (inverse) {
        uint64_t factor = cubf_oracle_mod_pow(n, q - 2, q);
        const uint64_t step = negacyclic ? cubf_oracle_mod_pow(root, q - 2, q) : 1;
        for (size_t j = 0; j < n; ++j) {
            values[j] = mod_mul(values[j], factor, q);
            factor = mod_mul(factor, step, q);
        }
    }
    if (output_bitrev) bitrev_permute(values, n, sizeof(uint64_t));
    return 0;
}

/* Batched RNS NTT over `count` polynomials stored contiguously (polynomial i
 * at i*n), polynomial i using (moduli[i], roots[i]). */
ORACLE_API int cubf_oracle_rns_ntt_batch(const uint64_t* input, uint64_t* output, unsigned log_n, size_t count,
                                         const uint64_t* moduli, const uint64_t* roots, int negacyclic,
                                         int inverse, int input_bitrev, int output_bitrev) {
    const size_t n = (size_t)1 << log_n;
    int status = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(| : status)
    for (size_t i = 0; i < count; ++i)
        status |= cubf_oracle_rns_ntt(input + i * n, output + i * n, log_n, moduli[i], roots[i], negacyclic, inverse,
                                      input_bitrev, output_bitrev);
    return status;
}

/* NTT of any length n over a prime q with 2n | q - 1, as the reference's
 * non-power-of-two NTT plans define it (src/bluestein_ntt.cu:42-57, :222-239):
 * psi = c^((q - 1) / 2n) for the first c = 2, 3, ... that makes it a
 * primitive 2n-th root, omega = psi^2 (its inverse for an inverse transform),
 * X[k] = sum_j (x[j] mod q) omega^(jk), times n^-1 for an inverse.  Rows of n
 * words, in place.  Returns 1 for an unusable modulus. */
ORACLE_API int cubf_oracle_ntt_any(uint64_t* values, size_t n, size_t batch, uint64_t q, int inverse) {
    if (n < 2 || !cubf_oracle_is_prime(q) || (q - 1) % (2 * n) != 0) return 1;
    const uint64_t order = 2 * n;
    uint64_t factors[64];
    int nf = 0;
    uint64_t v = order;
    for (uint64_t f = 2; f <= v / f; ++f) {
        if (v % f) continue;
        factors[nf++] = f;
        while (v % f == 0) v /= f;
    }
    if (v > 1) factors[nf++] = v;
    uint64_t psi = 0;
    for (uint64_t c = 2; c < (1ull << 20) && !psi; ++c) {
        const uint64_t r = cubf_oracle_mod_pow(c, (q - 1) / order, q);
        int primitive = cubf_oracle_mod_pow(r, order, q) == 1;
        for (int i = 0; i < nf && primitive; ++i) primitive = cubf_oracle_mod_pow(r, order / factors[i], q) != 1;
        if (primitive) psi = r;
    }
    if (!psi) return 1;
    uint64_t omega = mod_mul(psi, psi, q);
    if (inverse) omega = cubf_oracle_mod_pow(omega, q - 2, q);
    const uint64_t scale = inverse ? cubf_oracle_mod_pow(n % q, q - 2, q) : 1;
    uint64_t* pw = (uint64_t*)malloc(n * sizeof(uint64_t));
    uint64_t* x = (uint64_t*)malloc(n * sizeof(uint64_t));
    if (!pw || !x) {
        free(pw);
        free(x);
        return 1;
    }
    pw[0] = 1;
    for (size_t m = 1; m < n; ++m) pw[m] = mod_mul(pw[m - 1], omega, q);
    for (size_t b = 0; b < batch; ++b) {
        uint64_t* row = values + b * n;
        for (size_t j = 0; j < n; ++j) x[j] = row[j] % q;
        for (size_t k = 0; k < n; ++k) {
            u128 acc = 0;
            size_t m = 0; /* j k mod n */
            for (size_t j = 0; j < n; ++j) {
                acc += (u128)x[j] * pw[m];
                acc %= q;
                m += k;
                if (m >= n) m -= n;
            }
            row[k] = mod_mul((uint64_t)acc, scale, q);
        }
    }
    free(pw);
    free(x);
    return 0;
}

ORACLE_API int cubf_oracle_abi_version(void) { return 1; }
