/* C restatement of the two kernel-level configs (oracle side, TEST INFRASTRUCTURE).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
 * this library; the engine never does.
 *
 *  cref_gemm_chain  -- config 1, the RDNA4 WMMA GEMM of r_6_2 shape with the
 *                      FFMA reference consumer (run_pinned2.py:158-192): per
 *                      output an fma.rn.f32 chain over k = 0..K-1 starting
 *                      from C (16-wide WMMA steps chain through C, so the
 *                      whole K range is one sequential chain).
 *  cref_reduce      -- config 2, r_32_32_3_12288_32 (NOTES.md:67-83,
 *                      alu_opt.py:1-12): out[r] = sum_i x[r][i] * w[i], f32
 *                      accumulate in index order.
 *  cref_fill        -- the hash RNG the engine uses for its random-init
 *                      weights (SplitMix64 finaliser, Steele/Lea/Flood 2014).
 *
 * f16 -> f32 conversion is written out from the IEEE 754 binary16 format.
 * An f16*f16 product is exact in f32, so fmaf(a, b, c) == (a*b) + c here.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: value = man * 2^-24 */
            float v = (float)man * 5.9604644775390625e-08f;
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* round-to-nearest-even f32 -> f16 */
static inline uint16_t f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* overflow to inf */
    if (ax < 0x38800000u) { /* subnormal or zero in f16 */
        float a;
        memcpy(&a, &ax, 4);
        float s = a * 16777216.0f; /* a / 2^-24, exact scaling */
        float r = nearbyintf(s);   /* RNE under default rounding mode */
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t e = (ax >> 23) - 112;
    uint32_t m = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;
    return (uint16_t)(sign | h);
}

void cref_gemm_chain(const uint16_t* A, const uint16_t* B, float* C,
                     long M, long N, long K, int b_kmajor, int nthreads) {
    /* A: [M][K]; B: b_kmajor ? [N][K] : [K][N]; C: [M][N] in/out */
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (long m = 0; m < M; ++m) {
        for (long n = 0; n < N; ++n) {
            float acc = C[m * N + n];
            for (long k = 0; k < K; ++k) {
                float a = h2f(A[m * K + k]);
                float b = h2f(b_kmajor ? B[n * K + k] : B[k * N + n]);
                acc = fmaf(a, b, acc);
            }
            C[m * N + n] = acc;
        }
    }
}

void cref_reduce(const uint16_t* x, const uint16_t* w, float* out,
                 long rows, long len, int nthreads) {
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (long r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * len;
        float acc = 0.0f;
        for (long i = 0; i < len; ++i) acc = fmaf(h2f(xr[i]), h2f(w[i]), acc);
        out[r] = acc;
    }
}

static inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline float hash_uniform(uint64_t seed, uint64_t tid, uint64_t idx) {
    uint64_t h = splitmix64((seed << 48) | (tid << 32) | idx);
    return (float)(int32_t)(h >> 40) * 1.1920928955078125e-07f - 1.0f;
}

/* out_f16 != NULL: f16 weights; else out_f32: f32 values. */
void cref_fill(uint64_t seed, uint64_t tid, long count, float bound,
               uint16_t* out_f16, float* out_f32, int nthreads) {
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (long i = 0; i < count; ++i) {
        float v = hash_uniform(seed, tid, (uint64_t)i) * bound;
        if (out_f16) out_f16[i] = f2h(v);
        else out_f32[i] = v;
    }
}

/* f16 [rows][K] x f16 [N][K]^T -> f32 [rows][N]; blocked, used by the CPU
 * baseline when numpy's BLAS is not the thing being timed. */
void cref_f16_to_f32(const uint16_t* src, float* dst, long n, int nthreads) {
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (long i = 0; i < n; ++i) dst[i] = h2f(src[i]);
}
