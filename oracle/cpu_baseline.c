/*
 * cpu_baseline.c -- the reference's AVX2 CPU matvec kernels, restated in C and
 * threaded the way the reference threads them.
 *
 * TEST / MEASUREMENT INFRASTRUCTURE ONLY: bench.py times these as the CPU
 * baseline ("cpu_baseline" leg and --impl reference); tests check them against
 * the scalar oracle.  Nothing in the product library calls them.
 *
 *  - matvec_q4_k: crates/soso-llm-core/src/gemm.rs:842-894 (avx2::matvec_q4_k):
 *    per 32-element half of a pair, 4 groups of 8 lanes, coef = q*dsc + (-dm),
 *    acc = fma(coef, x, acc), one 8-lane accumulator per row, hsum at the end.
 *  - matvec_q8_0: gemm.rs:806-836 (avx2::matvec_q8_0): per block 4 groups of 8
 *    lanes into blk, then acc = fma(scale, blk, acc).
 *  - row split: crates/soso-llm-core/src/parallel.rs:22-31 (row_strip).
 */
#include <immintrin.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define OR_API __attribute__((visibility("default")))

float or_f16_to_f32(uint16_t bits);
void or_q4k_scale_min(const uint8_t *s, int j, uint8_t *sc, uint8_t *m);
int or_matvec_q6_k(const uint8_t *bytes, size_t rows, size_t cols, const float *x, float *out);

/* parallel.rs:22-31 */
OR_API void or_row_strip(size_t rows, size_t i, size_t n, size_t *start, size_t *end)
{
    if (n == 0 || i >= n) { *start = *end = 0; return; }
    size_t base = rows / n, rem = rows % n;
    *start = i * base + (i < rem ? i : rem);
    *end = *start + base + (i < rem ? 1 : 0);
}

/* gemm.rs:694-703 (hsum) */
__attribute__((target("avx2,fma"))) static inline float hsum(__m256 v)
{
    __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
    __m128 s = _mm_add_ps(lo, hi);
    s = _mm_add_ps(s, _mm_movehl_ps(s, s));
    s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 1));
    return _mm_cvtss_f32(s);
}

__attribute__((target("avx2,fma"))) static void q4k_rows(const uint8_t *bytes, size_t r0, size_t r1, size_t cols,
                                                        const float *x, float *out)
{
    size_t blocks = cols / 256, rb = blocks * 144;
    const __m256i mask = _mm256_set1_epi8(0x0F);
    for (size_t r = r0; r < r1; r++) {
        const uint8_t *row = bytes + r * rb;
        __m256 acc = _mm256_setzero_ps();
        for (size_t b = 0; b < blocks; b++) {
            const uint8_t *blk = row + b * 144;
            float d = or_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            float dmin = or_f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            for (int pair = 0; pair < 4; pair++) {
                uint8_t sc1, m1, sc2, m2;
                or_q4k_scale_min(blk + 4, 2 * pair, &sc1, &m1);
                or_q4k_scale_min(blk + 4, 2 * pair + 1, &sc2, &m2);
                __m256 dsc[2] = {_mm256_set1_ps(d * (float)sc1), _mm256_set1_ps(d * (float)sc2)};
                __m256 dm[2] = {_mm256_set1_ps(-dmin * (float)m1), _mm256_set1_ps(-dmin * (float)m2)};
                __m256i qv = _mm256_loadu_si256((const __m256i *)(blk + 16 + pair * 32));
                __m256i half[2] = {_mm256_and_si256(qv, mask), _mm256_and_si256(_mm256_srli_epi16(qv, 4), mask)};
                const float *xb = x + b * 256 + pair * 64;
                for (int h = 0; h < 2; h++) {
                    __m128i l0 = _mm256_castsi256_si128(half[h]), l1 = _mm256_extracti128_si256(half[h], 1);
                    __m128i quads[4] = {l0, _mm_srli_si128(l0, 8), l1, _mm_srli_si128(l1, 8)};
                    for (int g = 0; g < 4; g++) {
                        __m256 qf = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(quads[g]));
                        __m256 coef = _mm256_fmadd_ps(qf, dsc[h], dm[h]);
                        __m256 xv = _mm256_loadu_ps(xb + h * 32 + g * 8);
                        acc = _mm256_fmadd_ps(coef, xv, acc);
                    }
                }
            }
        }
        out[r] = hsum(acc);
    }
}

__attribute__((target("avx2,fma"))) static void q80_rows(const uint8_t *bytes, size_t r0, size_t r1, size_t cols,
                                                        const float *x, float *out)
{
    size_t blocks = cols / 32, rb = blocks * 36;
    for (size_t r = r0; r < r1; r++) {
        const uint8_t *row = bytes + r * rb;
        __m256 acc = _mm256_setzero_ps();
        for (size_t b = 0; b < blocks; b++) {
            const uint8_t *c = row + b * 36;
            float s;
            memcpy(&s, c, 4);
            __m256 scale = _mm256_set1_ps(s), blk = _mm256_setzero_ps();
            for (int g = 0; g < 4; g++) {
                __m128i qi = _mm_loadl_epi64((const __m128i *)(c + 4 + g * 8));
                __m256 qf = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(qi));
                blk = _mm256_fmadd_ps(qf, _mm256_loadu_ps(x + b * 32 + g * 8), blk);
            }
            acc = _mm256_fmadd_ps(scale, blk, acc);
        }
        out[r] = hsum(acc);
    }
}

typedef struct {
    uint8_t dtype;
    const uint8_t *bytes;
    size_t r0, r1, rows, cols;
    const float *x;
    float *out;
} job_t;

static void *run_job(void *p)
{
    job_t *j = (job_t *)p;
    size_t rb = j->dtype == 3 ? j->cols / 256 * 144 : j->dtype == 2 ? j->cols / 32 * 36 : j->cols / 256 * 210;
    if (j->dtype == 3) q4k_rows(j->bytes, j->r0, j->r1, j->cols, j->x, j->out);
    else if (j->dtype == 2) q80_rows(j->bytes, j->r0, j->r1, j->cols, j->x, j->out);
    else or_matvec_q6_k(j->bytes + j->r0 * rb, j->r1 - j->r0, j->cols, j->x, j->out + j->r0);
    return NULL;
}

/* Threaded AVX2 matvec (dtype 2 = Q8_0, 3 = Q4_K, 13 = Q6_K scalar). */
OR_API int or_cpu_matvec(uint8_t dtype, const uint8_t *bytes, size_t rows, size_t cols, const float *x, float *out,
                         int nthreads)
{
    if (dtype == 3 && cols % 256) return -1;
    if (dtype == 2 && cols % 32) return -1;
    if (dtype == 13 && cols % 256) return -1;
    if (dtype != 2 && dtype != 3 && dtype != 13) return -1;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    job_t jobs[256];
    pthread_t th[256];
    for (int i = 0; i < nthreads; i++) {
        jobs[i] = (job_t){dtype, bytes, 0, 0, rows, cols, x, out};
        or_row_strip(rows, (size_t)i, (size_t)nthreads, &jobs[i].r0, &jobs[i].r1);
    }
    for (int i = 1; i < nthreads; i++) pthread_create(&th[i], NULL, run_job, &jobs[i]);
    run_job(&jobs[0]);
    for (int i = 1; i < nthreads; i++) pthread_join(th[i], NULL);
    return 0;
}
