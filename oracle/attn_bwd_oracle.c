/*
 * TEST INFRASTRUCTURE ONLY. CPU checker for blackflash_b200's attention
 * backward; never on the product path.
 *
 * The reference has no backward pass (its l/m slots, include/flash_attn.cuh:27-28,
 * are declared for one). This restates the gradients of the forward the
 * reference tests define (tests/test_blackflash.py:16-19: S = scale Q K^T,
 * P = softmax(S), O = P V) for one upstream gradient dO:
 *
 *   dV = P^T dO
 *   dP = dO V^T
 *   dS = P o (dP - D),   D_i = sum_j P_ij dP_ij = sum_c dO_ic O_ic
 *   dQ = scale dS K
 *   dK = scale dS^T Q
 *
 * in double precision on bf16 inputs (raw uint16 bit patterns, [BH, N, d]),
 * rounded once to fp32. Parity of this restatement is pinned against torch
 * autograd of the fp32 forward in tests/test_oracle.py.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline double bf(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return (double)f;
}

typedef struct {
    const uint16_t *q, *k, *v, *dout;
    float *dq, *dk, *dv;
    long long s0, s1;
    int n, d;
    double scale;
} BwdJob;

static void bwd_slice(const BwdJob* j, long long s) {
    const int n = j->n, d = j->d;
    const size_t off = (size_t)s * n * d;
    double* P = (double*)malloc(sizeof(double) * (size_t)n * n);
    double* dP = (double*)malloc(sizeof(double) * (size_t)n * n);
    double* O = (double*)calloc((size_t)n * d, sizeof(double));
    double* D = (double*)malloc(sizeof(double) * (size_t)n);
    for (int i = 0; i < n; ++i) {
        double mx = -INFINITY;
        for (int c = 0; c < n; ++c) {
            double acc = 0.0;
            for (int e = 0; e < d; ++e) acc += bf(j->q[off + (size_t)i * d + e]) * bf(j->k[off + (size_t)c * d + e]);
            P[(size_t)i * n + c] = acc * j->scale;
            if (P[(size_t)i * n + c] > mx) mx = P[(size_t)i * n + c];
        }
        double sum = 0.0;
        for (int c = 0; c < n; ++c) {
            P[(size_t)i * n + c] = exp(P[(size_t)i * n + c] - mx);
            sum += P[(size_t)i * n + c];
        }
        for (int c = 0; c < n; ++c) P[(size_t)i * n + c] /= sum;
        for (int c = 0; c < n; ++c) {
            const double p = P[(size_t)i * n + c];
            for (int e = 0; e < d; ++e) O[(size_t)i * d + e] += p * bf(j->v[off + (size_t)c * d + e]);
        }
        double dd = 0.0;
        for (int e = 0; e < d; ++e) dd += bf(j->dout[off + (size_t)i * d + e]) * O[(size_t)i * d + e];
        D[i] = dd;
        for (int c = 0; c < n; ++c) {
            double acc = 0.0;
            for (int e = 0; e < d; ++e) acc += bf(j->dout[off + (size_t)i * d + e]) * bf(j->v[off + (size_t)c * d + e]);
            dP[(size_t)i * n + c] = P[(size_t)i * n + c] * (acc - D[i]);  // dS in place of dP
        }
    }
    for (int i = 0; i < n; ++i)
        for (int e = 0; e < d; ++e) {
            double a = 0.0;
            for (int c = 0; c < n; ++c) a += dP[(size_t)i * n + c] * bf(j->k[off + (size_t)c * d + e]);
            j->dq[off + (size_t)i * d + e] = (float)(a * j->scale);
        }
    for (int c = 0; c < n; ++c)
        for (int e = 0; e < d; ++e) {
            double a = 0.0, b = 0.0;
            for (int i = 0; i < n; ++i) {
                a += dP[(size_t)i * n + c] * bf(j->q[off + (size_t)i * d + e]);
                b += P[(size_t)i * n + c] * bf(j->dout[off + (size_t)i * d + e]);
            }
            j->dk[off + (size_t)c * d + e] = (float)(a * j->scale);
            j->dv[off + (size_t)c * d + e] = (float)b;
        }
    free(P);
    free(dP);
    free(O);
    free(D);
}

static void* bwd_worker(void* arg) {
    const BwdJob* j = (const BwdJob*)arg;
    for (long long s = j->s0; s < j->s1; ++s) bwd_slice(j, s);
    return NULL;
}

int oracle_attn_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* dout, float* dq, float* dk,
                    float* dv, long long bh, int n, int d, float scale, int nthreads) {
    if (bh <= 0 || n <= 0 || d <= 0) return 0;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > bh) nthreads = (int)bh;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
    BwdJob* jobs = (BwdJob*)malloc(sizeof(BwdJob) * (size_t)nthreads);
    for (int t = 0; t < nthreads; ++t) {
        BwdJob b = {q, k, v, dout, dq, dk, dv, bh * t / nthreads, bh * (t + 1) / nthreads, n, d, (double)scale};
        jobs[t] = b;
        pthread_create(&th[t], NULL, bwd_worker, &jobs[t]);
    }
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
    return 0;
}
