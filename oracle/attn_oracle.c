/*
 * TEST INFRASTRUCTURE ONLY. This is the CPU checker for blackflash_b200 and is
 * never on the product path. Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg may load it.
 *
 * CPU restatements of the reference's attention forward, on bf16 inputs given
 * as raw uint16 bit patterns in [BH, N, d] layout:
 *
 *  oracle_attn_exact  fp32 math attention as in reference tests/test_blackflash.py:16-19
 *                     and profile/gen_ref.py:80-84: S = (Q K^T) * scale, P = softmax(S),
 *                     O = P V. Dot products and the softmax sum are accumulated in
 *                     double, then rounded once to fp32. The result is the
 *                     "unrounded fp32" O that parity is measured against. It also
 *                     gives lse = log sum exp(S) and the row max of S.
 *
 *  oracle_attn_fa2    the reference kernel's own algorithm (kernel/flash_attn_mma.cu):
 *                     64-row Q tiles and 64-row KV tiles (:7-9, :105, :228), S scaled
 *                     after the product (:284-290), an online max with an every-tile
 *                     rescale by exp(m_old - m_new) (:326-339, :407-423), P rounded to
 *                     bf16 before the PV product (:359-378), l summed over fp32 p
 *                     (:340-357), and O = acc / l rounded to bf16 (:436-464). fp32
 *                     throughout, as on the GPU. Like the reference, it assumes
 *                     N % 64 == 0 (no tail masking).
 *
 *  oracle_attn_exact_causal  the same with a causal mask (key j visible to query i iff j <= i).
 *
 *  oracle_scores      S and P = softmax(S) of one slice in fp32, the quantities
 *                     gen_ref.py saves as s_ref.bin / p_ref.bin (:80-84, :183-184).
 *
 * Work is split over slices with pthreads.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float round_to_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) return x; /* inf / nan unchanged */
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb; /* round to nearest, ties to even */
    u &= 0xffff0000u;
    memcpy(&x, &u, 4);
    return x;
}

typedef struct {
    const uint16_t *q, *k, *v;
    float *o, *lse, *rowmax;
    uint16_t* o_bf16;
    long long bh0, bh1;
    int nq, nkv, d;
    float scale;
    int mode; /* 0 exact, 1 fa2 */
    int causal; /* exact mode: key j is visible to query i only if j <= i */
} Job;

static void exact_slice(const Job* j, long long s) {
    const int nq = j->nq, nkv = j->nkv, d = j->d;
    const uint16_t* q = j->q + (size_t)s * nq * d;
    const uint16_t* k = j->k + (size_t)s * nkv * d;
    const uint16_t* v = j->v + (size_t)s * nkv * d;
    float* kf = (float*)malloc(sizeof(float) * (size_t)nkv * d);
    float* vf = (float*)malloc(sizeof(float) * (size_t)nkv * d);
    double* srow = (double*)malloc(sizeof(double) * (size_t)nkv);
    double* acc = (double*)malloc(sizeof(double) * (size_t)d);
    float* qf = (float*)malloc(sizeof(float) * (size_t)d);
    for (size_t i = 0; i < (size_t)nkv * d; ++i) {
        kf[i] = bf16_to_f32(k[i]);
        vf[i] = bf16_to_f32(v[i]);
    }
    for (int i = 0; i < nq; ++i) {
        for (int c = 0; c < d; ++c) qf[c] = bf16_to_f32(q[(size_t)i * d + c]);
        double mx = -INFINITY;
        const int lim = j->causal ? (i + 1 < nkv ? i + 1 : nkv) : nkv;
        for (int jj = 0; jj < lim; ++jj) {
            double dot = 0.0;
            const float* kr = kf + (size_t)jj * d;
            for (int c = 0; c < d; ++c) dot += (double)qf[c] * (double)kr[c];
            srow[jj] = dot * (double)j->scale;
            if (srow[jj] > mx) mx = srow[jj];
        }
        double sum = 0.0;
        for (int c = 0; c < d; ++c) acc[c] = 0.0;
        for (int jj = 0; jj < lim; ++jj) {
            const double p = exp(srow[jj] - mx);
            sum += p;
            const float* vr = vf + (size_t)jj * d;
            for (int c = 0; c < d; ++c) acc[c] += p * (double)vr[c];
        }
        float* orow = j->o + ((size_t)s * nq + i) * d;
        for (int c = 0; c < d; ++c) orow[c] = (float)(acc[c] / sum);
        if (j->lse) j->lse[(size_t)s * nq + i] = (float)(mx + log(sum));
        if (j->rowmax) j->rowmax[(size_t)s * nq + i] = (float)mx;
    }
    free(kf);
    free(vf);
    free(srow);
    free(acc);
    free(qf);
}

/* The reference kernel's tiling (64 x 64), fp32 online softmax, bf16 P. */
static void fa2_slice(const Job* j, long long s) {
    enum { BR = 64, BC = 64 };
    const int n = j->nq, d = j->d;
    const uint16_t* q = j->q + (size_t)s * n * d;
    const uint16_t* k = j->k + (size_t)s * n * d;
    const uint16_t* v = j->v + (size_t)s * n * d;
    float sc[BC], p[BC];
    float* acc = (float*)malloc(sizeof(float) * (size_t)d);
    for (int i = 0; i < n; ++i) {
        float m = -INFINITY, l = 0.f;
        for (int c = 0; c < d; ++c) acc[c] = 0.f;
        for (int t0 = 0; t0 < n; t0 += BC) {
            const int tn = (n - t0) < BC ? (n - t0) : BC;
            float mt = -INFINITY;
            for (int jj = 0; jj < tn; ++jj) {
                float dot = 0.f;
                for (int c = 0; c < d; ++c)
                    dot = fmaf(bf16_to_f32(q[(size_t)i * d + c]), bf16_to_f32(k[(size_t)(t0 + jj) * d + c]), dot);
                sc[jj] = dot * j->scale;
                if (sc[jj] > mt) mt = sc[jj];
            }
            const float m_new = m > mt ? m : mt;
            const float alpha = expf(m - m_new);
            float rs = 0.f;
            for (int jj = 0; jj < tn; ++jj) {
                p[jj] = expf(sc[jj] - m_new);
                rs += p[jj];
                p[jj] = round_to_bf16(p[jj]);
            }
            for (int c = 0; c < d; ++c) {
                float pv = 0.f;
                for (int jj = 0; jj < tn; ++jj) pv = fmaf(p[jj], bf16_to_f32(v[(size_t)(t0 + jj) * d + c]), pv);
                acc[c] = acc[c] * alpha + pv;
            }
            l = l * alpha + rs;
            m = m_new;
        }
        for (int c = 0; c < d; ++c) {
            const float o = acc[c] / l;
            j->o[((size_t)s * n + i) * d + c] = round_to_bf16(o);
        }
        if (j->lse) j->lse[(size_t)s * n + i] = m + logf(l);
        if (j->rowmax) j->rowmax[(size_t)s * n + i] = m;
    }
    free(acc);
}

static void* worker(void* arg) {
    const Job* j = (const Job*)arg;
    for (long long s = j->bh0; s < j->bh1; ++s) {
        if (j->mode == 0)
            exact_slice(j, s);
        else
            fa2_slice(j, s);
    }
    return NULL;
}

static int run(Job base, long long bh, int nthreads) {
    if (bh <= 0 || base.nq <= 0 || base.nkv <= 0 || base.d <= 0) return 0;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > bh) nthreads = (int)bh;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
    Job* jobs = (Job*)malloc(sizeof(Job) * (size_t)nthreads);
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = base;
        jobs[t].bh0 = bh * t / nthreads;
        jobs[t].bh1 = bh * (t + 1) / nthreads;
        pthread_create(&th[t], NULL, worker, &jobs[t]);
    }
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
    return 0;
}

int oracle_attn_exact_causal(const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o, float* lse,
                             float* rowmax, long long bh, int nq, int nkv, int d, float scale, int causal, int nthreads);

int oracle_attn_exact(const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o, float* lse, float* rowmax,
                      long long bh, int nq, int nkv, int d, float scale, int nthreads) {
    return oracle_attn_exact_causal(q, k, v, o, lse, rowmax, bh, nq, nkv, d, scale, 0, nthreads);
}

/* Causal variant (key j visible to query i iff j <= i, top-left aligned). This is
 * not a reference feature. The reference is non-causal only, and its benchmark
 * times cuDNN with is_causal=True (tests/bench_blackflash.py:58-60). */
int oracle_attn_exact_causal(const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o, float* lse,
                             float* rowmax, long long bh, int nq, int nkv, int d, float scale, int causal, int nthreads) {
    Job b;
    memset(&b, 0, sizeof(b));
    b.q = q;
    b.k = k;
    b.v = v;
    b.o = o;
    b.lse = lse;
    b.rowmax = rowmax;
    b.nq = nq;
    b.nkv = nkv;
    b.d = d;
    b.scale = scale;
    b.mode = 0;
    b.causal = causal;
    return run(b, bh, nthreads);
}

int oracle_attn_fa2(const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o, float* lse, float* rowmax,
                    long long bh, int n, int d, float scale, int nthreads) {
    Job b;
    memset(&b, 0, sizeof(b));
    b.q = q;
    b.k = k;
    b.v = v;
    b.o = o;
    b.lse = lse;
    b.rowmax = rowmax;
    b.nq = n;
    b.nkv = n;
    b.d = d;
    b.scale = scale;
    b.mode = 1;
    return run(b, bh, nthreads);
}

int oracle_scores(const uint16_t* q, const uint16_t* k, float* s_out, float* p_out, int n, int d, float scale) {
    for (int i = 0; i < n; ++i) {
        float mx = -INFINITY;
        for (int jj = 0; jj < n; ++jj) {
            float dot = 0.f;
            for (int c = 0; c < d; ++c) dot = fmaf(bf16_to_f32(q[(size_t)i * d + c]), bf16_to_f32(k[(size_t)jj * d + c]), dot);
            const float sv = dot * scale;
            s_out[(size_t)i * n + jj] = sv;
            if (sv > mx) mx = sv;
        }
        if (p_out) {
            double sum = 0.0;
            for (int jj = 0; jj < n; ++jj) sum += exp((double)s_out[(size_t)i * n + jj] - mx);
            for (int jj = 0; jj < n; ++jj)
                p_out[(size_t)i * n + jj] = (float)(exp((double)s_out[(size_t)i * n + jj] - mx) / sum);
        }
    }
    return 0;
}
