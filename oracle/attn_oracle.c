/* attn_oracle.c — TEST INFRASTRUCTURE ONLY. CPU restatement of the reference's attention math.
 *
 * This file is the parity checker for the B200 kernels. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it. The product library never links it and
 * has no CPU fallback.
 *
 * It restates, in double precision:
 *   - causal prefill attention over the packed qkv[T, 3E] buffer, following the reference's CPU
 *     attention() in cpu/forward_cpu.c:83-116 (scale 1/sqrt(D) at :84, causal mask j<=i at :95,
 *     2-pass softmax max/exp/sum at :101-105, P·V at :108-112);
 *   - M=1 decode attention over the head-major KV cache [H][maxT][D] of one layer, following the
 *     reference's k_attn_decode in cuda/kvcache.cu:88-129 (keys 0..len-1, same scale, max/exp-sum,
 *     P·V), which the reference only has as a CUDA kernel.
 *
 * Pinning (how we know this restatement is right): tests/test_oracle.py compares it with the
 * reference's own attention() compiled from cpu/forward_cpu.c (oracle/_ref/libref_cpu.so, built by
 * oracle/Makefile) and with golden vectors under tests/golden/ that were produced by that compiled
 * reference (tests/golden/make_golden.py). The decode restatement is pinned by the identity
 * "decode of query i over keys 0..i == causal prefill row i", checked against the same reference.
 *
 * Inputs are fp32 (the caller feeds the exact fp16-rounded values the GPU sees); accumulation is
 * double, like the reference. OpenMP parallelises over independent (head, query) outputs, so the
 * result is bit-identical for any thread count (cpu/forward_cpu.h:9-10 makes the same promise).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Causal multi-head attention for one sequence.
 *   qkv: T rows of row_stride floats; q at column 0, k at E, v at 2E; head h at h*D inside each.
 *   att: T rows of out_stride floats; head h context written at h*D.
 * Returns 0, or -1 on bad arguments. */
int oracle_prefill_attention(float *att, const float *qkv, int T, int E, int H, int D,
                             long row_stride, long out_stride) {
    if (T < 1 || H < 1 || D < 1 || E != H * D || row_stride < 3L * E || out_stride < E) return -1;
    const double scale = 1.0 / sqrt((double)D);
    const long HT = (long)H * T;
    long hi;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 16)
#endif
    for (hi = 0; hi < HT; hi++) {
        const int h = (int)(hi / T), i = (int)(hi % T);
        const float *qi = qkv + (long)i * row_stride + h * D;
        double *sc = (double *)malloc(sizeof(double) * (size_t)(i + 1));
        double *acc = (double *)calloc((size_t)D, sizeof(double));
        double mx = -INFINITY;
        for (int j = 0; j <= i; j++) {
            const float *kj = qkv + (long)j * row_stride + E + h * D;
            double d = 0.0;
            for (int x = 0; x < D; x++) d += (double)qi[x] * (double)kj[x];
            d *= scale;
            sc[j] = d;
            if (d > mx) mx = d;
        }
        double sum = 0.0;
        for (int j = 0; j <= i; j++) { sc[j] = exp(sc[j] - mx); sum += sc[j]; }
        for (int j = 0; j <= i; j++) {
            const float *vj = qkv + (long)j * row_stride + 2L * E + h * D;
            for (int x = 0; x < D; x++) acc[x] += sc[j] * (double)vj[x];
        }
        const double inv = 1.0 / sum;
        float *o = att + (long)i * out_stride + h * D;
        for (int x = 0; x < D; x++) o[x] = (float)(acc[x] * inv);
        free(sc);
        free(acc);
    }
    return 0;
}

/* M=1 attention of one layer over the cache.
 *   q:   H*D floats (head h at h*D) — the first E entries of the step's qkv row.
 *   K,V: [H][maxT][D] floats (one layer's slabs of the reference arena, kvcache.cuh:31-33).
 *   att: H*D floats.
 * Attends to keys 0..len-1 (all of them: the reference's decode applies no mask beyond len). */
int oracle_decode_attention(float *att, const float *q, const float *K, const float *V,
                            int H, int maxT, int D, int len) {
    if (H < 1 || D < 1 || len < 1 || len > maxT) return -1;
    const double scale = 1.0 / sqrt((double)D);
    int h;
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
    for (h = 0; h < H; h++) {
        const float *qh = q + (long)h * D;
        const float *Kh = K + (long)h * maxT * D;
        const float *Vh = V + (long)h * maxT * D;
        double *sc = (double *)malloc(sizeof(double) * (size_t)len);
        double *acc = (double *)calloc((size_t)D, sizeof(double));
        double mx = -INFINITY;
        for (int j = 0; j < len; j++) {
            double d = 0.0;
            for (int x = 0; x < D; x++) d += (double)qh[x] * (double)Kh[(long)j * D + x];
            d *= scale;
            sc[j] = d;
            if (d > mx) mx = d;
        }
        double sum = 0.0;
        for (int j = 0; j < len; j++) { sc[j] = exp(sc[j] - mx); sum += sc[j]; }
        for (int j = 0; j < len; j++)
            for (int x = 0; x < D; x++) acc[x] += sc[j] * (double)Vh[(long)j * D + x];
        const double inv = 1.0 / sum;
        for (int x = 0; x < D; x++) att[(long)h * D + x] = (float)(acc[x] * inv);
        free(sc);
        free(acc);
    }
    return 0;
}

/* Reference cache writers, restated: the append of one position (cuda/kvcache.cu:57-64) and the
 * prefill scatter of T rows (cuda/kvcache.cu:67-76), on raw 16-bit words so the check is bit-exact.
 * K and V are one layer's [H][maxT][D] slabs; qkv rows are row_stride words long. */
int oracle_kv_scatter_u16(unsigned short *K, unsigned short *V, const unsigned short *qkv,
                          int T, int E, int H, int D, int maxT, long row_stride, int pos0) {
    if (T < 0 || E != H * D || pos0 < 0 || pos0 + T > maxT) return -1;
    for (int t = 0; t < T; t++)
        for (int i = 0; i < E; i++) {
            const int h = i / D, d = i % D;
            const long off = (long)h * maxT * D + (long)(pos0 + t) * D + d;
            K[off] = qkv[(long)t * row_stride + E + i];
            V[off] = qkv[(long)t * row_stride + 2L * E + i];
        }
    return 0;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
