/* ref_compose.c — the CPU MoE layer assembled from the reference's own kernels.
 * TEST INFRASTRUCTURE ONLY: linked with the reference's sources into
 * oracle/_ref/libkatali_ref.so; used as the fp32-activation parity oracle and
 * as the timed CPU baseline. The plugin never loads it.
 *
 * The reference's MoE CPU code is not in its checkout (README.md:13,17 describe
 * it). This composes the kernels that are there, each called through its public
 * entry point (vendor/katali_gguf_dense/ abbreviated V/):
 *   - router probabilities: katali_gguf_softmax (V/src/gguf_kernels.c:74-80);
 *   - gate and up of every selected expert in ONE dispatch:
 *     katali_ggml_matvec_fused (V/src/gguf_dtype.c:925-985), with the Q4_K
 *     activation-sum hoist (katali_ggml_q4k_sums, V/src/gguf_simd_x86.c:510-523);
 *   - silu(g)*u: katali_ggml_silu_mul_avx2 (V/src/gguf_simd_x86.c:744-773),
 *     scalar katali_gguf_silu (V/src/gguf_kernels.c:323) without AVX2;
 *   - down of every selected expert in one more fused dispatch;
 *   - the router-weighted sum in double, rounded once.
 * Top-k is taken on the logits (ties -> lower id), the same rule the plugin and
 * the restatement use, so all three pick the same experts.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "katali_gguf_dtype.h"
#include "katali_gguf_kernels.h"
#include "katali_gguf_simd.h"
#include "katali_gguf_threads.h"

static inline uint32_t order_key(float f) {
    if (f != f) return 0u;
    f = f + 0.0f;
    uint32_t u;
    memcpy(&u, &f, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/* y = W x through the reference's threaded GEMV, with the Q4_K sums hoist. */
int kref_matvec(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                const float *x, float *y, int n_threads) {
    uint64_t cap = KATALI_Q4K_SUMS_FLOATS(cols);
    float *scratch = cap ? (float *)malloc((size_t)cap * sizeof(float)) : NULL;
    katali_ggml_matvec(type, w, rows, cols, x, y, n_threads, NULL, scratch, cap);
    free(scratch);
    return 0;
}

/* Scratch for one layer call, sized once by the caller. */
typedef struct KrefMoeScratch {
    float *probs, *g, *u, *d, *q4k;
    uint64_t q4k_cap;
    KataliMatvecJob *jobs;
} KrefMoeScratch;

void *kref_moe_scratch_new(int n_experts, int hidden, int ffn, int top_k) {
    KrefMoeScratch *s = (KrefMoeScratch *)calloc(1, sizeof(*s));
    if (!s) return NULL;
    s->probs = (float *)malloc(sizeof(float) * (size_t)n_experts);
    s->g = (float *)malloc(sizeof(float) * (size_t)top_k * ffn);
    s->u = (float *)malloc(sizeof(float) * (size_t)top_k * ffn);
    s->d = (float *)malloc(sizeof(float) * (size_t)top_k * hidden);
    s->q4k_cap = KATALI_Q4K_SUMS_FLOATS(hidden > ffn ? hidden : ffn);
    s->q4k = (float *)malloc(sizeof(float) * (size_t)(s->q4k_cap ? s->q4k_cap : 1));
    s->jobs = (KataliMatvecJob *)malloc(sizeof(KataliMatvecJob) * (size_t)(2 * top_k));
    if (!s->probs || !s->g || !s->u || !s->d || !s->q4k || !s->jobs) {
        free(s->probs); free(s->g); free(s->u); free(s->d); free(s->q4k); free(s->jobs);
        free(s);
        return NULL;
    }
    return s;
}

void kref_moe_scratch_free(void *p) {
    KrefMoeScratch *s = (KrefMoeScratch *)p;
    if (!s) return;
    free(s->probs); free(s->g); free(s->u); free(s->d); free(s->q4k); free(s->jobs);
    free(s);
}

/* One MoE layer for one token with fp32 activations.
 * gate/up/down: arrays of n_experts host pointers to GGUF matrices
 * (gate/up: ffn x hidden, down: hidden x ffn). ids/w (top_k) may be NULL. */
int kref_moe_layer(int n_experts, int hidden, int ffn, int top_k, int norm_topk,
                   uint32_t gate_type, uint32_t up_type, uint32_t down_type,
                   const void *const *gate, const void *const *up,
                   const void *const *down, const float *x, const float *logits,
                   float *y, int n_threads, void *scratch, int32_t *ids_out,
                   float *w_out) {
    KrefMoeScratch *s = (KrefMoeScratch *)scratch;
    if (!s || top_k <= 0 || top_k > 64 || top_k > n_experts) return -1;
    int32_t ids[64];
    float w[64];
    unsigned char *taken = (unsigned char *)calloc((size_t)n_experts, 1);
    if (!taken) return -1;
    for (int t = 0; t < top_k; t++) {
        int best = -1;
        uint32_t bk = 0;
        for (int i = 0; i < n_experts; i++) {
            if (taken[i]) continue;
            const uint32_t k = order_key(logits[i]);
            if (best < 0 || k > bk) { best = i; bk = k; }
        }
        taken[best] = 1;
        ids[t] = best;
    }
    free(taken);
    memcpy(s->probs, logits, sizeof(float) * (size_t)n_experts);
    katali_gguf_softmax(s->probs, (size_t)n_experts);
    double S = 0.0;
    for (int t = 0; t < top_k; t++) S += (double)s->probs[ids[t]];
    for (int t = 0; t < top_k; t++)
        w[t] = norm_topk ? (float)((double)s->probs[ids[t]] / S) : s->probs[ids[t]];

    for (int t = 0; t < top_k; t++) {
        s->jobs[2 * t] = (KataliMatvecJob){ gate_type, gate[ids[t]], (uint64_t)ffn,
                                            s->g + (size_t)t * ffn, KATALI_ROLE_GATE };
        s->jobs[2 * t + 1] = (KataliMatvecJob){ up_type, up[ids[t]], (uint64_t)ffn,
                                                s->u + (size_t)t * ffn, KATALI_ROLE_UP };
    }
    katali_ggml_matvec_fused(s->jobs, 2 * top_k, (uint64_t)hidden, x, n_threads, NULL,
                             s->q4k, s->q4k_cap);
    for (int t = 0; t < top_k; t++) {
        float *g = s->g + (size_t)t * ffn, *u = s->u + (size_t)t * ffn;
        if (katali_ggml_silu_mul_avx2(g, u, (size_t)ffn) != 0)
            for (int j = 0; j < ffn; j++) g[j] = katali_gguf_silu(g[j]) * u[j];
    }
    /* Each expert's down projection reads its own h, so the jobs cannot share
     * one activation vector: one dispatch per expert. */
    for (int t = 0; t < top_k; t++) {
        katali_ggml_matvec(down_type, down[ids[t]], (uint64_t)hidden, (uint64_t)ffn,
                           s->g + (size_t)t * ffn, s->d + (size_t)t * hidden,
                           n_threads, NULL, s->q4k, s->q4k_cap);
    }
    for (int r = 0; r < hidden; r++) {
        double acc = 0.0;
        for (int t = 0; t < top_k; t++) acc += (double)w[t] * (double)s->d[(size_t)t * hidden + r];
        y[r] = (float)acc;
    }
    if (ids_out) memcpy(ids_out, ids, sizeof(int32_t) * (size_t)top_k);
    if (w_out) memcpy(w_out, w, sizeof(float) * (size_t)top_k);
    return 0;
}
