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

/* ------------------------------------------------------------------------ */
/* Dense decoder decode step composed from the reference's kernels, following */
/* gguf_forward_token (V/src/gguf_model.c:570-703) call by call: embedding     */
/* row (katali_ggml_dequant_ref), katali_gguf_rmsnorm, q/k/v through           */
/* katali_ggml_matvec, per-head katali_gguf_rmsnorm_inplace, RoPE with the      */
/* rope_prepare table (:466-475, rope_inv from :344) through                    */
/* katali_gguf_rope_apply, KV append, katali_gguf_gqa_decode_scratch, o + add,  */
/* gate/up, katali_ggml_silu_mul_avx2 (scalar silu without AVX2), down + add,   */
/* final norm and the LM head. Weights and norms are HOST arrays.               */
/* ------------------------------------------------------------------------ */
typedef struct KrefDenseLayer {
    const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
    const void *w[7]; /* wq wk wv wo gate up down */
    uint32_t t[7];
} KrefDenseLayer;

typedef struct KrefDense {
    int NL, H, F, NH, NKV, HD, vocab, cap, rd, n_threads;
    float eps, theta;
    const void *embed, *lm;
    uint32_t embed_t, lm_t;
    const float *out_norm;
    KrefDenseLayer *L;
    float *x, *xb, *q, *k, *v, *attn, *gate, *up, *down, *logits, *kv_k, *kv_v;
    float *scores, *rope_inv, *rope_cos, *rope_sin;
} KrefDense;

void *kref_dense_new(int NL, int H, int F, int NH, int NKV, int HD, int vocab, int cap,
                     int rope_dim, float eps, float theta, const void *embed, uint32_t embed_t,
                     const void *lm, uint32_t lm_t, const float *out_norm,
                     const float *const *attn_norm, const float *const *ffn_norm,
                     const float *const *q_norm, const float *const *k_norm,
                     const void *const *w /* 7 per layer */, const uint32_t *t, int n_threads) {
    KrefDense *m = (KrefDense *)calloc(1, sizeof(*m));
    if (!m) return NULL;
    m->NL = NL; m->H = H; m->F = F; m->NH = NH; m->NKV = NKV; m->HD = HD; m->vocab = vocab;
    m->cap = cap; m->eps = eps; m->theta = theta; m->n_threads = n_threads;
    m->rd = (rope_dim == 0 || rope_dim > HD) ? HD : rope_dim;
    m->embed = embed; m->embed_t = embed_t; m->lm = lm; m->lm_t = lm_t; m->out_norm = out_norm;
    m->L = (KrefDenseLayer *)calloc((size_t)NL, sizeof(KrefDenseLayer));
    for (int l = 0; l < NL; l++) {
        m->L[l].attn_norm = attn_norm[l];
        m->L[l].ffn_norm = ffn_norm[l];
        m->L[l].q_norm = q_norm ? q_norm[l] : NULL;
        m->L[l].k_norm = k_norm ? k_norm[l] : NULL;
        for (int i = 0; i < 7; i++) { m->L[l].w[i] = w[7 * l + i]; m->L[l].t[i] = t[7 * l + i]; }
    }
    m->x = (float *)calloc((size_t)H, 4); m->xb = (float *)calloc((size_t)H, 4);
    m->q = (float *)calloc((size_t)NH * HD, 4); m->k = (float *)calloc((size_t)NKV * HD, 4);
    m->v = (float *)calloc((size_t)NKV * HD, 4); m->attn = (float *)calloc((size_t)NH * HD, 4);
    m->gate = (float *)calloc((size_t)F, 4); m->up = (float *)calloc((size_t)F, 4);
    m->down = (float *)calloc((size_t)H, 4); m->logits = (float *)calloc((size_t)vocab, 4);
    m->kv_k = (float *)calloc((size_t)NL * NKV * cap * HD, 4);
    m->kv_v = (float *)calloc((size_t)NL * NKV * cap * HD, 4);
    m->scores = (float *)calloc((size_t)cap, 4);
    m->rope_inv = (float *)calloc((size_t)m->rd / 2, 4);
    m->rope_cos = (float *)calloc((size_t)m->rd / 2, 4);
    m->rope_sin = (float *)calloc((size_t)m->rd / 2, 4);
    for (int i = 0; i < m->rd / 2; i++)
        m->rope_inv[i] = 1.0f / powf(theta, (2.0f * (float)i) / (float)m->rd);
    return m;
}

void kref_dense_free(void *p) {
    KrefDense *m = (KrefDense *)p;
    if (!m) return;
    free(m->L); free(m->x); free(m->xb); free(m->q); free(m->k); free(m->v); free(m->attn);
    free(m->gate); free(m->up); free(m->down); free(m->logits); free(m->kv_k); free(m->kv_v);
    free(m->scores); free(m->rope_inv); free(m->rope_cos); free(m->rope_sin);
    free(m);
}

/* One step at position pos with input token; logits_out may be NULL. */
int kref_dense_step(void *p, int token, int pos, float *logits_out) {
    KrefDense *m = (KrefDense *)p;
    if (!m || token < 0 || token >= m->vocab || pos < 0 || pos >= m->cap) return -1;
    const int H = m->H, F = m->F, NH = m->NH, NKV = m->NKV, HD = m->HD, nt = m->n_threads;
    const uint64_t erb = katali_ggml_row_bytes(m->embed_t, (uint64_t)H);
    if (katali_ggml_dequant_ref(m->embed_t, (const uint8_t *)m->embed + (size_t)token * erb,
                                (uint64_t)H, m->x) != 0)
        return -1;
    const int half = m->rd / 2;
    for (int i = 0; i < half; i++) {
        float freq = (float)pos * m->rope_inv[i];
        m->rope_cos[i] = cosf(freq);
        m->rope_sin[i] = sinf(freq);
    }
    const size_t per_layer = (size_t)NKV * m->cap * HD;
    for (int l = 0; l < m->NL; l++) {
        const KrefDenseLayer *L = &m->L[l];
        katali_gguf_rmsnorm(m->x, L->attn_norm, (size_t)H, m->eps, m->xb);
        kref_matvec(L->t[0], L->w[0], (uint64_t)NH * HD, (uint64_t)H, m->xb, m->q, nt);
        kref_matvec(L->t[1], L->w[1], (uint64_t)NKV * HD, (uint64_t)H, m->xb, m->k, nt);
        kref_matvec(L->t[2], L->w[2], (uint64_t)NKV * HD, (uint64_t)H, m->xb, m->v, nt);
        if (L->q_norm)
            for (int h = 0; h < NH; h++)
                katali_gguf_rmsnorm_inplace(m->q + (size_t)h * HD, L->q_norm, (size_t)HD, m->eps);
        katali_gguf_rope_apply(m->q, (size_t)NH, (size_t)HD, (size_t)m->rd, m->rope_cos, m->rope_sin);
        if (L->k_norm)
            for (int h = 0; h < NKV; h++)
                katali_gguf_rmsnorm_inplace(m->k + (size_t)h * HD, L->k_norm, (size_t)HD, m->eps);
        katali_gguf_rope_apply(m->k, (size_t)NKV, (size_t)HD, (size_t)m->rd, m->rope_cos, m->rope_sin);
        float *lk = m->kv_k + (size_t)l * per_layer, *lv = m->kv_v + (size_t)l * per_layer;
        for (int h = 0; h < NKV; h++) {
            memcpy(lk + ((size_t)h * m->cap + pos) * HD, m->k + (size_t)h * HD, (size_t)HD * 4);
            memcpy(lv + ((size_t)h * m->cap + pos) * HD, m->v + (size_t)h * HD, (size_t)HD * 4);
        }
        katali_gguf_gqa_decode_scratch(m->q, lk, lv, (size_t)pos + 1, (size_t)m->cap, (size_t)NH,
                                       (size_t)NKV, (size_t)HD, m->attn, m->scores);
        kref_matvec(L->t[3], L->w[3], (uint64_t)H, (uint64_t)NH * HD, m->attn, m->down, nt);
        katali_gguf_add_inplace(m->x, m->down, (size_t)H);
        katali_gguf_rmsnorm(m->x, L->ffn_norm, (size_t)H, m->eps, m->xb);
        kref_matvec(L->t[4], L->w[4], (uint64_t)F, (uint64_t)H, m->xb, m->gate, nt);
        kref_matvec(L->t[5], L->w[5], (uint64_t)F, (uint64_t)H, m->xb, m->up, nt);
        if (katali_ggml_silu_mul_avx2(m->gate, m->up, (size_t)F) != 0)
            for (int i = 0; i < F; i++) m->gate[i] = katali_gguf_silu(m->gate[i]) * m->up[i];
        kref_matvec(L->t[6], L->w[6], (uint64_t)H, (uint64_t)F, m->gate, m->down, nt);
        katali_gguf_add_inplace(m->x, m->down, (size_t)H);
    }
    katali_gguf_rmsnorm(m->x, m->out_norm, (size_t)H, m->eps, m->xb);
    kref_matvec(m->lm_t, m->lm, (uint64_t)m->vocab, (uint64_t)H, m->xb, m->logits, nt);
    if (logits_out) memcpy(logits_out, m->logits, (size_t)m->vocab * 4);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Hybrid MoE decoder step (Qwen3.5/3.6-35B-A3B layer family; the reference   */
/* runs it only in its binaries, README.md:15,19,322-336). Composed from the  */
/* reference's kernels where the checkout has them — katali_gguf_rmsnorm[_    */
/* inplace], katali_ggml_matvec (Q4_K/Q6_K and the F32 router), katali_gguf_ */
/* rope_apply on the first rope_dim dimensions, katali_gguf_gqa_decode_       */
/* scratch, katali_gguf_sigmoid, katali_gguf_add_inplace and the composed MoE */
/* layer above — plus a RESTATEMENT of the Gated DeltaNet decode step, which  */
/* has no reference source: the published gated delta rule (Yang, Kautz,     */
/* Hatamizadeh, ICLR 2025) in the Qwen3-Next/Qwen3.5 layer layout:            */
/*   depthwise causal conv (kernel K) over q|k|v + SiLU; q, k L2-normalised   */
/*   per head (eps 1e-6), q scaled by 1/sqrt(dk); beta = sigmoid(b),          */
/*   g = -exp(A_log) softplus(a + dt_bias); S <- exp(g) S; kv = S^T k;        */
/*   S <- S + k (beta (v - kv))^T; o = S^T q; out = RMSNorm(o) w silu(z).     */
/* Parity of the GDN step and the gated attention is therefore unpinned by    */
/* the reference; the arithmetic order matches the plugin's kq_hybrid.cu.     */
/* ------------------------------------------------------------------------ */
typedef struct KrefHybridLayer {
    int32_t kind; /* 0 GDN, 1 gated attention */
    const float *attn_norm, *ffn_norm, *router;
    const void *w_qkv, *w_z, *w_b, *w_a, *w_out;
    uint32_t t_qkv, t_z, t_b, t_a, t_out;
    const float *conv, *a_log, *dt_bias, *ssm_norm;
    const void *wq, *wk, *wv, *wo;
    uint32_t tq, tk, tv, to;
    const float *q_norm, *k_norm;
    const void *const *gate;  /* n_experts host pointers each */
    const void *const *up;
    const void *const *down;
} KrefHybridLayer;

typedef struct KrefHybrid {
    int NL, H, vocab, cap, NH, NKV, HD, rd, nk, nv, dh, K, E, F, top_k, norm_topk, n_threads;
    uint32_t gate_t, up_t, down_t, embed_t, lm_t;
    float eps, theta;
    const void *embed, *lm;
    const float *out_norm;
    KrefHybridLayer *L;
    float *x, *xb, *tmp, *qkv, *cv, *z, *b, *a, *go, *qg, *q, *gt, *k, *v, *attn, *rl, *logits;
    float *kv_k, *kv_v, *ring, *state, *scores, *rope_inv, *rope_cos, *rope_sin;
    float *route_gap; /* per layer, last step: (top_k-th - (top_k+1)-th router logit) / |top_k-th| */
    void *moe_scratch;
} KrefHybrid;

void kref_hybrid_free(void *p) {
    KrefHybrid *m = (KrefHybrid *)p;
    if (!m) return;
    free(m->L); free(m->x); free(m->xb); free(m->tmp); free(m->qkv); free(m->cv); free(m->z);
    free(m->b); free(m->a); free(m->go); free(m->qg); free(m->q); free(m->gt); free(m->k);
    free(m->v); free(m->attn); free(m->rl); free(m->logits); free(m->kv_k); free(m->kv_v);
    free(m->ring); free(m->state); free(m->scores); free(m->rope_inv); free(m->rope_cos);
    free(m->rope_sin); free(m->route_gap);
    kref_moe_scratch_free(m->moe_scratch);
    free(m);
}

static int kh_count(const KrefHybrid *m, int kind) {
    int n = 0;
    for (int l = 0; l < m->NL; l++) n += m->L[l].kind == kind;
    return n;
}

void *kref_hybrid_new(const int32_t *dims /* NL H vocab cap NH NKV HD rope_dim nk nv dh K E F top_k norm_topk */,
                      float eps, float theta, const void *embed, uint32_t embed_t, const void *lm,
                      uint32_t lm_t, const float *out_norm, uint32_t gate_t, uint32_t up_t,
                      uint32_t down_t, const KrefHybridLayer *layers, int n_threads) {
    KrefHybrid *m = (KrefHybrid *)calloc(1, sizeof(*m));
    if (!m) return NULL;
    m->NL = dims[0]; m->H = dims[1]; m->vocab = dims[2]; m->cap = dims[3]; m->NH = dims[4];
    m->NKV = dims[5]; m->HD = dims[6]; m->nk = dims[8]; m->nv = dims[9]; m->dh = dims[10];
    m->K = dims[11]; m->E = dims[12]; m->F = dims[13]; m->top_k = dims[14]; m->norm_topk = dims[15];
    m->rd = (dims[7] == 0 || dims[7] > m->HD) ? m->HD : dims[7];
    m->eps = eps; m->theta = theta; m->embed = embed; m->embed_t = embed_t; m->lm = lm;
    m->lm_t = lm_t; m->out_norm = out_norm; m->gate_t = gate_t; m->up_t = up_t; m->down_t = down_t;
    m->n_threads = n_threads;
    m->L = (KrefHybridLayer *)malloc(sizeof(KrefHybridLayer) * (size_t)m->NL);
    memcpy(m->L, layers, sizeof(KrefHybridLayer) * (size_t)m->NL);
    const size_t H = (size_t)m->H, C = (size_t)(2 * m->nk + m->nv) * m->dh, VD = (size_t)m->nv * m->dh;
    const size_t QD = (size_t)m->NH * m->HD, KD = (size_t)m->NKV * m->HD;
    const int n_gdn = kh_count(m, 0), n_attn = kh_count(m, 1);
    m->x = calloc(H, 4); m->xb = calloc(H, 4); m->tmp = calloc(H, 4);
    m->qkv = calloc(C + 1, 4); m->cv = calloc(C + 1, 4); m->z = calloc(VD + 1, 4);
    m->b = calloc((size_t)m->nv + 1, 4); m->a = calloc((size_t)m->nv + 1, 4); m->go = calloc(VD + 1, 4);
    m->qg = calloc(2 * QD + 1, 4); m->q = calloc(QD + 1, 4); m->gt = calloc(QD + 1, 4);
    m->k = calloc(KD + 1, 4); m->v = calloc(KD + 1, 4); m->attn = calloc(QD + 1, 4);
    m->rl = calloc((size_t)m->E, 4); m->logits = calloc((size_t)m->vocab, 4);
    m->kv_k = calloc((size_t)n_attn * KD * m->cap + 1, 4);
    m->kv_v = calloc((size_t)n_attn * KD * m->cap + 1, 4);
    m->ring = calloc((size_t)n_gdn * m->K * C + 1, 4);
    m->state = calloc((size_t)n_gdn * VD * m->dh + 1, 4);
    m->scores = calloc((size_t)m->cap, 4);
    m->rope_inv = calloc((size_t)m->rd / 2 + 1, 4); m->rope_cos = calloc((size_t)m->rd / 2 + 1, 4);
    m->rope_sin = calloc((size_t)m->rd / 2 + 1, 4);
    for (int i = 0; i < m->rd / 2; i++)
        m->rope_inv[i] = 1.0f / powf(theta, (2.0f * (float)i) / (float)m->rd);
    m->moe_scratch = kref_moe_scratch_new(m->E, m->H, m->F, m->top_k);
    m->route_gap = calloc((size_t)m->NL + 1, 4);
    if (!m->x || !m->route_gap || !m->state || !m->ring || !m->kv_k || !m->kv_v || !m->moe_scratch) {
        kref_hybrid_free(m);
        return NULL;
    }
    return m;
}

void kref_hybrid_reset(void *p) {
    KrefHybrid *m = (KrefHybrid *)p;
    const size_t C = (size_t)(2 * m->nk + m->nv) * m->dh, VD = (size_t)m->nv * m->dh;
    const int n_gdn = kh_count(m, 0);
    memset(m->ring, 0, (size_t)n_gdn * m->K * C * 4);
    memset(m->state, 0, (size_t)n_gdn * VD * m->dh * 4);
}

static float kh_silu(float x) { return x / (1.0f + expf(-x)); }

/* The Gated DeltaNet decode step (restatement, see above) of one layer at position pos:
 * qkv (C), z (nv dh), b / a (nv) in; out (nv dh) = the gated RMSNorm of the recurrence. */
static void kref_gdn_step(const KrefHybrid *m, const KrefHybridLayer *L, int pos, float *ring,
                          float *state, float *out) {
    const int nk = m->nk, nv = m->nv, dh = m->dh, K = m->K, ratio = nv / nk;
    const int C = (2 * nk + nv) * dh;
    for (int c = 0; c < C; c++) {
        float acc = 0.0f;
        for (int j = 0; j < K - 1; j++) {
            const int t = pos - (K - 1) + j;
            const int slot = ((t % K) + K) % K;
            acc = acc + L->conv[(size_t)c * K + j] * ring[(size_t)slot * C + c];
        }
        acc = acc + L->conv[(size_t)c * K + K - 1] * m->qkv[c];
        m->cv[c] = kh_silu(acc);
    }
    for (int c = 0; c < C; c++) ring[(size_t)(pos % K) * C + c] = m->qkv[c];
    const float scale = 1.0f / sqrtf((float)dh);
    for (int h = 0; h < 2 * nk; h++) {
        float *v = m->cv + (size_t)h * dh;
        double ss = 0.0;
        for (int i = 0; i < dh; i++) ss += (double)v[i] * (double)v[i];
        const float inv = 1.0f / sqrtf((float)ss + 1e-6f);
        for (int i = 0; i < dh; i++) v[i] = h < nk ? v[i] * inv * scale : v[i] * inv;
    }
    float *o = m->tmp; /* dh floats (H >= dh) */
    for (int vh = 0; vh < nv; vh++) {
        const int kh = vh / ratio;
        const float *q = m->cv + (size_t)kh * dh, *k = m->cv + (size_t)(nk + kh) * dh;
        const float *v = m->cv + (size_t)(2 * nk) * dh + (size_t)vh * dh;
        const float beta = 1.0f / (1.0f + expf(-m->b[vh]));
        const float xa = m->a[vh] + L->dt_bias[vh];
        const float sp = xa > 20.0f ? xa : log1pf(expf(xa));
        const float g = -(expf(L->a_log[vh]) * sp);
        const float decay = expf(g);
        float *S = state + (size_t)vh * dh * dh;
        for (int j = 0; j < dh; j++) {
            float *col = S + (size_t)j * dh;
            double kv = 0.0;
            for (int i = 0; i < dh; i++) {
                col[i] = col[i] * decay;
                kv += (double)col[i] * (double)k[i];
            }
            const float delta = (v[j] - (float)kv) * beta;
            double acc = 0.0;
            for (int i = 0; i < dh; i++) {
                col[i] = col[i] + k[i] * delta;
                acc += (double)col[i] * (double)q[i];
            }
            o[j] = (float)acc;
        }
        double ss = 0.0;
        for (int j = 0; j < dh; j++) ss += (double)o[j] * (double)o[j];
        const float inv = 1.0f / sqrtf((float)(ss / (double)dh) + m->eps);
        for (int j = 0; j < dh; j++)
            out[(size_t)vh * dh + j] = o[j] * inv * L->ssm_norm[j] * kh_silu(m->z[(size_t)vh * dh + j]);
    }
}

/* Margin of a routing decision: (k-th largest - (k+1)-th largest logit) / |k-th largest|.
 * Two implementations whose router logits differ by a relative ~1e-7 can select different
 * experts only where this margin is of that order. */
static float kref_route_gap(const float *lg, int n, int k) {
    if (k <= 0 || k >= n || k > 16) return 1.0f;
    float top[17];  /* the k + 1 largest logits so far, descending */
    int cnt = 0;
    for (int i = 0; i < n; i++) {
        const float v = lg[i];
        if (cnt == k + 1 && !(v > top[k])) continue;
        int j = cnt < k + 1 ? cnt++ : k;
        while (j > 0 && top[j - 1] < v) { top[j] = top[j - 1]; j--; }
        top[j] = v;
    }
    const float a = fabsf(top[k - 1]);
    return (top[k - 1] - top[k]) / (a > 0.0f ? a : 1.0f);
}

/* The routing margins of every layer at the last step (NL floats). */
void kref_hybrid_route_gaps(const void *p, float *out) {
    const KrefHybrid *m = (const KrefHybrid *)p;
    memcpy(out, m->route_gap, (size_t)m->NL * 4);
}

/* One step at position pos with input token; logits_out may be NULL. */
int kref_hybrid_step(void *p, int token, int pos, float *logits_out) {
    KrefHybrid *m = (KrefHybrid *)p;
    if (!m || token < 0 || token >= m->vocab || pos < 0 || pos >= m->cap) return -1;
    const int H = m->H, NH = m->NH, NKV = m->NKV, HD = m->HD, nt = m->n_threads;
    const int nv = m->nv, dh = m->dh, C = (2 * m->nk + nv) * dh;
    const uint64_t erb = katali_ggml_row_bytes(m->embed_t, (uint64_t)H);
    if (katali_ggml_dequant_ref(m->embed_t, (const uint8_t *)m->embed + (size_t)token * erb,
                                (uint64_t)H, m->x) != 0)
        return -1;
    const int half = m->rd / 2;
    for (int i = 0; i < half; i++) {
        const float freq = (float)pos * m->rope_inv[i];
        m->rope_cos[i] = cosf(freq);
        m->rope_sin[i] = sinf(freq);
    }
    const size_t KD = (size_t)NKV * HD, QD = (size_t)NH * HD;
    int gi = 0, ai = 0;
    for (int l = 0; l < m->NL; l++) {
        const KrefHybridLayer *L = &m->L[l];
        katali_gguf_rmsnorm(m->x, L->attn_norm, (size_t)H, m->eps, m->xb);
        if (L->kind == 0) {
            kref_matvec(L->t_qkv, L->w_qkv, (uint64_t)C, (uint64_t)H, m->xb, m->qkv, nt);
            kref_matvec(L->t_z, L->w_z, (uint64_t)nv * dh, (uint64_t)H, m->xb, m->z, nt);
            kref_matvec(L->t_b, L->w_b, (uint64_t)nv, (uint64_t)H, m->xb, m->b, nt);
            kref_matvec(L->t_a, L->w_a, (uint64_t)nv, (uint64_t)H, m->xb, m->a, nt);
            float *ring = m->ring + (size_t)gi * m->K * C;
            float *state = m->state + (size_t)gi * nv * dh * dh;
            gi++;
            kref_gdn_step(m, L, pos, ring, state, m->go);
            kref_matvec(L->t_out, L->w_out, (uint64_t)H, (uint64_t)nv * dh, m->go, m->tmp, nt);
        } else {
            kref_matvec(L->tq, L->wq, (uint64_t)2 * QD, (uint64_t)H, m->xb, m->qg, nt);
            for (int h = 0; h < NH; h++) {
                memcpy(m->q + (size_t)h * HD, m->qg + (size_t)h * 2 * HD, (size_t)HD * 4);
                memcpy(m->gt + (size_t)h * HD, m->qg + (size_t)h * 2 * HD + HD, (size_t)HD * 4);
            }
            kref_matvec(L->tk, L->wk, (uint64_t)KD, (uint64_t)H, m->xb, m->k, nt);
            kref_matvec(L->tv, L->wv, (uint64_t)KD, (uint64_t)H, m->xb, m->v, nt);
            if (L->q_norm)
                for (int h = 0; h < NH; h++)
                    katali_gguf_rmsnorm_inplace(m->q + (size_t)h * HD, L->q_norm, (size_t)HD, m->eps);
            katali_gguf_rope_apply(m->q, (size_t)NH, (size_t)HD, (size_t)m->rd, m->rope_cos, m->rope_sin);
            if (L->k_norm)
                for (int h = 0; h < NKV; h++)
                    katali_gguf_rmsnorm_inplace(m->k + (size_t)h * HD, L->k_norm, (size_t)HD, m->eps);
            katali_gguf_rope_apply(m->k, (size_t)NKV, (size_t)HD, (size_t)m->rd, m->rope_cos, m->rope_sin);
            float *lk = m->kv_k + (size_t)ai * KD * m->cap, *lv = m->kv_v + (size_t)ai * KD * m->cap;
            ai++;
            for (int h = 0; h < NKV; h++) {
                memcpy(lk + ((size_t)h * m->cap + pos) * HD, m->k + (size_t)h * HD, (size_t)HD * 4);
                memcpy(lv + ((size_t)h * m->cap + pos) * HD, m->v + (size_t)h * HD, (size_t)HD * 4);
            }
            katali_gguf_gqa_decode_scratch(m->q, lk, lv, (size_t)pos + 1, (size_t)m->cap, (size_t)NH,
                                           (size_t)NKV, (size_t)HD, m->attn, m->scores);
            for (size_t i = 0; i < QD; i++) m->attn[i] = m->attn[i] * katali_gguf_sigmoid(m->gt[i]);
            kref_matvec(L->to, L->wo, (uint64_t)H, (uint64_t)QD, m->attn, m->tmp, nt);
        }
        katali_gguf_add_inplace(m->x, m->tmp, (size_t)H);
        katali_gguf_rmsnorm(m->x, L->ffn_norm, (size_t)H, m->eps, m->xb);
        kref_matvec(KGGML_F32, L->router, (uint64_t)m->E, (uint64_t)H, m->xb, m->rl, nt);
        m->route_gap[l] = kref_route_gap(m->rl, m->E, m->top_k);
        if (kref_moe_layer(m->E, H, m->F, m->top_k, m->norm_topk, m->gate_t, m->up_t, m->down_t,
                           L->gate, L->up, L->down, m->xb, m->rl, m->tmp, nt, m->moe_scratch,
                           NULL, NULL) != 0)
            return -1;
        katali_gguf_add_inplace(m->x, m->tmp, (size_t)H);
    }
    katali_gguf_rmsnorm(m->x, m->out_norm, (size_t)H, m->eps, m->xb);
    kref_matvec(m->lm_t, m->lm, (uint64_t)m->vocab, (uint64_t)H, m->xb, m->logits, nt);
    if (logits_out) memcpy(logits_out, m->logits, (size_t)m->vocab * 4);
    return 0;
}

/* T decode steps of one Gated DeltaNet mixer from zero conv and recurrent state (the
 * restatement above, for the CPU test that checks it against a matrix-form formulation):
 * qkv [T][(2 nk + nv) dh], z [T][nv dh], b / a [T][nv] in, out [T][nv dh]. */
int kref_gdn_apply(int nk, int nv, int dh, int K, int T, float eps, const float *conv,
                   const float *a_log, const float *dt_bias, const float *norm_w,
                   const float *qkv, const float *z, const float *b, const float *a, float *out) {
    KrefHybrid m;
    memset(&m, 0, sizeof m);
    m.nk = nk; m.nv = nv; m.dh = dh; m.K = K; m.eps = eps;
    const size_t C = (size_t)(2 * nk + nv) * dh, VD = (size_t)nv * dh;
    KrefHybridLayer L;
    memset(&L, 0, sizeof L);
    L.conv = conv; L.a_log = a_log; L.dt_bias = dt_bias; L.ssm_norm = norm_w;
    m.qkv = calloc(C, 4); m.cv = calloc(C, 4); m.z = calloc(VD, 4); m.b = calloc((size_t)nv, 4);
    m.a = calloc((size_t)nv, 4); m.tmp = calloc((size_t)dh, 4);
    float *ring = calloc((size_t)K * C, 4), *state = calloc(VD * (size_t)dh, 4);
    int rc = (m.qkv && m.cv && m.z && m.b && m.a && m.tmp && ring && state) ? 0 : -1;
    for (int t = 0; rc == 0 && t < T; t++) {
        memcpy(m.qkv, qkv + (size_t)t * C, C * 4);
        memcpy(m.z, z + (size_t)t * VD, VD * 4);
        memcpy(m.b, b + (size_t)t * nv, (size_t)nv * 4);
        memcpy(m.a, a + (size_t)t * nv, (size_t)nv * 4);
        kref_gdn_step(&m, &L, t, ring, state, out + (size_t)t * VD);
    }
    free(m.qkv); free(m.cv); free(m.z); free(m.b); free(m.a); free(m.tmp); free(ring); free(state);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* The reference's GGUF reader (V/src/gguf_reader.c, katali_gguf_open and the */
/* getters of V/include/katali_gguf.h:117-152) behind a handle, so the tests  */
/* can compare the plugin's reader with it on the same files.                 */
/* ------------------------------------------------------------------------ */
#include "katali_gguf.h"

void *kref_gguf_open(const char *path, char *err, int err_cap) {
    KataliGgufFile *f = (KataliGgufFile *)calloc(1, sizeof(*f));
    if (!f) return NULL;
    if (katali_gguf_open(f, path, 1, err, (size_t)err_cap) != 0) {
        free(f);
        return NULL;
    }
    return f;
}

void kref_gguf_close(void *p) {
    if (!p) return;
    katali_gguf_close((KataliGgufFile *)p);
    free(p);
}

void kref_gguf_counts(void *p, uint64_t *nt, uint64_t *nkv, uint32_t *version) {
    const KataliGgufFile *f = (const KataliGgufFile *)p;
    *nt = f->tensor_count;
    *nkv = f->kv_count;
    *version = f->version;
}

/* Tensor i: name, type, n_dims, dims[4], absolute file offset of its data (or 0 when
 * the reader exposes no data pointer), nbytes. */
int kref_gguf_tensor(void *p, uint64_t i, const char **name, uint32_t *type, uint32_t *n_dims,
                     uint64_t *dims, uint64_t *abs_off, uint64_t *nbytes) {
    const KataliGgufFile *f = (const KataliGgufFile *)p;
    if (i >= f->tensor_count) return -1;
    const KataliGgufTensor *t = &f->tensors[i];
    *name = t->name;
    *type = t->type;
    *n_dims = t->n_dims;
    for (uint32_t d = 0; d < 4; d++) dims[d] = d < t->n_dims ? t->dims[d] : 1;
    *abs_off = t->data ? (uint64_t)(t->data - f->map) : 0;
    *nbytes = t->nbytes;
    return 0;
}

int64_t kref_gguf_get_int(void *p, const char *key, int64_t def) {
    return katali_gguf_get_int((const KataliGgufFile *)p, key, def);
}
double kref_gguf_get_float(void *p, const char *key, double def) {
    return katali_gguf_get_float((const KataliGgufFile *)p, key, def);
}
const char *kref_gguf_get_str(void *p, const char *key, size_t *len) {
    return katali_gguf_get_str((const KataliGgufFile *)p, key, NULL, len);
}
int64_t kref_gguf_array_len(void *p, const char *key, uint32_t *et) {
    return katali_gguf_array_len((const KataliGgufFile *)p, key, et);
}
int64_t kref_gguf_array_int(void *p, const char *key, uint64_t i) {
    return katali_gguf_array_int((const KataliGgufFile *)p, key, i);
}
