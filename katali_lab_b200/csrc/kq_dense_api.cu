// kq_dense_api.cu — host side of the on-device dense decoder (katali_cuda_dense_*):
// validation, device buffers, the RoPE table, the per-layer GEMV jobs and greedy
// generation by replaying one captured CUDA graph per step.
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <vector>

#include "katali_cuda.h"
#include "kq_launch.h"

namespace kq {
int ensure_runtime();
void set_status_message(const char *msg);
cudaStream_t current_stream();
volatile uint32_t *device_status_word();
int take_status_after_sync();
}  // namespace kq

namespace {

uint64_t rbytes(uint32_t type, uint64_t cols) {
    if (cols % 256) return 0;
    if (type == KATALI_TYPE_Q4_K) return cols / 256 * 144;
    if (type == KATALI_TYPE_Q6_K) return cols / 256 * 210;
    return 0;
}
bool a16(const void *p) { return p && ((uintptr_t)p & 15u) == 0; }

int bad(const char *why) {
    kq::set_status_message(why);
    return KATALI_ERR_BAD_ARG;
}

}  // namespace

struct KataliDense {
    KataliDenseDesc d;
    std::vector<KataliDenseLayerW> lw;
    std::vector<kq::DenseLayer> L;
    std::vector<kq::GemvParams> g;  // 4 per layer + LM head
    kq::DenseParams p;
    void *mem = nullptr;            // one allocation for all buffers
    const float **qn_dev = nullptr, **kn_dev = nullptr;
    int pos = 0;                    // host copy of the next position
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaStream_t graph_stream = nullptr;
    void *weights = nullptr;        // weight memory owned for the caller (a decoder made from a file)
};

namespace kq {
// A decoder created from a model file owns the device memory its weights were uploaded to.
void dense_adopt_weights(KataliDense *m, void *mem) { m->weights = mem; }
}  // namespace kq

namespace {

kq::GemvParams gemv_job(const float *x, uint64_t cols, int n, const void *const *w,
                        const uint32_t *types, const uint64_t *rows, float *const *y, int accum,
                        const float *norm_w = nullptr, float eps = 0.0f,
                        const float *x_mul = nullptr) {
    kq::GemvParams g = {};
    g.njobs = n;
    g.cols = (uint32_t)cols;
    g.x = x;
    g.norm_w = norm_w;
    g.norm_eps = eps;
    g.x_mul = x_mul;
    g.status = kq::device_status_word();
    g.pdl = 1;  // programmatic dependent of the previous launch of the decode step
    for (int j = 0; j < n; ++j) {
        g.job[j].w = (const uint8_t *)w[j];
        g.job[j].y = y[j];
        g.job[j].rows = rows[j];
        g.job[j].type = types[j];
        g.job[j].rb = (uint32_t)rbytes(types[j], cols);
        g.job[j].accum = (uint32_t)accum;
    }
    return g;
}

}  // namespace

extern "C" {

int katali_cuda_dense_create(const KataliDenseDesc *d, KataliDense **out) {
    if (!d || !out || !d->layers) return KATALI_ERR_BAD_ARG;
    *out = nullptr;
    // device, own stream and mapped status word (KATALI_ERR_NO_DEVICE without a usable GPU)
    if (const int rs = kq::ensure_runtime()) return rs;
    const uint32_t H = d->hidden, F = d->ffn, NH = d->n_heads, NKV = d->n_kv_heads, HD = d->head_dim;
    if (!d->n_layers || !H || !F || !NH || !NKV || !HD || !d->vocab || !d->kv_cap)
        return bad("katali_cuda_dense_create: zero dimension");
    if (NH % NKV || HD > 512 || HD % 32 || H % 256 || F % 256 || (NH * HD) % 256)
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    if (d->flags & ~KATALI_DENSE_Q8_1) return bad("katali_cuda_dense_create: unknown flags");
    // widest projection input (fp32 staging in the GEMV): fp32 24576 columns, q8_1 65536
    if ((d->flags & KATALI_DENSE_Q8_1) ? (F > 65536 || NH * HD > 65536) : (F > 24576 || NH * HD > 24576))
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    const uint32_t rd = (d->rope_dim == 0 || d->rope_dim > HD) ? HD : d->rope_dim;
    if ((uint64_t)d->kv_cap * 4 > 200 * 1024) return KATALI_ERR_UNSUPPORTED_SHAPE;  // scores in smem
    if (!rbytes(d->embed_type, H) || !rbytes(d->lm_head_type, H) || !a16(d->embed) ||
        !a16(d->lm_head) || !d->out_norm)
        return bad("katali_cuda_dense_create: embedding / LM head");
    for (uint32_t l = 0; l < d->n_layers; ++l) {
        const KataliDenseLayerW &w = d->layers[l];
        if (!w.attn_norm || !w.ffn_norm) return bad("katali_cuda_dense_create: layer norms");
        const void *m[7] = {w.wq, w.wk, w.wv, w.wo, w.gate, w.up, w.down};
        const uint32_t t[7] = {w.wq_type, w.wk_type, w.wv_type, w.wo_type, w.gate_type, w.up_type,
                               w.down_type};
        const uint32_t cols[7] = {H, H, H, NH * HD, H, H, F};
        for (int i = 0; i < 7; ++i) {
            if (!a16(m[i])) return bad("katali_cuda_dense_create: weight pointer");
            if (!rbytes(t[i], cols[i]) || rbytes(t[i], cols[i]) % 2)
                return KATALI_ERR_UNSUPPORTED_TYPE;
        }
    }
    KataliDense *m = new KataliDense();
    m->d = *d;
    m->lw.assign(d->layers, d->layers + d->n_layers);
    m->d.layers = m->lw.data();

    // one device allocation: activations, KV cache, RoPE table, control words
    const size_t NL = d->n_layers, cap = d->kv_cap, rh = rd / 2;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) & ~(size_t)255;
        return o;
    };
    const size_t o_x = take(4 * H), o_xb = take(4 * H), o_q = take(4ull * NH * HD),
                 o_k = take(4ull * NKV * HD), o_v = take(4ull * NKV * HD), o_attn = take(4ull * NH * HD),
                 o_gate = take(4ull * F), o_up = take(4ull * F), o_logits = take(4ull * d->vocab),
                 o_kk = take(4 * NL * NKV * cap * HD), o_kv = take(4 * NL * NKV * cap * HD),
                 o_cos = take(4 * cap * rh), o_sin = take(4 * cap * rh), o_ctl = take(64),
                 o_forced = take(4 * cap), o_out = take(4 * cap), o_av = take(4 * 148),
                 o_ai = take(4 * 148), o_qn = take(8 * NL), o_kn = take(8 * NL);
    cudaError_t e = cudaMalloc(&m->mem, off);
    if (e != cudaSuccess) {
        delete m;
        kq::set_status_message(cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : KATALI_ERR_CUDA;
    }
    unsigned char *b = (unsigned char *)m->mem;
    kq::DenseParams &p = m->p;
    memset(&p, 0, sizeof p);
    p.H = (int)H;
    p.F = (int)F;
    p.NH = (int)NH;
    p.NKV = (int)NKV;
    p.HD = (int)HD;
    p.NL = (int)NL;
    p.vocab = (int)d->vocab;
    p.kv_cap = (int)cap;
    p.rope_half = (int)rh;
    p.eps = d->rms_eps;
    p.gemv_mode = (d->flags & KATALI_DENSE_Q8_1) ? 0 : 2;
    p.attn_scale = 1.0f / sqrtf((float)HD);  // as the reference's attention (gguf_kernels.c)
    p.embed = (const uint8_t *)d->embed;
    p.embed_type = d->embed_type;
    p.embed_rb = (uint32_t)rbytes(d->embed_type, H);
    p.out_norm = d->out_norm;
    p.x = (float *)(b + o_x);
    p.xb = (float *)(b + o_xb);
    p.q = (float *)(b + o_q);
    p.k = (float *)(b + o_k);
    p.v = (float *)(b + o_v);
    p.attn = (float *)(b + o_attn);
    p.gate = (float *)(b + o_gate);
    p.up = (float *)(b + o_up);
    p.logits = (float *)(b + o_logits);
    p.kv_k = (float *)(b + o_kk);
    p.kv_v = (float *)(b + o_kv);
    p.rope_cos = (const float *)(b + o_cos);
    p.rope_sin = (const float *)(b + o_sin);
    int *ctl = (int *)(b + o_ctl);
    p.tok = ctl;
    p.pos = ctl + 1;
    p.step = ctl + 2;
    p.n_forced = ctl + 3;
    p.forced = (const int *)(b + o_forced);
    p.out_tokens = (int *)(b + o_out);
    p.out_cap = (int)cap;
    p.arg_v = (float *)(b + o_av);
    p.arg_i = (int *)(b + o_ai);
    m->qn_dev = (const float **)(b + o_qn);
    m->kn_dev = (const float **)(b + o_kn);
    p.q_norm_dev = m->qn_dev;
    p.k_norm_dev = m->kn_dev;

    // RoPE table with the reference's own libm calls (rope_prepare, gguf_model.c:466-475;
    // rope_inv from :344): bit-identical cos/sin on every position.
    std::vector<float> inv(rh), cs(cap * rh), sn(cap * rh);
    for (size_t i = 0; i < rh; ++i)
        inv[i] = 1.0f / powf(d->rope_theta, (2.0f * (float)i) / (float)rd);
    for (size_t t = 0; t < cap; ++t)
        for (size_t i = 0; i < rh; ++i) {
            const float f = (float)t * inv[i];
            cs[t * rh + i] = cosf(f);
            sn[t * rh + i] = sinf(f);
        }
    std::vector<const float *> qn(NL), kn(NL);
    m->L.resize(NL);
    for (size_t l = 0; l < NL; ++l) {
        qn[l] = m->lw[l].q_norm;
        kn[l] = m->lw[l].k_norm;
        m->L[l] = kq::DenseLayer{m->lw[l].attn_norm, m->lw[l].ffn_norm};
    }
    p.L = m->L.data();
    cudaStream_t st = kq::current_stream();
    e = cudaMemcpyAsync((void *)p.rope_cos, cs.data(), 4 * cap * rh, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync((void *)p.rope_sin, sn.data(), 4 * cap * rh, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->qn_dev, qn.data(), 8 * NL, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->kn_dev, kn.data(), 8 * NL, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctl, 0, 64, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) e = kq::dense_set_attention_smem((int)cap);
    if (e != cudaSuccess) {
        kq::set_status_message(cudaGetErrorString(e));
        katali_cuda_dense_destroy(m);
        return KATALI_ERR_CUDA;
    }

    // GEMV jobs: per layer qkv (x = xb), o (+= into x), gate/up (x = xb), down (+= into x)
    m->g.resize(4 * NL + 1);
    for (size_t l = 0; l < NL; ++l) {
        const KataliDenseLayerW &w = m->lw[l];
        {
            const void *ws[3] = {w.wq, w.wk, w.wv};
            const uint32_t ts[3] = {w.wq_type, w.wk_type, w.wv_type};
            const uint64_t rows[3] = {(uint64_t)NH * HD, (uint64_t)NKV * HD, (uint64_t)NKV * HD};
            float *ys[3] = {p.q, p.k, p.v};
            m->g[4 * l] = gemv_job(p.x, H, 3, ws, ts, rows, ys, 0, w.attn_norm, d->rms_eps);
        }
        {
            const void *ws[1] = {w.wo};
            const uint32_t ts[1] = {w.wo_type};
            const uint64_t rows[1] = {H};
            float *ys[1] = {p.x};
            m->g[4 * l + 1] = gemv_job(p.attn, (uint64_t)NH * HD, 1, ws, ts, rows, ys, 1);
        }
        {
            const void *ws[2] = {w.gate, w.up};
            const uint32_t ts[2] = {w.gate_type, w.up_type};
            const uint64_t rows[2] = {F, F};
            float *ys[2] = {p.gate, p.up};
            m->g[4 * l + 2] = gemv_job(p.x, H, 2, ws, ts, rows, ys, 0, w.ffn_norm, d->rms_eps);
        }
        {
            const void *ws[1] = {w.down};
            const uint32_t ts[1] = {w.down_type};
            const uint64_t rows[1] = {H};
            float *ys[1] = {p.x};
            m->g[4 * l + 3] = gemv_job(p.gate, F, 1, ws, ts, rows, ys, 1);
        }
    }
    {
        const void *ws[1] = {d->lm_head};
        const uint32_t ts[1] = {d->lm_head_type};
        const uint64_t rows[1] = {d->vocab};
        float *ys[1] = {p.logits};
        m->g[4 * NL] = gemv_job(p.x, H, 1, ws, ts, rows, ys, 0, d->out_norm, d->rms_eps);
    }
    *out = m;
    return KATALI_OK;
}

int katali_cuda_dense_destroy(KataliDense *m) {
    if (!m) return KATALI_OK;
    cudaStream_t st = kq::current_stream();
    if (st) cudaStreamSynchronize(st);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    cudaFree(m->mem);
    cudaFree(m->weights);
    delete m;
    return KATALI_OK;
}

int katali_cuda_dense_reset(KataliDense *m) {
    if (!m) return KATALI_ERR_BAD_ARG;
    m->pos = 0;
    const cudaError_t e = cudaMemsetAsync(m->p.pos, 0, sizeof(int), kq::current_stream());
    return e == cudaSuccess ? KATALI_OK : KATALI_ERR_CUDA;
}

int katali_cuda_dense_generate(KataliDense *m, const int32_t *prompt, uint32_t n_prompt,
                               uint32_t n_gen, int32_t *out_tokens) {
    if (!m || !prompt || n_prompt == 0 || n_gen == 0 || !out_tokens) return KATALI_ERR_BAD_ARG;
    const uint64_t steps = (uint64_t)n_prompt + n_gen - 1;
    if ((uint64_t)m->pos + steps > (uint64_t)m->p.kv_cap) {
        kq::set_status_message("katali_cuda_dense_generate: KV cache full (kv_cap)");
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    }
    for (uint32_t i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || (uint32_t)prompt[i] >= m->d.vocab) return KATALI_ERR_BAD_ARG;
    cudaStream_t st = kq::current_stream();
    const int ctl[4] = {prompt[0], m->pos, 0, (int)n_prompt};
    // control words: tok, pos (unchanged), step = 0, n_forced
    cudaError_t e = cudaMemcpyAsync((void *)m->p.forced, prompt, 4ull * n_prompt,
                                    cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->p.tok, ctl, sizeof ctl, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return KATALI_ERR_CUDA;
    for (uint64_t s = 0; s < steps; ++s) {
        if (!m->exec || m->graph_stream != st) {
            // First step on this stream: run it eagerly (sets kernel attributes), then
            // capture the same launch sequence once for the following steps.
            e = kq::launch_dense_step(m->p, m->g.data(), st);
            if (e != cudaSuccess) break;
            if (m->exec) {
                cudaGraphExecDestroy(m->exec);
                cudaGraphDestroy(m->graph);
                m->exec = nullptr;
                m->graph = nullptr;
            }
            cudaStream_t cap;
            e = cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking);
            if (e != cudaSuccess) break;
            cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
            cudaError_t le = kq::launch_dense_step(m->p, m->g.data(), cap);
            e = cudaStreamEndCapture(cap, &m->graph);
            cudaStreamDestroy(cap);
            if (le != cudaSuccess) e = le;
            if (e == cudaSuccess) e = cudaGraphInstantiate(&m->exec, m->graph, 0);
            if (e != cudaSuccess) break;
            m->graph_stream = st;
            continue;
        }
        e = cudaGraphLaunch(m->exec, st);
        if (e != cudaSuccess) break;
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(out_tokens, m->p.out_tokens + (n_prompt - 1), 4ull * n_gen,
                            cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        kq::set_status_message(cudaGetErrorString(e));
        return KATALI_ERR_CUDA;
    }
    m->pos += (int)steps;
    return kq::take_status_after_sync();
}

int katali_cuda_dense_logits(KataliDense *m, const float **logits_dev, int32_t *position) {
    if (!m) return KATALI_ERR_BAD_ARG;
    if (logits_dev) *logits_dev = m->p.logits;
    if (position) *position = m->pos;
    return KATALI_OK;
}

}  // extern "C"
