// kq_hybrid_api.cu — host side of the on-device hybrid MoE decoder (katali_cuda_hybrid_*):
// validation, one device allocation for activations / states / KV cache / RoPE table, the
// per-layer GEMV jobs and fused MoE launches, and greedy generation by replaying one captured
// CUDA graph per step.
#include <cuda_runtime.h>
#include <math.h>
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
int moe_fused_params(KataliMoe *m, uint32_t mode, MoeParams *p, int *grid);
int moe_ep_fused_params(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens, uint32_t n_tokens,
                        const float *x, const float *router_logits, float *y, const EpPeer *pp,
                        double *ret_scratch, MoeParams *out, int *grid);
int ep_peer_prepare(KataliEp *ep, KataliMoe *m, uint32_t max_tokens, uint32_t *n_ranks,
                    const EpPeer **pp, double **ret);
// Resources a decoder made from a file owns: device allocations, the MoE objects, page-locked
// host ranges; with a cache, its experts are fed through it (keys layer * n_experts + e).
void hybrid_adopt(KataliHybrid *m, std::vector<void *> allocs, std::vector<KataliMoe *> moes,
                  std::vector<void *> pinned, KataliExpertCache *cache);
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
int unsupported(const char *why) {
    kq::set_status_message(why);
    return KATALI_ERR_UNSUPPORTED_SHAPE;
}

kq::GemvParams gemv_jobs(const float *x, uint64_t cols, int n, const void *const *w,
                         const uint32_t *types, const uint64_t *rows, float *const *y, int accum,
                         const float *norm_w, float eps) {
    kq::GemvParams g = {};
    g.njobs = n;
    g.cols = (uint32_t)cols;
    g.x = x;
    g.norm_w = norm_w;
    g.norm_eps = eps;
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

struct KataliHybrid;
namespace {
int bind_routed(void *ctx, int layer);
}

struct KataliHybrid {
    KataliHybridDesc d;
    std::vector<KataliHybridLayerW> lw;
    std::vector<kq::HybridLayer> L;
    std::vector<kq::GemvParams> g;  // 2 per layer + LM head
    std::vector<kq::MoeParams> moe;       // the launches the step uses
    std::vector<int> moe_grid;
    std::vector<kq::MoeParams> moe_local;  // single-GPU launches (kept while expert-parallel)
    std::vector<int> grid_local;
    std::vector<kq::MoeParams> moe_sep;    // the same with the router as its own kernel
    // owned when made from a file (katali_cuda_hybrid_create_from_gguf)
    std::vector<void *> own_allocs, own_pinned;
    std::vector<KataliMoe *> own_moe;
    KataliExpertCache *cache = nullptr;    // residency mode: experts bound per step
    int32_t *route_dev = nullptr;          // [2 * top_k]: one routing decision (ids, weights)
    uint32_t n_experts = 0, top_k = 0;
    kq::HybridParams p;
    void *mem = nullptr;
    size_t state_off = 0, state_bytes = 0;  // GDN states + conv rings (zeroed by reset)
    int pos = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaStream_t graph_stream = nullptr;
};

namespace {
// Residency mode, after layer l's router: the routing decision of the MoE kernel itself
// (its route-only launch on the router logits), read back, then every selected expert bound
// through the cache (uploaded from the host mapping when not on the device; the MoE launch
// that follows waits for the upload).
int bind_routed(void *ctx, int layer) {
    KataliHybrid *m = (KataliHybrid *)ctx;
    KataliMoe *moe = m->lw[(size_t)layer].moe;
    const uint32_t K = m->top_k;
    int s = katali_cuda_debug_route(moe, m->p.rlogits, m->route_dev, (float *)(m->route_dev + K));
    if (s) return s;
    int32_t ids[kq::MOE_MAX_K];
    cudaStream_t st = kq::current_stream();
    cudaError_t e = cudaMemcpyAsync(ids, m->route_dev, 4ull * K, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        kq::set_status_message(cudaGetErrorString(e));
        return KATALI_ERR_CUDA;
    }
    for (uint32_t k = 0; k < K; ++k) {
        if (ids[k] < 0 || (uint32_t)ids[k] >= m->n_experts) return KATALI_ERR_CUDA;
        s = katali_cuda_expert_bind(m->cache, (uint64_t)layer * m->n_experts + (uint64_t)ids[k], moe,
                                    (uint32_t)ids[k]);
        if (s) return s;
    }
    return KATALI_OK;
}
}  // namespace

namespace kq {
void hybrid_adopt(KataliHybrid *m, std::vector<void *> allocs, std::vector<KataliMoe *> moes,
                  std::vector<void *> pinned, KataliExpertCache *cache) {
    m->own_allocs = std::move(allocs);
    m->own_moe = std::move(moes);
    m->own_pinned = std::move(pinned);
    m->cache = cache;
}
}  // namespace kq

extern "C" {

int katali_cuda_hybrid_create(const KataliHybridDesc *d, KataliHybrid **out) {
    if (!d || !out || !d->layers) return KATALI_ERR_BAD_ARG;
    *out = nullptr;
    // device, own stream and mapped status word (KATALI_ERR_NO_DEVICE without a usable GPU)
    if (const int rs = kq::ensure_runtime()) return rs;
    const uint32_t H = d->hidden, NH = d->n_heads, NKV = d->n_kv_heads, HD = d->head_dim;
    const uint32_t nk = d->ssm_k_heads, nv = d->ssm_v_heads, dh = d->ssm_head_dim, ck = d->ssm_conv;
    if (!d->n_layers || !H || !d->vocab || !d->kv_cap) return bad("katali_cuda_hybrid_create: zero dimension");
    if (d->flags & ~KATALI_DENSE_Q8_1) return bad("katali_cuda_hybrid_create: unknown flags");
    if (H % 256 || H > 8192) return unsupported("katali_cuda_hybrid_create: hidden");
    uint32_t n_gdn = 0, n_attn = 0, n_experts = 0;
    for (uint32_t l = 0; l < d->n_layers; ++l) {
        const KataliHybridLayerW &w = d->layers[l];
        if (w.kind == KATALI_HYBRID_GDN) ++n_gdn;
        else if (w.kind == KATALI_HYBRID_ATTN) ++n_attn;
        else return bad("katali_cuda_hybrid_create: layer kind");
    }
    if (n_gdn && (dh != 128 || !nk || !nv || nv % nk || ck < 2 || ck > 8))
        return unsupported("katali_cuda_hybrid_create: GDN heads (head dim 128, v heads a multiple of k heads, conv 2..8)");
    if (n_attn && (!NH || !NKV || NH % NKV || HD == 0 || HD > 256 || HD % 32 || (NH * HD) % 256))
        return unsupported("katali_cuda_hybrid_create: attention heads (head_dim <= 256)");
    if (n_attn && (uint64_t)d->kv_cap * 4 > 200 * 1024)
        return unsupported("katali_cuda_hybrid_create: kv_cap (attention scores in shared memory)");
    const bool q8 = (d->flags & KATALI_DENSE_Q8_1) != 0;
    const uint64_t max_cols = q8 ? 65536 : 24576;  // widest GEMV input staged per CTA
    if ((uint64_t)nv * dh > max_cols || (uint64_t)NH * HD > max_cols)
        return unsupported("katali_cuda_hybrid_create: projection width");
    if (!rbytes(d->embed_type, H) || !rbytes(d->lm_head_type, H) || !a16(d->embed) ||
        !a16(d->lm_head) || !d->out_norm)
        return bad("katali_cuda_hybrid_create: embedding / LM head");
    const uint32_t C = 2 * nk * dh + nv * dh;
    for (uint32_t l = 0; l < d->n_layers; ++l) {
        const KataliHybridLayerW &w = d->layers[l];
        if (!w.attn_norm || !w.ffn_norm || !a16(w.router) || !w.moe)
            return bad("katali_cuda_hybrid_create: layer norms / router / MoE");
        if (w.kind == KATALI_HYBRID_GDN) {
            if (!w.ssm_conv || (!w.ssm_a_log && !w.ssm_decay) || !w.ssm_dt_bias || !w.ssm_norm)
                return bad("katali_cuda_hybrid_create: GDN parameters");
            const void *m[5] = {w.ssm_qkv, w.ssm_z, w.ssm_b, w.ssm_a, w.ssm_out};
            const uint32_t t[5] = {w.ssm_qkv_type, w.ssm_z_type, w.ssm_b_type, w.ssm_a_type, w.ssm_out_type};
            const uint64_t cols[5] = {H, H, H, H, (uint64_t)nv * dh};
            for (int i = 0; i < 5; ++i) {
                if (!a16(m[i])) return bad("katali_cuda_hybrid_create: GDN weight pointer");
                if (!rbytes(t[i], cols[i]) || rbytes(t[i], cols[i]) % 2) return KATALI_ERR_UNSUPPORTED_TYPE;
            }
        } else {
            const void *m[4] = {w.wq, w.wk, w.wv, w.wo};
            const uint32_t t[4] = {w.wq_type, w.wk_type, w.wv_type, w.wo_type};
            const uint64_t cols[4] = {H, H, H, (uint64_t)NH * HD};
            for (int i = 0; i < 4; ++i) {
                if (!a16(m[i])) return bad("katali_cuda_hybrid_create: attention weight pointer");
                if (!rbytes(t[i], cols[i]) || rbytes(t[i], cols[i]) % 2) return KATALI_ERR_UNSUPPORTED_TYPE;
            }
        }
        kq::MoeParams mp;
        int grid = 0;
        const int s = kq::moe_fused_params(w.moe, q8 ? KATALI_MOE_Q8_1 : KATALI_MOE_F32, &mp, &grid);
        if (s) return s == KATALI_ERR_UNSUPPORTED_SHAPE
                          ? unsupported("katali_cuda_hybrid_create: MoE layer has no fused plan")
                          : s;
        if ((uint32_t)mp.H != H) return bad("katali_cuda_hybrid_create: MoE hidden size");
        if (l == 0) n_experts = (uint32_t)mp.n_experts;
        else if ((uint32_t)mp.n_experts != n_experts)
            return unsupported("katali_cuda_hybrid_create: expert count differs between layers");
    }

    KataliHybrid *m = new KataliHybrid();
    m->d = *d;
    m->lw.assign(d->layers, d->layers + d->n_layers);
    m->d.layers = m->lw.data();
    const size_t NL = d->n_layers, cap = d->kv_cap;
    const uint32_t rd = (d->rope_dim == 0 || d->rope_dim > HD) ? HD : d->rope_dim;
    const size_t rh = n_attn ? rd / 2 : 0;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) & ~(size_t)255;
        return o;
    };
    const size_t o_x = take(4ull * H), o_xb = take(4ull * H), o_q = take(8ull * NH * HD + 16),
                 o_k = take(4ull * NKV * HD + 16), o_v = take(4ull * NKV * HD + 16),
                 o_attn = take(4ull * NH * HD + 16), o_logits = take(4ull * d->vocab),
                 o_qkv = take(4ull * C + 16), o_z = take(4ull * nv * dh + 16), o_ba = take(8ull * nv + 16),
                 o_go = take(4ull * nv * dh + 16), o_rl = take(4ull * n_experts),
                 o_kk = take(4 * (size_t)n_attn * NKV * cap * HD + 16),
                 o_kv = take(4 * (size_t)n_attn * NKV * cap * HD + 16),
                 o_cos = take(4 * cap * rh + 16), o_sin = take(4 * cap * rh + 16), o_ctl = take(64),
                 o_forced = take(4 * cap), o_out = take(4 * cap), o_av = take(4 * 148),
                 o_ai = take(4 * 148);
    const size_t ring_bytes = 4ull * ck * C, state_bytes = 4ull * nv * dh * dh;
    m->state_bytes = (ring_bytes + state_bytes) * n_gdn + 16;
    m->state_off = take(m->state_bytes);
    cudaError_t e = cudaMalloc(&m->mem, off);
    if (e != cudaSuccess) {
        delete m;
        kq::set_status_message(cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : KATALI_ERR_CUDA;
    }
    unsigned char *b = (unsigned char *)m->mem;
    kq::HybridParams &hp = m->p;
    memset(&hp, 0, sizeof hp);
    kq::DenseParams &p = hp.d;
    p.H = (int)H;
    p.NH = (int)NH;
    p.NKV = (int)NKV;
    p.HD = (int)HD;
    p.NL = (int)NL;
    p.vocab = (int)d->vocab;
    p.kv_cap = (int)cap;
    p.rope_half = (int)rh;
    p.eps = d->rms_eps;
    p.gemv_mode = q8 ? 0 : 2;
    p.attn_scale = HD ? 1.0f / sqrtf((float)HD) : 0.0f;
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
    hp.nk = (int)nk;
    hp.nv = (int)nv;
    hp.dk = hp.dv = (int)dh;
    hp.conv_k = (int)ck;
    hp.n_experts = (int)n_experts;
    hp.qkv = (float *)(b + o_qkv);
    hp.z = (float *)(b + o_z);
    hp.ba = (float *)(b + o_ba);
    hp.go = (float *)(b + o_go);
    hp.rlogits = (float *)(b + o_rl);

    // RoPE table with the same libm calls as the reference's rope_prepare
    // (V/src/gguf_model.c:466-475): bit-identical cos/sin at every position.
    std::vector<float> cs(cap * rh), sn(cap * rh);
    for (size_t i = 0; i < rh; ++i) {
        const float inv = 1.0f / powf(d->rope_theta, (2.0f * (float)i) / (float)rd);
        for (size_t t = 0; t < cap; ++t) {
            const float f = (float)t * inv;
            cs[t * rh + i] = cosf(f);
            sn[t * rh + i] = sinf(f);
        }
    }
    cudaStream_t st = kq::current_stream();
    if (rh) {
        e = cudaMemcpyAsync((void *)p.rope_cos, cs.data(), 4 * cap * rh, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync((void *)p.rope_sin, sn.data(), 4 * cap * rh, cudaMemcpyHostToDevice, st);
    }
    if (e == cudaSuccess) e = cudaMemsetAsync(ctl, 0, 64, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(b + m->state_off, 0, m->state_bytes, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess && n_attn) e = kq::hybrid_set_attention_smem((int)cap);
    if (e != cudaSuccess) {
        kq::set_status_message(cudaGetErrorString(e));
        katali_cuda_hybrid_destroy(m);
        return KATALI_ERR_CUDA;
    }

    // Per layer: input projections (mixer RMSNorm in the GEMV staging), the output
    // projection added into x, and the fused MoE launch (x = xb, logits = rlogits, y += x).
    m->L.resize(NL);
    m->g.resize(2 * NL + 1);
    m->moe.resize(NL);
    m->moe_grid.resize(NL);
    unsigned char *st_base = b + m->state_off;
    uint32_t gi = 0, ai = 0;
    for (size_t l = 0; l < NL; ++l) {
        const KataliHybridLayerW &w = m->lw[l];
        kq::HybridLayer &hl = m->L[l];
        hl = kq::HybridLayer{};
        hl.ffn_norm = w.ffn_norm;
        hl.router = w.router;
        if (w.kind == KATALI_HYBRID_GDN) {
            hl.kind = 0;
            hl.conv_w = w.ssm_conv;
            hl.a_log = w.ssm_a_log;
            hl.a_neg = w.ssm_decay;
            hl.dt_bias = w.ssm_dt_bias;
            hl.ssm_norm = w.ssm_norm;
            hl.ring = (float *)(st_base + (size_t)gi * (ring_bytes + state_bytes));
            hl.state = (float *)(st_base + (size_t)gi * (ring_bytes + state_bytes) + ring_bytes);
            ++gi;
            const void *ws[4] = {w.ssm_qkv, w.ssm_z, w.ssm_b, w.ssm_a};
            const uint32_t ts[4] = {w.ssm_qkv_type, w.ssm_z_type, w.ssm_b_type, w.ssm_a_type};
            const uint64_t rows[4] = {C, (uint64_t)nv * dh, nv, nv};
            float *ys[4] = {hp.qkv, hp.z, hp.ba, hp.ba + nv};
            m->g[2 * l] = gemv_jobs(p.x, H, 4, ws, ts, rows, ys, 0, w.attn_norm, d->rms_eps);
            const void *wo[1] = {w.ssm_out};
            const uint32_t to[1] = {w.ssm_out_type};
            const uint64_t ro[1] = {H};
            float *yo[1] = {p.x};
            m->g[2 * l + 1] = gemv_jobs(hp.go, (uint64_t)nv * dh, 1, wo, to, ro, yo, 1, nullptr, 0.0f);
        } else {
            hl.kind = 1;
            hl.q_norm = w.q_norm;
            hl.k_norm = w.k_norm;
            hl.kv_k = p.kv_k + (size_t)ai * NKV * cap * HD;
            hl.kv_v = p.kv_v + (size_t)ai * NKV * cap * HD;
            ++ai;
            const void *ws[3] = {w.wq, w.wk, w.wv};
            const uint32_t ts[3] = {w.wq_type, w.wk_type, w.wv_type};
            const uint64_t rows[3] = {2ull * NH * HD, (uint64_t)NKV * HD, (uint64_t)NKV * HD};
            float *ys[3] = {p.q, p.k, p.v};
            m->g[2 * l] = gemv_jobs(p.x, H, 3, ws, ts, rows, ys, 0, w.attn_norm, d->rms_eps);
            const void *wo[1] = {w.wo};
            const uint32_t to[1] = {w.wo_type};
            const uint64_t ro[1] = {H};
            float *yo[1] = {p.x};
            m->g[2 * l + 1] = gemv_jobs(p.attn, (uint64_t)NH * HD, 1, wo, to, ro, yo, 1, nullptr, 0.0f);
        }
        kq::MoeParams &mp = m->moe[l];
        kq::moe_fused_params(w.moe, q8 ? KATALI_MOE_Q8_1 : KATALI_MOE_F32, &mp, &m->moe_grid[l]);
        mp.logits = hp.rlogits;
        mp.y = p.x;
        mp.accum = 1;
        mp.pdl = 1;
        mp.x = p.xb;  // RMSNorm and router logits from the router kernel
        m->moe_sep.push_back(mp);
        const int grid = m->moe_grid[l];
        if (H <= 4u * 512u && (n_experts + grid - 1) / grid <= (uint32_t)kq::MOE_RT_ROWS) {
            // the router runs inside the MoE launch: x is the residual stream itself (read by
            // every CTA before the launch's first grid barrier, added to after the last)
            mp.x = p.x;
            mp.rt_w = w.router;
            mp.rt_norm = w.ffn_norm;
            mp.rt_eps = d->rms_eps;
        } else {
            mp.x = p.xb;  // RMSNorm and router logits from the router kernel
        }
    }
    {
        const void *ws[1] = {d->lm_head};
        const uint32_t ts[1] = {d->lm_head_type};
        const uint64_t rows[1] = {d->vocab};
        float *ys[1] = {p.logits};
        m->g[2 * NL] = gemv_jobs(p.x, H, 1, ws, ts, rows, ys, 0, d->out_norm, d->rms_eps);
    }
    m->moe_local = m->moe;
    m->grid_local = m->moe_grid;
    m->n_experts = n_experts;
    m->top_k = (uint32_t)m->moe[0].K;
    *out = m;
    return KATALI_OK;
}

int katali_cuda_hybrid_set_ep(KataliHybrid *m, KataliEp *ep) {
    if (!m) return KATALI_ERR_BAD_ARG;
    cudaStream_t st = kq::current_stream();
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return KATALI_ERR_CUDA;
    if (m->exec) {  // the step's launches change: capture again at the next generate
        cudaGraphExecDestroy(m->exec);
        cudaGraphDestroy(m->graph);
        m->exec = nullptr;
        m->graph = nullptr;
    }
    if (!ep) {
        m->moe = m->moe_local;
        m->moe_grid = m->grid_local;
        m->p.moe_ep = 0;
        return KATALI_OK;
    }
    if (m->p.d.gemv_mode != 0) {
        kq::set_status_message("katali_cuda_hybrid_set_ep: expert parallelism needs q8_1 activations "
                               "(KATALI_DENSE_Q8_1)");
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    }
    std::vector<kq::MoeParams> mp(m->lw.size());
    std::vector<int> grid(m->lw.size());
    for (size_t l = 0; l < m->lw.size(); ++l) {
        uint32_t G = 0;
        const kq::EpPeer *pp = nullptr;
        double *ret = nullptr;
        int s = kq::ep_peer_prepare(ep, m->lw[l].moe, 1, &G, &pp, &ret);
        if (s) return s;
        s = kq::moe_ep_fused_params(m->lw[l].moe, G, 1, 1, m->p.d.xb, m->p.rlogits, m->p.d.x, pp,
                                    ret, &mp[l], &grid[l]);
        if (s) return s;
        mp[l].accum = 1;
    }
    m->moe = mp;
    m->moe_grid = grid;
    m->p.moe_ep = 1;
    return KATALI_OK;
}

int katali_cuda_hybrid_destroy(KataliHybrid *m) {
    if (!m) return KATALI_OK;
    cudaStream_t st = kq::current_stream();
    if (st) cudaStreamSynchronize(st);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    cudaFree(m->mem);
    cudaFree(m->route_dev);
    for (KataliMoe *moe : m->own_moe) katali_cuda_moe_destroy(moe);
    for (void *a : m->own_allocs) cudaFree(a);
    for (void *h : m->own_pinned) cudaHostUnregister(h);
    delete m;
    return KATALI_OK;
}

int katali_cuda_hybrid_reset(KataliHybrid *m) {
    if (!m) return KATALI_ERR_BAD_ARG;
    m->pos = 0;
    cudaStream_t st = kq::current_stream();
    cudaError_t e = cudaMemsetAsync(m->p.d.pos, 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaMemsetAsync((unsigned char *)m->mem + m->state_off, 0, m->state_bytes, st);
    return e == cudaSuccess ? KATALI_OK : KATALI_ERR_CUDA;
}

int katali_cuda_hybrid_generate(KataliHybrid *m, const int32_t *prompt, uint32_t n_prompt,
                                uint32_t n_gen, int32_t *out_tokens) {
    if (!m || !prompt || n_prompt == 0 || n_gen == 0 || !out_tokens) return KATALI_ERR_BAD_ARG;
    const uint64_t steps = (uint64_t)n_prompt + n_gen - 1;
    if ((uint64_t)m->pos + steps > (uint64_t)m->p.d.kv_cap) {
        kq::set_status_message("katali_cuda_hybrid_generate: KV cache full (kv_cap)");
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    }
    for (uint32_t i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || (uint32_t)prompt[i] >= m->d.vocab) return KATALI_ERR_BAD_ARG;
    cudaStream_t st = kq::current_stream();
    const int ctl[4] = {prompt[0], m->pos, 0, (int)n_prompt};
    cudaError_t e = cudaMemcpyAsync((void *)m->p.d.forced, prompt, 4ull * n_prompt,
                                    cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->p.d.tok, ctl, sizeof ctl, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return KATALI_ERR_CUDA;
    if (m->cache) {  // residency mode: each step layer by layer, experts bound after the router
        if (!m->route_dev && (e = cudaMalloc((void **)&m->route_dev, 8ull * kq::MOE_MAX_K)) != cudaSuccess) {
            m->route_dev = nullptr;
            return KATALI_ERR_OOM;
        }
        for (uint64_t s = 0; s < steps; ++s) {
            int hs = 0;
            e = kq::launch_hybrid_step(m->p, m->L.data(), m->g.data(), m->moe_sep.data(),
                                       m->grid_local.data(), st, bind_routed, m, &hs);
            if (hs) return hs;
            if (e != cudaSuccess) break;
        }
    }
    for (uint64_t s = 0; s < steps && !m->cache; ++s) {
        if (!m->exec || m->graph_stream != st) {
            // First step on this stream: run it eagerly (sets kernel attributes), then
            // capture the same launch sequence once for the following steps.
            e = kq::launch_hybrid_step(m->p, m->L.data(), m->g.data(), m->moe.data(),
                                       m->moe_grid.data(), st);
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
            cudaError_t le = kq::launch_hybrid_step(m->p, m->L.data(), m->g.data(), m->moe.data(),
                                                    m->moe_grid.data(), cap);
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
        e = cudaMemcpyAsync(out_tokens, m->p.d.out_tokens + (n_prompt - 1), 4ull * n_gen,
                            cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        kq::set_status_message(cudaGetErrorString(e));
        return KATALI_ERR_CUDA;
    }
    m->pos += (int)steps;
    return kq::take_status_after_sync();
}

int katali_cuda_hybrid_logits(KataliHybrid *m, const float **logits_dev, int32_t *position) {
    if (!m) return KATALI_ERR_BAD_ARG;
    if (logits_dev) *logits_dev = m->p.d.logits;
    if (position) *position = m->pos;
    return KATALI_OK;
}

}  // extern "C"
