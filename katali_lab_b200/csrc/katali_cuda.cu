// katali_cuda.cu — the C ABI of libkatali_cuda.so (declared in include/katali_cuda.h).
//
// Host side of the plugin: device probe, allocation and copies, argument
// checks, launch of the kernels in kq_gemv.cu / kq_moe.cu on the plugin stream,
// and error reporting. No CPU fallback: a call that cannot run on the GPU
// returns a status code and the caller decides (the reference's caller falls
// back to its CPU kernels, vendor/katali_gguf_dense/src/gguf_model.c:500-504).
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "katali_cuda.h"
#include "kq_launch.h"

namespace {

int g_probed = -1;
char g_status[512] = "not probed";
int g_dev = 0;
int g_num_sms = 148;
int g_max_smem = 0;
cudaStream_t g_own_stream = nullptr;
cudaStream_t g_stream = nullptr;
int g_async = 0;
uint32_t *g_status_host = nullptr;  // mapped pinned word the kernels set on a device-side timeout
uint32_t *g_status_dev = nullptr;

int probe_impl() {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        snprintf(g_status, sizeof g_status, "CUDA unavailable: %s", cudaGetErrorString(e));
        return 0;
    }
    if (n <= 0) {
        snprintf(g_status, sizeof g_status, "no CUDA device");
        return 0;
    }
    cudaGetDevice(&g_dev);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, g_dev) != cudaSuccess) {
        snprintf(g_status, sizeof g_status, "cannot query device %d", g_dev);
        return 0;
    }
    if (prop.major != 10 || prop.minor != 0) {
        snprintf(g_status, sizeof g_status,
                 "device %d (%s) is sm_%d%d; this plugin is built for sm_100a (B200)", g_dev,
                 prop.name, prop.major, prop.minor);
        return 0;
    }
    g_num_sms = prop.multiProcessorCount;
    g_max_smem = (int)prop.sharedMemPerBlockOptin;
    snprintf(g_status, sizeof g_status, "ok: device %d %s sm_%d%d, %d SMs, %.1f GiB", g_dev,
             prop.name, prop.major, prop.minor, prop.multiProcessorCount,
             prop.totalGlobalMem / 1073741824.0);
    return 1;
}

int ensure() {
    if (g_probed < 0) g_probed = probe_impl();
    if (!g_probed) return KATALI_ERR_NO_DEVICE;
    if (!g_own_stream) {
        if (cudaStreamCreateWithFlags(&g_own_stream, cudaStreamNonBlocking) != cudaSuccess)
            return KATALI_ERR_CUDA;
        if (!g_stream) g_stream = g_own_stream;
    }
    if (!g_status_host) {
        if (cudaHostAlloc((void **)&g_status_host, sizeof(uint32_t), cudaHostAllocMapped) !=
            cudaSuccess)
            return KATALI_ERR_CUDA;
        *g_status_host = 0;
        if (cudaHostGetDevicePointer((void **)&g_status_dev, g_status_host, 0) != cudaSuccess)
            return KATALI_ERR_CUDA;
    }
    return KATALI_OK;
}

int cuda_fail(cudaError_t e) {
    snprintf(g_status, sizeof g_status, "CUDA error: %s", cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : KATALI_ERR_CUDA;
}

int take_device_status() {
    if (!g_status_host) return KATALI_OK;  // no call has launched work yet
    const uint32_t s = *(volatile uint32_t *)g_status_host;
    if (s) {
        *(volatile uint32_t *)g_status_host = 0;
        if (s & kq::KQ_STATUS_NOT_RESIDENT) {
            snprintf(g_status, sizeof g_status, "a selected expert is not resident (bits 0x%x)", s);
            return KATALI_ERR_NOT_RESIDENT;
        }
        snprintf(g_status, sizeof g_status, "device-side wait timed out (bits 0x%x)", s);
        return KATALI_ERR_TIMEOUT;
    }
    return KATALI_OK;
}

// After a launch: in synchronous mode wait for the stream and report errors.
int finish(cudaError_t e) {
    if (e != cudaSuccess) return cuda_fail(e);
    if (g_async) return KATALI_OK;
    e = cudaStreamSynchronize(g_stream);
    if (e != cudaSuccess) return cuda_fail(e);
    return take_device_status();
}

bool aligned16(const void *p) { return p && ((uintptr_t)p & 15u) == 0; }

uint64_t row_bytes(uint32_t type, uint64_t cols) {
    switch (type) {
        case KATALI_TYPE_Q4_K: return cols % 256 ? 0 : cols / 256 * 144;
        case KATALI_TYPE_Q6_K: return cols % 256 ? 0 : cols / 256 * 210;
        case KATALI_TYPE_Q8_1: return cols % 32 ? 0 : cols / 32 * 36;
        default: return 0;
    }
}

bool gemv_type(uint32_t t) { return t == KATALI_TYPE_Q4_K || t == KATALI_TYPE_Q6_K; }

// fp32-activation GEMV by default, as the reference's dense path; the q8_1
// (DP4A) path when KATALI_CUDA_DP4A=1 (the reference's switch, README.md:17).
int dense_mode() {
    const char *e = getenv("KATALI_CUDA_DP4A");
    return (e && (e[0] == '1' || e[0] == 'y' || e[0] == 'Y')) ? 0 : 2;
}

int max_cols_for_smem(int mode) {
    // activations staged per CTA next to the weight ring (~100 KB)
    return mode == 2 ? 24576 : 65536;
}

}  // namespace

namespace kq {
// The plugin's runtime state (device probe, own stream, mapped status word), created on the
// first call that needs it; the entry points of the other translation units call this first.
int ensure_runtime() { return ensure(); }
// Lets other translation units of the plugin report a reason via katali_cuda_status().
void set_status_message(const char *msg) { snprintf(g_status, sizeof g_status, "%s", msg); }
cudaStream_t current_stream() { return g_stream; }
volatile uint32_t *device_status_word() { return g_status_dev; }
// After the stream was synchronised: KATALI_OK or the device-side status.
int take_status_after_sync() { return take_device_status(); }
}  // namespace kq

struct KataliMoe {
    kq::MoeParams plan[2];  // per activation mode
    int plan_ok[2];
    std::vector<const uint8_t *> table;  // host copy of the device pointer table
    const uint8_t **d_table;
    float *hbuf;
    uint32_t *sync;
    int32_t *dbg_ids;
    float *dbg_w;
    uint64_t *trace;
    int grid;
    // Ragged-batch scratch, grown on demand (katali_cuda_moe_batch, the EP stages).
    unsigned char *bscratch;
    size_t bscratch_bytes;
    int32_t *ep_src_ids;  // routing of the last katali_cuda_moe_ep_dispatch
    uint32_t ep_src_cap;  // tokens
    uint64_t *ep_route;   // the single-launch layer's tagged routing record (zeroed when made)
    uint32_t ep_route_cap;
    KataliExpertCache *cache;  // the residency cache this layer's experts are bound to
};

namespace kq {
void cache_forget_layer(KataliExpertCache *c, KataliMoe *m);

// Stream-ordered update of expert e's pointers (no host wait): calls enqueued
// before keep the old pointers, calls enqueued after see the new ones.
int moe_set_expert_async(KataliMoe *m, uint32_t e, const void *g, const void *u, const void *d) {
    if (!m || e >= m->table.size() / 3) return KATALI_ERR_BAD_ARG;
    m->table[3 * e] = (const uint8_t *)g;
    m->table[3 * e + 1] = (const uint8_t *)u;
    m->table[3 * e + 2] = (const uint8_t *)d;
    // pageable source: the three pointers are captured before cudaMemcpyAsync returns
    const cudaError_t err = cudaMemcpyAsync(m->d_table + 3 * e, &m->table[3 * e], 3 * sizeof(void *),
                                            cudaMemcpyHostToDevice, g_stream);
    return err == cudaSuccess ? KATALI_OK : cuda_fail(err);
}
uint32_t moe_n_experts(const KataliMoe *m) { return (uint32_t)(m->table.size() / 3); }
KataliExpertCache *moe_cache(const KataliMoe *m) { return m->cache; }
void moe_set_cache(KataliMoe *m, KataliExpertCache *c) { m->cache = c; }
}  // namespace kq

namespace {

// Carves the ragged-batch scratch for T tokens out of one allocation; with base ==
// nullptr it only returns the size. Every array starts on a 256-byte boundary.
size_t moe_batch_layout(const kq::MoeParams &pl, int T, unsigned char *base, kq::MoeBatchParams *b) {
    const size_t P = (size_t)T * pl.K, H = pl.H, F = pl.F, E = pl.n_experts;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        unsigned char *ptr = base ? base + off : nullptr;
        off += (bytes + 255) & ~(size_t)255;
        return ptr;
    };
    // First, at an offset that does not depend on T: the group count and the item
    // counters (a call never reads what a call of another batch size left there).
    unsigned char *ng = take(32);
    unsigned char *ids = take(4 * P), *w = take(4 * P);
    unsigned char *xq = take(T * H), *xd = take(4 * T * H / 32), *xs32 = take(4 * T * H / 32),
                  *xs16 = take(4 * T * H / 16);
    unsigned char *ge = take(4 * E), *go = take(4 * (E + 1)), *ps = take(4 * P),
                  *po = take(4 * P), *tcg = take(4 * E);
    unsigned char *h = take(4 * P * F), *hq = take(P * F), *hd = take(4 * P * F / 32),
                  *hs32 = take(4 * P * F / 32), *hs16 = take(4 * P * F / 16);
    unsigned char *part = take(4 * P * H);
    unsigned char *hu = take(4 * P * F), *ptc = take(P);
    if (b) {
        b->ids = (int32_t *)ids;
        b->w = (float *)w;
        b->xq = (int8_t *)xq;
        b->xd = (float *)xd;
        b->xs32 = (int *)xs32;
        b->xs16 = (int *)xs16;
        b->grp_expert = (int *)ge;
        b->grp_off = (int *)go;
        b->tc_groups = (int *)tcg;
        b->hu = (float *)hu;
        b->pair_tc = (uint8_t *)ptc;
        b->n_groups = (int *)ng;
        b->work = (uint32_t *)(ng + 4);
        b->pair_src = (int *)ps;
        b->pos_of = (int *)po;
        b->h = (float *)h;
        b->hq = (int8_t *)hq;
        b->hd = (float *)hd;
        b->hs32 = (int *)hs32;
        b->hs16 = (int *)hs16;
        b->part = (float *)part;
    }
    return off;
}

}  // namespace

namespace kq {
// The fused single-launch call of MoE layer m in activation mode `mode`, for a decoder that
// launches it from its own step (kq_hybrid.cu): every field but x, logits, y and accum.
int moe_fused_params(KataliMoe *m, uint32_t mode, MoeParams *p, int *grid) {
    if (!m || mode > 1) return KATALI_ERR_BAD_ARG;
    if (!m->plan_ok[mode]) return KATALI_ERR_UNSUPPORTED_SHAPE;
    *p = m->plan[mode];
    p->experts = m->d_table;
    p->hbuf = m->hbuf;
    p->sync = m->sync;
    p->status = g_status_dev;
    p->trace = nullptr;
    p->route_only = 0;
    *grid = m->grid;
    return KATALI_OK;
}
}  // namespace kq

extern "C" {

int katali_cuda_probe(void) {
    if (g_probed < 0) g_probed = probe_impl();
    return g_probed;
}

const char *katali_cuda_status(void) {
    if (g_probed < 0) g_probed = probe_impl();
    return g_status;
}

const char *katali_cuda_strerror(int s) {
    switch (s) {
        case KATALI_OK: return "ok";
        case KATALI_ERR_NO_DEVICE: return "no usable sm_100 device";
        case KATALI_ERR_OOM: return "out of device memory";
        case KATALI_ERR_BAD_ARG: return "bad argument";
        case KATALI_ERR_UNSUPPORTED_TYPE: return "unsupported tensor type";
        case KATALI_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
        case KATALI_ERR_TIMEOUT: return "device-side wait timed out";
        case KATALI_ERR_NOT_RESIDENT: return "selected expert not resident";
        case KATALI_ERR_CUDA: return "CUDA error";
        case KATALI_ERR_NCCL: return "NCCL error";
        default: return "unknown status";
    }
}

int katali_cuda_malloc(void **ptr, size_t bytes) {
    if (!ptr) return KATALI_ERR_BAD_ARG;
    *ptr = nullptr;
    int s = ensure();
    if (s) return s;
    cudaError_t e = cudaMalloc(ptr, bytes ? bytes : 1);
    if (e != cudaSuccess) {
        *ptr = nullptr;
        return cuda_fail(e);
    }
    return KATALI_OK;
}

int katali_cuda_free(void *ptr) {
    if (!ptr) return KATALI_OK;
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? KATALI_OK : cuda_fail(e);
}

int katali_cuda_upload(void *dev, const void *host, size_t bytes) {
    if ((!dev || !host) && bytes) return KATALI_ERR_BAD_ARG;
    int s = ensure();
    if (s) return s;
    cudaError_t e = cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, g_stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(g_stream);
    return e == cudaSuccess ? KATALI_OK : cuda_fail(e);
}

int katali_cuda_download(void *host, const void *dev, size_t bytes) {
    if ((!dev || !host) && bytes) return KATALI_ERR_BAD_ARG;
    int s = ensure();
    if (s) return s;
    cudaError_t e = cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, g_stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(g_stream);
    if (e != cudaSuccess) return cuda_fail(e);
    return take_device_status();
}

int katali_cuda_supports_type(uint32_t type) { return gemv_type(type) ? 1 : 0; }

int katali_cuda_set_stream(void *stream) {
    int s = ensure();
    if (s) return s;
    g_stream = stream ? (cudaStream_t)stream : g_own_stream;
    return KATALI_OK;
}

int katali_cuda_set_async(int on) {
    g_async = on ? 1 : 0;
    return KATALI_OK;
}

int katali_cuda_sync(void) {
    int s = ensure();
    if (s) return s;
    cudaError_t e = cudaStreamSynchronize(g_stream);
    if (e != cudaSuccess) return cuda_fail(e);
    return take_device_status();
}

static int matvec_common(int n, const uint32_t *types, const void *const *w, const uint64_t *rows,
                         uint64_t cols, const float *x, const uint8_t *xq, float *const *y,
                         int mode) {
    if (n <= 0 || n > 8 || !types || !w || !rows || !y) return KATALI_ERR_BAD_ARG;
    if (mode == 1 ? !xq : !aligned16(x)) return KATALI_ERR_BAD_ARG;
    if (cols == 0 || cols % 256 || cols > (uint64_t)max_cols_for_smem(mode))
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    int s = ensure();
    if (s) return s;
    kq::GemvParams p = {};
    p.njobs = n;
    p.cols = (uint32_t)cols;
    p.x = x;
    p.xq = xq;
    p.status = g_status_dev;
    for (int j = 0; j < n; ++j) {
        if (!gemv_type(types[j])) return KATALI_ERR_UNSUPPORTED_TYPE;
        if (!aligned16(w[j]) || !y[j] || rows[j] == 0 || rows[j] > 0xFFFFFFFFull)
            return KATALI_ERR_BAD_ARG;
        p.job[j].w = (const uint8_t *)w[j];
        p.job[j].y = y[j];
        p.job[j].rows = rows[j];
        p.job[j].type = types[j];
        p.job[j].rb = (uint32_t)row_bytes(types[j], cols);
    }
    return finish(kq::launch_gemv(p, mode, g_stream));
}

int katali_cuda_matvec(uint32_t type, const void *w, uint64_t rows, uint64_t cols, const float *x,
                       float *y) {
    if (!gemv_type(type)) return KATALI_ERR_UNSUPPORTED_TYPE;
    if (!x) return KATALI_ERR_BAD_ARG;
    const void *wl[1] = {w};
    float *yl[1] = {y};
    return matvec_common(1, &type, wl, &rows, cols, x, nullptr, yl, dense_mode());
}

int katali_cuda_matvec_multi(int n, const uint32_t *types, const void *const *w,
                             const uint64_t *rows, uint64_t cols, const float *x, float *const *y) {
    if (!x) return KATALI_ERR_BAD_ARG;
    return matvec_common(n, types, w, rows, cols, x, nullptr, y, dense_mode());
}

int katali_cuda_matvec_q8_1(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                            const void *xq, float *y) {
    if (!gemv_type(type)) return KATALI_ERR_UNSUPPORTED_TYPE;
    const void *wl[1] = {w};
    float *yl[1] = {y};
    return matvec_common(1, &type, wl, &rows, cols, nullptr, (const uint8_t *)xq, yl, 1);
}

int katali_cuda_quantize_q8_1(const float *x, uint64_t n, void *xq) {
    if (!x || !xq || n == 0 || n % 32 || ((uintptr_t)xq & 3u)) return KATALI_ERR_BAD_ARG;
    int s = ensure();
    if (s) return s;
    return finish(kq::launch_quantize_q8_1(x, n, xq, g_stream));
}

int katali_cuda_quantize_rows(uint32_t type, const float *src, uint64_t rows, uint64_t cols,
                              void *dst) {
    if (type != KATALI_TYPE_Q4_K && type != KATALI_TYPE_Q6_K && type != KATALI_TYPE_Q8_1)
        return KATALI_ERR_UNSUPPORTED_TYPE;
    if (!src || !dst || rows == 0 || row_bytes(type, cols) == 0) return KATALI_ERR_BAD_ARG;
    if (type == KATALI_TYPE_Q8_1 && ((uintptr_t)dst & 3u)) return KATALI_ERR_BAD_ARG;
    int s = ensure();
    if (s) return s;
    return finish(kq::launch_encode(type, src, rows * cols, dst, g_stream));
}

int katali_cuda_debug_row_isums(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                                const void *xq, int32_t *isum, int32_t *xsum) {
    if (!gemv_type(type)) return KATALI_ERR_UNSUPPORTED_TYPE;
    if (!w || !xq || !isum || rows == 0 || cols == 0 || cols % 256) return KATALI_ERR_BAD_ARG;
    if (type == KATALI_TYPE_Q4_K && !xsum) return KATALI_ERR_BAD_ARG;
    int s = ensure();
    if (s) return s;
    return finish(kq::launch_row_isums(type, w, rows, cols, (uint32_t)row_bytes(type, cols), xq,
                                       isum, xsum, g_stream));
}

// ---------------------------------------------------------------------------
// MoE
// ---------------------------------------------------------------------------
int katali_cuda_moe_create(const KataliMoeDesc *d, KataliMoe **out) {
    if (!d || !out) return KATALI_ERR_BAD_ARG;
    *out = nullptr;
    if (d->n_experts == 0 || d->n_experts > 1024 || d->top_k == 0 || d->top_k > kq::MOE_MAX_K ||
        d->top_k > d->n_experts)
        return KATALI_ERR_BAD_ARG;
    if (!gemv_type(d->gate_type) || !gemv_type(d->up_type) || !gemv_type(d->down_type))
        return KATALI_ERR_UNSUPPORTED_TYPE;
    const uint64_t rbg = row_bytes(d->gate_type, d->hidden), rbu = row_bytes(d->up_type, d->hidden);
    const uint64_t rbd = row_bytes(d->down_type, d->ffn);
    if (!rbg || !rbu || !rbd || rbg % 16 || rbu % 16)
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    int s = ensure();
    if (s) return s;
    KataliMoe *m = new KataliMoe();
    m->grid = g_num_sms;
    for (int mode = 0; mode < 2; ++mode) {
        kq::MoeParams &p = m->plan[mode];
        p = kq::MoeParams{};
        p.n_experts = (int)d->n_experts;
        p.H = (int)d->hidden;
        p.F = (int)d->ffn;
        p.K = (int)d->top_k;
        p.norm = (d->flags & KATALI_MOE_NORM_TOPK) ? 1 : 0;
        p.mode = mode;
        p.gate_type = d->gate_type;
        p.up_type = d->up_type;
        p.down_type = d->down_type;
        p.rbg = (uint32_t)rbg;
        p.rbu = (uint32_t)rbu;
        p.rbd = (uint32_t)rbd;
        m->plan_ok[mode] = kq::moe_plan(p, m->grid, g_max_smem) == 0;
    }
    m->table.assign(3 * (size_t)d->n_experts, nullptr);
    if (d->experts) {
        for (size_t i = 0; i < m->table.size(); ++i) {
            if (d->experts[i] && !aligned16(d->experts[i])) {
                delete m;
                return KATALI_ERR_BAD_ARG;
            }
            m->table[i] = (const uint8_t *)d->experts[i];
        }
    }
    // +1 pointer: the kernel copies the table in 16-byte pairs
    cudaError_t e = cudaMalloc((void **)&m->d_table, (m->table.size() + 1) * sizeof(void *));
    // h scratch: top_k * ffn floats (fp32 mode), or the q8_1 records (48 B per 32 values) of up
    // to MOE_EP_MAX_SLOTS * top_k expert-parallel pairs
    const size_t hbuf_bytes = std::max(sizeof(float) * d->top_k * d->ffn,
                                       (size_t)kq::MOE_EP_MAX_SLOTS * d->top_k * d->ffn / 32 * 48);
    if (e == cudaSuccess) e = cudaMalloc((void **)&m->hbuf, hbuf_bytes);
    if (e == cudaSuccess) e = cudaMalloc((void **)&m->sync, 16);
    if (e == cudaSuccess) e = cudaMalloc((void **)&m->dbg_ids, 4 * kq::MOE_MAX_K);
    if (e == cudaSuccess) e = cudaMalloc((void **)&m->dbg_w, 4 * kq::MOE_MAX_K);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->sync, 0, 16, g_stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->d_table, m->table.data(), m->table.size() * sizeof(void *),
                            cudaMemcpyHostToDevice, g_stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(g_stream);
    if (e != cudaSuccess) {
        katali_cuda_moe_destroy(m);
        return cuda_fail(e);
    }
    *out = m;
    return KATALI_OK;
}

int katali_cuda_moe_set_expert(KataliMoe *m, uint32_t e, const void *gate, const void *up,
                               const void *down) {
    if (!m || e >= m->table.size() / 3) return KATALI_ERR_BAD_ARG;
    if (!aligned16(gate) || !aligned16(up) || !aligned16(down)) return KATALI_ERR_BAD_ARG;
    m->table[3 * e] = (const uint8_t *)gate;
    m->table[3 * e + 1] = (const uint8_t *)up;
    m->table[3 * e + 2] = (const uint8_t *)down;
    // Stream-ordered: calls already enqueued keep the pointers they were launched with.
    cudaError_t err = cudaMemcpyAsync(m->d_table + 3 * e, &m->table[3 * e], 3 * sizeof(void *),
                                      cudaMemcpyHostToDevice, g_stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(g_stream);
    return err == cudaSuccess ? KATALI_OK : cuda_fail(err);
}

int katali_cuda_moe_destroy(KataliMoe *m) {
    if (!m) return KATALI_OK;
    if (m->cache) kq::cache_forget_layer(m->cache, m);
    if (g_stream) cudaStreamSynchronize(g_stream);
    cudaFree(m->d_table);
    cudaFree(m->hbuf);
    cudaFree(m->sync);
    cudaFree(m->dbg_ids);
    cudaFree(m->dbg_w);
    cudaFree(m->bscratch);
    cudaFree(m->ep_src_ids);
    cudaFree(m->ep_route);
    delete m;
    return KATALI_OK;
}

static int grow_batch_scratch(KataliMoe *m, int T);
static kq::MoeBatchParams batch_params(KataliMoe *m, int T);

static int moe_run(KataliMoe *m, const float *x, const float *logits, const int32_t *ids,
                   const float *w, float *y, uint32_t mode, int route_only) {
    if (!m || mode > 1) return KATALI_ERR_BAD_ARG;
    if (!m->plan_ok[mode]) {
        // Shapes whose fused single-launch plan does not fit shared memory (e.g. FFN 768):
        // the ragged-batch pipeline with one token, q8_1 activations.
        if (mode != KATALI_MOE_Q8_1 || route_only) return KATALI_ERR_UNSUPPORTED_SHAPE;
        int s = grow_batch_scratch(m, 1);
        if (s) return s;
        kq::MoeBatchParams b = batch_params(m, 1);
        b.X = x;
        b.logits = logits;
        b.ids_in = ids;
        b.w_in = w;
        b.Y = y;
        return finish(kq::launch_moe_batch(b, g_stream));
    }
    kq::MoeParams p = m->plan[mode];
    p.experts = m->d_table;
    p.x = x;
    p.logits = logits;
    p.ids = ids;
    p.w = w;
    p.y = y;
    p.hbuf = m->hbuf;
    p.sync = m->sync;
    p.status = g_status_dev;
    p.dbg_ids = m->dbg_ids;
    p.dbg_w = m->dbg_w;
    p.route_only = route_only;
    p.trace = route_only ? nullptr : m->trace;
    p.pdl = 1;  // overlaps this launch's prologue with the end of the previous kernel
    return finish(kq::launch_moe(p, route_only ? 1 : m->grid, g_stream));
}

int katali_cuda_moe_layer(KataliMoe *m, const float *x, const float *router_logits, float *y,
                          uint32_t mode) {
    if (!aligned16(x) || !router_logits || !y) return KATALI_ERR_BAD_ARG;
    return moe_run(m, x, router_logits, nullptr, nullptr, y, mode, 0);
}

int katali_cuda_moe_layer_routed(KataliMoe *m, const float *x, const int32_t *ids, const float *w,
                                 float *y, uint32_t mode) {
    if (!aligned16(x) || !ids || !w || !y) return KATALI_ERR_BAD_ARG;
    return moe_run(m, x, nullptr, ids, w, y, mode, 0);
}

static int grow_batch_scratch(KataliMoe *m, int T) {
    const size_t need = moe_batch_layout(m->plan[0], T, nullptr, nullptr);
    if (need <= m->bscratch_bytes) return KATALI_OK;
    // Grow: earlier calls on the stream may still read the old scratch.
    cudaError_t e = cudaStreamSynchronize(g_stream);
    if (e != cudaSuccess) return cuda_fail(e);
    cudaFree(m->bscratch);
    m->bscratch = nullptr;
    m->bscratch_bytes = 0;
    e = cudaMalloc((void **)&m->bscratch, need);
    if (e != cudaSuccess) {
        m->bscratch = nullptr;
        return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : cuda_fail(e);
    }
    m->bscratch_bytes = need;
    return KATALI_OK;
}

static kq::MoeBatchParams batch_params(KataliMoe *m, int T) {
    const kq::MoeParams &pl = m->plan[0];
    kq::MoeBatchParams b = {};
    moe_batch_layout(pl, T, m->bscratch, &b);
    b.experts = m->d_table;
    b.T = T;
    b.n_experts = pl.n_experts;
    b.H = pl.H;
    b.F = pl.F;
    b.K = pl.K;
    b.norm = pl.norm;
    b.gate_type = pl.gate_type;
    b.up_type = pl.up_type;
    b.down_type = pl.down_type;
    b.rbg = pl.rbg;
    b.rbu = pl.rbu;
    b.rbd = pl.rbd;
    b.status = g_status_dev;
    b.sms = g_num_sms;
    // Groups of >= 16 tokens run gate/up on the tensor cores (Q4_K gate and up only; fp32
    // block terms, so its bar against the restatement is looser), groups of >= 8 tokens the
    // down projection (Q6_K down whose 128-row tile fits the kernel's staging; rows equal to
    // the restatement's dot): a tensor-core item costs the same for 1 to 32 tokens, and from
    // about 8 tokens it is shorter than the DP4A items of the same group.
    // KATALI_CUDA_NO_TC=1 keeps every group on the DP4A kernels.
    const char *no_tc = getenv("KATALI_CUDA_NO_TC");
    const bool tc = !(no_tc && no_tc[0] == '1');
    b.tc_min = (pl.gate_type == KATALI_TYPE_Q4_K && pl.up_type == KATALI_TYPE_Q4_K && pl.F % 128 == 0 && tc)
                   ? 16
                   : 0;
    b.tc_down_min = (pl.down_type == KATALI_TYPE_Q6_K && pl.H % 128 == 0 &&
                     128ull * pl.rbd <= kq::TC_DOWN_RAW_MAX && tc)
                        ? 8
                        : 0;
    return b;
}

int katali_cuda_moe_batch(KataliMoe *m, uint32_t n_tokens, const float *x,
                          const float *router_logits, float *y, uint32_t mode) {
    if (!m || mode > 1) return KATALI_ERR_BAD_ARG;
    if (n_tokens == 0) return KATALI_OK;
    if (!x || !router_logits || !y || !aligned16(x) || n_tokens > KATALI_MOE_BATCH_MAX_TOKENS)
        return KATALI_ERR_BAD_ARG;
    if (mode != KATALI_MOE_Q8_1) return KATALI_ERR_UNSUPPORTED_TYPE;
    int s = grow_batch_scratch(m, (int)n_tokens);
    if (s) return s;
    kq::MoeBatchParams b = batch_params(m, (int)n_tokens);
    b.X = x;
    b.logits = router_logits;
    b.Y = y;
    return finish(kq::launch_moe_batch(b, g_stream));
}

// ---------------------------------------------------------------------------
// Expert parallelism: the three stages around the two exchanges
// ---------------------------------------------------------------------------
static uint32_t ep_hdr_bytes(int K) { return (uint32_t)(16 + 8 * K + 15) & ~15u; }
static uint32_t ep_slot_bytes(const kq::MoeParams &pl) { return ep_hdr_bytes(pl.K) + pl.H / 32 * 36; }

// The experts stage runs in the fused kernel (pairs mode) for up to MOE_EP_MAX_SLOTS
// received slots when the layer has a q8_1 fused plan with decoded Q6_K down rows and
// one phase-A block per CTA per round (K * F / 32 <= grid); KATALI_CUDA_NO_EP_FUSED=1
// keeps the ragged-batch pipeline.
static bool ep_fused_ok(const KataliMoe *m, int slots) {
    const char *off = getenv("KATALI_CUDA_NO_EP_FUSED");
    if (off && off[0] == '1') return false;
    const kq::MoeParams &pl = m->plan[KATALI_MOE_Q8_1];
    const bool pow2_f = pl.F == 256 || pl.F == 512 || pl.F == 1024 || pl.F == 2048;
    return m->plan_ok[KATALI_MOE_Q8_1] && slots <= kq::MOE_EP_MAX_SLOTS && pl.dec_enabled &&
           pl.down_type == KATALI_TYPE_Q6_K && pow2_f && pl.K * pl.F / 32 <= m->grid;
}

static int ep_check(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens) {
    if (!m || n_ranks == 0 || n_ranks > 64 || max_tokens == 0 ||
        (uint64_t)n_ranks * max_tokens > KATALI_MOE_BATCH_MAX_TOKENS)
        return KATALI_ERR_BAD_ARG;
    if (m->plan[0].n_experts % (int)n_ranks) return KATALI_ERR_UNSUPPORTED_SHAPE;
    return KATALI_OK;
}

static void ep_fill(kq::MoeBatchParams &b, KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens) {
    b.ep_ranks = (int)n_ranks;
    b.ep_tmax = (int)max_tokens;
    b.ep_hdr_bytes = ep_hdr_bytes(m->plan[0].K);
    b.ep_slot_bytes = ep_slot_bytes(m->plan[0]);
    b.ep_src_ids = m->ep_src_ids;
}

int katali_cuda_moe_ep_slot_bytes(KataliMoe *m, uint64_t *slot_bytes, uint64_t *ret_slot_bytes) {
    if (!m) return KATALI_ERR_BAD_ARG;
    if (slot_bytes) *slot_bytes = ep_slot_bytes(m->plan[0]);
    if (ret_slot_bytes) *ret_slot_bytes = 8ull * m->plan[0].H;
    return KATALI_OK;
}

}  // extern "C"

static void ep_peer_fill(kq::MoeBatchParams &b, const kq::EpPeer *pp) {
    if (!pp) return;
    b.ep_p2p = 1;
    b.ep_rank = pp->rank;
    b.ep_peer_recv = pp->recv;
    b.ep_peer_back = pp->back;
    b.ep_peer_flags = pp->flags;
    b.ep_epoch = pp->epoch;
    b.ep_done = pp->done;
}

namespace kq {
// The three stages; pp != nullptr selects the exchange over peer memory (the
// buffers are the communicator's windows then, and send / recv / ret / back unused).
int moe_ep_dispatch(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens, uint32_t n_tokens,
                    const float *x, const float *router_logits, void *send, const EpPeer *pp) {
    int s = ep_check(m, n_ranks, max_tokens);
    if (s) return s;
    if (n_tokens > max_tokens || (!pp && (!send || !aligned16(send)))) return KATALI_ERR_BAD_ARG;
    if (n_tokens && (!x || !router_logits || !aligned16(x))) return KATALI_ERR_BAD_ARG;
    const uint32_t K = (uint32_t)m->plan[0].K;
    if (max_tokens > m->ep_src_cap) {
        cudaError_t e = cudaStreamSynchronize(g_stream);
        if (e != cudaSuccess) return cuda_fail(e);
        cudaFree(m->ep_src_ids);
        m->ep_src_cap = 0;
        e = cudaMalloc((void **)&m->ep_src_ids, 4ull * K * max_tokens);
        if (e != cudaSuccess) {
            m->ep_src_ids = nullptr;
            return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : cuda_fail(e);
        }
        m->ep_src_cap = max_tokens;
    }
    kq::MoeBatchParams b = batch_params(m, 0);
    ep_fill(b, m, n_ranks, max_tokens);
    ep_peer_fill(b, pp);
    b.ep_tokens = (int)n_tokens;
    b.X = x;
    b.logits = router_logits;
    b.ep_send = (uint8_t *)send;
    return finish(kq::launch_moe_ep_dispatch(b, g_stream));
}

int moe_ep_experts(KataliMoe *m, uint32_t n_ranks, uint32_t rank, uint32_t max_tokens,
                   const void *recv, void *ret, const EpPeer *pp) {
    int s = ep_check(m, n_ranks, max_tokens);
    if (s) return s;
    if (rank >= n_ranks || (!pp && (!recv || !ret || !aligned16(recv) || !aligned16(ret))))
        return KATALI_ERR_BAD_ARG;
    const int T = (int)(n_ranks * max_tokens);
    if (!pp && ep_fused_ok(m, T)) {  // the fused kernel over the received pairs
        kq::MoeParams p = m->plan[KATALI_MOE_Q8_1];
        kq::moe_plan_dec_apart(p, g_max_smem);  // rounds overlap when shared memory allows
        p.experts = m->d_table;
        p.x = nullptr;
        p.logits = nullptr;
        p.ids = nullptr;
        p.w = nullptr;
        p.y = nullptr;
        p.hbuf = m->hbuf;
        p.sync = m->sync;
        p.status = g_status_dev;
        p.dbg_ids = m->dbg_ids;
        p.dbg_w = m->dbg_w;
        p.route_only = 0;
        p.trace = nullptr;
        p.ep_recv = (const uint8_t *)recv;
        p.ep_ret = (double *)ret;
        p.ep_slots = (uint32_t)T;
        p.ep_slot_bytes = ep_slot_bytes(m->plan[0]);
        p.ep_hdr_bytes = ep_hdr_bytes(m->plan[0].K);
        return finish(kq::launch_moe_ep(p, m->grid, g_stream));
    }
    s = grow_batch_scratch(m, T);
    if (s) return s;
    kq::MoeBatchParams b = batch_params(m, T);
    ep_fill(b, m, n_ranks, max_tokens);
    ep_peer_fill(b, pp);
    b.ep_recv = (const uint8_t *)recv;
    b.ep_ret = (double *)ret;
    return finish(kq::launch_moe_ep_experts(b, g_stream));
}

// The whole layer over peer memory in one launch (dispatch, experts in the fused kernel,
// return, combine), when the exchange is small enough for it; KATALI_OK when it ran,
// KATALI_ERR_UNSUPPORTED_SHAPE when the caller should run the three stages instead.
// The single-launch expert-parallel layer's parameters (moe_ep_layer_fused without the
// launch); allocates the layer's routing record on first use, so it runs before any capture.
int moe_ep_fused_params(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens, uint32_t n_tokens,
                        const float *x, const float *router_logits, float *y, const EpPeer *pp,
                        double *ret_scratch, MoeParams *out, int *grid) {
    int s = ep_check(m, n_ranks, max_tokens);
    if (s) return s;
    if (!pp || !ret_scratch || !ep_fused_ok(m, (int)(n_ranks * max_tokens)))
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    if (n_tokens > max_tokens) return KATALI_ERR_BAD_ARG;
    if (n_tokens && (!x || !router_logits || !y || !aligned16(x))) return KATALI_ERR_BAD_ARG;
    const uint32_t K = (uint32_t)m->plan[0].K;
    if (max_tokens > m->ep_route_cap) {
        // Zeroed: a word of it counts only once it carries the current call number (>= 1).
        cudaError_t e = cudaStreamSynchronize(g_stream);
        if (e != cudaSuccess) return cuda_fail(e);
        cudaFree(m->ep_route);
        m->ep_route_cap = 0;
        e = cudaMalloc((void **)&m->ep_route, 8ull * K * max_tokens);
        if (e == cudaSuccess) e = cudaMemsetAsync(m->ep_route, 0, 8ull * K * max_tokens, g_stream);
        if (e != cudaSuccess) {
            cudaFree(m->ep_route);
            m->ep_route = nullptr;
            return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : cuda_fail(e);
        }
        m->ep_route_cap = max_tokens;
    }
    kq::MoeParams p = m->plan[KATALI_MOE_Q8_1];
    kq::moe_plan_dec_apart(p, g_max_smem);  // rounds overlap when shared memory allows
    p.experts = m->d_table;
    p.x = x;
    p.logits = router_logits;
    p.ids = nullptr;
    p.w = nullptr;
    p.y = y;
    p.hbuf = m->hbuf;
    p.sync = m->sync;
    p.status = g_status_dev;
    p.dbg_ids = m->dbg_ids;
    p.dbg_w = m->dbg_w;
    p.route_only = 0;
    p.trace = m->trace;  // optional per-stage timestamps (katali_cuda_debug_moe_trace)
    p.ep_recv = nullptr;  // this rank's window, chosen on the device
    p.ep_ret = ret_scratch;
    p.ep_slots = n_ranks * max_tokens;
    p.ep_slot_bytes = ep_slot_bytes(m->plan[0]);
    p.ep_hdr_bytes = ep_hdr_bytes(K);
    p.ep_rank = pp->rank;
    p.ep_ranks = (int)n_ranks;
    p.ep_tmax = (int)max_tokens;
    p.ep_tokens = (int)n_tokens;
    p.ep_route_rec = m->ep_route;
    p.ep_peer_recv = pp->recv;
    p.ep_peer_back = pp->back;
    p.ep_peer_flags = pp->flags;
    p.ep_epoch = pp->epoch;
    p.ep_done = pp->done;
    p.ep_peer_trecv = pp->trecv;
    p.ep_peer_tback = pp->tback;
    p.ep_peer_tdone = pp->tdone;
    p.ep_tslot_words = pp->tslot_words;
    if (!pp->trecv) return KATALI_ERR_UNSUPPORTED_SHAPE;  // window without the tagged regions
    *out = p;
    *grid = m->grid;
    return KATALI_OK;
}

int moe_ep_layer_fused(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens, uint32_t n_tokens,
                       const float *x, const float *router_logits, float *y, const EpPeer *pp,
                       double *ret_scratch) {
    kq::MoeParams p;
    int grid = 0;
    const int s = moe_ep_fused_params(m, n_ranks, max_tokens, n_tokens, x, router_logits, y, pp,
                                      ret_scratch, &p, &grid);
    if (s) return s;
    return finish(kq::launch_moe_ep_layer(p, grid, g_stream));
}

int moe_ep_combine(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens, uint32_t n_tokens,
                   const void *back, float *y, const EpPeer *pp) {
    int s = ep_check(m, n_ranks, max_tokens);
    if (s) return s;
    if (n_tokens > max_tokens || n_tokens > m->ep_src_cap || (!pp && (!back || !aligned16(back))))
        return KATALI_ERR_BAD_ARG;
    if (n_tokens == 0 && !pp) return KATALI_OK;  // over peer memory the call must still close
    if (n_tokens && !y) return KATALI_ERR_BAD_ARG;
    kq::MoeBatchParams b = batch_params(m, 0);
    ep_fill(b, m, n_ranks, max_tokens);
    ep_peer_fill(b, pp);
    b.ep_tokens = (int)n_tokens;
    b.ep_back = (const double *)back;
    b.Y = y;
    return finish(kq::launch_moe_ep_combine(b, g_stream));
}
}  // namespace kq

extern "C" {

int katali_cuda_moe_ep_dispatch(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens,
                                uint32_t n_tokens, const float *x, const float *router_logits,
                                void *send) {
    return kq::moe_ep_dispatch(m, n_ranks, max_tokens, n_tokens, x, router_logits, send, nullptr);
}

int katali_cuda_moe_ep_experts(KataliMoe *m, uint32_t n_ranks, uint32_t rank,
                               uint32_t max_tokens, const void *recv, void *ret) {
    return kq::moe_ep_experts(m, n_ranks, rank, max_tokens, recv, ret, nullptr);
}

int katali_cuda_moe_ep_combine(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens,
                               uint32_t n_tokens, const void *back, float *y) {
    return kq::moe_ep_combine(m, n_ranks, max_tokens, n_tokens, back, y, nullptr);
}

int katali_cuda_debug_moe_trace(KataliMoe *m, uint64_t *trace, int *grid) {
    if (!m) return KATALI_ERR_BAD_ARG;
    m->trace = trace;
    if (grid) *grid = m->grid;
    return KATALI_OK;
}

int katali_cuda_debug_route(KataliMoe *m, const float *router_logits, int32_t *ids, float *w) {
    if (!m || !router_logits || !ids || !w) return KATALI_ERR_BAD_ARG;
    int s = moe_run(m, nullptr, router_logits, nullptr, nullptr, nullptr,
                    0, 1);
    if (s) return s;
    const int K = m->plan[0].K;
    cudaError_t e = cudaMemcpyAsync(ids, m->dbg_ids, 4 * K, cudaMemcpyDeviceToDevice, g_stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(w, m->dbg_w, 4 * K, cudaMemcpyDeviceToDevice, g_stream);
    return finish(e);
}

}  // extern "C"
