// kq_ep_nccl.cu — expert-parallel MoE layer with the two token exchanges done by
// NCCL inside the plugin (katali_cuda_ep_* / katali_cuda_moe_ep_layer).
//
// One process per GPU; rank r holds experts [r*E/G, (r+1)*E/G) of every layer.
// Per layer call: dispatch (route + q8_1 + one slot per destination rank) ->
// grouped ncclSend/ncclRecv of the slots -> the owned experts of every received
// slot -> grouped ncclSend/ncclRecv of the per-slot partial sums -> combine.
// Slots have a fixed capacity (max_tokens per rank) so no counts are exchanged
// and the whole call can be captured in a CUDA graph.
//
// NCCL is opened at run time (libnccl.so.2): in a process that already loaded an
// NCCL with that soname (a PyTorch host) the same library is shared.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <string.h>

#include <vector>

#include "katali_cuda.h"
#include "kq_launch.h"

namespace kq {
int ensure_runtime();
void set_status_message(const char *msg);
cudaStream_t current_stream();
int moe_ep_dispatch(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens, uint32_t n_tokens,
                    const float *x, const float *router_logits, void *send, const EpPeer *pp);
int moe_ep_experts(KataliMoe *m, uint32_t n_ranks, uint32_t rank, uint32_t max_tokens,
                   const void *recv, void *ret, const EpPeer *pp);
int moe_ep_combine(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens, uint32_t n_tokens,
                   const void *back, float *y, const EpPeer *pp);
int moe_ep_layer_fused(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens, uint32_t n_tokens,
                       const float *x, const float *router_logits, float *y, const EpPeer *pp,
                       double *ret_scratch);
}  // namespace kq

namespace {

struct Nccl {
    void *lib = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

Nccl g_nccl;

template <typename F>
bool sym(F &f, const char *name) {
    f = reinterpret_cast<F>(dlsym(g_nccl.lib, name));
    return f != nullptr;
}

int load_nccl() {
    if (g_nccl.lib) return KATALI_OK;
    const char *names[] = {"libnccl.so.2", "libnccl.so"};
    void *lib = nullptr;
    for (const char *n : names)
        if ((lib = dlopen(n, RTLD_NOW | RTLD_GLOBAL))) break;
    if (!lib) {
        kq::set_status_message("NCCL not found (dlopen libnccl.so.2 failed)");
        return KATALI_ERR_NCCL;
    }
    g_nccl.lib = lib;
    bool ok = sym(g_nccl.GetUniqueId, "ncclGetUniqueId") && sym(g_nccl.CommInitRank, "ncclCommInitRank") &&
              sym(g_nccl.CommDestroy, "ncclCommDestroy") && sym(g_nccl.CommAbort, "ncclCommAbort") &&
              sym(g_nccl.CommGetAsyncError, "ncclCommGetAsyncError") &&
              sym(g_nccl.GroupStart, "ncclGroupStart") && sym(g_nccl.GroupEnd, "ncclGroupEnd") &&
              sym(g_nccl.Send, "ncclSend") && sym(g_nccl.Recv, "ncclRecv") &&
              sym(g_nccl.AllGather, "ncclAllGather") &&
              sym(g_nccl.GetErrorString, "ncclGetErrorString");
    if (!ok) {
        kq::set_status_message("libnccl.so.2 lacks a required symbol");
        g_nccl.lib = nullptr;
        return KATALI_ERR_NCCL;
    }
    return KATALI_OK;
}

int cuda_err(cudaError_t e, const char *what) {
    char msg[200];
    snprintf(msg, sizeof msg, "%s: %s", what, cudaGetErrorString(e));
    kq::set_status_message(msg);
    return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : KATALI_ERR_CUDA;
}

int nccl_fail(ncclResult_t r) {
    char msg[200];
    snprintf(msg, sizeof msg, "NCCL: %s", g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "error");
    kq::set_status_message(msg);
    return KATALI_ERR_NCCL;
}

}  // namespace

struct KataliEp {
    ncclComm_t comm;
    int n_ranks, rank;
    // exchange buffers, grown on demand
    unsigned char *send, *recv, *ret, *back;
    size_t slot_cap, ret_cap;  // bytes per buffer
    // exchange over peer memory (katali_cuda_ep_use_peer_memory)
    int peer_mode;
    unsigned char *win;        // this rank's window: recv, back, flags
    uint64_t win_slot;
    uint32_t win_h, win_tmax;
    std::vector<void *> opened;  // other ranks' windows mapped here
    void *dev_arrays;          // recv[G], back[G], flags[G] pointers, then epoch + 3 counters
    kq::EpPeer peer;
};

namespace {

int grow(unsigned char *&p, size_t &cap, size_t need) {
    if (need <= cap) return KATALI_OK;
    cudaError_t e = cudaStreamSynchronize(kq::current_stream());
    if (e == cudaSuccess) {
        cudaFree(p);
        p = nullptr;
        cap = 0;
        e = cudaMalloc((void **)&p, need);
        if (e != cudaSuccess) p = nullptr;
    }
    if (e != cudaSuccess) {
        kq::set_status_message(cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : KATALI_ERR_CUDA;
    }
    cap = need;
    return KATALI_OK;
}

// Every rank sends `chunk` bytes from buf_out + d * chunk to rank d and receives
// rank d's chunk into buf_in + d * chunk.
int exchange(KataliEp *ep, const unsigned char *out, unsigned char *in, size_t chunk, cudaStream_t st) {
    ncclResult_t r = g_nccl.GroupStart();
    for (int d = 0; d < ep->n_ranks && r == ncclSuccess; ++d) {
        r = g_nccl.Send(out + d * chunk, chunk, ncclUint8, d, ep->comm, st);
        if (r == ncclSuccess) r = g_nccl.Recv(in + d * chunk, chunk, ncclUint8, d, ep->comm, st);
    }
    const ncclResult_t r2 = g_nccl.GroupEnd();
    if (r != ncclSuccess) return nccl_fail(r);
    if (r2 != ncclSuccess) return nccl_fail(r2);
    return KATALI_OK;
}

// Collective: every rank allocates its window, the IPC handles are all-gathered over
// the communicator and every other rank's window is mapped into this process.
int peer_setup(KataliEp *ep, uint64_t slot, uint32_t H, uint32_t tmax, cudaStream_t st) {
    if (ep->win) {
        if (ep->win_slot == slot && ep->win_h == H && ep->win_tmax == tmax) return KATALI_OK;
        kq::set_status_message("peer-memory exchange: layer shape or max_tokens differs from the window");
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    }
    const size_t G = (size_t)ep->n_ranks;
    auto r256 = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t recv = r256(2 * G * tmax * slot), back = r256(2 * G * tmax * (size_t)H * 8),
                 flags = r256(4 * G * sizeof(uint32_t));
    // tagged regions for the single-launch layer, when the exchange is small enough for it
    const bool tagged = G * tmax <= (size_t)kq::MOE_EP_MAX_SLOTS;
    const uint32_t tsw = kq::ep_tslot_words(H);
    const size_t trecv = tagged ? r256(2 * G * tmax * tsw * 8) : 0,
                 tback = tagged ? r256(2 * G * tmax * (size_t)H * 16) : 0,
                 tdone = tagged ? r256(2 * G * 8) : 0;
    const size_t total = recv + back + flags + trecv + tback + tdone;
    cudaError_t e = cudaMalloc((void **)&ep->win, total);
    if (e == cudaSuccess) e = cudaMemsetAsync(ep->win, 0, total, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_err(e, "peer window");
    cudaIpcMemHandle_t mine;
    e = cudaIpcGetMemHandle(&mine, ep->win);
    if (e != cudaSuccess) return cuda_err(e, "cudaIpcGetMemHandle");
    unsigned char *hbuf = nullptr;  // [own handle][G handles]
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    e = cudaMalloc((void **)&hbuf, hb * (G + 1));
    if (e == cudaSuccess) e = cudaMemcpyAsync(hbuf, &mine, hb, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_err(e, "peer handles");
    ncclResult_t r = g_nccl.AllGather(hbuf, hbuf + hb, hb, ncclUint8, ep->comm, st);
    if (r != ncclSuccess) {
        cudaFree(hbuf);
        return nccl_fail(r);
    }
    std::vector<cudaIpcMemHandle_t> all(G);
    e = cudaMemcpyAsync(all.data(), hbuf + hb, hb * G, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFree(hbuf);
    if (e != cudaSuccess) return cuda_err(e, "peer handles");
    std::vector<unsigned char *> base(G);
    for (size_t d = 0; d < G; ++d) {
        if ((int)d == ep->rank) {
            base[d] = ep->win;
            continue;
        }
        void *p = nullptr;
        e = cudaIpcOpenMemHandle(&p, all[d], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_err(e, "cudaIpcOpenMemHandle");
        ep->opened.push_back(p);
        base[d] = (unsigned char *)p;
    }
    std::vector<void *> arrays(6 * G);
    for (size_t d = 0; d < G; ++d) {
        unsigned char *b = base[d];
        arrays[d] = b;
        arrays[G + d] = b + recv;
        arrays[2 * G + d] = b + recv + back;
        arrays[3 * G + d] = tagged ? b + recv + back + flags : nullptr;
        arrays[4 * G + d] = tagged ? b + recv + back + flags + trecv : nullptr;
        arrays[5 * G + d] = tagged ? b + recv + back + flags + trecv + tback : nullptr;
    }
    e = cudaMalloc(&ep->dev_arrays, 6 * G * sizeof(void *) + 64);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(ep->dev_arrays, arrays.data(), 6 * G * sizeof(void *), cudaMemcpyHostToDevice, st);
    uint32_t *words = (uint32_t *)((unsigned char *)ep->dev_arrays + 6 * G * sizeof(void *));
    if (e == cudaSuccess) e = cudaMemsetAsync(words, 0, 64, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_err(e, "peer arrays");
    void **arr = (void **)ep->dev_arrays;
    ep->peer = kq::EpPeer{ep->rank, (uint8_t *const *)arr, (double *const *)(arr + G),
                          (uint32_t *const *)(arr + 2 * G), words, words + 1,
                          tagged ? (uint64_t *const *)(arr + 3 * G) : nullptr,
                          tagged ? (uint64_t *const *)(arr + 4 * G) : nullptr,
                          tagged ? (uint64_t *const *)(arr + 5 * G) : nullptr, tsw};
    ep->win_slot = slot;
    ep->win_h = H;
    ep->win_tmax = tmax;
    return KATALI_OK;
}

}  // namespace

namespace kq {
// For a decoder that launches the single-launch expert-parallel layer from its own step
// (kq_hybrid_api.cu): maps the peer windows (collective on the first call, as the first
// katali_cuda_moe_ep_layer call) and sizes the per-slot scratch for layer m with max_tokens
// tokens per rank; returns the communicator's rank count, peer arrays and scratch.
int ep_peer_prepare(KataliEp *ep, KataliMoe *m, uint32_t max_tokens, uint32_t *n_ranks,
                    const EpPeer **pp, double **ret) {
    if (!ep || !m || max_tokens == 0) return KATALI_ERR_BAD_ARG;
    if (!ep->peer_mode) {
        set_status_message("expert-parallel decode needs the peer-memory exchange "
                           "(katali_cuda_ep_use_peer_memory)");
        return KATALI_ERR_BAD_ARG;
    }
    uint64_t slot = 0, rslot = 0;
    int s = katali_cuda_moe_ep_slot_bytes(m, &slot, &rslot);
    if (s) return s;
    cudaStream_t st = current_stream();
    if ((s = peer_setup(ep, slot, (uint32_t)(rslot / 8), max_tokens, st))) return s;
    size_t r0 = ep->ret_cap, r1 = ep->ret_cap;
    if ((s = grow(ep->ret, r0, rslot * max_tokens * ep->n_ranks)) ||
        (s = grow(ep->back, r1, rslot * max_tokens * ep->n_ranks)))
        return s;
    ep->ret_cap = r0 < r1 ? r0 : r1;
    *n_ranks = (uint32_t)ep->n_ranks;
    *pp = &ep->peer;
    *ret = (double *)ep->ret;
    return KATALI_OK;
}
}  // namespace kq

extern "C" {

int katali_cuda_ep_use_peer_memory(KataliEp *ep, int on) {
    if (!ep) return KATALI_ERR_BAD_ARG;
    ep->peer_mode = on ? 1 : 0;
    return KATALI_OK;
}

int katali_cuda_ep_unique_id(void *id) {
    if (!id) return KATALI_ERR_BAD_ARG;
    int s = load_nccl();
    if (s) return s;
    ncclUniqueId u;
    ncclResult_t r = g_nccl.GetUniqueId(&u);
    if (r != ncclSuccess) return nccl_fail(r);
    memcpy(id, u.internal, sizeof u.internal);
    return KATALI_OK;
}

int katali_cuda_ep_create(uint32_t n_ranks, uint32_t rank, const void *id, KataliEp **out) {
    if (!out || !id || n_ranks == 0 || n_ranks > 64 || rank >= n_ranks) return KATALI_ERR_BAD_ARG;
    *out = nullptr;
    // device, own stream and mapped status word (KATALI_ERR_NO_DEVICE without a usable GPU)
    if (const int rs = kq::ensure_runtime()) return rs;
    int s = load_nccl();
    if (s) return s;
    ncclUniqueId u;
    memcpy(u.internal, id, sizeof u.internal);
    KataliEp *ep = new KataliEp();
    ep->n_ranks = (int)n_ranks;
    ep->rank = (int)rank;
    ncclResult_t r = g_nccl.CommInitRank(&ep->comm, (int)n_ranks, u, (int)rank);
    if (r != ncclSuccess) {
        delete ep;
        return nccl_fail(r);
    }
    *out = ep;
    return KATALI_OK;
}

int katali_cuda_ep_destroy(KataliEp *ep) {
    if (!ep) return KATALI_OK;
    cudaStream_t st = kq::current_stream();
    cudaStreamSynchronize(st);
    ncclResult_t async = ncclSuccess;
    g_nccl.CommGetAsyncError(ep->comm, &async);
    if (ep->win) {
        // no rank may still write into a window that is released: meet first
        if (async == ncclSuccess) {
            void *tmp = nullptr;
            if (cudaMalloc(&tmp, 4 * ep->n_ranks) == cudaSuccess) {
                g_nccl.AllGather(tmp, tmp, 4, ncclUint8, ep->comm, st);  // in place: slot `rank`
                cudaStreamSynchronize(st);
                cudaFree(tmp);
            }
        }
        for (void *p : ep->opened) cudaIpcCloseMemHandle(p);
        cudaFree(ep->dev_arrays);
        cudaFree(ep->win);
    }
    // A communicator with an error pending cannot be destroyed cleanly: abort it.
    if (async != ncclSuccess) g_nccl.CommAbort(ep->comm);
    else g_nccl.CommDestroy(ep->comm);
    cudaFree(ep->send);
    cudaFree(ep->recv);
    cudaFree(ep->ret);
    cudaFree(ep->back);
    delete ep;
    return KATALI_OK;
}

int katali_cuda_moe_ep_layer(KataliMoe *m, KataliEp *ep, uint32_t max_tokens, uint32_t n_tokens,
                             const float *x, const float *router_logits, float *y) {
    if (!m || !ep) return KATALI_ERR_BAD_ARG;
    uint64_t slot = 0, rslot = 0;
    int s = katali_cuda_moe_ep_slot_bytes(m, &slot, &rslot);
    if (s) return s;
    if (max_tokens == 0 || (uint64_t)max_tokens * ep->n_ranks > KATALI_MOE_BATCH_MAX_TOKENS)
        return KATALI_ERR_BAD_ARG;
    cudaStream_t st = kq::current_stream();
    const uint32_t G = (uint32_t)ep->n_ranks;
    if (ep->peer_mode) {  // both exchanges inside the kernels, over NVLink peer memory
        if ((s = peer_setup(ep, slot, (uint32_t)(rslot / 8), max_tokens, st))) return s;
        // small exchanges: the whole layer in one launch (local scratch for the per-slot sums)
        size_t r0 = ep->ret_cap, r1 = ep->ret_cap;
        if ((s = grow(ep->ret, r0, rslot * max_tokens * ep->n_ranks)) ||
            (s = grow(ep->back, r1, rslot * max_tokens * ep->n_ranks)))
            return s;
        ep->ret_cap = r0 < r1 ? r0 : r1;
        s = kq::moe_ep_layer_fused(m, G, max_tokens, n_tokens, x, router_logits, y, &ep->peer,
                                   (double *)ep->ret);
        if (s != KATALI_ERR_UNSUPPORTED_SHAPE) return s;
        if ((s = kq::moe_ep_dispatch(m, G, max_tokens, n_tokens, x, router_logits, nullptr, &ep->peer)))
            return s;
        if ((s = kq::moe_ep_experts(m, G, (uint32_t)ep->rank, max_tokens, nullptr, nullptr, &ep->peer)))
            return s;
        return kq::moe_ep_combine(m, G, max_tokens, n_tokens, nullptr, y, &ep->peer);
    }
    const size_t chunk = slot * max_tokens, rchunk = rslot * max_tokens;
    size_t c0 = ep->slot_cap, c1 = ep->slot_cap;
    if ((s = grow(ep->send, c0, chunk * ep->n_ranks)) || (s = grow(ep->recv, c1, chunk * ep->n_ranks)))
        return s;
    ep->slot_cap = c0 < c1 ? c0 : c1;
    size_t r0 = ep->ret_cap, r1 = ep->ret_cap;
    if ((s = grow(ep->ret, r0, rchunk * ep->n_ranks)) || (s = grow(ep->back, r1, rchunk * ep->n_ranks)))
        return s;
    ep->ret_cap = r0 < r1 ? r0 : r1;
    if ((s = katali_cuda_moe_ep_dispatch(m, G, max_tokens, n_tokens, x, router_logits, ep->send)))
        return s;
    if ((s = exchange(ep, ep->send, ep->recv, chunk, st))) return s;
    if ((s = katali_cuda_moe_ep_experts(m, G, (uint32_t)ep->rank, max_tokens, ep->recv, ep->ret)))
        return s;
    if ((s = exchange(ep, ep->ret, ep->back, rchunk, st))) return s;
    return katali_cuda_moe_ep_combine(m, G, max_tokens, n_tokens, ep->back, y);
}

}  // extern "C"
