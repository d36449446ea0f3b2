// kq_expert_cache.cu — the expert residency tier (katali_cuda_expert_*).
//
// A fixed pool of device slots, each holding one expert's gate, up and down
// matrices in native GGUF bytes, fed from host memory (typically an mmap'd GGUF
// file) by asynchronous copies on the cache's own side stream, so uploads
// overlap the layer kernels on the compute stream. The reference engine pages
// experts between SSD, host RAM and VRAM and names its bottleneck the uploads
// and syncs around them (README.md:13,21,260,329-333); here:
//   - host ranges are page-locked once (cudaHostRegister) so copies are truly
//     asynchronous;
//   - a slot is reused least-recently-used first, and its new copy waits (by an
//     event, not the host) for every compute call enqueued before the reuse;
//   - binding an expert of a layer to a slot makes the compute stream wait for
//     that slot's copy (event) and updates the layer's pointer table in stream
//     order; an evicted slot's bindings become NULL, so a later call that
//     selects the expert reports KATALI_ERR_NOT_RESIDENT instead of reading
//     another expert's bytes.
#include <cuda_runtime.h>
#include <stdio.h>

#include <map>
#include <unordered_map>
#include <utility>
#include <vector>

#include "katali_cuda.h"

namespace kq {
int ensure_runtime();
void set_status_message(const char *msg);
cudaStream_t current_stream();
int moe_set_expert_async(KataliMoe *m, uint32_t e, const void *g, const void *u, const void *d);
uint32_t moe_n_experts(const KataliMoe *m);
KataliExpertCache *moe_cache(const KataliMoe *m);
void moe_set_cache(KataliMoe *m, KataliExpertCache *c);
}  // namespace kq

namespace {

uint64_t align16(uint64_t v) { return (v + 15) & ~uint64_t(15); }

struct HostExpert {
    const void *ptr[3];
    uint64_t bytes[3];
};

struct Slot {
    bool used = false;
    uint64_t key = 0, last_use = 0;
    cudaEvent_t ready = nullptr;  // recorded on the side stream after the slot's copy
};

int fail(cudaError_t e, const char *what) {
    char msg[200];
    snprintf(msg, sizeof msg, "%s: %s", what, cudaGetErrorString(e));
    kq::set_status_message(msg);
    return e == cudaErrorMemoryAllocation ? KATALI_ERR_OOM : KATALI_ERR_CUDA;
}

}  // namespace

struct KataliExpertCache {
    uint64_t slot_bytes = 0;
    unsigned char *base = nullptr;
    cudaStream_t side = nullptr;
    cudaEvent_t reuse = nullptr;  // recorded on the compute stream before a slot is refilled
    std::vector<Slot> slots;
    std::unordered_map<uint64_t, HostExpert> host;
    std::unordered_map<uint64_t, int> resident;  // key -> slot
    std::map<std::pair<KataliMoe *, uint32_t>, int> bound;  // (layer, expert) -> slot
    std::vector<const void *> pinned;  // host ranges this cache registered
    uint64_t clock = 0;

    unsigned char *slot_ptr(int s, int which, const HostExpert &h) const {
        uint64_t off = 0;
        for (int i = 0; i < which; ++i) off += align16(h.bytes[i]);
        return base + (size_t)s * slot_bytes + off;
    }

    // NULL every layer entry bound to slot s (stream-ordered).
    int unbind_slot(int s) {
        for (auto it = bound.begin(); it != bound.end();) {
            if (it->second == s) {
                int r = kq::moe_set_expert_async(it->first.first, it->first.second, nullptr, nullptr,
                                                 nullptr);
                if (r) return r;
                it = bound.erase(it);
            } else {
                ++it;
            }
        }
        return KATALI_OK;
    }

    int load(uint64_t key, int *slot_out) {
        auto r = resident.find(key);
        if (r != resident.end()) {
            slots[r->second].last_use = ++clock;
            *slot_out = r->second;
            return KATALI_OK;
        }
        auto h = host.find(key);
        if (h == host.end()) {
            kq::set_status_message("katali_cuda_expert: key not registered");
            return KATALI_ERR_BAD_ARG;
        }
        int s = -1;
        for (int i = 0; i < (int)slots.size() && s < 0; ++i)
            if (!slots[i].used) s = i;
        if (s < 0) {  // least recently used
            s = 0;
            for (int i = 1; i < (int)slots.size(); ++i)
                if (slots[i].last_use < slots[s].last_use) s = i;
            int rc = unbind_slot(s);
            if (rc) return rc;
            resident.erase(slots[s].key);
            slots[s].used = false;
        }
        // The refill waits for every compute call enqueued so far (they may read the slot).
        cudaStream_t cs = kq::current_stream();
        cudaError_t e = cudaEventRecord(reuse, cs);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(side, reuse, 0);
        for (int i = 0; i < 3 && e == cudaSuccess; ++i)
            e = cudaMemcpyAsync(slot_ptr(s, i, h->second), h->second.ptr[i], h->second.bytes[i],
                                cudaMemcpyHostToDevice, side);
        if (e == cudaSuccess) e = cudaEventRecord(slots[s].ready, side);
        if (e != cudaSuccess) return fail(e, "expert upload");
        slots[s].used = true;
        slots[s].key = key;
        slots[s].last_use = ++clock;
        resident[key] = s;
        *slot_out = s;
        return KATALI_OK;
    }
};

namespace kq {
void cache_forget_layer(KataliExpertCache *c, KataliMoe *m) {
    for (auto it = c->bound.begin(); it != c->bound.end();)
        it = it->first.first == m ? c->bound.erase(it) : std::next(it);
}
}  // namespace kq

extern "C" {

int katali_cuda_expert_cache_create(uint64_t slot_bytes, uint32_t n_slots, KataliExpertCache **out) {
    if (!out || slot_bytes == 0 || n_slots == 0) return KATALI_ERR_BAD_ARG;
    *out = nullptr;
    // device, own stream and mapped status word (KATALI_ERR_NO_DEVICE without a usable GPU)
    if (const int rs = kq::ensure_runtime()) return rs;
    KataliExpertCache *c = new KataliExpertCache();
    c->slot_bytes = align16(slot_bytes);
    c->slots.resize(n_slots);
    cudaError_t e = cudaMalloc((void **)&c->base, c->slot_bytes * n_slots);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->reuse, cudaEventDisableTiming);
    for (uint32_t i = 0; i < n_slots && e == cudaSuccess; ++i)
        e = cudaEventCreateWithFlags(&c->slots[i].ready, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        int rc = fail(e, "katali_cuda_expert_cache_create");
        katali_cuda_expert_cache_destroy(c);
        return rc;
    }
    *out = c;
    return KATALI_OK;
}

int katali_cuda_expert_cache_destroy(KataliExpertCache *c) {
    if (!c) return KATALI_OK;
    // Layers still bound lose their entries (NULL: not resident) before the slots go.
    for (auto &b : c->bound) {
        kq::moe_set_expert_async(b.first.first, b.first.second, nullptr, nullptr, nullptr);
        kq::moe_set_cache(b.first.first, nullptr);
    }
    c->bound.clear();
    if (kq::current_stream()) cudaStreamSynchronize(kq::current_stream());
    if (c->side) cudaStreamSynchronize(c->side);
    for (const void *p : c->pinned) cudaHostUnregister(const_cast<void *>(p));
    for (auto &s : c->slots)
        if (s.ready) cudaEventDestroy(s.ready);
    if (c->reuse) cudaEventDestroy(c->reuse);
    if (c->side) cudaStreamDestroy(c->side);
    cudaFree(c->base);
    delete c;
    return KATALI_OK;
}

int katali_cuda_expert_register(KataliExpertCache *c, uint64_t key, const void *gate,
                                uint64_t gate_bytes, const void *up, uint64_t up_bytes,
                                const void *down, uint64_t down_bytes) {
    if (!c || !gate || !up || !down || !gate_bytes || !up_bytes || !down_bytes)
        return KATALI_ERR_BAD_ARG;
    if (align16(gate_bytes) + align16(up_bytes) + align16(down_bytes) > c->slot_bytes) {
        kq::set_status_message("katali_cuda_expert_register: expert larger than a slot");
        return KATALI_ERR_BAD_ARG;
    }
    HostExpert h{{gate, up, down}, {gate_bytes, up_bytes, down_bytes}};
    // Page-lock the ranges so the side-stream copies are asynchronous. A range that
    // is already registered (by the caller or an overlapping expert) is fine; one
    // that cannot be registered still copies, synchronously with the host.
    for (int i = 0; i < 3; ++i) {
        cudaError_t e = cudaHostRegister(const_cast<void *>(h.ptr[i]), h.bytes[i],
                                         cudaHostRegisterReadOnly);
        if (e == cudaSuccess) c->pinned.push_back(h.ptr[i]);
        else cudaGetLastError();  // clear it, so later calls do not report it
    }
    c->host[key] = h;
    return KATALI_OK;
}

int katali_cuda_expert_prefetch_async(KataliExpertCache *c, uint64_t key) {
    if (!c) return KATALI_ERR_BAD_ARG;
    int s;
    return c->load(key, &s);
}

int katali_cuda_expert_bind(KataliExpertCache *c, uint64_t key, KataliMoe *m, uint32_t e) {
    if (!c || !m || e >= kq::moe_n_experts(m)) return KATALI_ERR_BAD_ARG;
    if (kq::moe_cache(m) && kq::moe_cache(m) != c) {
        kq::set_status_message("katali_cuda_expert_bind: layer is bound to another cache");
        return KATALI_ERR_BAD_ARG;
    }
    int s;
    int rc = c->load(key, &s);
    if (rc) return rc;
    const HostExpert &h = c->host[key];
    cudaError_t err = cudaStreamWaitEvent(kq::current_stream(), c->slots[s].ready, 0);
    if (err != cudaSuccess) return fail(err, "katali_cuda_expert_bind");
    rc = kq::moe_set_expert_async(m, e, c->slot_ptr(s, 0, h), c->slot_ptr(s, 1, h),
                                  c->slot_ptr(s, 2, h));
    if (rc) return rc;
    c->bound[{m, e}] = s;
    kq::moe_set_cache(m, c);
    return KATALI_OK;
}

int katali_cuda_expert_evict(KataliExpertCache *c, uint64_t key) {
    if (!c) return KATALI_ERR_BAD_ARG;
    auto r = c->resident.find(key);
    if (r == c->resident.end()) return KATALI_OK;
    const int s = r->second;
    int rc = c->unbind_slot(s);
    if (rc) return rc;
    c->slots[s].used = false;
    c->resident.erase(r);
    return KATALI_OK;
}

int katali_cuda_expert_lookup(KataliExpertCache *c, uint64_t key, int *resident, void **gate,
                              void **up, void **down) {
    if (!c || !resident) return KATALI_ERR_BAD_ARG;
    auto r = c->resident.find(key);
    *resident = r != c->resident.end();
    if (!*resident) return KATALI_OK;
    const HostExpert &h = c->host[key];
    if (gate) *gate = c->slot_ptr(r->second, 0, h);
    if (up) *up = c->slot_ptr(r->second, 1, h);
    if (down) *down = c->slot_ptr(r->second, 2, h);
    return KATALI_OK;
}

int katali_cuda_expert_sync(KataliExpertCache *c) {
    if (!c) return KATALI_ERR_BAD_ARG;
    cudaError_t e = cudaStreamSynchronize(c->side);
    return e == cudaSuccess ? KATALI_OK : fail(e, "katali_cuda_expert_sync");
}

}  // extern "C"
