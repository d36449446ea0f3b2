// kq_moe_static.cu — katali_cuda_moe_layer_static: the fused MoE layer for callers
// that cannot allocate device memory.
//
// Some hosts cannot call cudaMalloc from the code path that runs a layer: an
// engine whose device memory is owned by another allocator or runtime, a plugin
// loaded into a process that forbids new device allocations after start-up, or
// code that must not grow the memory footprint after a budget check (the
// reference refuses unsafe contexts up front, README.md:62-90). This entry point
// runs the same kernel as katali_cuda_moe_layer but allocates nothing: the
// layer's expert-pointer table, the h records and the grid-barrier counters live
// in the file-scope array below, which every GPU that loads the library holds
// until the process exits.
//
// Use rules: the first call on a device looks the array up for that device
// (cudaGetSymbolAddress), so make that first call before any stream capture.
// Every call shares the one array and overwrites what the previous call left
// there; calls that overlap on the GPU (different streams, or two host threads)
// race on it and must be serialised by the caller. A call is synchronous: it
// copies the expert table from host memory, launches the layer, reads the
// kernel's status word back and waits for its stream before it returns.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include "katali_cuda.h"
#include "kq_launch.h"

namespace kq {
void set_status_message(const char *msg);
}

namespace {

// Every error return names its reason for katali_cuda_status().
int fail(int code, const char *msg) {
    kq::set_status_message(msg);
    return code;
}
int fail_cuda(const char *what, cudaError_t e) {
    char msg[200];
    snprintf(msg, sizeof msg, "katali_cuda_moe_layer_static: %s: %s", what, cudaGetErrorString(e));
    kq::set_status_message(msg);
    return KATALI_ERR_CUDA;
}

constexpr size_t TABLE_BYTES = 3u * KATALI_MOE_STATIC_MAX_EXPERTS * sizeof(void *) + 256;
constexpr size_t H_BYTES = (size_t)KATALI_MOE_STATIC_MAX_TOPK_FFN * sizeof(float);
constexpr size_t SYNC_OFF = TABLE_BYTES + H_BYTES;  // barrier counter, unused, status word, counter base
constexpr size_t SCRATCH_BYTES = SYNC_OFF + 256;

static __device__ __align__(256) unsigned char g_moe_scratch[SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
unsigned char *g_scratch[MAX_DEVICES];  // device address of g_moe_scratch, per device
int g_sms[MAX_DEVICES];
int g_smem[MAX_DEVICES];

uint64_t rbytes(uint32_t type, uint64_t cols) {
    if (cols % 256) return 0;
    if (type == KATALI_TYPE_Q4_K) return cols / 256 * 144;
    if (type == KATALI_TYPE_Q6_K) return cols / 256 * 210;
    return 0;
}

// Per-device set-up on first use: the scratch array's device address (a host-side
// reference to g_moe_scratch is not a device address) and the launch limits.
int setup_device(int dev) {
    if (g_scratch[dev]) return KATALI_OK;
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_moe_scratch);
    if (e != cudaSuccess || !ptr) {
        char msg[160];
        snprintf(msg, sizeof msg, "cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        kq::set_status_message(msg);
        return KATALI_ERR_CUDA;
    }
    int sms = 0, smem = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return fail_cuda("device attribute query", e);
    g_sms[dev] = sms;
    g_smem[dev] = smem;
    g_scratch[dev] = static_cast<unsigned char *>(ptr);
    return KATALI_OK;
}

}  // namespace

extern "C" int katali_cuda_moe_layer_static(const KataliMoeDesc *d, const float *x,
                                            const float *router_logits, float *y, uint32_t mode,
                                            void *stream) {
    if (!d || !d->experts || !x || !router_logits || !y || mode > 1)
        return fail(KATALI_ERR_BAD_ARG, "katali_cuda_moe_layer_static: NULL argument or mode > 1");
    if (((uintptr_t)x & 15u) != 0)
        return fail(KATALI_ERR_BAD_ARG, "katali_cuda_moe_layer_static: x is not 16-byte aligned");
    if (d->top_k == 0 || d->top_k > (uint32_t)kq::MOE_MAX_K || d->top_k > d->n_experts)
        return fail(KATALI_ERR_BAD_ARG, "katali_cuda_moe_layer_static: top_k out of range");
    if (d->n_experts > KATALI_MOE_STATIC_MAX_EXPERTS ||
        (uint64_t)d->top_k * d->ffn > KATALI_MOE_STATIC_MAX_TOPK_FFN) {
        char msg[200];
        snprintf(msg, sizeof msg,
                 "katali_cuda_moe_layer_static: n_experts %u / top_k*ffn %llu exceed the static "
                 "scratch (max %d experts, top_k*ffn <= %d)",
                 d->n_experts, (unsigned long long)d->top_k * d->ffn,
                 KATALI_MOE_STATIC_MAX_EXPERTS, KATALI_MOE_STATIC_MAX_TOPK_FFN);
        kq::set_status_message(msg);
        return KATALI_ERR_UNSUPPORTED_SHAPE;
    }
    const uint64_t rbg = rbytes(d->gate_type, d->hidden), rbu = rbytes(d->up_type, d->hidden);
    const uint64_t rbd = rbytes(d->down_type, d->ffn);
    if (!rbg || !rbu || !rbd || rbg % 16 || rbu % 16)
        return fail(KATALI_ERR_UNSUPPORTED_SHAPE,
                    "katali_cuda_moe_layer_static: gate/up must be Q4_K and down Q4_K or Q6_K, "
                    "with hidden and ffn multiples of 256");
    for (uint32_t i = 0; i < 3 * d->n_experts; ++i)  // NULL: not resident (checked on device)
        if ((uintptr_t)d->experts[i] & 15u)
            return fail(KATALI_ERR_BAD_ARG, "katali_cuda_moe_layer_static: expert tensor not 16-byte aligned");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES)
        return fail(KATALI_ERR_NO_DEVICE, "katali_cuda_moe_layer_static: no current CUDA device");
    int s = setup_device(dev);
    if (s) return s;

    kq::MoeParams p = {};
    p.n_experts = (int)d->n_experts;
    p.H = (int)d->hidden;
    p.F = (int)d->ffn;
    p.K = (int)d->top_k;
    p.norm = (d->flags & KATALI_MOE_NORM_TOPK) ? 1 : 0;
    p.mode = (int)mode;
    p.gate_type = d->gate_type;
    p.up_type = d->up_type;
    p.down_type = d->down_type;
    p.rbg = (uint32_t)rbg;
    p.rbu = (uint32_t)rbu;
    p.rbd = (uint32_t)rbd;
    const int grid = g_sms[dev];
    if (kq::moe_plan(p, grid, g_smem[dev]) != 0)
        return fail(KATALI_ERR_UNSUPPORTED_SHAPE,
                    "katali_cuda_moe_layer_static: the layer does not fit the fused kernel's shared memory");

    unsigned char *base = g_scratch[dev];
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t *sync = reinterpret_cast<uint32_t *>(base + SYNC_OFF);
    // The table is the caller's; the counters and the status word must start at zero.
    cudaError_t e = cudaMemcpyAsync(base, d->experts, 3u * d->n_experts * sizeof(void *),
                                    cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(sync, 0, 16, st);
    if (e != cudaSuccess) return fail_cuda("table copy / counter reset", e);
    p.experts = reinterpret_cast<const uint8_t *const *>(base);
    p.x = x;
    p.logits = router_logits;
    p.y = y;
    p.hbuf = reinterpret_cast<float *>(base + TABLE_BYTES);
    p.sync = sync;
    p.status = sync + 2;
    e = kq::launch_moe(p, grid, st);
    if (e != cudaSuccess) return fail_cuda("launch", e);
    uint32_t status = 0;  // a device-side wait that gave up leaves a bit here
    e = cudaMemcpyAsync(&status, sync + 2, sizeof status, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail_cuda("status read-back", e);
    if (status) {
        char msg[160];
        const bool nr = (status & kq::KQ_STATUS_NOT_RESIDENT) != 0;
        snprintf(msg, sizeof msg, "katali_cuda_moe_layer_static: %s (bits 0x%x)",
                 nr ? "a selected expert is not resident" : "device-side wait timed out", status);
        kq::set_status_message(msg);
        return nr ? KATALI_ERR_NOT_RESIDENT : KATALI_ERR_TIMEOUT;
    }
    return KATALI_OK;
}
