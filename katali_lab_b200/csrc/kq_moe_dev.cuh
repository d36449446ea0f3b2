// kq_moe_dev.cuh — device pieces of the fused MoE kernel (kq_moe.cu): barrier and timer
// primitives, the phase trace, the split bulk copy, routing (top-k over the router logits
// with deterministic ties, softmax weights) and the Q4_K x q8_1 unit dot with the
// activation unit held in registers.
#pragma once

#include "kq_device.cuh"
#include "kq_launch.h"

namespace kq {

constexpr int MOE_WARPS = 16;
constexpr int MOE_THREADS = MOE_WARPS * 32;

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void trace(const MoeParams &p, int slot) {
    if (p.trace && threadIdx.x == 0) {
        p.trace[blockIdx.x * TRACE_SLOTS + slot] = globaltimer();
        if (slot == 0 || slot == 8)  // SM cycle counter beside the first and last stamps
            p.trace[blockIdx.x * TRACE_SLOTS + 16 + (slot == 8)] = (uint64_t)clock64();
    }
}

__device__ __forceinline__ void bulk_g2s_split(uint8_t *dst, const uint8_t *src, uint32_t bytes,
                                               uint64_t *bar, uint64_t pol,
                                               volatile uint32_t *status = nullptr) {
    if (!src) {  // expert not resident: account for the bytes, report, copy nothing
        if (status) atomicOr((uint32_t *)status, KQ_STATUS_NOT_RESIDENT);
        mbar_complete_tx(bar, bytes);
        return;
    }
    while (bytes) {
        const uint32_t n = bytes > 32768u ? 32768u : bytes;
        bulk_g2s_hint(dst, src, n, bar, pol);
        dst += n;
        src += n;
        bytes -= n;
    }
}

// Router logits are read through the read-only path, except when this launch wrote them
// itself (router folded into the launch: other CTAs' stores, seen after a grid barrier).
template <int RT>
__device__ __forceinline__ float ld_logit(const float *a) {
    if constexpr (RT != 0) return __ldcg(a);
    else return __ldg(a);
}
template <int RT>
__device__ __forceinline__ float4 ld_logit4(const float *a) {
    if constexpr (RT != 0) return __ldcg(reinterpret_cast<const float4 *>(a));
    else return __ldg(reinterpret_cast<const float4 *>(a));
}

// Softmax weights of the chosen ids (lane 0 writes s_w); shared by both top-k paths.
template <int RT = 0>
__device__ __forceinline__ void route_weights(const MoeParams &p, const float *L, const float *lg, int npl,
                                              int lane, int32_t *s_ids, float *s_w) {
    const int n = p.n_experts, K = p.K;
    const float m = ld_logit<RT>(&L[s_ids[0]]);
    double S = 0.0;
    if (!p.norm) {  // sum over all n logits (lane-owned contiguous ranges)
        const int per = (n + 31) >> 5;
        for (int i = 0; i < per; ++i) {
            const int idx = lane * per + i;
            if (idx < n) S += (double)kq_expf(__fsub_rn(lg ? lg[i] : ld_logit<RT>(&L[idx]), m));
        }
        S = warp_sum_d(S);
    }
    // lane t < K: e_t; every lane then sums e_0..e_{K-1} in order (the
    // restatement's order) and lane t divides its own weight.
    const float e = lane < K ? kq_expf(__fsub_rn(ld_logit<RT>(&L[s_ids[lane]]), m)) : 0.0f;
    if (p.norm) {
        S = 0.0;
        for (int t = 0; t < K; ++t) S += (double)__shfl_sync(KQ_FULL, e, t);
    }
    if (lane < K) s_w[lane] = (float)((double)e / S);
    __syncwarp();
}

// Composite routing key: order_key(logit) in the high word, ~id in the low word,
// so a larger key is a larger logit or, for equal logits, a lower expert id.
__device__ __forceinline__ uint64_t route_key(float f, int idx) {
    return ((uint64_t)order_key(f) << 32) | (uint32_t)(~idx);
}
__device__ __forceinline__ void ce_desc(uint64_t &a, uint64_t &b) {
    const uint64_t hi = a > b ? a : b, lo = a > b ? b : a;
    a = hi;
    b = lo;
}

// Top-k by one warp for n <= 256: lane l owns ids [8l, 8l+8), sorts its 8 keys
// (Batcher odd-even merge network), then each round takes the warp maximum of
// the lane heads with two redux steps and the winning lane pops its head. The lane's
// logits stay in lv, so route_weights_regs can form the weights without a second read
// of the logits from global memory.
template <int RT = 0>
__device__ __forceinline__ void route_regs(const MoeParams &p, const float *L, int lane, int32_t *s_ids,
                                           float *s_w, bool weights, float (&lv)[8]) {
    const int n = p.n_experts, K = p.K;
    const int npl = (n + 31) >> 5;
    uint64_t v[8];
    if (n == 256) {  // two 16-byte loads per lane, contiguous across the warp
        const float4 l0 = ld_logit4<RT>(L + 8 * lane);
        const float4 l1 = ld_logit4<RT>(L + 8 * lane + 4);
        lv[0] = l0.x; lv[1] = l0.y; lv[2] = l0.z; lv[3] = l0.w;
        lv[4] = l1.x; lv[5] = l1.y; lv[6] = l1.z; lv[7] = l1.w;
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = route_key(lv[i], 8 * lane + i);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = lane * npl + i;
            const bool live = i < npl && idx < n;
            lv[i] = live ? ld_logit<RT>(&L[idx]) : 0.0f;
            v[i] = live ? route_key(lv[i], idx) : 0ull;
        }
    }
    trace(p, 9);
    ce_desc(v[0], v[1]); ce_desc(v[2], v[3]); ce_desc(v[4], v[5]); ce_desc(v[6], v[7]);
    ce_desc(v[0], v[2]); ce_desc(v[1], v[3]); ce_desc(v[4], v[6]); ce_desc(v[5], v[7]);
    ce_desc(v[1], v[2]); ce_desc(v[5], v[6]);
    ce_desc(v[0], v[4]); ce_desc(v[1], v[5]); ce_desc(v[2], v[6]); ce_desc(v[3], v[7]);
    ce_desc(v[2], v[4]); ce_desc(v[3], v[5]);
    ce_desc(v[1], v[2]); ce_desc(v[3], v[4]); ce_desc(v[5], v[6]);
    trace(p, 10);
    for (int t = 0; t < K; ++t) {
        const uint32_t hi = (uint32_t)(v[0] >> 32), lo = (uint32_t)v[0];
        const uint32_t Mh = __reduce_max_sync(KQ_FULL, hi);
        const uint32_t Ml = __reduce_max_sync(KQ_FULL, hi == Mh ? lo : 0u);
        const bool won = (hi == Mh) && (lo == Ml) && (v[0] != 0ull);
#pragma unroll
        for (int i = 0; i < 7; ++i) v[i] = won ? v[i + 1] : v[i];
        v[7] = won ? 0ull : v[7];
        if (lane == 0) s_ids[t] = (int32_t)(~Ml);
    }
    __syncwarp();
    trace(p, 11);
    if (weights) route_weights<RT>(p, L, nullptr, 0, lane, s_ids, s_w);
}

// Softmax weights of the chosen ids from route_regs' registers: the same arithmetic as
// route_weights (m = the top logit, e_t = exp(l_t - m), S = sum of e over the top-k in
// order, or over all n logits in the lanes' contiguous ranges), with no global read: the
// chosen logits come from their owners' registers by a shuffle each.
__device__ __forceinline__ void route_weights_regs(const MoeParams &p, int lane, const float (&lv)[8],
                                                   const int32_t *s_ids, float *s_w) {
    const int n = p.n_experts, K = p.K;
    const int npl = (n + 31) >> 5;
    // lane t < K: the t-th chosen logit, fetched from its owner lane by eight independent
    // shuffles (one per register slot) and a select
    float mine = 0.0f;
    {
        const int id = lane < K ? s_ids[lane] : 0, src = id / npl, slot = id % npl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float v = __shfl_sync(KQ_FULL, lv[j], src);
            mine = slot == j ? v : mine;
        }
        if (lane >= K) mine = 0.0f;
    }
    const float m = __shfl_sync(KQ_FULL, mine, 0);
    double S = 0.0;
    if (!p.norm) {
        const int per = (n + 31) >> 5;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < per && lane * per + i < n) S += (double)kq_expf(__fsub_rn(lv[i], m));
        S = warp_sum_d(S);
    }
    const float e = lane < K ? kq_expf(__fsub_rn(mine, m)) : 0.0f;
    if (p.norm) {
        S = 0.0;
        for (int t = 0; t < K; ++t) S += (double)__shfl_sync(KQ_FULL, e, t);
    }
    if (lane < K) s_w[lane] = (float)((double)e / S);
    __syncwarp();
}

// Generic top-k for n_experts > 256: logits staged in shared memory.
template <int RT = 0>
__device__ void route_smem(const MoeParams &p, const float *L, float *s_logits, int32_t *s_ids, float *s_w,
                           int lane, bool weights) {
    const int n = p.n_experts, K = p.K;
    for (int i = lane; i < n; i += 32) s_logits[i] = ld_logit<RT>(&L[i]);
    __syncwarp();
    const int npl = (n + 31) >> 5;
    uint32_t taken = 0;
    for (int t = 0; t < K; ++t) {
        uint32_t bk = 0;
        int bi = -1;
        for (int i = 0; i < npl; ++i) {
            const int idx = lane * npl + i;
            if (idx < n && !((taken >> i) & 1u)) {
                const uint32_t key = order_key(s_logits[idx]);
                if (bi < 0 || key > bk) {
                    bk = key;
                    bi = i;
                }
            }
        }
        const uint32_t M = __reduce_max_sync(KQ_FULL, bi >= 0 ? bk : 0u);
        const uint32_t ball = __ballot_sync(KQ_FULL, bi >= 0 && bk == M);
        const int win = __ffs((int)ball) - 1;
        const int widx = __shfl_sync(KQ_FULL, lane * npl + bi, win);
        if (lane == win) taken |= 1u << bi;
        if (lane == 0) s_ids[t] = widx;
    }
    __syncwarp();
    float lg[32];
    for (int i = 0; i < npl; ++i) {
        const int idx = lane * npl + i;
        lg[i] = idx < n ? s_logits[idx] : 0.0f;
    }
    if (weights) route_weights<RT>(p, L, lg, npl, lane, s_ids, s_w);
}

// Top-k routing by warp 0. n <= 256: the registered path (lv, s_lg filled, so the caller
// may form the weights later with route_weights_regs); else logits staged in shared memory.
// weights: form the softmax weights now.
template <int RT = 0>
__device__ __forceinline__ void route(const MoeParams &p, const float *L, float *s_logits, int32_t *s_ids,
                                      float *s_w, int lane, bool weights = true) {
    float lv[8];
    if (p.n_experts <= 256) route_regs<RT>(p, L, lane, s_ids, s_w, weights, lv);
    else route_smem<RT>(p, L, s_logits, s_ids, s_w, lane, weights);
}

// This lane's Q4_K unit of x held in registers (phase A reuses it for every row).
struct Q4Act {
    uint4 a0, a1, a2, a3;
    double dx0, dx1;
    int xs0, xs1;
};
__device__ __forceinline__ Q4Act load_q4act(const ActQ8 &a, int u) {
    const int g = 8 * (u >> 2) + 2 * (u & 3);
    const uint4 *ap = reinterpret_cast<const uint4 *>(a.q + 32 * g);
    return Q4Act{ap[0], ap[1], ap[2], ap[3], (double)a.d[g], (double)a.d[g + 1], a.s32[g], a.s32[g + 1]};
}
// q4k_q8_unit with register activations: identical terms.
// The unit's arithmetic on its bytes in registers: block header h, the 32 bytes of nibbles
// w0, w1 of sub-block pair c.
__device__ __forceinline__ double q4k_q8_unit_v(const uint4 &h, const uint4 &w0, const uint4 &w1, int c,
                                                const Q4Act &A) {
    const uint32_t M = 0x0F0F0F0Fu;
    int lo = 0, hi = 0;
    lo = __dp4a((int)(w0.x & M), (int)A.a0.x, lo);
    hi = __dp4a((int)((w0.x >> 4) & M), (int)A.a2.x, hi);
    lo = __dp4a((int)(w0.y & M), (int)A.a0.y, lo);
    hi = __dp4a((int)((w0.y >> 4) & M), (int)A.a2.y, hi);
    lo = __dp4a((int)(w0.z & M), (int)A.a0.z, lo);
    hi = __dp4a((int)((w0.z >> 4) & M), (int)A.a2.z, hi);
    lo = __dp4a((int)(w0.w & M), (int)A.a0.w, lo);
    hi = __dp4a((int)((w0.w >> 4) & M), (int)A.a2.w, hi);
    lo = __dp4a((int)(w1.x & M), (int)A.a1.x, lo);
    hi = __dp4a((int)((w1.x >> 4) & M), (int)A.a3.x, hi);
    lo = __dp4a((int)(w1.y & M), (int)A.a1.y, lo);
    hi = __dp4a((int)((w1.y >> 4) & M), (int)A.a3.y, hi);
    lo = __dp4a((int)(w1.z & M), (int)A.a1.z, lo);
    hi = __dp4a((int)((w1.z >> 4) & M), (int)A.a3.z, hi);
    lo = __dp4a((int)(w1.w & M), (int)A.a1.w, lo);
    hi = __dp4a((int)((w1.w >> 4) & M), (int)A.a3.w, hi);
    int sc0, m0, sc1, m1;
    q4k_scales(h, c, sc0, m0, sc1, m1);
    const double d = (double)h2f(h.x), dmin = (double)h2f(h.x >> 16);
    return ((d * A.dx0) * (double)(sc0 * lo) - (dmin * A.dx0) * (double)(m0 * A.xs0)) +
           ((d * A.dx1) * (double)(sc1 * hi) - (dmin * A.dx1) * (double)(m1 * A.xs1));
}
// Unit u of a Q4_K row in shared memory.
__device__ __forceinline__ double q4k_q8_unit_r(const uint8_t *row, int u, const Q4Act &A) {
    const int b = u >> 2, c = u & 3;
    const uint8_t *blk = row + Q4K_BYTES * b;
    return q4k_q8_unit_v(*reinterpret_cast<const uint4 *>(blk),
                         *reinterpret_cast<const uint4 *>(blk + 16 + 32 * c),
                         *reinterpret_cast<const uint4 *>(blk + 32 + 32 * c), c, A);
}

}  // namespace kq
