// kq_device.cuh — device building blocks of the katali_cuda plugin (sm_100a).
//
// GGUF block layouts (vendor/katali_gguf_dense/src/gguf_dtype.c, V/ below):
//   Q4_K 144 B / 256 w: d f16 @0, dmin f16 @2, 12 B packed 6-bit scales/mins @4,
//        128 B nibbles @16; 64-element chunk c: low nibbles of bytes 32c..32c+31
//        are elements 64c..64c+31, high nibbles 64c+32..64c+63 (V:429-452,350-358)
//   Q6_K 210 B / 256 w: ql[128] @0, qh[64] @128, 16 int8 scales @192, d f16 @208;
//        element e = 128h + 32*quarter + l takes ql[64h + 32(quarter&1) + l]
//        (low nibble for quarter<2, high otherwise) and bits 2*quarter of
//        qh[32h + l]; value d * sc[e/16] * (q - 32) (V:487-512)
//   q8_1  36 B / 32:  d f16 @0, s f16 @2, 32 int8 @4 (V:328-335)
//
// Exactness contract shared with the CPU restatement (oracle/kq_oracle.c):
// integer block sums are exact; each per-q8-block float term is a product of
// values exact in double, rounded once; terms are summed in double and each
// row rounds once to float. kq_expf and the encoders use only IEEE-rounded
// single operations (explicit __f*_rn intrinsics, so nvcc cannot contract
// them), which makes routing weights, silu(g)*u and the q8_1 bytes
// bit-identical to the CPU restatement.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#define KQ_FULL 0xFFFFFFFFu

namespace kq {

constexpr int Q4K_BYTES = 144;
constexpr int Q6K_BYTES = 210;
constexpr int Q81_BYTES = 36;
constexpr uint32_t T_Q8_1 = 9, T_Q4_K = 12, T_Q6_K = 14;

// Bounded waits: iterations of a poll loop with a short sleep. ~2^24 polls of
// >= 64 ns each is well above a second; a wait that runs out sets a status bit
// and returns instead of hanging the GPU.
constexpr uint32_t SPIN_LIMIT = 1u << 24;
constexpr uint32_t ERR_TIMEOUT_TMA = 1u;
constexpr uint32_t ERR_TIMEOUT_GRID = 2u;

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}
__device__ __forceinline__ uint16_t f2h(float f) {
    return __half_as_ushort(__float2half_rn(f));
}

// e^x: Cody-Waite reduction by ln2 (hi/lo split) and a degree-7 Taylor
// polynomial for e^r, |r| <= 0.35. Same operations, in the same order, as
// kqo_expf in the CPU restatement.
__device__ __forceinline__ float kq_expf(float x) {
    if (x != x) return x;
    x = fminf(fmaxf(x, -87.0f), 88.0f);
    const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
    float r = __fmaf_rn(-n, 0.693145751953125f, x);
    r = __fmaf_rn(-n, 1.42860682030941723e-6f, r);
    float p = 1.98412698412698413e-4f;
    p = __fmaf_rn(p, r, 1.38888888888888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333333333333e-3f);
    p = __fmaf_rn(p, r, 4.16666666666666667e-2f);
    p = __fmaf_rn(p, r, 1.66666666666666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const float s = __uint_as_float((uint32_t)((int)n + 127) << 23);
    return __fmul_rn(p, s);
}

__device__ __forceinline__ float kq_silu(float x) {
    return __fdiv_rn(x, __fadd_rn(1.0f, kq_expf(-x)));
}

// Total order for top-k: NaN lowest, -0 == +0, then by value.
__device__ __forceinline__ uint32_t order_key(float f) {
    if (f != f) return 0u;
    const uint32_t u = __float_as_uint(__fadd_rn(f, 0.0f));
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(KQ_FULL, v, o);
    return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(KQ_FULL, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch. A kernel launched with the programmatic stream
// serialization attribute may start before the previous kernel on its stream has
// finished; pdl_wait() blocks the calling thread until that kernel has completed
// and its memory is visible (a no-op for an ordinary launch). pdl_trigger() lets
// the next such kernel be scheduled once every CTA of this grid has issued it.
// Rule for every kernel that is launched this way: read only constant data
// (weights) before pdl_wait(); every read of a predecessor's output and every
// global write comes after it, in at least one thread of every CTA.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// mbarrier + bulk (TMA, non-tensor) copies, no multicast.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait on phase `parity`: 64 quick tries, then tries spaced by a short
// sleep (tight polling of an mbarrier slows the TMA transfers completing on it).
// Returns false (and the caller records a timeout) when the limit runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t it = 0; it < SPIN_LIMIT; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if (it > 64) __nanosleep(64);
    }
    return false;
}
// Same, called by all lanes of a warp together (all lanes poll one address).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity) {
    return mbar_wait(bar, parity);
}
// Global -> shared bulk copy completing on `bar`. dst/src 16-byte aligned,
// bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Completes `bytes` of a barrier's expected transaction count without a copy (an
// expert that is not resident: its copy is skipped and the call reports it).
__device__ __forceinline__ void mbar_complete_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// L2 policy for streamed weights: read once per call, so they are marked
// evict-first and do not push code, pointer tables and activations out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes,
                                              uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// ---------------------------------------------------------------------------
// Loads
// ---------------------------------------------------------------------------
// 16 bytes at a 2-byte aligned address: five aligned words, funnel-shifted.
// Reads at most 2 bytes before and 2 after the range; callers keep that inside
// the weight block (every Q6_K sub-range used here is).
__device__ __forceinline__ void load16_a2(const uint8_t *p, uint32_t out[4]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(a & 3u) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
    out[0] = __funnelshift_r(w0, w1, sh);
    out[1] = __funnelshift_r(w1, w2, sh);
    out[2] = __funnelshift_r(w2, w3, sh);
    out[3] = __funnelshift_r(w3, w4, sh);
}
__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p) {
    return *reinterpret_cast<const uint16_t *>(p);
}

// Q4_K sub-scale and sub-min for groups 2c and 2c+1 from the 16-byte block
// header (h.y = scale bytes 0..3, h.z = 4..7, h.w = 8..11).
__device__ __forceinline__ void q4k_scales(const uint4 &h, int c, int &sc0, int &m0, int &sc1,
                                           int &m1) {
    const int j0 = 2 * c, j1 = 2 * c + 1;
    auto byte = [](uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFFu); };
    if (j0 < 4) {  // c = 0, 1: both groups < 4
        sc0 = byte(h.y, j0) & 63;
        m0 = byte(h.z, j0) & 63;
        sc1 = byte(h.y, j1) & 63;
        m1 = byte(h.z, j1) & 63;
    } else {  // c = 2, 3: both groups >= 4
        sc0 = (byte(h.w, j0 - 4) & 0x0F) | ((byte(h.y, j0 - 4) >> 6) << 4);
        m0 = (byte(h.w, j0 - 4) >> 4) | ((byte(h.z, j0 - 4) >> 6) << 4);
        sc1 = (byte(h.w, j1 - 4) & 0x0F) | ((byte(h.y, j1 - 4) >> 6) << 4);
        m1 = (byte(h.w, j1 - 4) >> 4) | ((byte(h.z, j1 - 4) >> 6) << 4);
    }
}

// Activations staged in shared memory in a split q8_1 layout: int8 values
// contiguous (16-byte aligned), the fp16 scale of each 32-block widened to
// float, the exact integer sum of each 32-block and of each 16-half.
struct ActQ8 {
    const int8_t *q;
    const float *d;
    const int *s32;
    const int *s16;
    int pad;  // 1: q holds element e at e + 16 * (e / 64) (bank-spread layout)
};
// Position of q8 activation element e (a multiple of 16) in an ActQ8 array.
__device__ __forceinline__ int qpos(const ActQ8 &a, int e) { return e + (a.pad ? ((e >> 6) << 4) : 0); }
// fp32 activations staged with the same spreading: element e at e + 4 * (e / 64).
__device__ __forceinline__ int fpos(int pad, int e) { return e + (pad ? ((e >> 6) << 2) : 0); }

// ---------------------------------------------------------------------------
// Block dots by "unit": 64 consecutive elements of a row whose bytes one lane
// loads once and uses fully.
//   Q4_K unit u: block b = u/4, chunk c = u%4 -> the 32 nibble bytes of chunk c,
//                low nibbles = q8_1 block 8b+2c, high nibbles = 8b+2c+1.
//   Q6_K unit u: block b = u/4, half h = (u/2)%2, quarter pair {qo, qo+2} with
//                qo = u%2 -> 32 ql bytes (low nibbles quarter qo, high nibbles
//                quarter qo+2) and the 32 qh bytes of half h;
//                q8_1 blocks 8b+4h+qo and 8b+4h+qo+2.
// Each unit returns the sum of its two exact per-q8-block double terms.
// ---------------------------------------------------------------------------
// A unit's weight bytes, loaded once and dotted with several activations.
struct Q4Unit {
    uint4 h, w0, w1;  // block header (d, dmin, scales), the chunk's 32 nibble bytes
};
struct Q6Unit {
    uint32_t ql[8], qh[8];
    uint32_t sc;  // sub-scales 2qo, 2qo+1, 2qo+4, 2qo+5 of half h (one byte each)
    float d;
};

__device__ __forceinline__ Q4Unit q4k_load_unit(const uint8_t *row, int u) {
    const int b = u >> 2, c = u & 3;
    const uint8_t *blk = row + Q4K_BYTES * b;
    Q4Unit w;
    w.h = *reinterpret_cast<const uint4 *>(blk);
    w.w0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * c);
    w.w1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * c);
    return w;
}

// A Q4_K unit with its nibbles split (lo: first 32 elements, hi: next 32) and its
// scales decoded, for dotting with several activations.
struct Q4Dec {
    uint32_t lo[8], hi[8];
    int sc0, m0, sc1, m1;
    double d, dmin;
};
__device__ __forceinline__ Q4Dec q4k_decode(const Q4Unit &wt, int u) {
    const uint32_t M = 0x0F0F0F0Fu;
    const uint32_t w[8] = {wt.w0.x, wt.w0.y, wt.w0.z, wt.w0.w, wt.w1.x, wt.w1.y, wt.w1.z, wt.w1.w};
    Q4Dec r;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        r.lo[i] = w[i] & M;
        r.hi[i] = (w[i] >> 4) & M;
    }
    q4k_scales(wt.h, u & 3, r.sc0, r.m0, r.sc1, r.m1);
    r.d = (double)h2f(wt.h.x);
    r.dmin = (double)h2f(wt.h.x >> 16);
    return r;
}
__device__ __forceinline__ double q4k_q8_dec(const Q4Dec &w, int u, const ActQ8 &a) {
    const int g = 8 * (u >> 2) + 2 * (u & 3);
    const uint4 *ap = reinterpret_cast<const uint4 *>(a.q + qpos(a, 32 * g));
    const uint4 a0 = ap[0], a1 = ap[1], a2 = ap[2], a3 = ap[3];
    int lo = 0, hi = 0;
    lo = __dp4a((int)w.lo[0], (int)a0.x, lo);
    hi = __dp4a((int)w.hi[0], (int)a2.x, hi);
    lo = __dp4a((int)w.lo[1], (int)a0.y, lo);
    hi = __dp4a((int)w.hi[1], (int)a2.y, hi);
    lo = __dp4a((int)w.lo[2], (int)a0.z, lo);
    hi = __dp4a((int)w.hi[2], (int)a2.z, hi);
    lo = __dp4a((int)w.lo[3], (int)a0.w, lo);
    hi = __dp4a((int)w.hi[3], (int)a2.w, hi);
    lo = __dp4a((int)w.lo[4], (int)a1.x, lo);
    hi = __dp4a((int)w.hi[4], (int)a3.x, hi);
    lo = __dp4a((int)w.lo[5], (int)a1.y, lo);
    hi = __dp4a((int)w.hi[5], (int)a3.y, hi);
    lo = __dp4a((int)w.lo[6], (int)a1.z, lo);
    hi = __dp4a((int)w.hi[6], (int)a3.z, hi);
    lo = __dp4a((int)w.lo[7], (int)a1.w, lo);
    hi = __dp4a((int)w.hi[7], (int)a3.w, hi);
    const double dx0 = (double)a.d[g], dx1 = (double)a.d[g + 1];
    return ((w.d * dx0) * (double)(w.sc0 * lo) - (w.dmin * dx0) * (double)(w.m0 * a.s32[g])) +
           ((w.d * dx1) * (double)(w.sc1 * hi) - (w.dmin * dx1) * (double)(w.m1 * a.s32[g + 1]));
}
__device__ __forceinline__ double q4k_q8_unit_w(const Q4Unit &wt, int u, const ActQ8 &a) {
    return q4k_q8_dec(q4k_decode(wt, u), u, a);
}

__device__ __forceinline__ double q4k_q8_unit(const uint8_t *row, int u, const ActQ8 &a) {
    return q4k_q8_unit_w(q4k_load_unit(row, u), u, a);
}

__device__ __forceinline__ Q6Unit q6k_load_unit(const uint8_t *row, int u) {
    const int b = u >> 2, h = (u >> 1) & 1, qo = u & 1;
    const uint8_t *blk = row + Q6K_BYTES * b;
    Q6Unit w;
    load16_a2(blk + 64 * h + 32 * qo, w.ql);
    load16_a2(blk + 64 * h + 32 * qo + 16, w.ql + 4);
    load16_a2(blk + 128 + 32 * h, w.qh);
    load16_a2(blk + 128 + 32 * h + 16, w.qh + 4);
    const uint8_t *sc = blk + 192 + 8 * h;
    w.sc = (uint32_t)sc[2 * qo] | ((uint32_t)sc[2 * qo + 1] << 8) | ((uint32_t)sc[2 * qo + 4] << 16) |
           ((uint32_t)sc[2 * qo + 5] << 24);
    w.d = h2f(ld_u16(blk + 208));
    return w;
}

// A Q6_K unit with its 6-bit values assembled (vA: quarter qo, vB: quarter qo+2,
// unsigned 0..63 in bytes) and its scales decoded.
struct Q6Dec {
    uint32_t vA[8], vB[8];
    int s0, s1, s4, s5;
    double d;
};
__device__ __forceinline__ Q6Dec q6k_decode(const Q6Unit &wt, int u) {
    const int qo = u & 1, shA = 2 * qo, shB = 2 * qo + 4;
    Q6Dec r;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        r.vA[i] = (wt.ql[i] & 0x0F0F0F0Fu) | (((wt.qh[i] >> shA) & 0x03030303u) << 4);
        r.vB[i] = ((wt.ql[i] >> 4) & 0x0F0F0F0Fu) | (((wt.qh[i] >> shB) & 0x03030303u) << 4);
    }
    r.s0 = (int)(int8_t)(wt.sc & 0xFFu);
    r.s1 = (int)(int8_t)((wt.sc >> 8) & 0xFFu);
    r.s4 = (int)(int8_t)((wt.sc >> 16) & 0xFFu);
    r.s5 = (int)(int8_t)(wt.sc >> 24);
    r.d = (double)wt.d;
    return r;
}
__device__ __forceinline__ double q6k_q8_dec(const Q6Dec &w, int u, const ActQ8 &a) {
    const int b = u >> 2, h = (u >> 1) & 1, qo = u & 1;
    const int jA = 8 * b + 4 * h + qo, jB = jA + 2;
    const uint4 *aA = reinterpret_cast<const uint4 *>(a.q + qpos(a, 32 * jA));
    const uint4 *aB = reinterpret_cast<const uint4 *>(a.q + qpos(a, 32 * jB));
    const uint4 xA0 = aA[0], xA1 = aA[1], xB0 = aB[0], xB1 = aB[1];
    const uint32_t wa[8] = {xA0.x, xA0.y, xA0.z, xA0.w, xA1.x, xA1.y, xA1.z, xA1.w};
    const uint32_t wb[8] = {xB0.x, xB0.y, xB0.z, xB0.w, xB1.x, xB1.y, xB1.z, xB1.w};
    int sA0 = 0, sA1 = 0, sB0 = 0, sB1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        sA0 = __dp4a((int)w.vA[i], (int)wa[i], sA0);
        sB0 = __dp4a((int)w.vB[i], (int)wb[i], sB0);
    }
#pragma unroll
    for (int i = 4; i < 8; ++i) {
        sA1 = __dp4a((int)w.vA[i], (int)wa[i], sA1);
        sB1 = __dp4a((int)w.vB[i], (int)wb[i], sB1);
    }
    const int IA = w.s0 * (sA0 - 32 * a.s16[2 * jA]) + w.s1 * (sA1 - 32 * a.s16[2 * jA + 1]);
    const int IB = w.s4 * (sB0 - 32 * a.s16[2 * jB]) + w.s5 * (sB1 - 32 * a.s16[2 * jB + 1]);
    return (w.d * (double)a.d[jA]) * (double)IA + (w.d * (double)a.d[jB]) * (double)IB;
}
__device__ __forceinline__ double q6k_q8_unit_w(const Q6Unit &wt, int u, const ActQ8 &a) {
    return q6k_q8_dec(q6k_decode(wt, u), u, a);
}

__device__ __forceinline__ double q6k_q8_unit(const uint8_t *row, int u, const ActQ8 &a) {
    return q6k_q8_unit_w(q6k_load_unit(row, u), u, a);
}

// Weight unit of either type, for code templated on the row type.
template <uint32_t T>
struct UnitOf {
    using type = Q4Unit;
};
template <>
struct UnitOf<T_Q6_K> {
    using type = Q6Unit;
};
template <uint32_t T>
__device__ __forceinline__ typename UnitOf<T>::type load_unit(const uint8_t *row, int u) {
    if constexpr (T == T_Q4_K) return q4k_load_unit(row, u);
    else return q6k_load_unit(row, u);
}
template <uint32_t T>
__device__ __forceinline__ double unit_dot(const typename UnitOf<T>::type &w, int u, const ActQ8 &a) {
    if constexpr (T == T_Q4_K) return q4k_q8_unit_w(w, u, a);
    else return q6k_q8_unit_w(w, u, a);
}
// Activations with the per-block scale and 32-element sum already widened to
// double (both exact), so a dot needs no conversion for them: (double)(m * s32)
// equals (double)m * (double)s32 because the product is an exact integer.
struct ActQ8D {
    const int8_t *q;
    const double *d, *s32;
    const int *s16;
    int pad;
};
__device__ __forceinline__ int qposd(const ActQ8D &a, int e) { return e + (a.pad ? ((e >> 6) << 4) : 0); }

__device__ __forceinline__ double q4k_q8_decd(const Q4Dec &w, int u, const ActQ8D &a) {
    const int g = 8 * (u >> 2) + 2 * (u & 3);
    const uint4 *ap = reinterpret_cast<const uint4 *>(a.q + qposd(a, 32 * g));
    const uint4 a0 = ap[0], a1 = ap[1], a2 = ap[2], a3 = ap[3];
    int lo = 0, hi = 0;
    lo = __dp4a((int)w.lo[0], (int)a0.x, lo);
    hi = __dp4a((int)w.hi[0], (int)a2.x, hi);
    lo = __dp4a((int)w.lo[1], (int)a0.y, lo);
    hi = __dp4a((int)w.hi[1], (int)a2.y, hi);
    lo = __dp4a((int)w.lo[2], (int)a0.z, lo);
    hi = __dp4a((int)w.hi[2], (int)a2.z, hi);
    lo = __dp4a((int)w.lo[3], (int)a0.w, lo);
    hi = __dp4a((int)w.hi[3], (int)a2.w, hi);
    lo = __dp4a((int)w.lo[4], (int)a1.x, lo);
    hi = __dp4a((int)w.hi[4], (int)a3.x, hi);
    lo = __dp4a((int)w.lo[5], (int)a1.y, lo);
    hi = __dp4a((int)w.hi[5], (int)a3.y, hi);
    lo = __dp4a((int)w.lo[6], (int)a1.z, lo);
    hi = __dp4a((int)w.hi[6], (int)a3.z, hi);
    lo = __dp4a((int)w.lo[7], (int)a1.w, lo);
    hi = __dp4a((int)w.hi[7], (int)a3.w, hi);
    const double dx0 = a.d[g], dx1 = a.d[g + 1];
    return ((w.d * dx0) * (double)(w.sc0 * lo) - (w.dmin * dx0) * ((double)w.m0 * a.s32[g])) +
           ((w.d * dx1) * (double)(w.sc1 * hi) - (w.dmin * dx1) * ((double)w.m1 * a.s32[g + 1]));
}
__device__ __forceinline__ double q6k_q8_decd(const Q6Dec &w, int u, const ActQ8D &a) {
    const int b = u >> 2, h = (u >> 1) & 1, qo = u & 1;
    const int jA = 8 * b + 4 * h + qo, jB = jA + 2;
    const uint4 *aA = reinterpret_cast<const uint4 *>(a.q + qposd(a, 32 * jA));
    const uint4 *aB = reinterpret_cast<const uint4 *>(a.q + qposd(a, 32 * jB));
    const uint4 xA0 = aA[0], xA1 = aA[1], xB0 = aB[0], xB1 = aB[1];
    const uint32_t wa[8] = {xA0.x, xA0.y, xA0.z, xA0.w, xA1.x, xA1.y, xA1.z, xA1.w};
    const uint32_t wb[8] = {xB0.x, xB0.y, xB0.z, xB0.w, xB1.x, xB1.y, xB1.z, xB1.w};
    int sA0 = 0, sA1 = 0, sB0 = 0, sB1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        sA0 = __dp4a((int)w.vA[i], (int)wa[i], sA0);
        sB0 = __dp4a((int)w.vB[i], (int)wb[i], sB0);
    }
#pragma unroll
    for (int i = 4; i < 8; ++i) {
        sA1 = __dp4a((int)w.vA[i], (int)wa[i], sA1);
        sB1 = __dp4a((int)w.vB[i], (int)wb[i], sB1);
    }
    const int IA = w.s0 * (sA0 - 32 * a.s16[2 * jA]) + w.s1 * (sA1 - 32 * a.s16[2 * jA + 1]);
    const int IB = w.s4 * (sB0 - 32 * a.s16[2 * jB]) + w.s5 * (sB1 - 32 * a.s16[2 * jB + 1]);
    return (w.d * a.d[jA]) * (double)IA + (w.d * a.d[jB]) * (double)IB;
}

template <uint32_t T>
struct DecOf {
    using type = Q4Dec;
};
template <>
struct DecOf<T_Q6_K> {
    using type = Q6Dec;
};
template <uint32_t T>
__device__ __forceinline__ typename DecOf<T>::type load_dec(const uint8_t *row, int u) {
    if constexpr (T == T_Q4_K) return q4k_decode(q4k_load_unit(row, u), u);
    else return q6k_decode(q6k_load_unit(row, u), u);
}
template <uint32_t T>
__device__ __forceinline__ double dec_dot(const typename DecOf<T>::type &w, int u, const ActQ8 &a) {
    if constexpr (T == T_Q4_K) return q4k_q8_dec(w, u, a);
    else return q6k_q8_dec(w, u, a);
}
template <uint32_t T>
__device__ __forceinline__ double dec_dot(const typename DecOf<T>::type &w, int u, const ActQ8D &a) {
    if constexpr (T == T_Q4_K) return q4k_q8_decd(w, u, a);
    else return q6k_q8_decd(w, u, a);
}

// 16-byte asynchronous global -> shared copy (cp.async, L2 only); completes at
// cp_async_wait_all().
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// fp32 activations x (shared) with per-32-group sums xs.
// Byte k (0..3) of w, an integer below 2^23, as float minus `bias`: the byte is
// placed under the exponent of 2^23 (0x4B000000) by one byte permute and one
// float add removes 2^23 + bias. Exact, and cheaper than an int -> float conversion.
__device__ __forceinline__ float byte_as_float(uint32_t w, int k, float bias2p23) {
    return __fsub_rn(__int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)k)), bias2p23);
}
constexpr float TWO23 = 8388608.0f;         // 2^23
constexpr float TWO23_P32 = 8388640.0f;     // 2^23 + 32 (Q6_K values are stored + 32)

// Two fp32 values in one 64-bit register, for sm_100's packed f32x2 instructions: each element
// of fma.rn.f32x2 / sub.rn.f32x2 is exactly fmaf / __fsub_rn on that element, so two independent
// accumulation chains advance in one instruction with the same results.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 f2_pack(float a, float b) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(f32x2 v, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ f32x2 f2_fma(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ f32x2 f2_sub(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 f2_mul(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// byte_as_float of byte k of wa and of wb, as one pair.
__device__ __forceinline__ f32x2 bytes_as_f2(uint32_t wa, uint32_t wb, int k, f32x2 bias2) {
    return f2_sub(f2_pack(__int_as_float((int)__byte_perm(wa, 0x4B000000u, 0x7440u | (uint32_t)k)),
                          __int_as_float((int)__byte_perm(wb, 0x4B000000u, 0x7440u | (uint32_t)k))),
                  bias2);
}

__device__ __forceinline__ double q4k_f32_unit(const uint8_t *row, int u, const float *x,
                                               const float *xs, int pad = 0) {
    const int b = u >> 2, c = u & 3;
    const uint8_t *blk = row + Q4K_BYTES * b;
    const uint4 h = *reinterpret_cast<const uint4 *>(blk);
    const uint4 w0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * c);
    const uint4 w1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * c);
    const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const float *xl = x + fpos(pad, 256 * b + 64 * c);
    // lo (low nibbles, first 32 elements) and hi (high nibbles, next 32) as one pair
    const f32x2 bias = f2_pack(TWO23, TWO23);
    f32x2 acc = f2_pack(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 xa = *reinterpret_cast<const float4 *>(xl + 4 * i);
        const float4 xb = *reinterpret_cast<const float4 *>(xl + 32 + 4 * i);
        const uint32_t wl = ww[i] & 0x0F0F0F0Fu, wh = (ww[i] >> 4) & 0x0F0F0F0Fu;
        acc = f2_fma(bytes_as_f2(wl, wh, 0, bias), f2_pack(xa.x, xb.x), acc);
        acc = f2_fma(bytes_as_f2(wl, wh, 1, bias), f2_pack(xa.y, xb.y), acc);
        acc = f2_fma(bytes_as_f2(wl, wh, 2, bias), f2_pack(xa.z, xb.z), acc);
        acc = f2_fma(bytes_as_f2(wl, wh, 3, bias), f2_pack(xa.w, xb.w), acc);
    }
    float lo, hi;
    f2_unpack(acc, lo, hi);
    int sc0, m0, sc1, m1;
    q4k_scales(h, c, sc0, m0, sc1, m1);
    const float d = h2f(h.x), dmin = h2f(h.x >> 16);
    const int g = 8 * b + 2 * c;
    return ((double)(d * (float)sc0) * (double)lo - (double)(dmin * (float)m0) * (double)xs[g]) +
           ((double)(d * (float)sc1) * (double)hi - (double)(dmin * (float)m1) * (double)xs[g + 1]);
}

__device__ __forceinline__ double q6k_f32_unit(const uint8_t *row, int u, const float *x,
                                               int pad = 0) {
    const int b = u >> 2, h = (u >> 1) & 1, qo = u & 1;
    const uint8_t *blk = row + Q6K_BYTES * b;
    uint32_t ql[8], qh[8];
    load16_a2(blk + 64 * h + 32 * qo, ql);
    load16_a2(blk + 64 * h + 32 * qo + 16, ql + 4);
    load16_a2(blk + 128 + 32 * h, qh);
    load16_a2(blk + 128 + 32 * h + 16, qh + 4);
    const float *xA = x + fpos(pad, 256 * b + 128 * h + 32 * qo);
    const float *xB = x + fpos(pad, 256 * b + 128 * h + 32 * qo + 64);
    const int shA = 2 * qo, shB = 2 * qo + 4;
    // quarter qo (A) and quarter qo + 2 (B) as one pair, per 16-element half: acc[0] over
    // elements 0-15 of each quarter, acc[1] over 16-31
    const f32x2 bias = f2_pack(TWO23_P32, TWO23_P32);
    f32x2 acc[2] = {f2_pack(0.0f, 0.0f), f2_pack(0.0f, 0.0f)};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t vA = (ql[i] & 0x0F0F0F0Fu) | (((qh[i] >> shA) & 0x03030303u) << 4);
        const uint32_t vB = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> shB) & 0x03030303u) << 4);
        const float4 a4 = *reinterpret_cast<const float4 *>(xA + 4 * i);
        const float4 b4 = *reinterpret_cast<const float4 *>(xB + 4 * i);
        f32x2 &ab = acc[i >> 2];
        ab = f2_fma(bytes_as_f2(vA, vB, 0, bias), f2_pack(a4.x, b4.x), ab);
        ab = f2_fma(bytes_as_f2(vA, vB, 1, bias), f2_pack(a4.y, b4.y), ab);
        ab = f2_fma(bytes_as_f2(vA, vB, 2, bias), f2_pack(a4.z, b4.z), ab);
        ab = f2_fma(bytes_as_f2(vA, vB, 3, bias), f2_pack(a4.w, b4.w), ab);
    }
    float fA[2], fB[2];
    f2_unpack(acc[0], fA[0], fB[0]);
    f2_unpack(acc[1], fA[1], fB[1]);
    const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * h);
    const float d = h2f(ld_u16(blk + 208));
    return ((double)(d * (float)sc[2 * qo]) * (double)fA[0] +
            (double)(d * (float)sc[2 * qo + 1]) * (double)fA[1]) +
           ((double)(d * (float)sc[2 * qo + 4]) * (double)fB[0] +
            (double)(d * (float)sc[2 * qo + 5]) * (double)fB[1]);
}

template <uint32_t T>
__device__ __forceinline__ double unit_q8(const uint8_t *row, int u, const ActQ8 &a) {
    return T == T_Q4_K ? q4k_q8_unit(row, u, a) : q6k_q8_unit(row, u, a);
}
template <uint32_t T>
__device__ __forceinline__ double unit_f32(const uint8_t *row, int u, const float *x,
                                           const float *xs, int pad = 0) {
    return T == T_Q4_K ? q4k_f32_unit(row, u, x, xs, pad) : q6k_f32_unit(row, u, x, pad);
}

// One warp per row: this lane's double partial over units lane, lane+32, ...
// (cols/64 units per row); the caller reduces across the warp and rounds once.
__device__ __forceinline__ double q4k_q8_partial(const uint8_t *row, int nb, const ActQ8 &a,
                                                 int lane) {
    double acc = 0.0;
    for (int u = lane; u < 4 * nb; u += 32) acc += q4k_q8_unit(row, u, a);
    return acc;
}
__device__ __forceinline__ double q6k_q8_partial(const uint8_t *row, int nb, const ActQ8 &a,
                                                 int lane) {
    double acc = 0.0;
    for (int u = lane; u < 4 * nb; u += 32) acc += q6k_q8_unit(row, u, a);
    return acc;
}
__device__ __forceinline__ double q4k_f32_partial(const uint8_t *row, int nb, const float *x,
                                                  const float *xs, int lane, int pad = 0) {
    double acc = 0.0;
    for (int u = lane; u < 4 * nb; u += 32) acc += q4k_f32_unit(row, u, x, xs, pad);
    return acc;
}
__device__ __forceinline__ double q6k_f32_partial(const uint8_t *row, int nb, const float *x,
                                                  int lane, int pad = 0) {
    double acc = 0.0;
    for (int u = lane; u < 4 * nb; u += 32) acc += q6k_f32_unit(row, u, x, pad);
    return acc;
}

// ---------------------------------------------------------------------------
// q8_1 quantisation of one 32-element block by one warp (lane = element).
// Writes the split shared layout (q/d_out/s32_out may be NULL), and the GGUF
// block at gblk (4-byte aligned) when non-NULL.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void quant_block_q8(float v, int lane, int8_t *q, float *d_out,
                                               int *s32_out, int *s16_out, uint8_t *gblk) {
    const float av = fabsf(v);
    const float amax = __uint_as_float(__reduce_max_sync(KQ_FULL, __float_as_uint(av)));
    const float d = __fdiv_rn(amax, 127.0f);
    int qi = 0;
    if (amax != 0.0f) qi = max(-127, min(127, (int)roundf(__fdiv_rn(v, d))));
    const int sum = __reduce_add_sync(KQ_FULL, qi);
    const int sum_lo = __reduce_add_sync(KQ_FULL, lane < 16 ? qi : 0);
    if (q) q[lane] = (int8_t)qi;
    const uint16_t dh = f2h(d);
    if (lane == 0 && d_out) {
        *d_out = h2f(dh);
        *s32_out = sum;
        if (s16_out) {
            s16_out[0] = sum_lo;
            s16_out[1] = sum - sum_lo;
        }
    }
    if (gblk) {  // GGUF block, written as aligned 32-bit words (gblk is 4-byte aligned)
        const uint32_t b = (uint32_t)qi & 0xFFu;
        const uint32_t b1 = __shfl_down_sync(KQ_FULL, b, 1);
        const uint32_t b2 = __shfl_down_sync(KQ_FULL, b, 2);
        const uint32_t b3 = __shfl_down_sync(KQ_FULL, b, 3);
        if ((lane & 3) == 0)
            *reinterpret_cast<uint32_t *>(gblk + 4 + lane) = b | (b1 << 8) | (b2 << 16) | (b3 << 24);
        if (lane == 0) {
            const uint32_t sh = f2h(__fmul_rn(d, (float)sum));
            *reinterpret_cast<uint32_t *>(gblk) = (uint32_t)dh | (sh << 16);
        }
    }
}

}  // namespace kq
