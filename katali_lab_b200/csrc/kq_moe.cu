// kq_moe.cu — the fused MoE layer, one launch per layer (README.md:13,17 of the
// reference describe its "one GPU call per MoE layer": routing, q8_1 activation
// quantisation, Q4_K gate/up, SiLU-gate multiply, Q6_K down, router-weighted
// sum; the reference ships that kernel only in binary form).
//
// B200 design: a persistent cooperative grid, one 16-warp CTA per SM.
//  1. Every CTA routes redundantly (warp 0: softmax top-k over the router
//     logits, deterministic ties) while warps 1-15 quantise x to q8_1 in shared
//     memory.
//  2. Thread 0 then requests ALL of the CTA's expert bytes at once with
//     cp.async.bulk into shared memory: its slice of the K*F gate/up row pairs
//     (phase A, one mbarrier per chunk) and its slice of the H down rows for all
//     K selected experts (phase B, one mbarrier). At the C2 shape (H 2048,
//     F 512, top-8) that is ~110 KB per SM, so the whole 16.3 MB layer is in
//     flight from the first microsecond.
//  3. Phase A: a warp per row pair computes gate and up against q8_1(x) with
//     DP4A, applies silu(g)*u and writes h to a small global scratch.
//  4. Grid barrier (one counter, bounded spin, error bit on timeout).
//  5. Phase B: every CTA quantises h (K*F values, from L2) to q8_1, then a warp
//     per output row dots the K down rows (already resident in shared memory)
//     and forms sum_k w_k * down_k in a fixed order, so the output is
//     deterministic and needs no atomics.
#include "kq_device.cuh"
#include "kq_launch.h"

namespace kq {

constexpr int MOE_WARPS = 16;
constexpr int MOE_THREADS = MOE_WARPS * 32;

struct Chunk {
    uint32_t u0;   // first unit (row pair) of the chunk, global unit index
    uint32_t n;    // units
    uint32_t off;  // byte offset in the phase-A staging area
    uint32_t pad;
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ double dot_q8(uint32_t type, const uint8_t *row, int nb,
                                         const ActQ8 &a, int lane) {
    return type == T_Q4_K ? q4k_q8_partial(row, nb, a, lane) : q6k_q8_partial(row, nb, a, lane);
}
__device__ __forceinline__ double dot_f32(uint32_t type, const uint8_t *row, int nb,
                                          const float *x, const float *xs, int lane) {
    return type == T_Q4_K ? q4k_f32_partial(row, nb, x, xs, lane)
                          : q6k_f32_partial(row, nb, x, lane);
}

__device__ __forceinline__ void bulk_g2s_split(uint8_t *dst, const uint8_t *src, uint32_t bytes,
                                               uint64_t *bar) {
    while (bytes) {
        const uint32_t n = bytes > 32768u ? 32768u : bytes;
        bulk_g2s(dst, src, n, bar);
        dst += n;
        src += n;
        bytes -= n;
    }
}

// Softmax top-k by one warp: lane l owns logits [l*npl, (l+1)*npl). Each round
// takes the largest remaining key; equal keys go to the lower expert id.
__device__ void route_warp(const MoeParams &p, float *s_logits, int32_t *s_ids, float *s_w,
                           int lane) {
    const int n = p.n_experts, K = p.K;
    for (int i = lane; i < n; i += 32) s_logits[i] = p.logits[i];
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
    const float m = s_logits[s_ids[0]];
    double S = 0.0;
    if (!p.norm) {
        for (int i = 0; i < npl; ++i) {
            const int idx = lane * npl + i;
            if (idx < n) S += (double)kq_expf(__fsub_rn(s_logits[idx], m));
        }
        S = warp_sum_d(S);
    }
    if (lane == 0) {
        float e[MOE_MAX_K];
        for (int t = 0; t < K; ++t) e[t] = kq_expf(__fsub_rn(s_logits[s_ids[t]], m));
        if (p.norm) {
            S = 0.0;
            for (int t = 0; t < K; ++t) S += (double)e[t];
        }
        for (int t = 0; t < K; ++t) s_w[t] = (float)((double)e[t] / S);
    }
    __syncwarp();
}

__global__ void __launch_bounds__(MOE_THREADS, 1) moe_kernel(const __grid_constant__ MoeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const int H = p.H, F = p.F, K = p.K;

    uint8_t *sa = smem;
    uint8_t *sb = smem + p.sb_off;
    uint8_t *act = smem + p.act_off;
    uint8_t *hact = smem + p.hact_off;
    uint8_t *misc = smem + p.misc_off;
    uint64_t *bars = reinterpret_cast<uint64_t *>(misc);  // MOE_MAX_CHUNKS + 1
    Chunk *chunks = reinterpret_cast<Chunk *>(misc + 8 * (MOE_MAX_CHUNKS + 1));
    int32_t *s_ids = reinterpret_cast<int32_t *>(chunks + MOE_MAX_CHUNKS);
    float *s_w = reinterpret_cast<float *>(s_ids + MOE_MAX_K);
    int *s_nch = reinterpret_cast<int *>(s_w + MOE_MAX_K);
    float *s_logits = reinterpret_cast<float *>(s_nch + 4);

    const uint32_t U = (uint32_t)K * F;
    const uint32_t u0 = (uint32_t)((uint64_t)U * c / G), u1 = (uint32_t)((uint64_t)U * (c + 1) / G);
    const uint32_t Q = (uint32_t)H / p.rg;  // phase-B row groups (16-byte aligned copies)
    const uint32_t q0 = (uint32_t)((uint64_t)Q * c / G), q1 = (uint32_t)((uint64_t)Q * (c + 1) / G);
    const uint32_t rB0 = p.rg * q0, nrB = p.rg * (q1 - q0);

    if (p.route_only) {  // check entry point: the routing decision only
        if (warp == 0) {
            route_warp(p, s_logits, s_ids, s_w, lane);
            if (c == 0 && lane < K) {
                p.dbg_ids[lane] = s_ids[lane];
                p.dbg_w[lane] = s_w[lane];
            }
        }
        return;
    }
    if (tid == 0) {
        for (int i = 0; i <= MOE_MAX_CHUNKS; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }

    // ---- 1. routing (warp 0) and x staging (warps 1..) ----------------------
    int8_t *xq = reinterpret_cast<int8_t *>(act);
    float *xd = reinterpret_cast<float *>(act + H);
    int *xs32 = reinterpret_cast<int *>(xd + H / 32);
    int *xs16 = xs32 + H / 32;
    float *xf = reinterpret_cast<float *>(act);
    float *xfs = xf + H;
    if (warp == 0) {
        if (p.ids) {
            if (lane < K) {
                s_ids[lane] = p.ids[lane];
                s_w[lane] = p.w[lane];
            }
            __syncwarp();
        } else {
            route_warp(p, s_logits, s_ids, s_w, lane);
        }
    } else if (p.mode == 0) {
        for (int g = warp - 1; g < H / 32; g += MOE_WARPS - 1)
            quant_block_q8(__ldg(&p.x[32 * g + lane]), lane, xq + 32 * g, xd + g, xs32 + g,
                           xs16 + 2 * g, nullptr);
    } else {
        for (int i = tid - 32; i < H / 4; i += MOE_THREADS - 32)
            reinterpret_cast<float4 *>(xf)[i] = __ldg(reinterpret_cast<const float4 *>(p.x) + i);
    }
    __syncthreads();
    if (p.mode != 0 && warp > 0) {
        for (int g = warp - 1; g < H / 32; g += MOE_WARPS - 1) {
            const float v = warp_sum_f(xf[32 * g + lane]);
            if (lane == 0) xfs[g] = v;
        }
    }
    // ---- 2. request every expert byte this CTA needs ------------------------
    if (tid == 0) {
        int nch = 0;
        uint32_t off = 0;
        for (uint32_t u = u0; u < u1;) {
            const uint32_t k = u / F, j = u % F;
            uint32_t n = u1 - u;
            if (n > p.chunk_units) n = p.chunk_units;
            if (n > (uint32_t)F - j) n = (uint32_t)F - j;
            const int e = s_ids[k];
            const uint8_t *gsrc = p.experts[3 * e] + (size_t)j * p.rbg;
            const uint8_t *usrc = p.experts[3 * e + 1] + (size_t)j * p.rbu;
            const uint32_t gb = n * p.rbg, ub = n * p.rbu;
            mbar_arrive_expect_tx(&bars[nch], gb + ub);
            bulk_g2s_split(sa + off, gsrc, gb, &bars[nch]);
            bulk_g2s_split(sa + off + gb, usrc, ub, &bars[nch]);
            chunks[nch] = Chunk{u, n, off, 0};
            off += gb + ub;
            ++nch;
            u += n;
        }
        *s_nch = nch;
        if (nrB) {
            const uint32_t per = nrB * p.rbd;
            mbar_arrive_expect_tx(&bars[MOE_MAX_CHUNKS], per * (uint32_t)K);
            for (int k = 0; k < K; ++k)
                bulk_g2s_split(sb + (size_t)k * per, p.experts[3 * s_ids[k] + 2] + (size_t)rB0 * p.rbd,
                               per, &bars[MOE_MAX_CHUNKS]);
        }
    }
    __syncthreads();

    // ---- 3. phase A: gate/up row pairs -> h = silu(g) * u --------------------
    bool ok = true;
    {
        const int nbh = H / 256;
        const ActQ8 ax{xq, xd, xs32, xs16};
        int ci = 0;
        for (uint32_t v = u0 + warp; v < u1; v += MOE_WARPS) {
            while (v >= chunks[ci].u0 + chunks[ci].n) ++ci;
            const Chunk ch = chunks[ci];
            if (!mbar_wait(&bars[ci], 0)) {
                ok = false;
                break;
            }
            const uint32_t jj = v - ch.u0;
            const uint8_t *grow = sa + ch.off + (size_t)jj * p.rbg;
            const uint8_t *urow = sa + ch.off + (size_t)ch.n * p.rbg + (size_t)jj * p.rbu;
            double pg, pu;
            if (p.mode == 0) {
                pg = dot_q8(p.gate_type, grow, nbh, ax, lane);
                pu = dot_q8(p.up_type, urow, nbh, ax, lane);
            } else {
                pg = dot_f32(p.gate_type, grow, nbh, xf, xfs, lane);
                pu = dot_f32(p.up_type, urow, nbh, xf, xfs, lane);
            }
            pg = warp_sum_d(pg);
            pu = warp_sum_d(pu);
            if (lane == 0) {
                const float g = (float)pg, u = (float)pu;
                p.hbuf[v] = __fmul_rn(kq_silu(g), u);  // unit v = k*F + j
            }
        }
    }
    if (!ok && lane == 0) *p.status |= ERR_TIMEOUT_TMA;

    // ---- 4. grid barrier ----------------------------------------------------
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        atomicAdd(&p.sync[0], 1u);
        uint32_t it = 0;
        while (ld_acquire_gpu(&p.sync[0]) < G) {
            if (++it > SPIN_LIMIT) {
                *p.status |= ERR_TIMEOUT_GRID;
                break;
            }
            __nanosleep(32);
        }
    }
    __syncthreads();

    // ---- 5. phase B: quantise h, then the K down rows per output row ---------
    int8_t *hq = reinterpret_cast<int8_t *>(hact);
    float *hd = reinterpret_cast<float *>(hact + (size_t)K * F);
    int *hs32 = reinterpret_cast<int *>(hd + (size_t)K * F / 32);
    int *hs16 = hs32 + (size_t)K * F / 32;
    float *hf = reinterpret_cast<float *>(hact);
    float *hfs = hf + (size_t)K * F;
    const int nblk = K * F / 32;
    for (int g = warp; g < nblk; g += MOE_WARPS) {
        const float v = __ldcg(&p.hbuf[32 * g + lane]);
        if (p.mode == 0) {
            quant_block_q8(v, lane, hq + 32 * g, hd + g, hs32 + g, hs16 + 2 * g, nullptr);
        } else {
            hf[32 * g + lane] = v;
            const float s = warp_sum_f(v);
            if (lane == 0) hfs[g] = s;
        }
    }
    __syncthreads();

    if (nrB) {
        if (!mbar_wait(&bars[MOE_MAX_CHUNKS], 0)) {
            if (lane == 0) *p.status |= ERR_TIMEOUT_TMA;
        } else {
            const int nbf = F / 256;
            const uint32_t per = nrB * p.rbd;
            for (uint32_t rr = warp; rr < nrB; rr += MOE_WARPS) {
                double part[MOE_MAX_K];
#pragma unroll
                for (int k = 0; k < MOE_MAX_K; ++k) {
                    if (k < K) {
                        const uint8_t *row = sb + (size_t)k * per + (size_t)rr * p.rbd;
                        if (p.mode == 0) {
                            const ActQ8 ah{hq + (size_t)k * F, hd + (size_t)k * F / 32,
                                           hs32 + (size_t)k * F / 32, hs16 + (size_t)k * F / 16};
                            part[k] = dot_q8(p.down_type, row, nbf, ah, lane);
                        } else {
                            part[k] = dot_f32(p.down_type, row, nbf, hf + (size_t)k * F,
                                              hfs + (size_t)k * F / 32, lane);
                        }
                    }
                }
#pragma unroll
                for (int k = 0; k < MOE_MAX_K; ++k)
                    if (k < K) part[k] = warp_sum_d(part[k]);
                if (lane == 0) {
                    double acc = 0.0;
                    for (int k = 0; k < K; ++k) acc += (double)s_w[k] * (double)(float)part[k];
                    p.y[rB0 + rr] = (float)acc;
                }
            }
        }
    }

    // ---- 6. the last CTA out re-arms the barrier counters --------------------
    __syncthreads();
    if (tid == 0) {
        const uint32_t prev = atomicAdd(&p.sync[1], 1u);
        if (prev == G - 1) {
            atomicExch(&p.sync[0], 0u);
            atomicExch(&p.sync[1], 0u);
        }
    }
}

static inline uint32_t al128(uint32_t v) { return (v + 127u) & ~127u; }

// Shared-memory plan for `grid` CTAs. Returns 0, or -1 when the layer does not
// fit (the caller reports KATALI_ERR_UNSUPPORTED_SHAPE).
int moe_plan(MoeParams &p, int grid, int max_smem) {
    const uint32_t U = (uint32_t)p.K * p.F;
    const uint32_t upc = (U + grid - 1) / grid;
    uint32_t ch = (upc + 15) / 16;
    if (ch < 4) ch = 4;
    p.chunk_units = ch;
    if ((upc + ch - 1) / ch + (uint32_t)p.K + 1 > (uint32_t)MOE_MAX_CHUNKS) return -1;
    p.sa_bytes = upc * (p.rbg + p.rbu);
    p.sb_off = al128(p.sa_bytes);
    uint32_t rg = 16;  // rows per phase-B group: 16 / gcd(rbd, 16)
    for (uint32_t v = p.rbd; v % 2 == 0 && rg > 1; v /= 2) rg /= 2;
    if (p.H % rg) return -1;
    p.rg = rg;
    const uint32_t Q = (uint32_t)p.H / rg;
    const uint32_t qpc = (Q + grid - 1) / grid;
    p.sb_bytes = (uint32_t)p.K * rg * qpc * p.rbd;
    p.act_off = al128(p.sb_off + p.sb_bytes);
    const uint32_t act = p.mode == 0 ? p.H + p.H / 32 * 8 + p.H / 16 * 4 : p.H * 4 + p.H / 32 * 4;
    p.hact_off = al128(p.act_off + act);
    const uint32_t KF = (uint32_t)p.K * p.F;
    const uint32_t hact = p.mode == 0 ? KF + KF / 32 * 8 + KF / 16 * 4 : KF * 4 + KF / 32 * 4;
    p.misc_off = al128(p.hact_off + hact);
    const uint32_t misc = 8 * (MOE_MAX_CHUNKS + 1) + (uint32_t)sizeof(Chunk) * MOE_MAX_CHUNKS +
                          4 * MOE_MAX_K * 2 + 16 + 4 * (uint32_t)p.n_experts;
    p.smem_bytes = al128(p.misc_off + misc);
    return p.smem_bytes <= (uint32_t)max_smem ? 0 : -1;
}

cudaError_t launch_moe(MoeParams &p, int grid, cudaStream_t st) {
    // Raise the dynamic shared-memory limit once per size (never during a graph capture
    // that follows a first eager call with the same plan).
    static uint32_t set_bytes = 0;
    if (p.smem_bytes > set_bytes) {
        cudaError_t e = cudaFuncSetAttribute(moe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)p.smem_bytes);
        if (e != cudaSuccess) return e;
        set_bytes = p.smem_bytes;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(MOE_THREADS);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = p.route_only ? 0 : 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, moe_kernel, p);
}

}  // namespace kq
