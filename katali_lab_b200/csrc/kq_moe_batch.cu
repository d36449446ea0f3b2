// kq_moe_batch.cu — the MoE layer for a ragged batch of tokens (continuous batching).
//
// T tokens are routed independently (the same top-k and softmax weights as the
// batch-1 kernel). The T*K (token, expert) pairs are then grouped by expert, so
// every selected expert's gate/up/down rows are read from HBM once per call and
// dotted with all of that expert's tokens. Every per-pair dot uses the same
// exact block terms as the batch-1 kernel and each token's output is the same
// fixed-order weighted sum, so a token's row of Y equals its batch-1 result.
//
// Pipeline (one stream, six launches):
//   route  : one CTA per token: top-k + weights, x -> q8_1 (split layout)
//   group  : one CTA: counting sort of the pairs by expert id
//   gateup : item = (group, a tile of up to 16 rows of F); the grid is the resident CTAs, which
//            take items from a counter; loop over the group's tokens; h = silu(g) * u
//   hquant : h -> q8_1 per pair (split layout with 16-element sums)
//   down   : item = (group, up to 64 output rows), scheduled the same way
//   combine: y[t] = sum_k w[t][k] * part[pair(t,k)] in k order
#include "kq_device.cuh"
#include "kq_launch.h"

namespace kq {

constexpr int BT = 256;  // threads per CTA for the batch kernels

// ---------------------------------------------------------------------------
// route: routing decision and q8_1 activations of one token per CTA
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t bkey(float f, int idx) {
    return ((uint64_t)order_key(f) << 32) | (uint32_t)(~idx);
}

// Routing of one token by one warp: top-k of E logits (each round takes the warp
// maximum of per-lane maxima of the composite key: larger logit, then lower id)
// and the softmax weights with the batch-1 kernel's summation order. Lane k < K
// returns id k in *id_out and its weight in *w_out.
__device__ __forceinline__ void route_token(const float *lg, int E, int K, int norm, int lane,
                                            int *id_out, float *w_out) {
    uint32_t mine = 0;  // taken ids of this lane (bit i = id lane + 32 i)
    const int npl = (E + 31) / 32;
    int my_id = 0;
    for (int r = 0; r < K; ++r) {
        uint64_t best = 0;
        for (int i = 0; i < npl; ++i) {
            const int e = lane + 32 * i;
            if (e < E && !((mine >> i) & 1u)) {
                const uint64_t kk = bkey(lg[e], e);
                if (kk > best) best = kk;
            }
        }
        const uint32_t hi = (uint32_t)(best >> 32), lo = (uint32_t)best;
        const uint32_t Mh = __reduce_max_sync(KQ_FULL, hi);
        const uint32_t Ml = __reduce_max_sync(KQ_FULL, hi == Mh ? lo : 0u);
        const int e = (int)(~Ml);
        if ((e & 31) == lane) mine |= 1u << (e >> 5);
        if (lane == r) my_id = e;
    }
    const float m = lg[__shfl_sync(KQ_FULL, my_id, 0)];
    double S = 0.0;
    if (!norm) {  // lane-owned contiguous ranges, the batch-1 kernel's order
        const int per = (E + 31) >> 5;
        for (int i = 0; i < per; ++i) {
            const int idx = lane * per + i;
            if (idx < E) S += (double)kq_expf(__fsub_rn(lg[idx], m));
        }
        S = warp_sum_d(S);
    }
    const float ev = lane < K ? kq_expf(__fsub_rn(lg[my_id], m)) : 0.0f;
    if (norm) {
        S = 0.0;
        for (int r = 0; r < K; ++r) S += (double)__shfl_sync(KQ_FULL, ev, r);
    }
    *id_out = my_id;
    *w_out = (float)((double)ev / S);
}

// Token t by the whole CTA (s_lg: 1024 floats of shared memory).
__device__ __forceinline__ void route_one(const MoeBatchParams &p, int t, float *s_lg) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = p.H, K = p.K;
    const float *x = p.X + (size_t)t * H;
    if (!p.ids_in)
        for (int i = threadIdx.x; i < p.n_experts; i += BT) s_lg[i] = p.logits[(size_t)t * p.n_experts + i];
    __syncthreads();
    if (warp == 0) {
        int id = 0;
        float w = 0.0f;
        if (p.ids_in) {  // routing given by the caller
            if (lane < K) {
                id = p.ids_in[t * K + lane];
                w = p.w_in[t * K + lane];
            }
        } else {
            route_token(s_lg, p.n_experts, K, p.norm, lane, &id, &w);
        }
        if (lane < K) {
            p.ids[t * K + lane] = id;
            p.w[t * K + lane] = w;
        }
    } else {
        const int nblk = H / 32;
        int8_t *q = p.xq + (size_t)t * H;
        float *d = p.xd + (size_t)t * nblk;
        int *s32 = p.xs32 + (size_t)t * nblk, *s16 = p.xs16 + (size_t)t * 2 * nblk;
        for (int g = warp - 1; g < nblk; g += BT / 32 - 1)
            quant_block_q8(x[32 * g + lane], lane, q + 32 * g, d + g, s32 + g, s16 + 2 * g, nullptr);
    }
}

__global__ void __launch_bounds__(BT) moe_batch_route(MoeBatchParams p) {
    __shared__ float s_lg[1024];
    pdl_trigger();
    pdl_wait();
    route_one(p, blockIdx.x, s_lg);
}

// ---------------------------------------------------------------------------
// group: counting sort of the T*K pairs by expert (one CTA)
// ---------------------------------------------------------------------------
// Exclusive block scan over blockDim.x (<= 1024) values; also returns the total.
__device__ __forceinline__ int block_exscan(int v, int *wsum, int &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(KQ_FULL, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nw ? wsum[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(KQ_FULL, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nw) wsum[lane] = w;
    }
    __syncthreads();
    total = wsum[nw - 1];
    const int excl = x - v + (warp ? wsum[warp - 1] : 0);
    __syncthreads();
    return excl;
}

// One CTA (any size up to 1024 threads; n_experts <= 1024): per-expert counts,
// offsets, the list of selected experts in ascending id, and each pair's slot
// (order within an expert is arbitrary; every pair is computed independently).
// Pairs with id < 0 are skipped. Thread i owns the contiguous experts
// [i * epT, (i + 1) * epT), epT = ceil(E / blockDim.x), so the scans keep id order.
__device__ void group_body(const MoeBatchParams &p, int *cnt, int *off, int *wsum) {
    const int P = p.T * p.K, E = p.n_experts;
    const int epT = (E + (int)blockDim.x - 1) / (int)blockDim.x, e0 = threadIdx.x * epT;
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < P; i += blockDim.x)
        if (p.ids[i] >= 0) atomicAdd(&cnt[p.ids[i]], 1);
    __syncthreads();
    // Groups the tensor-core kernels take (n >= the smaller of their positive thresholds)
    // are also listed, in group order, so those kernels size their work to them.
    const int thr = p.tc_min > 0 && (p.tc_down_min <= 0 || p.tc_min <= p.tc_down_min) ? p.tc_min
                                                                                      : p.tc_down_min;
    int c = 0, nz = 0, ntc = 0;
    for (int e = e0; e < e0 + epT && e < E; ++e) {
        c += cnt[e];
        nz += cnt[e] > 0;
        ntc += thr > 0 && cnt[e] >= thr;
    }
    int total, ngroups, ntcg;
    int o = block_exscan(c, wsum, total);
    int gi = block_exscan(nz, wsum, ngroups);
    int ti = block_exscan(ntc, wsum, ntcg);
    for (int e = e0; e < e0 + epT && e < E; ++e) {
        const int ce = cnt[e];
        off[e] = o;
        if (ce > 0) {
            p.grp_expert[gi] = e;
            p.grp_off[gi] = o;
            if (thr > 0 && ce >= thr) p.tc_groups[ti++] = gi;
            ++gi;
        }
        o += ce;
    }
    __syncthreads();  // every count read before the second pass reuses cnt
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    if (threadIdx.x == 0) {
        p.grp_off[ngroups] = total;
        *p.n_groups = ngroups;
        p.work[0] = 0u;  // the item counters of this call's gate/up and down kernels
        p.work[1] = 0u;
        p.work[2] = (uint32_t)ntcg;  // listed tensor-core groups
    }
    __syncthreads();
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int ex = p.ids[i];
        if (ex < 0) continue;  // a pair this rank does not own (expert-parallel slots)
        const int pos = off[ex] + atomicAdd(&cnt[ex], 1);
        p.pair_src[pos] = i;  // i = t * K + k
        p.pos_of[i] = pos;
        const int n_ex = (ex + 1 < E ? off[ex + 1] : total) - off[ex];  // the expert's group size
        p.pair_tc[pos] = p.tc_min > 0 && n_ex >= p.tc_min;
    }
}

__global__ void __launch_bounds__(1024) moe_batch_group(MoeBatchParams p) {
    __shared__ int cnt[1024], off[1024], wsum[32];
    pdl_trigger();
    pdl_wait();
    group_body(p, cnt, off, wsum);
}

// ---------------------------------------------------------------------------
// Row tiles: a CTA takes `rows` consecutive rows of one selected expert matrix
// (gate and up together for gateup), copies them into shared memory with one
// bulk copy per matrix and computes them for every token of the expert's group.
// LPR = 256 / rows lanes per row, each lane a strided share of the row's units;
// tokens in chunks of BTC with one double accumulator each, so a weight unit is
// read from shared memory once per chunk.
// ---------------------------------------------------------------------------
constexpr int BTC = 2;  // tokens per register chunk

__device__ __forceinline__ ActQ8 x_act(const MoeBatchParams &p, int t) {
    const int nblk = p.H / 32;
    return ActQ8{p.xq + (size_t)t * p.H, p.xd + (size_t)t * nblk, p.xs32 + (size_t)t * nblk,
                 p.xs16 + (size_t)t * 2 * nblk, 0};
}
__device__ __forceinline__ ActQ8 h_act(const MoeBatchParams &p, int q) {
    const int nblk = p.F / 32;
    return ActQ8{p.hq + (size_t)q * p.F, p.hd + (size_t)q * nblk, p.hs32 + (size_t)q * nblk,
                 p.hs16 + (size_t)q * 2 * nblk, 0};
}
// Sum over the LPR lanes of a row (LPR a power of two, lanes of a row adjacent).
__device__ __forceinline__ double row_sum(double v, int lpr) {
    for (int o = 1; o < lpr; o <<= 1) v += __shfl_xor_sync(KQ_FULL, v, o);
    return v;
}

// Copies the q8_1 activations of `n` rows (row i = src_row(i)) of length L into
// shared memory: values in the bank-spread layout (16 bytes of padding after every
// 64), scales, 32- and 16-element sums. Returns the slot stride of the values.
constexpr int ACT_TOKS = 4;  // activation rows staged at a time
__host__ __device__ constexpr int act_q_stride(int L) { return L + L / 4; }
__host__ __device__ constexpr int act_slot_bytes(int L) { return act_q_stride(L) + L / 32 * 16 + L / 16 * 4; }

struct SmemAct {
    int8_t *q;
    double *d, *s32;
    int *s16;
    int L;
    __device__ ActQ8D at(int i) const {
        return ActQ8D{q + (size_t)i * act_q_stride(L), d + (size_t)i * (L / 32),
                      s32 + (size_t)i * (L / 32), s16 + (size_t)i * (L / 16), 1};
    }
};
__device__ __forceinline__ SmemAct smem_act(uint8_t *base, int L) {
    SmemAct a;
    a.L = L;
    a.q = reinterpret_cast<int8_t *>(base);
    a.d = reinterpret_cast<double *>(base + (size_t)ACT_TOKS * act_q_stride(L));
    a.s32 = a.d + ACT_TOKS * (L / 32);
    a.s16 = reinterpret_cast<int *>(a.s32 + ACT_TOKS * (L / 32));
    return a;
}
// Issues the copies (cp.async) of n activation rows into `sa`; the caller waits
// with cp_async_wait_all() and a CTA barrier.
template <typename RowOf>
__device__ __forceinline__ void stage_act(const SmemAct &sa, int n, RowOf row_of) {
    const int L = sa.L, nv = L / 16, nb = L / 32;
    for (int idx = threadIdx.x; idx < n * nv; idx += BT) {
        const int i = idx / nv, v = idx % nv;
        cp_async16(sa.q + (size_t)i * act_q_stride(L) + 16 * v + 16 * (v >> 2), row_of(i).q + 16 * v);
    }
    for (int idx = threadIdx.x; idx < n * nb; idx += BT) {
        const int i = idx / nb, b = idx % nb;
        const ActQ8 src = row_of(i);
        cp_async4(sa.s16 + (i * nb + b) * 2, src.s16 + 2 * b);
        cp_async4(sa.s16 + (i * nb + b) * 2 + 1, src.s16 + 2 * b + 1);
        sa.d[i * nb + b] = (double)src.d[b];
        sa.s32[i * nb + b] = (double)src.s32[b];
    }
}

// Thread 0 arms `bar` for the next phase and starts the weight-tile copies on it.
// The barrier is initialised once per CTA (init_tiles_bar) and reused: every item
// toggles the phase the CTA waits on.
__device__ __forceinline__ void init_tiles_bar(uint64_t *bar) {
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
}
__device__ __forceinline__ void issue_tiles(uint64_t *bar, int n, uint8_t *const *dst,
                                            const uint8_t *const *src, const uint32_t *bytes) {
    if (threadIdx.x == 0) {
        uint32_t total = 0;
        for (int i = 0; i < n; ++i) total += bytes[i];
        mbar_arrive_expect_tx(bar, total);
        const uint64_t pol = l2_evict_first_policy();
        for (int i = 0; i < n; ++i) bulk_g2s_hint(dst[i], src[i], bytes[i], bar, pol);
    }
}
// All threads wait for phase `parity`; the outcome is made uniform across the CTA
// so that a timeout ends every thread (and is recorded once).
__device__ __forceinline__ bool wait_tiles(uint64_t *bar, uint32_t parity,
                                           volatile uint32_t *status) {
    const bool ok = mbar_wait(bar, parity);
    if (!__syncthreads_or(!ok)) return true;
    if (threadIdx.x == 0 && status) atomicOr((uint32_t *)status, 4u);
    return false;
}

// Item scheduling of the gate/up and down kernels: the grid is sized to the resident
// CTAs (not to the worst-case group count). A CTA starts on item blockIdx.x and then
// takes items gridDim.x, gridDim.x + 1, ... from a counter in arrival order, so CTAs
// that drew small groups take more items and no CTA exists for a group the batch
// does not have. Thread 0 asks for the next item when it starts the current one
// and hands it over after the item, so the atomic's latency is hidden.
__device__ __forceinline__ uint32_t next_item_async(uint32_t *counter) {
    return threadIdx.x == 0 ? gridDim.x + atomicAdd(counter, 1u) : 0u;
}
// Two slots, used in turn: a thread still reading the previous hand-over's slot
// cannot be overtaken, since thread 0 passes the next hand-over's CTA barrier only
// after every thread has read it.
__device__ __forceinline__ int hand_over_item(uint32_t next, int *s_next, int &slot) {
    if (threadIdx.x == 0) s_next[slot] = (int)next;
    __syncthreads();
    const int v = s_next[slot];
    slot ^= 1;
    return v;
}

// Shared memory of an item kernel: the tile barrier, the weight tile (128-byte
// aligned), then the staged activations of ACT_TOKS rows of length L.
struct ItemSmem {
    uint64_t *bar;
    uint8_t *tile;
    uint8_t *act;
};
__host__ __device__ constexpr size_t align128(size_t v) { return (v + 127) & ~(size_t)127; }
__host__ __device__ constexpr size_t item_smem_bytes(size_t tile_bytes, int L) {
    return 128 + align128(tile_bytes) + (size_t)ACT_TOKS * act_slot_bytes(L);
}
__device__ __forceinline__ ItemSmem item_smem(uint8_t *sm, size_t tile_bytes) {
    return ItemSmem{reinterpret_cast<uint64_t *>(sm), sm + 128, sm + 128 + align128(tile_bytes)};
}
// Per-CTA state that carries across item loops: the tile barrier's next parity and
// the hand-over slot.
struct ItemState {
    uint32_t phase;
    int slot;
};

// ---------------------------------------------------------------------------
// gate/up: work item = (group g, p.gu_rows rows of F). Returns false when a tile
// wait timed out (the whole CTA then stops).
// ---------------------------------------------------------------------------
template <uint32_t GT, uint32_t UT>
__device__ bool gateup_items(const MoeBatchParams &p, const ItemSmem &S, int *s_next, ItemState &st) {
    const int rows = p.gu_rows, lpr = BT / rows;
    const int nrb = (p.F + rows - 1) / rows;
    const int items = *p.n_groups * nrb;
    const int F = p.F, K = p.K, U = p.H / 64;
    uint8_t *sg = S.tile, *su = S.tile + (size_t)rows * p.rbg;
    const SmemAct sa = smem_act(S.act, p.H);
    const int sub = threadIdx.x % lpr, jr = threadIdx.x / lpr;
    for (int it = blockIdx.x; it < items;) {
        const uint32_t next = next_item_async(&p.work[0]);
        const int g = it / nrb, rb = it % nrb;
        const int e = p.grp_expert[g], p0 = p.grp_off[g], p1 = p.grp_off[g + 1];
        const bool tc = p.tc_min > 0 && p1 - p0 >= p.tc_min;  // the tensor-core kernel takes it
        const bool resident = p.experts[3 * e] && p.experts[3 * e + 1];
        if (!resident && threadIdx.x == 0 && p.status)  // not resident: report, skip
            atomicOr((uint32_t *)p.status, KQ_STATUS_NOT_RESIDENT);
        if (p1 <= p0 || tc || !resident) {
            it = hand_over_item(next, s_next, st.slot);
            continue;
        }
        const int j0 = rb * rows, nrows = min(rows, F - j0), j = j0 + jr;
        const bool valid = jr < nrows;
        __syncthreads();  // barrier init visible; the previous item's tiles are no longer read
        {
            uint8_t *dst[2] = {sg, su};
            const uint8_t *src[2] = {p.experts[3 * e] + (size_t)j0 * p.rbg,
                                     p.experts[3 * e + 1] + (size_t)j0 * p.rbu};
            const uint32_t bytes[2] = {(uint32_t)nrows * p.rbg, (uint32_t)nrows * p.rbu};
            issue_tiles(S.bar, 2, dst, src, bytes);
        }
        const uint8_t *grow = sg + (size_t)(valid ? jr : 0) * p.rbg;
        const uint8_t *urow = su + (size_t)(valid ? jr : 0) * p.rbu;
        bool tiles_in = false;
        for (int c0 = p0; c0 < p1; c0 += ACT_TOKS) {
            const int nc = min(ACT_TOKS, p1 - c0);
            if (c0 != p0) __syncthreads();  // the previous chunk is no longer read
            stage_act(sa, nc, [&](int i) { return x_act(p, p.pair_src[c0 + i] / K); });
            cp_async_wait_all();
            __syncthreads();
            if (!tiles_in) {
                if (!wait_tiles(S.bar, st.phase, p.status)) return false;
                st.phase ^= 1u;
                tiles_in = true;
            }
            for (int i0 = 0; i0 < nc; i0 += BTC) {
                const int nq = min(BTC, nc - i0);
                double ag[BTC], au[BTC];
#pragma unroll
                for (int i = 0; i < BTC; ++i) ag[i] = au[i] = 0.0;
                if (valid) {
                    for (int u = sub; u < U; u += lpr) {
                        const auto wg = load_dec<GT>(grow, u);
                        const auto wu = load_dec<UT>(urow, u);
#pragma unroll
                        for (int i = 0; i < BTC; ++i) {
                            if (i < nq) {
                                const ActQ8D a = sa.at(i0 + i);
                                ag[i] += dec_dot<GT>(wg, u, a);
                                au[i] += dec_dot<UT>(wu, u, a);
                            }
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < BTC; ++i) {
                    const double dg = row_sum(ag[i], lpr), du = row_sum(au[i], lpr);
                    if (valid && sub == 0 && i < nq)
                        p.h[(size_t)(c0 + i0 + i) * F + j] = __fmul_rn(kq_silu((float)dg), (float)du);
                }
            }
        }
        it = hand_over_item(next, s_next, st.slot);
    }
    return true;
}

template <uint32_t GT, uint32_t UT>
__global__ void __launch_bounds__(BT, 3) moe_batch_gateup(MoeBatchParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ int s_next[2];
    pdl_trigger();
    pdl_wait();
    const ItemSmem S = item_smem(sm, (size_t)p.gu_rows * (p.rbg + p.rbu));
    init_tiles_bar(S.bar);
    ItemState st{0u, 0};
    gateup_items<GT, UT>(p, S, s_next, st);
}

// ---------------------------------------------------------------------------
// hquant: one warp per 32-element block of one pair's h (warps w0, w0 + ws, ...)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void hquant_range(const MoeBatchParams &p, int w0, int ws) {
    const int lane = threadIdx.x & 31;
    const int nblk = p.F / 32;
    const int P = p.grp_off[*p.n_groups];  // grouped pairs (<= T * K)
    for (int wg = w0; wg < P * nblk; wg += ws) {
        const int q = wg / nblk, b = wg % nblk;
        const size_t i = (size_t)q * p.F + 32 * b + lane;
        // pairs whose gate/up ran on the tensor cores: h holds the gate sums, hu the up sums
        const float v = p.pair_tc[q] ? __fmul_rn(kq_silu(p.h[i]), p.hu[i]) : p.h[i];
        quant_block_q8(v, lane, p.hq + (size_t)q * p.F + 32 * b, p.hd + (size_t)q * nblk + b,
                       p.hs32 + (size_t)q * nblk + b, p.hs16 + ((size_t)q * nblk + b) * 2, nullptr);
    }
}
__global__ void __launch_bounds__(BT) moe_batch_hquant(MoeBatchParams p) {
    pdl_trigger();
    pdl_wait();
    hquant_range(p, (blockIdx.x * BT + threadIdx.x) >> 5, gridDim.x * (BT / 32));
}

// ---------------------------------------------------------------------------
// down: work item = (group g, p.dn_rows output rows), same scheme as gateup
// ---------------------------------------------------------------------------
template <uint32_t DT>
__device__ bool down_items(const MoeBatchParams &p, const ItemSmem &S, int *s_next, ItemState &st) {
    const int rows = p.dn_rows, lpr = BT / rows;
    const int nrb = (p.H + rows - 1) / rows;
    const int items = *p.n_groups * nrb;
    const int U = p.F / 64;
    const SmemAct sa = smem_act(S.act, p.F);
    const int sub = threadIdx.x % lpr, rr = threadIdx.x / lpr;
    for (int it = blockIdx.x; it < items;) {
        const uint32_t next = next_item_async(&p.work[1]);
        const int g = it / nrb, rb = it % nrb;
        const int e = p.grp_expert[g], p0 = p.grp_off[g], p1 = p.grp_off[g + 1];
        const bool tc = p.tc_down_min > 0 && p1 - p0 >= p.tc_down_min;  // the tensor-core kernel takes it
        const bool resident = p.experts[3 * e + 2] != nullptr;
        if (!resident && threadIdx.x == 0 && p.status)  // not resident: report, skip
            atomicOr((uint32_t *)p.status, KQ_STATUS_NOT_RESIDENT);
        if (p1 <= p0 || tc || !resident) {
            it = hand_over_item(next, s_next, st.slot);
            continue;
        }
        const int r0 = rb * rows, nrows = min(rows, p.H - r0), r = r0 + rr;
        const bool valid = rr < nrows;
        __syncthreads();  // barrier init visible; the previous item's tile is no longer read
        {
            uint8_t *dst[1] = {S.tile};
            const uint8_t *src[1] = {p.experts[3 * e + 2] + (size_t)r0 * p.rbd};
            const uint32_t bytes[1] = {(uint32_t)nrows * p.rbd};
            issue_tiles(S.bar, 1, dst, src, bytes);
        }
        const uint8_t *row = S.tile + (size_t)(valid ? rr : 0) * p.rbd;
        bool tiles_in = false;
        for (int c0 = p0; c0 < p1; c0 += ACT_TOKS) {
            const int nc = min(ACT_TOKS, p1 - c0);
            if (c0 != p0) __syncthreads();
            stage_act(sa, nc, [&](int i) { return h_act(p, c0 + i); });
            cp_async_wait_all();
            __syncthreads();
            if (!tiles_in) {
                if (!wait_tiles(S.bar, st.phase, p.status)) return false;
                st.phase ^= 1u;
                tiles_in = true;
            }
            for (int i0 = 0; i0 < nc; i0 += BTC) {
                const int nq = min(BTC, nc - i0);
                double acc[BTC];
#pragma unroll
                for (int i = 0; i < BTC; ++i) acc[i] = 0.0;
                if (valid) {
                    for (int u = sub; u < U; u += lpr) {
                        const auto w = load_dec<DT>(row, u);
#pragma unroll
                        for (int i = 0; i < BTC; ++i)
                            if (i < nq) acc[i] += dec_dot<DT>(w, u, sa.at(i0 + i));
                    }
                }
#pragma unroll
                for (int i = 0; i < BTC; ++i) {
                    const double v = row_sum(acc[i], lpr);
                    if (valid && sub == 0 && i < nq)
                        p.part[(size_t)(c0 + i0 + i) * p.H + r] = (float)v;
                }
            }
        }
        it = hand_over_item(next, s_next, st.slot);
    }
    return true;
}

template <uint32_t DT>
__global__ void __launch_bounds__(BT, 4) moe_batch_down(MoeBatchParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ int s_next[2];
    pdl_trigger();
    pdl_wait();
    const ItemSmem S = item_smem(sm, (size_t)p.dn_rows * p.rbd);
    init_tiles_bar(S.bar);
    ItemState st{0u, 0};
    down_items<DT>(p, S, s_next, st);
}

// ---------------------------------------------------------------------------
// combine: y[t][r] = sum_k w[t][k] * part[pos(t,k)][r], k in rank order
// ---------------------------------------------------------------------------
__device__ __forceinline__ void combine_range(const MoeBatchParams &p, int i0, int is) {
    for (int i = i0; i < p.T * p.H; i += is) {
        const int t = i / p.H, r = i % p.H;
        double acc = 0.0;
        for (int k = 0; k < p.K; ++k)
            acc += (double)p.w[t * p.K + k] * (double)p.part[(size_t)p.pos_of[t * p.K + k] * p.H + r];
        p.Y[i] = (float)acc;
    }
}
__global__ void __launch_bounds__(BT) moe_batch_combine(MoeBatchParams p) {
    pdl_trigger();
    pdl_wait();
    combine_range(p, blockIdx.x * BT + threadIdx.x, gridDim.x * BT);
}

// ---------------------------------------------------------------------------
// Expert parallelism: experts split over G ranks in contiguous blocks of E/G.
//
// Slot (dest rank d, source token t) of a send buffer [G][Tmax][slot_bytes]:
//   int32 n_owned, int32 t, int32 pad[2], int32 ids[K], float w[K]   (ep_hdr_bytes)
//   the token's q8_1 row as GGUF blocks (H/32 x 36 B), present when n_owned > 0
// ids[k] is the global expert id when rank d owns it, else -1. A return buffer
// [G][Tmax][H] of doubles carries back, per slot, the weighted sum over the
// slot's owned pairs in k order.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint8_t *ep_slot(const MoeBatchParams &p, uint8_t *buf, int d, int t) {
    return buf + ((size_t)d * p.ep_tmax + t) * p.ep_slot_bytes;
}

// --- peer-memory exchange -----------------------------------------------------
// Call e (= *ep_epoch + 1, the same on every rank) uses parity e & 1 of every
// window. A slot written for call e is reused at call e + 2 only: the writer gets
// there after its combine of call e + 1, which waited for the reader's return of
// e + 1, which the reader sent after consuming call e.
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait until *flag == e; false (status bit 2) when the limit runs out.
__device__ __forceinline__ bool wait_flag(const MoeBatchParams &p, const uint32_t *flag, uint32_t e) {
    for (uint32_t it = 0; it < SPIN_LIMIT; ++it) {
        if (ld_acquire_sys(flag) == e) return true;
        if (it > 16) __nanosleep(128);
    }
    if (p.status) atomicOr((uint32_t *)p.status, 2u);
    return false;
}
__device__ __forceinline__ uint32_t *flag_at(uint32_t *flags, int kind, uint32_t par, int G, int d) {
    return flags + ((size_t)kind * 2 + par) * G + d;  // kind 0: recv, 1: back
}
// After every CTA's stores to peer memory: the last CTA to finish raises this
// rank's flag of `kind` in every peer's window.
__device__ __forceinline__ void signal_peers(const MoeBatchParams &p, int counter, int kind, uint32_t e) {
    __syncthreads();
    if (threadIdx.x != 0) return;
    __threadfence_system();
    const uint32_t prev = atomicAdd(&p.ep_done[counter], 1u);
    if (prev != gridDim.x * gridDim.y * gridDim.z - 1) return;
    p.ep_done[counter] = 0u;
    __threadfence_system();
    for (int d = 0; d < p.ep_ranks; ++d)
        st_release_sys(flag_at(p.ep_peer_flags[d], kind, e & 1u, p.ep_ranks, p.ep_rank), e);
}

// CTA per source token slot t < Tmax: route, quantise x to a GGUF q8_1 row in
// shared memory, write one slot per destination rank (empty headers for t >= T).
__global__ void __launch_bounds__(BT) moe_ep_dispatch(MoeBatchParams p) {
    extern __shared__ __align__(16) uint8_t ep_row[];
    __shared__ int s_ids[MOE_MAX_K];
    __shared__ float s_w[MOE_MAX_K];
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = p.H, K = p.K, G = p.ep_ranks, per = p.n_experts / G;
    const uint32_t e = p.ep_p2p ? *p.ep_epoch + 1 : 0u;
    // slot (d, t): the send buffer, or rank d's receive window (this rank's row) over peer memory
    auto dst = [&](int d) {
        if (!p.ep_p2p) return ep_slot(p, p.ep_send, d, t);
        return p.ep_peer_recv[d] + (((size_t)(e & 1u) * G + p.ep_rank) * p.ep_tmax + t) * p.ep_slot_bytes;
    };
    if (t >= p.ep_tokens) {
        for (int d = threadIdx.x; d < G; d += BT) *reinterpret_cast<int4 *>(dst(d)) = make_int4(0, t, 0, 0);
        if (p.ep_p2p) signal_peers(p, 0, 0, e);
        return;
    }
    __shared__ float s_lg[1024];
    for (int i = threadIdx.x; i < p.n_experts; i += BT) s_lg[i] = p.logits[(size_t)t * p.n_experts + i];
    __syncthreads();
    if (warp == 0) {
        int id;
        float w;
        route_token(s_lg, p.n_experts, K, p.norm, lane, &id, &w);
        if (lane < K) {
            s_ids[lane] = id;
            s_w[lane] = w;
            p.ep_src_ids[t * K + lane] = id;
        }
    } else {
        const float *x = p.X + (size_t)t * H;
        for (int g = warp - 1; g < H / 32; g += BT / 32 - 1)
            quant_block_q8(x[32 * g + lane], lane, nullptr, nullptr, nullptr, nullptr, ep_row + 36 * g);
    }
    __syncthreads();
    const int row_bytes = H / 32 * 36;
    for (int d = 0; d < G; ++d) {
        uint8_t *slot = dst(d);
        int n = 0;
        for (int k = 0; k < K; ++k) n += s_ids[k] / per == d;
        if (threadIdx.x < K) {
            const int id = s_ids[threadIdx.x];
            reinterpret_cast<int *>(slot + 16)[threadIdx.x] = id / per == d ? id : -1;
            reinterpret_cast<float *>(slot + 16 + 4 * K)[threadIdx.x] = s_w[threadIdx.x];
        }
        if (threadIdx.x == 0) *reinterpret_cast<int4 *>(slot) = make_int4(n, t, 0, 0);
        if (n == 0) continue;
        uint8_t *row = slot + p.ep_hdr_bytes;
        for (int i = threadIdx.x; i < row_bytes / 16; i += BT)
            reinterpret_cast<int4 *>(row)[i] = reinterpret_cast<const int4 *>(ep_row)[i];
    }
    if (p.ep_p2p) signal_peers(p, 0, 0, e);
}

// Received slot s by the whole CTA: header -> pair ids/weights (ids -1 for empty
// slots); GGUF q8_1 row -> split activations with integer 32- and 16-element sums.
// s_ok: one int of shared memory.
__device__ void unpack_slot(const MoeBatchParams &p, int s, int *s_ok) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = p.H, K = p.K, nblk = H / 32;
    const uint8_t *slot = p.ep_recv + (size_t)s * p.ep_slot_bytes;
    if (p.ep_p2p) {  // this rank's window, current parity; wait for the source's flag
        const uint32_t e = *p.ep_epoch + 1;
        const int G = p.ep_ranks, src = s / p.ep_tmax;
        slot = p.ep_peer_recv[p.ep_rank] + ((size_t)(e & 1u) * G * p.ep_tmax + s) * p.ep_slot_bytes;
        if (threadIdx.x == 0)
            *s_ok = wait_flag(p, flag_at(p.ep_peer_flags[p.ep_rank], 0, e & 1u, G, src), e);
        __syncthreads();
        const bool ok = *s_ok;
        __syncthreads();  // s_ok may be rewritten for the next slot
        if (!ok) {  // treated as an empty slot; the call reports the timeout
            if (threadIdx.x < K) p.ids[s * K + threadIdx.x] = -1;
            return;
        }
    }
    // slots written by other GPUs (or by NCCL): L2 loads, no stale L1 lines
    const int n = __ldcg(reinterpret_cast<const int *>(slot));
    if (threadIdx.x < K) {
        p.ids[s * K + threadIdx.x] = n > 0 ? __ldcg(reinterpret_cast<const int *>(slot + 16) + threadIdx.x) : -1;
        p.w[s * K + threadIdx.x] = __ldcg(reinterpret_cast<const float *>(slot + 16 + 4 * K) + threadIdx.x);
    }
    if (n == 0) return;
    const uint8_t *row = slot + p.ep_hdr_bytes;
    for (int g = warp; g < nblk; g += BT / 32) {
        const uint8_t *blk = row + 36 * g;
        const int qi = (int)__ldcg(reinterpret_cast<const signed char *>(blk) + 4 + lane);
        const int sum = __reduce_add_sync(KQ_FULL, qi);
        const int sum_lo = __reduce_add_sync(KQ_FULL, lane < 16 ? qi : 0);
        p.xq[(size_t)s * H + 32 * g + lane] = (int8_t)qi;
        if (lane == 0) {
            p.xd[(size_t)s * nblk + g] = h2f(__ldcg(reinterpret_cast<const unsigned short *>(blk)));
            p.xs32[(size_t)s * nblk + g] = sum;
            p.xs16[((size_t)s * nblk + g) * 2] = sum_lo;
            p.xs16[((size_t)s * nblk + g) * 2 + 1] = sum - sum_lo;
        }
    }
}
__global__ void __launch_bounds__(BT) moe_ep_unpack(MoeBatchParams p) {
    __shared__ int s_ok;
    unpack_slot(p, blockIdx.x, &s_ok);
}

// ret[s][r] = sum over the slot's owned pairs k (in k order) of w_k * part[pair][r],
// for the (slot, row) indices i = s * H + r in i0, i0 + is, ...
__device__ __forceinline__ void combine_slots_range(const MoeBatchParams &p, int i0, int is) {
    const int K = p.K;
    for (int i = i0; i < p.T * p.H; i += is) {
        const int s = i / p.H, r = i % p.H;
        int any = 0;
        double acc = 0.0;
        for (int k = 0; k < K; ++k) {
            if (p.ids[s * K + k] < 0) continue;
            any = 1;
            acc += (double)p.w[s * K + k] * (double)p.part[(size_t)p.pos_of[s * K + k] * p.H + r];
        }
        if (any) {
            if (!p.ep_p2p) {
                p.ep_ret[(size_t)s * p.H + r] = acc;
            } else {  // straight into the source rank's back window, this rank's row
                const uint32_t e = *p.ep_epoch + 1;
                const int G = p.ep_ranks, src = s / p.ep_tmax, t = s % p.ep_tmax;
                p.ep_peer_back[src][(((size_t)(e & 1u) * G + p.ep_rank) * p.ep_tmax + t) * p.H + r] = acc;
            }
        }
    }
}
__global__ void __launch_bounds__(BT) moe_ep_combine_slots(MoeBatchParams p) {
    const int r = blockIdx.x * BT + threadIdx.x;  // grid (H / BT, slots): one (slot, row) each
    if (r < p.H) combine_slots_range(p, blockIdx.y * p.H + r, p.T * p.H);
    if (p.ep_p2p) signal_peers(p, 1, 1, *p.ep_epoch + 1);
}

// y[t][r] = sum over ranks d that own one of t's experts (rank order) of back[d][t][r].
__global__ void __launch_bounds__(BT) moe_ep_combine_tokens(MoeBatchParams p) {
    const int i = blockIdx.x * BT + threadIdx.x;
    const double *back = p.ep_back;
    uint32_t e = 0;
    if (p.ep_p2p) {  // every rank's return for this call has landed in this rank's window
        e = *p.ep_epoch + 1;
        const int G = p.ep_ranks;
        back = p.ep_peer_back[p.ep_rank] + (size_t)(e & 1u) * G * p.ep_tmax * p.H;
        if (threadIdx.x < G) wait_flag(p, flag_at(p.ep_peer_flags[p.ep_rank], 1, e & 1u, G, threadIdx.x), e);
        __syncthreads();
    }
    if (i < p.ep_tokens * p.H) {
        const int t = i / p.H, r = i % p.H, K = p.K, per = p.n_experts / p.ep_ranks;
        double acc = 0.0;
        for (int d = 0; d < p.ep_ranks; ++d) {
            bool own = false;
            for (int k = 0; k < K; ++k) own |= p.ep_src_ids[t * K + k] / per == d;
            if (own) acc += __ldcg(back + ((size_t)d * p.ep_tmax + t) * p.H + r);
        }
        p.Y[i] = (float)acc;
    }
    if (p.ep_p2p) {  // the last CTA out advances the epoch: the next call uses the other parity
        __syncthreads();
        if (threadIdx.x == 0) {
            const uint32_t prev = atomicAdd(&p.ep_done[2], 1u);
            if (prev == gridDim.x - 1) {
                p.ep_done[2] = 0u;
                __threadfence();
                *p.ep_epoch = e;
            }
        }
    }
}

// Largest power-of-two row count in [8, 64] whose tile fits `budget` bytes.
static int tile_rows(uint32_t bytes_per_row, int cap, size_t budget) {
    int r = cap;
    while (r > 8 && (size_t)r * bytes_per_row > budget) r >>= 1;
    return r;
}

template <typename KernelT>
static void set_smem(KernelT k, size_t bytes) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// Launches a grid-stride item kernel on min(worst-case items, resident CTAs) CTAs.
template <typename KernelT>
static void launch_items(KernelT k, int max_items, size_t smem, int sms, const MoeBatchParams &p,
                         cudaStream_t st, int pdl) {
    // The limit is set on every launch: another layer shape may have lowered it.
    set_smem(k, smem);
    // resident CTAs per SM, asked once per (kernel, shared-memory size) and thread
    struct Occ { const void *fn; size_t smem; int per_sm; };
    thread_local Occ cache[16];
    thread_local int ncache = 0;
    int per_sm = 0;
    for (int i = 0; i < ncache && i < 16 && !per_sm; ++i)
        if (cache[i].fn == (const void *)k && cache[i].smem == smem) per_sm = cache[i].per_sm;
    if (!per_sm) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, BT, smem) != cudaSuccess ||
            per_sm < 1)
            per_sm = 1;
        cache[ncache % 16] = Occ{(const void *)k, smem, per_sm};
        ++ncache;
    }
    const int resident = per_sm * (sms > 0 ? sms : 1);
    const int grid = max_items < resident ? max_items : resident;
    if (grid > 0) launch_k(k, dim3(grid), dim3(BT), smem, st, pdl, p);
}

// Tile heights: three CTAs per SM, each weight tile + staged activations within ~70 KB.
static void plan_tiles(MoeBatchParams &p) {
    const size_t budget = 70 * 1024 - (size_t)ACT_TOKS * act_slot_bytes(p.H > p.F ? p.H : p.F);
    p.gu_rows = tile_rows(p.rbg + p.rbu, 16, budget);
    p.dn_rows = tile_rows(p.rbd, 64, budget);
}

// group -> gate/up -> h quantisation -> down for the pairs in p.ids (T = tokens or slots).
// pdl: every launch a programmatic dependent of the one before (each kernel waits for its
// predecessor before its first statement); the tensor-core gate/up and down launches stay ordinary.
static void launch_experts(MoeBatchParams &p, int max_groups, cudaStream_t st, int pdl = 0) {
    plan_tiles(p);
    launch_k(moe_batch_group, dim3(1), dim3((p.n_experts + 31) / 32 * 32), 0, st, pdl, p);
    const int gitems = max_groups * ((p.F + p.gu_rows - 1) / p.gu_rows);
    const size_t gsm = item_smem_bytes((size_t)p.gu_rows * (p.rbg + p.rbu), p.H);
    if (p.gate_type == T_Q4_K && p.up_type == T_Q4_K)
        launch_items(moe_batch_gateup<T_Q4_K, T_Q4_K>, gitems, gsm, p.sms, p, st, pdl);
    else if (p.gate_type == T_Q4_K)
        launch_items(moe_batch_gateup<T_Q4_K, T_Q6_K>, gitems, gsm, p.sms, p, st, pdl);
    else if (p.up_type == T_Q4_K)
        launch_items(moe_batch_gateup<T_Q6_K, T_Q4_K>, gitems, gsm, p.sms, p, st, pdl);
    else
        launch_items(moe_batch_gateup<T_Q6_K, T_Q6_K>, gitems, gsm, p.sms, p, st, pdl);
    if (p.tc_min > 0) launch_gateup_tc(p, max_groups, st);
    const int P = p.T * p.K;
    launch_k(moe_batch_hquant, dim3((P * (p.F / 32) * 32 + BT - 1) / BT), dim3(BT), 0, st, pdl, p);
    const int ditems = max_groups * ((p.H + p.dn_rows - 1) / p.dn_rows);
    const size_t dsm = item_smem_bytes((size_t)p.dn_rows * p.rbd, p.F);
    if (p.down_type == T_Q6_K)
        launch_items(moe_batch_down<T_Q6_K>, ditems, dsm, p.sms, p, st, pdl);
    else
        launch_items(moe_batch_down<T_Q4_K>, ditems, dsm, p.sms, p, st, pdl);
    if (p.tc_down_min > 0) launch_down_tc(p, max_groups, st);
}

cudaError_t launch_moe_batch(MoeBatchParams &p, cudaStream_t st) {
    const int P = p.T * p.K;
    moe_batch_route<<<p.T, BT, 0, st>>>(p);
    launch_experts(p, P < p.n_experts ? P : p.n_experts, st, 1);
    launch_k(moe_batch_combine, dim3((p.T * p.H + BT - 1) / BT), dim3(BT), 0, st, 1, p);
    return cudaGetLastError();
}

cudaError_t launch_moe_ep_dispatch(MoeBatchParams &p, cudaStream_t st) {
    moe_ep_dispatch<<<p.ep_tmax, BT, p.H / 32 * 36, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_moe_ep_experts(MoeBatchParams &p, cudaStream_t st) {
    // p.T = ranks * Tmax received slots
    const int P = p.T * p.K, local = p.n_experts / p.ep_ranks;
    moe_ep_unpack<<<p.T, BT, 0, st>>>(p);
    launch_experts(p, P < local ? P : local, st);
    moe_ep_combine_slots<<<dim3((p.H + BT - 1) / BT, p.T), BT, 0, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_moe_ep_combine(MoeBatchParams &p, cudaStream_t st) {
    // over peer memory it always runs (also with no tokens): it closes the call's epoch
    const int grid = (p.ep_tokens * p.H + BT - 1) / BT;
    if (grid == 0 && !p.ep_p2p) return cudaSuccess;
    moe_ep_combine_tokens<<<grid > 0 ? grid : 1, BT, 0, st>>>(p);
    return cudaGetLastError();
}

}  // namespace kq
