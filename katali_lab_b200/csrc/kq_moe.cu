// kq_moe.cu — the fused MoE layer, one launch per layer (README.md:13,17 of the
// reference describe its "one GPU call per MoE layer": routing, q8_1 activation
// quantisation, Q4_K gate/up, SiLU-gate multiply, Q6_K down, router-weighted
// sum; the reference ships that kernel only in binary form).
//
// B200 design: a persistent cooperative grid, one 16-warp CTA per SM.
//  1. Every CTA routes redundantly (warp 0: top-k over the router logits held
//     in registers, deterministic ties) while the other warps stage x in
//     shared memory with one vector load per thread.
//  2. Warp 0 then requests ALL of the CTA's expert bytes at once with cp.async.bulk
//     (TMA, no multicast) into shared memory, one copy per lane: its
//     phase-A blocks (32 gate/up row pairs each, two 16-pair chunks with one
//     mbarrier each) first, then its slice of the H down rows for each of the K
//     selected experts (one mbarrier per expert). At the C2 shape (H 2048, F 512,
//     top-8) that is ~120 KB per SM, so the whole 16.3 MB layer is in flight.
//  3. Phase A: each warp computes two gate/up row pairs against q8_1(x) with
//     DP4A; silu(g)*u lands in shared memory and the CTA quantises its
//     32-value block of h to q8_1 itself, writing one 48-byte record.
//  4. Grid barrier (one counter, bounded spin, error bit on timeout); while it
//     waits, the CTA decodes each expert's Q6_K down rows to 6-bit values as
//     they arrive.
//  5. Phase B: every CTA loads the K*F/32 h records (6 KB at C2) with one vector
//     load per thread, dots each expert's decoded rows with its h (both in a
//     chunk-major order that keeps the lanes' 16-byte reads conflict-free) and
//     forms sum_k w_k * down_k in a fixed order: deterministic, no atomics.
// Optional tracing: when p.trace is set, thread 0 of every CTA records
// %globaltimer at the phase boundaries (TRACE_SLOTS per CTA).
#include "kq_moe_dev.cuh"

namespace kq {
constexpr int HB = 32;        // row pairs per phase-A block = one q8_1 block of h
constexpr int HCH = 16;       // row pairs per TMA chunk
constexpr int NCH = HB / HCH; // chunks per block
constexpr int MAX_ABLK = 8;   // phase-A blocks per CTA
constexpr int DBAR = MAX_ABLK * NCH;       // first down-row barrier (one per selected expert)
constexpr int NBARS = DBAR + MOE_MAX_K;
constexpr int BAR_SLOTS = (NBARS + 2) & ~1;  // barriers + a spare, an even count of 8-byte slots
constexpr int REC_BYTES = 48; // q8_1 record of h: 32 x int8, d, sum32, sum16[2]
// The misc region holds, from a 128-byte boundary: the expert table (48-byte pairs), the
// barriers, ids, weights, h values and the q8_1 records of h, which are read as 16-byte
// vectors and so must start on a 16-byte boundary.
static_assert((8 * BAR_SLOTS + 8 * MOE_MAX_K + 4 * MAX_ABLK * HB) % 16 == 0,
              "q8_1 records of h must start 16-byte aligned");

// Decode Q6_K unit u of a raw row (quarter pair {qo, qo+2} of half h of block b)
// into its unsigned 6-bit values q at vals, and, once per block, its 16 int8
// sub-scales and fp16 scale (as float). nun = 0: element order. nun = F / 64:
// chunk-major order, the 16-element chunk c of unit v at 16 * (c * nun + v), so
// that eight lanes reading chunk c of eight consecutive units touch 128
// contiguous bytes (no bank conflicts).
__device__ __forceinline__ void q6k_decode_unit(const uint8_t *row, int u, int8_t *vals,
                                                int8_t *scales, float *dd, int nun = 0) {
    const int b = u >> 2, h = (u >> 1) & 1, qo = u & 1;
    const uint8_t *blk = row + Q6K_BYTES * b;
    uint32_t ql[8], qh[8];
    load16_a2(blk + 64 * h + 32 * qo, ql);
    load16_a2(blk + 64 * h + 32 * qo + 16, ql + 4);
    load16_a2(blk + 128 + 32 * h, qh);
    load16_a2(blk + 128 + 32 * h + 16, qh + 4);
    const int shA = 2 * qo, shB = 2 * qo + 4;
    uint32_t va[8], vb[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        va[i] = (ql[i] & 0x0F0F0F0Fu) | (((qh[i] >> shA) & 0x03030303u) << 4);
        vb[i] = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> shB) & 0x03030303u) << 4);
    }
    // va: elements [32 qo, 32 qo + 32) of unit 4b + 2h; vb: the same of unit 4b + 2h + 1
    const int va0 = nun ? 16 * (2 * qo * nun + 4 * b + 2 * h) : 256 * b + 128 * h + 32 * qo;
    const int vb0 = nun ? va0 + 16 : va0 + 64;
    const int c1 = nun ? 16 * nun : 16;  // from chunk 2qo to chunk 2qo + 1
    *reinterpret_cast<uint4 *>(vals + va0) = make_uint4(va[0], va[1], va[2], va[3]);
    *reinterpret_cast<uint4 *>(vals + va0 + c1) = make_uint4(va[4], va[5], va[6], va[7]);
    *reinterpret_cast<uint4 *>(vals + vb0) = make_uint4(vb[0], vb[1], vb[2], vb[3]);
    *reinterpret_cast<uint4 *>(vals + vb0 + c1) = make_uint4(vb[4], vb[5], vb[6], vb[7]);
    if ((u & 3) == 0) {
        uint32_t sc[4];
        load16_a2(blk + 192, sc);
        *reinterpret_cast<uint4 *>(scales + 16 * b) = make_uint4(sc[0], sc[1], sc[2], sc[3]);
        dd[b] = h2f(ld_u16(blk + 208));
    }
}

// Dot of 64 decoded elements [64u, 64u+64) of a row against q8_1 activations:
// the same exact per-q8-block terms as q6k_q8_unit (sum (q-32)x = sum qx - 32 sum x).
__device__ __forceinline__ double dec_q8_unit(const uint8_t *drow, int F, int u, const ActQ8 &a) {
    const uint4 *w = reinterpret_cast<const uint4 *>(drow + 64 * u);
    const uint4 *x = reinterpret_cast<const uint4 *>(a.q + 64 * u);
    int s[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const uint4 wv = w[g], xv = x[g];
        int acc = __dp4a((int)wv.x, (int)xv.x, 0);
        acc = __dp4a((int)wv.y, (int)xv.y, acc);
        acc = __dp4a((int)wv.z, (int)xv.z, acc);
        s[g] = __dp4a((int)wv.w, (int)xv.w, acc);
    }
    const int8_t *sc = reinterpret_cast<const int8_t *>(drow + F) + 4 * u;
    const float d = reinterpret_cast<const float *>(drow + F + F / 16)[u >> 2];
    const int *x16 = a.s16 + 4 * u;
    const int I0 = (int)sc[0] * (s[0] - 32 * x16[0]) + (int)sc[1] * (s[1] - 32 * x16[1]);
    const int I1 = (int)sc[2] * (s[2] - 32 * x16[2]) + (int)sc[3] * (s[3] - 32 * x16[3]);
    return ((double)d * (double)a.d[2 * u]) * (double)I0 +
           ((double)d * (double)a.d[2 * u + 1]) * (double)I1;
}

// fp32-activation phase B: the lanes of one expert take a row's units in the order 0, 2, 4, ...
// then 1, 3, 5, ... (i-th unit -> this unit), so that lanes reading x at the same time start on
// different banks (units 2j and 2j + 1 are 32 floats apart: the same bank).
__device__ __forceinline__ int f32_unit(int i, int nunits) {
    const int half = nunits >> 1;
    return (i % half) * 2 + i / half;
}
// The fp32-activation Q6_K unit u (block b = u/4, half h, quarter pair {qo, qo+2}: the unit
// of q6k_f32_unit) from an element-order decoded row (16-byte aligned 6-bit values, sub-scales,
// d per block): the same terms in the same order, so the same result.
__device__ __forceinline__ double dec_f32_unit(const uint8_t *drow, int F, int u, const float *x) {
    const int b = u >> 2, h = (u >> 1) & 1, qo = u & 1;
    const int eA = 256 * b + 128 * h + 32 * qo, eB = eA + 64;
    const uint4 a0 = *reinterpret_cast<const uint4 *>(drow + eA);
    const uint4 a1 = *reinterpret_cast<const uint4 *>(drow + eA + 16);
    const uint4 b0 = *reinterpret_cast<const uint4 *>(drow + eB);
    const uint4 b1 = *reinterpret_cast<const uint4 *>(drow + eB + 16);
    const uint32_t vA[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t vB[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    const float *xA = x + fpos(1, eA), *xB = x + fpos(1, eB);
    const f32x2 bias = f2_pack(TWO23_P32, TWO23_P32);
    f32x2 acc[2] = {f2_pack(0.0f, 0.0f), f2_pack(0.0f, 0.0f)};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 a4 = *reinterpret_cast<const float4 *>(xA + 4 * i);
        const float4 b4 = *reinterpret_cast<const float4 *>(xB + 4 * i);
        f32x2 &ab = acc[i >> 2];
        ab = f2_fma(bytes_as_f2(vA[i], vB[i], 0, bias), f2_pack(a4.x, b4.x), ab);
        ab = f2_fma(bytes_as_f2(vA[i], vB[i], 1, bias), f2_pack(a4.y, b4.y), ab);
        ab = f2_fma(bytes_as_f2(vA[i], vB[i], 2, bias), f2_pack(a4.z, b4.z), ab);
        ab = f2_fma(bytes_as_f2(vA[i], vB[i], 3, bias), f2_pack(a4.w, b4.w), ab);
    }
    float fA[2], fB[2];
    f2_unpack(acc[0], fA[0], fB[0]);
    f2_unpack(acc[1], fA[1], fB[1]);
    const int8_t *sc = reinterpret_cast<const int8_t *>(drow + F) + 16 * b + 8 * h;
    const float d = reinterpret_cast<const float *>(drow + F + F / 16)[b];
    return ((double)(d * (float)sc[2 * qo]) * (double)fA[0] +
            (double)(d * (float)sc[2 * qo + 1]) * (double)fA[1]) +
           ((double)(d * (float)sc[2 * qo + 4]) * (double)fB[0] +
            (double)(d * (float)sc[2 * qo + 5]) * (double)fB[1]);
}

__device__ __forceinline__ void mbar_inval(uint64_t *bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Grid barriers count arrivals on p.sync[0], which only grows (32-bit, compared modulo
// 2^32): the n-th barrier of a launch waits until it reaches base + n * gridDim.x, where base
// (p.sync[3]) is where the previous launch left it; CTA 0 records the new value at the end of
// a launch. Thread 0 of every CTA reads base after the programmatic wait.
__device__ __forceinline__ uint32_t sync_base(const MoeParams &p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.sync + 3) : "memory");
    return v;
}
__device__ __forceinline__ void grid_wait(const MoeParams &p, uint32_t target) {
    uint32_t it = 0;
    while ((int32_t)(ld_acquire_gpu(&p.sync[0]) - target) < 0) {
        if (++it > SPIN_LIMIT) {
            *p.status |= ERR_TIMEOUT_GRID;
            break;
        }
        if (it > 32) __nanosleep(20);
    }
}
__device__ void grid_barrier(const MoeParams &p, int &nbar, uint32_t sbase) {
    __syncthreads();
    if (threadIdx.x == 0) {
        red_release_gpu_add(&p.sync[0], 1u);
        grid_wait(p, sbase + (uint32_t)(nbar + 1) * gridDim.x);
    }
    ++nbar;
    __syncthreads();
}

// --- the whole expert-parallel layer over peer memory (EP 2) --------------------
// Call e (= *ep_epoch + 1, the same on every rank) uses parity e & 1 of the windows' tagged
// regions (EpPeer): every word a rank stores into another rank's window is 8 bytes, 32 bits
// of payload and the call number e, so a receiver polls the data itself until it carries e
// (no flag, no system-scope fence; a release flag cost ~6 us per exchange here). A rank
// stores its slots (header, and the q8_1 row where the owner has pairs) straight into the
// owners' windows (NVLink stores; peer loads are long dependent chains here), the owners
// store each slot's final per-row sums (two words per double) into the source's window,
// and each rank writes a "done" word into every window once none of its CTAs reads its own
// window of call e any more. A window part of call e is rewritten at call e + 2 only: a
// rank's call e + 1 ends after it has seen every rank's done word of e + 1, which each
// rank writes after it has finished call e.
// Tagged words: a plain (relaxed, system-scope) 8-byte store and load are single-copy atomic,
// so payload and call number arrive together.
__device__ __forceinline__ uint64_t tag_word(uint32_t payload, uint32_t e) {
    return ((uint64_t)e << 32) | payload;
}
__device__ __forceinline__ void st_tagged(uint64_t *a, uint32_t payload, uint32_t e) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(tag_word(payload, e)) : "memory");
}
// Two tagged words (16-byte aligned) in one vector store; each word is single-copy atomic on
// its own and the reader checks both tags.
__device__ __forceinline__ void st_tagged2(uint64_t *a, uint32_t p0, uint32_t p1, uint32_t e) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(a), "l"(tag_word(p0, e)),
                 "l"(tag_word(p1, e)) : "memory");
}
__device__ __forceinline__ uint64_t ld_tagged(const uint64_t *a) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ void ld_tagged2(const uint64_t *a, uint64_t &v0, uint64_t &v1) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v0), "=l"(v1) : "l"(a) : "memory");
}
// The payload of a tagged word once it carries call e, starting from a value v already
// loaded from it (bounded; once any wait of the call has given up the others give up at
// their next check).
__device__ __forceinline__ uint32_t tagged_value(const uint64_t *a, uint64_t v, uint32_t e,
                                                 volatile uint32_t *status) {
    for (uint32_t it = 0; (uint32_t)(v >> 32) != e; ++it) {
        if (it > SPIN_LIMIT || ((it & 1023u) == 1023u && (*status & ERR_TIMEOUT_GRID))) {
            atomicOr((uint32_t *)status, ERR_TIMEOUT_GRID);
            break;
        }
        if (it > 16) __nanosleep(32);
        v = ld_tagged(a);
    }
    return (uint32_t)v;
}
__device__ __forceinline__ uint32_t poll_tagged(const uint64_t *a, uint32_t e, volatile uint32_t *status) {
    return tagged_value(a, ld_tagged(a), e, status);
}
// Tagged slot (source src, token t) of call e in rank d's window.
__device__ __forceinline__ uint64_t *ep2_tslot(const MoeParams &p, int d, uint32_t e, int src, int t) {
    return p.ep_peer_trecv[d] + (((size_t)(e & 1u) * p.ep_ranks + src) * p.ep_tmax + t) * p.ep_tslot_words;
}
// Dispatch of call e. Warp 0 of CTA t (< tmax) routes this rank's token t, records the
// routing (tagged, for the combine) and stores slot (this rank, t)'s header into every rank's
// window: n_owned, ids[K] (-1 where another rank owns the expert), then w[K] once the softmax
// weights are formed (a receiver needs them only for its sums); a token t >= ep_tokens has
// n_owned 0, ids -1 and w 0. The other warps, spread over the CTAs, quantise the
// tokens' x block by block to GGUF q8_1 (9 words per 32 values) and store each block into
// every rank's window (only the owners of one of the token's experts read it).
__device__ void ep2_dispatch(const MoeParams &p, uint32_t e, int K, int H, float *s_logits,
                             int32_t *s_ids, float *s_w, uint8_t *blkbuf) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = p.ep_ranks, me = p.ep_rank, tmax = p.ep_tmax, per = p.n_experts / G;
    uint64_t *route_rec = p.ep_route_rec;
    if (warp == 0) {
        for (int t = blockIdx.x; t < tmax; t += gridDim.x) {
            const bool live = t < p.ep_tokens;
            const float *L = p.logits + (size_t)t * p.n_experts;
            float lv[8];
            const bool regs = p.n_experts <= 256;  // weights formed after the ids are out
            if (live) {
                if (regs) route_regs(p, L, lane, s_ids, s_w, false, lv);
                else route_smem(p, L, s_logits, s_ids, s_w, lane, true);
            }
            __syncwarp();
            trace(p, 20);
            const int id = live && lane < K ? s_ids[lane] : -1;
            if (lane < K) st_tagged(route_rec + (size_t)t * K + lane, (uint32_t)id, e);
            for (int d = 0; d < G; ++d) {
                uint64_t *slot = ep2_tslot(p, d, e, me, t);
                const bool mine = id >= 0 && id / per == d;
                const int n = __popc(__ballot_sync(KQ_FULL, lane < K && mine));
                if (lane < K) st_tagged(slot + EPT_IDS + lane, (uint32_t)(mine ? id : -1), e);
                if (lane == 0) st_tagged(slot, (uint32_t)n, e);
            }
            if (live && regs) route_weights_regs(p, lane, lv, s_ids, s_w);
            __syncwarp();
            const float w = live && lane < K ? s_w[lane] : 0.0f;
            if (lane < K)
                for (int d = 0; d < G; ++d) st_tagged(ep2_tslot(p, d, e, me, t) + EPT_W + lane, __float_as_uint(w), e);
            __syncwarp();
        }
    } else {
        const int nblk = H / 32, items = p.ep_tokens * nblk;
        uint8_t *b = blkbuf + 36 * (warp - 1);
        for (int i = (warp - 1) * (int)gridDim.x + (int)blockIdx.x; i < items;
             i += (MOE_WARPS - 1) * (int)gridDim.x) {
            const int t = i / nblk, g = i - t * nblk;
            quant_block_q8(__ldg(p.x + (size_t)t * H + 32 * g + lane), lane, nullptr, nullptr, nullptr,
                           nullptr, b);
            __syncwarp();
            if (lane < 9) {
                const uint32_t wv = reinterpret_cast<const uint32_t *>(b)[lane];
                for (int d = 0; d < G; ++d) st_tagged(ep2_tslot(p, d, e, me, t) + EPT_ROW + 9 * g + lane, wv, e);
            }
            __syncwarp();
        }
    }
}
// Word i of the received slot headers of call e (this rank's window): slot s = i / (1 + K),
// then n_owned, ids[K] (the weights are read later, per round).
__device__ __forceinline__ const uint64_t *ep2_hdr_word(const MoeParams &p, uint32_t e, int K, int i) {
    const int s = i / (1 + K), j = i - s * (1 + K);
    return ep2_tslot(p, p.ep_rank, e, s / p.ep_tmax, s % p.ep_tmax) + (j == 0 ? 0 : EPT_IDS + j - 1);
}
// Every thread of the CTA polls its words of the received headers (all loads issued before
// any wait) into hw[nslots][1 + K].
__device__ void ep2_headers(const MoeParams &p, uint32_t e, int nslots, int K, uint32_t *hw) {
    const int n = nslots * (1 + K);
    for (int i0 = threadIdx.x; i0 < n; i0 += 2 * MOE_THREADS) {
        const int i1 = i0 + MOE_THREADS;
        const uint64_t *a0 = ep2_hdr_word(p, e, K, i0);
        const uint64_t *a1 = i1 < n ? ep2_hdr_word(p, e, K, i1) : a0;
        const uint64_t v0 = ld_tagged(a0), v1 = ld_tagged(a1);
        hw[i0] = tagged_value(a0, v0, e, p.status);
        if (i1 < n) hw[i1] = tagged_value(a1, v1, e, p.status);
    }
}
// x of a phase-A block's token (warps 1..15): slot sl's q8_1 row from this rank's window of
// call e, polled in parallel into raw (9 words per 32 values: d | sum, then 32 int8 four to a
// word), then unpacked into the activation area.
__device__ void ep2_stage_x(const MoeParams &p, uint32_t e, int H, int sl, uint32_t *raw, int8_t *xq,
                            float *xd, int *xs32, int *xs16) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint64_t *trow = ep2_tslot(p, p.ep_rank, e, sl / p.ep_tmax, sl % p.ep_tmax) + EPT_ROW;
    const int nw = H / 32 * 9, nt = MOE_THREADS - 32;
    for (int i0 = tid - 32; i0 < nw; i0 += 2 * nt) {
        const int i1 = i0 + nt;
        const uint64_t v0 = ld_tagged(trow + i0), v1 = ld_tagged(trow + (i1 < nw ? i1 : i0));
        raw[i0] = tagged_value(trow + i0, v0, e, p.status);
        if (i1 < nw) raw[i1] = tagged_value(trow + i1, v1, e, p.status);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(MOE_THREADS - 32) : "memory");
    for (int g = warp - 1; g < H / 32; g += MOE_WARPS - 1) {
        const int qi = (int)(signed char)(raw[9 * g + 1 + (lane >> 2)] >> (8 * (lane & 3)));
        const int sum = __reduce_add_sync(KQ_FULL, qi);
        const int sum_lo = __reduce_add_sync(KQ_FULL, lane < 16 ? qi : 0);
        xq[32 * g + lane] = (int8_t)qi;
        if (lane == 0) {
            xd[g] = h2f(raw[9 * g] & 0xFFFFu);
            xs32[g] = sum;
            xs16[2 * g] = sum_lo;
            xs16[2 * g + 1] = sum - sum_lo;
        }
    }
}
// Combine: y[t][r] = sum over ranks d owning one of t's experts (rank order) of the sum rank d
// stored for slot (this rank, t), two tagged words per double in this rank's window. s_own:
// the owner ranks of each token (from the tagged routing record); a token whose experts are
// all on this rank was written by phase B and is skipped.
__device__ void ep2_combine(const MoeParams &p, uint32_t e, int H, const uint32_t *s_own) {
    const int G = p.ep_ranks, me = p.ep_rank, tmax = p.ep_tmax;
    const uint64_t *back = p.ep_peer_tback[me] + (size_t)(e & 1u) * G * tmax * H * 2;
    const size_t n = (size_t)p.ep_tokens * H;
    for (size_t i = (size_t)blockIdx.x * MOE_THREADS + threadIdx.x; i < n;
         i += (size_t)gridDim.x * MOE_THREADS) {
        const int t = (int)(i / H), r = (int)(i % H);
        const uint32_t owners = s_own[t];
        if (owners == (1u << me)) continue;
        double acc = 0.0;
        for (int d0 = 0; d0 < G; d0 += 4) {  // four owners' words in flight at a time
            uint64_t v[4][2];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (d0 + j < G && ((owners >> (d0 + j)) & 1u))
                    ld_tagged2(back + (((size_t)(d0 + j) * tmax + t) * H + r) * 2, v[j][0], v[j][1]);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (d0 + j < G && ((owners >> (d0 + j)) & 1u)) {
                    const uint64_t *w = back + (((size_t)(d0 + j) * tmax + t) * H + r) * 2;
                    const uint32_t hi = tagged_value(w, v[j][0], e, p.status);
                    const uint32_t lo = tagged_value(w + 1, v[j][1], e, p.status);
                    acc += __hiloint2double((int)hi, (int)lo);
                }
        }
        p.y[i] = p.accum ? __fadd_rn(p.y[i], (float)acc) : (float)acc;
    }
}
// EP 2 pairs from the polled headers hw (warp 0): in slot then k order; pw holds each pair's
// k (as int bits) until its round reads the weight; s_nown[s] = n_owned.
__device__ void ep2_pairs(const uint32_t *hw, int nslots, int K, int lane, int *pslot, int *pid,
                          float *pw, int *np, int *s_nown) {
    int base = 0;
    for (int s0 = 0; s0 < nslots; s0 += 32) {
        const int s = s0 + lane;
        const uint32_t *h = hw + (size_t)s * (1 + K);
        const int n = s < nslots ? (int)h[0] : 0;
        if (s < nslots) s_nown[s] = n;
        int cnt = 0;
        if (n > 0)
            for (int k = 0; k < K; ++k) cnt += (int)h[1 + k] >= 0;
        int incl = cnt;
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(KQ_FULL, incl, o);
            if (lane >= o) incl += y;
        }
        int off = base + incl - cnt;
        if (n > 0)
            for (int k = 0; k < K; ++k)
                if ((int)h[1 + k] >= 0) {
                    pslot[off] = s;
                    pid[off] = (int)h[1 + k];
                    pw[off] = __int_as_float(k);
                    ++off;
                }
        base += __shfl_sync(KQ_FULL, incl, 31);
    }
    if (lane == 0) *np = base;
    __syncwarp();
}
// Expert-parallel pairs of the received slots (EP 1), in slot then k order (warp 0): a slot
// header holds n_owned, t, pad[2], ids[K] (global expert id, or -1 when another rank owns
// it), w[K]; slots with n_owned == 0 carry no pairs.
__device__ void ep_pairs(const MoeParams &p, const uint8_t *recv, int nslots, int K, int lane,
                         int *pslot, int *pid, float *pw, int *np) {
    int base = 0;
    for (int s0 = 0; s0 < nslots; s0 += 32) {
        const int s = s0 + lane;
        int idv[MOE_MAX_K];
        float wv[MOE_MAX_K];
        bool live = false;
        if (s < nslots) {  // every header word loaded before any is used
            const uint8_t *slot = recv + (size_t)s * p.ep_slot_bytes;
            const int *ids = reinterpret_cast<const int *>(slot + 16);
            const float *ws = reinterpret_cast<const float *>(slot + 16 + 4 * K);
            const int n = __ldcg(reinterpret_cast<const int *>(slot));
#pragma unroll
            for (int k = 0; k < MOE_MAX_K; ++k)
                if (k < K) {
                    idv[k] = __ldcg(ids + k);
                    wv[k] = __ldcg(ws + k);
                }
            live = n > 0;
        }
        int cnt = 0;
        if (live)
#pragma unroll
            for (int k = 0; k < MOE_MAX_K; ++k)
                if (k < K) cnt += idv[k] >= 0;
        int incl = cnt;
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(KQ_FULL, incl, o);
            if (lane >= o) incl += y;
        }
        int off = base + incl - cnt;
        if (live)
#pragma unroll
            for (int k = 0; k < MOE_MAX_K; ++k)
                if (k < K && idv[k] >= 0) {
                    pslot[off] = s;
                    pid[off] = idv[k];
                    pw[off] = wv[k];
                    ++off;
                }
        base += __shfl_sync(KQ_FULL, incl, 31);
    }
    if (lane == 0) *np = base;
    __syncwarp();
}
// A slot's sum for one row: in ep_ret (a run of the slot's pairs continues from it in the
// next round; EP 2 keeps only such partial sums there) and, EP 2, once the sum is final: into the source rank's window as two tagged
// words (the source takes the first value that carries the call number), or, for a token of
// this rank whose experts are all here (local), straight into y as the combine would.
template <int EP>
__device__ __forceinline__ void ep_store_t(const MoeParams &p, uint32_t e, int slot, int H, uint32_t row,
                                           double v, bool final_sum, bool local) {
    if (EP != 2 || !final_sum) p.ep_ret[(size_t)slot * H + row] = v;
    if (EP == 2 && final_sum) {  // tback[e & 1][this rank][t][row], slot = src * tmax + t
        const int src = slot / p.ep_tmax, t = slot % p.ep_tmax;
        if (local) {
            float *y = p.y + (size_t)t * H + row;
            *y = p.accum ? __fadd_rn(*y, (float)v) : (float)v;
            return;
        }
        uint64_t *w = p.ep_peer_tback[src] +
                      ((((size_t)(e & 1u) * p.ep_ranks + p.ep_rank) * p.ep_tmax + t) * H + row) * 2;
        st_tagged2(w, (uint32_t)__double2hiint(v), (uint32_t)__double2loint(v), e);
    }
}

// SHAPE 1: the layer shape is compile-time (hidden 2048, FFN 512, top-8, Q4_K gate/up, Q6_K
// down: C2 and its family), so shape-dependent branches and loop bounds fold away; SHAPE 0
// reads every size from the parameters.
// EP 1: the experts stage of an expert-parallel layer. The (slot, k) pairs this rank owns
// come from the received slots instead of routing, each pair with its own token's q8_1 x;
// they run in rounds of K pairs (phase A, grid barrier, phase B per round) and each slot's
// weighted sum over its pairs, in k order, accumulates in double into p.ep_ret.
template <int MODE, uint32_t DT, int SHAPE, int EP, int RT = 0>
__global__ void __launch_bounds__(MOE_THREADS, 1) moe_kernel(const __grid_constant__ MoeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const int H = SHAPE ? 2048 : p.H, F = SHAPE ? 512 : p.F, K = SHAPE ? 8 : p.K;
    trace(p, 0);
    pdl_trigger();  // a following programmatic launch (a decoder's next GEMV) may be scheduled

    uint8_t *sa = smem;
    uint8_t *sb = smem + p.sb_off;
    uint8_t *act = smem + p.act_off;
    uint8_t *hact = smem + p.hact_off;
    uint8_t *misc = smem + p.misc_off;
    const uint8_t **s_tab = reinterpret_cast<const uint8_t **>(misc);  // 3 * n_experts pointers
    uint64_t *bars = reinterpret_cast<uint64_t *>(misc + 24 * ((p.n_experts + 1) & ~1));
    int32_t *s_ids = reinterpret_cast<int32_t *>(bars + BAR_SLOTS);
    float *s_w = reinterpret_cast<float *>(s_ids + MOE_MAX_K);
    float *s_h = s_w + MOE_MAX_K;                                   // MAX_ABLK * HB floats
    uint8_t *s_rec = reinterpret_cast<uint8_t *>(s_h + MAX_ABLK * HB);  // MAX_ABLK * REC_BYTES
    float *s_logits = reinterpret_cast<float *>(s_rec + MAX_ABLK * REC_BYTES);
    // expert-parallel pairs: slot, expert, weight of each owned pair; their count; n_owned of
    // each received slot; owner ranks of each of this rank's tokens
    int *s_pslot = reinterpret_cast<int *>(s_logits + p.n_experts);
    int *s_pid = s_pslot + MOE_EP_MAX_PAIRS;
    float *s_pw = reinterpret_cast<float *>(s_pid + MOE_EP_MAX_PAIRS);
    int *s_np = reinterpret_cast<int *>(s_pw + MOE_EP_MAX_PAIRS);
    int *s_nown = s_np + 4;
    uint32_t *s_own = reinterpret_cast<uint32_t *>(s_nown + MOE_EP_MAX_SLOTS);

    const uint32_t Q = (uint32_t)H / p.rg;  // phase-B row groups (16-byte aligned copies)
    const uint32_t q0 = Q * c / G, q1 = Q * (c + 1) / G;
    const uint32_t rB0 = p.rg * q0, nrB = p.rg * (q1 - q0);
    const uint32_t rbg = SHAPE ? 1152u : p.rbg, rbu = SHAPE ? 1152u : p.rbu,
                   rbd = SHAPE ? 420u : p.rbd;
    const uint32_t blk_bytes = HB * (rbg + rbu);

    if (tid == 32 && !p.route_only) {  // warp 1: keep warp 0 free for routing
        for (int i = 0; i < NBARS; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }

    if (p.route_only) {  // check entry point: the routing decision only
        pdl_wait();
        if (warp == 0) {
            route(p, p.logits, s_logits, s_ids, s_w, lane);
            if (c == 0 && lane < K) {
                p.dbg_ids[lane] = s_ids[lane];
                p.dbg_w[lane] = s_w[lane];
            }
        }
        return;
    }

    // Warp 0 keeps its logits in registers from the top-k to the softmax weights (formed after
    // the copies are issued): a second read of the logits would wait behind the weight stream.
    float route_lv[8];
    const bool route_in_regs = p.n_experts <= 256;
    // ---- 1. routing (warp 0) and x staging (all other threads) --------------
    float *xf = reinterpret_cast<float *>(act);  // fp32 x, H floats
    int8_t *xq = reinterpret_cast<int8_t *>(act + 4 * H);
    float *xd = reinterpret_cast<float *>(act + 5 * H);
    int *xs32 = reinterpret_cast<int *>(xd + H / 32);
    int *xs16 = xs32 + H / 32;
    // fp32 mode: x bank-spread (element i at fpos(1, i): 16 bytes of padding after every 64
    // floats, so the lanes' 64-element units fall on distinct banks), then the per-32 sums
    float *xfs = reinterpret_cast<float *>(act + (MODE == 1 ? 4 * (H + H / 16) : 4 * H));
    auto xfi = [&](int i) { return MODE == 1 ? fpos(1, i) : i; };
    int npairs = K, nrounds = 1;
    int nbar = 0;        // grid barriers passed
    uint32_t sbase = 0;  // thread 0: the barrier counter at launch (sync_base)
    const uint8_t *ep_recv = p.ep_recv;
    int ep_nslots = (int)p.ep_slots;
    uint32_t ep_e = 0;
    if constexpr (EP == 2) {
        pdl_wait();
        if (tid == 0) sbase = sync_base(p);
        ep_e = *p.ep_epoch + 1;
        ep_nslots = p.ep_ranks * p.ep_tmax;  // slot s = source rank * tmax + token
        ep2_dispatch(p, ep_e, K, H, s_logits, s_ids, s_w, act);
        if (c < (uint32_t)p.ep_tmax) trace(p, 1);
        // the expert pointer table, then every header word of the call in parallel, and the
        // owner ranks of this rank's tokens from the routing record (for the combine)
        const int npair = (3 * p.n_experts + 1) / 2;  // 2 pointers per 16 B
        for (int i = tid; i < npair; i += MOE_THREADS)
            reinterpret_cast<uint4 *>(s_tab)[i] = __ldg(reinterpret_cast<const uint4 *>(p.experts) + i);
        if (tid < MOE_EP_MAX_SLOTS) s_own[tid] = 0u;
        __syncthreads();  // the dispatch's staging in act is free again
        uint32_t *hw = reinterpret_cast<uint32_t *>(act);
        ep2_headers(p, ep_e, ep_nslots, K, hw);
        {
            const uint64_t *route_rec = p.ep_route_rec;
            const int per = p.n_experts / p.ep_ranks;
            for (int i = tid; i < p.ep_tokens * K; i += MOE_THREADS)
                atomicOr(&s_own[i / K], 1u << ((int)poll_tagged(route_rec + i, ep_e, p.status) / per));
        }
        __syncthreads();
        if (warp == 0) ep2_pairs(hw, ep_nslots, K, lane, s_pslot, s_pid, s_pw, s_np, s_nown);
        __syncthreads();
    } else if constexpr (EP == 1) {
        pdl_wait();
        if (tid == 0) sbase = sync_base(p);
        if (warp == 0) {
            ep_pairs(p, ep_recv, ep_nslots, K, lane, s_pslot, s_pid, s_pw, s_np);
        } else {
            const int npair = (3 * p.n_experts + 1) / 2;  // expert pointer table, 2 per 16 B
            for (int i = tid - 32; i < npair; i += MOE_THREADS - 32)
                reinterpret_cast<uint4 *>(s_tab)[i] = __ldg(reinterpret_cast<const uint4 *>(p.experts) + i);
        }
        __syncthreads();
    }
    if constexpr (EP != 0) {
        npairs = *s_np;
        nrounds = (npairs + K - 1) / K;
        trace(p, 11);
    } else if (RT) {
        // Router folded into the launch: this CTA's router rows [r0, r0 + nr) are loaded into
        // registers before pdl_wait() (constant weights), then every CTA forms xb = RMSNorm(x) *
        // rt_norm in xf (the order of the reference's rmsnorm: (x * inv) * w), dots its rows
        // with it (double sums), publishes the logits, and after a grid barrier warp 0 routes
        // on the whole vector.
        const int E = p.n_experts, r0 = E * (int)c / (int)G, nr = E * ((int)c + 1) / (int)G - r0;
        const bool xl = tid < H / 4;
        float4 rw[MOE_RT_ROWS];
#pragma unroll
        for (int i = 0; i < MOE_RT_ROWS; ++i)
            rw[i] = (i < nr && xl) ? __ldcs(reinterpret_cast<const float4 *>(p.rt_w + (size_t)(r0 + i) * H) + tid)
                                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        const int npair = (3 * p.n_experts + 1) / 2;  // expert pointer table, 2 per 16 B
        for (int i = tid; i < npair; i += MOE_THREADS)
            reinterpret_cast<uint4 *>(s_tab)[i] = __ldg(reinterpret_cast<const uint4 *>(p.experts) + i);
        const float4 nw = xl ? __ldg(reinterpret_cast<const float4 *>(p.rt_norm) + tid)
                             : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        pdl_wait();
        if (tid == 0) sbase = sync_base(p);
        double *red = reinterpret_cast<double *>(s_h);  // MOE_WARPS doubles, free until phase A
        auto block_sum = [&](double v) {
            v = warp_sum_d(v);
            if (lane == 0) red[warp] = v;
            __syncthreads();
            double t = 0.0;
            for (int w = 0; w < MOE_WARPS; ++w) t += red[w];
            __syncthreads();
            return t;
        };
        float4 xv = xl ? __ldcg(reinterpret_cast<const float4 *>(p.x) + tid) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        double ss = (double)xv.x * (double)xv.x;
        ss += (double)xv.y * (double)xv.y;
        ss += (double)xv.z * (double)xv.z;
        ss += (double)xv.w * (double)xv.w;
        ss = block_sum(ss);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(ss / (double)H), p.rt_eps)));
        if (xl) {
            xv.x = __fmul_rn(__fmul_rn(xv.x, inv), nw.x);
            xv.y = __fmul_rn(__fmul_rn(xv.y, inv), nw.y);
            xv.z = __fmul_rn(__fmul_rn(xv.z, inv), nw.z);
            xv.w = __fmul_rn(__fmul_rn(xv.w, inv), nw.w);
            *reinterpret_cast<float4 *>(xf + xfi(4 * tid)) = xv;
        }
#pragma unroll
        for (int i = 0; i < MOE_RT_ROWS; ++i) {
            if (i < nr) {  // uniform across the CTA
                double d = (double)rw[i].x * (double)xv.x;
                d += (double)rw[i].y * (double)xv.y;
                d += (double)rw[i].z * (double)xv.z;
                d += (double)rw[i].w * (double)xv.w;
                d = block_sum(xl ? d : 0.0);
                if (tid == 0) const_cast<float *>(p.logits)[r0 + i] = (float)d;
            }
        }
        grid_barrier(p, nbar, sbase);  // every CTA's logits published
        if (warp == 0) {
            if (route_in_regs) route_regs<RT>(p, p.logits, lane, s_ids, s_w, false, route_lv);
            else route<RT>(p, p.logits, s_logits, s_ids, s_w, lane, false);  // weights after the copies are issued
            trace(p, 1);
        }
    } else if (warp == 0) {
        pdl_wait();  // under a programmatic launch: x, logits / ids, scratch only after this
        if (lane == 0) sbase = sync_base(p);
        if (p.ids) {
            if (lane < K) {
                s_ids[lane] = p.ids[lane];
                s_w[lane] = p.w[lane];
            }
            __syncwarp();
        } else if (route_in_regs) {  // weights after the copies are issued
            route_regs(p, p.logits, lane, s_ids, s_w, false, route_lv);
        } else {
            route(p, p.logits, s_logits, s_ids, s_w, lane, false);
        }
        trace(p, 1);
    } else {
        // The expert pointer table changes only through stream-ordered copies (a copy ends
        // any programmatic overlap), so it is read before pdl_wait(); x after it.
        const int npair = (3 * p.n_experts + 1) / 2;  // expert pointer table, 2 per 16 B
        for (int i = tid - 32; i < npair; i += MOE_THREADS - 32)
            reinterpret_cast<uint4 *>(s_tab)[i] = __ldg(reinterpret_cast<const uint4 *>(p.experts) + i);
        pdl_wait();
        for (int i = tid - 32; i < H / 4; i += MOE_THREADS - 32)
            *reinterpret_cast<float4 *>(xf + xfi(4 * i)) = __ldg(reinterpret_cast<const float4 *>(p.x) + i);
    }
    if constexpr (!EP) __syncthreads();
    trace(p, 2);

    // Expert-parallel rounds overlap when the decoded down rows have their own area: round
    // rd + 1's gate/up rows are requested (and its x rows staged) once round rd's phase A is
    // done, its down rows once round rd's rows are decoded.
    const bool pipe = EP && MODE == 0 && DT == T_Q6_K && p.dec_enabled && p.dec_off != 0 && nrB != 0;
    const uint32_t per = nrB * rbd;  // down-row bytes of one expert for this CTA
    // Request round r's bytes (warp 0, one copy per lane): gate/up chunks (what & 1), then
    // each selected expert's down rows on its own barrier (what & 2), decoded as they arrive.
    // One warp keeps that order (copies issued from every warp interleave and delay the
    // first gate/up chunk).
    auto issue_round = [&](int r, int what) {
        const int KRr = EP ? min(K, npairs - r * K) : K;
        const int32_t *rids = EP ? s_pid + r * K : s_ids;
        const uint32_t BAr = (uint32_t)KRr * F / HB, b0r = BAr * c / G;
        const int nchunk = (int)(BAr * (c + 1) / G - b0r) * NCH;
        if ((what & 1) && lane < nchunk) mbar_arrive_expect_tx(&bars[lane], HCH * (rbg + rbu));
        if ((what & 2) && nrB && lane < KRr) mbar_arrive_expect_tx(&bars[DBAR + lane], per);
        __syncwarp();
        const uint64_t pol = l2_evict_first_policy();
        const int q0 = (what & 1) ? 0 : 2 * nchunk;
        const int ncopy = (what & 2) ? 2 * nchunk + (nrB ? KRr : 0) : 2 * nchunk;
        for (int q = q0 + lane; q < ncopy; q += 32) {
            if (q < 2 * nchunk) {  // gate (even) or up (odd) rows of one chunk
                const int ci = q >> 1, a = ci / NCH, ch = ci % NCH, up = q & 1;
                const uint32_t blk = b0r + a;
                const int k = (int)(blk / (F / HB));
                const uint32_t j0 = (blk % (F / HB)) * HB + ch * HCH;
                const uint32_t rb = up ? rbu : rbg;
                const uint8_t *base = s_tab[3 * rids[k] + up];
                const uint8_t *src = base ? base + (size_t)j0 * rb : nullptr;
                uint8_t *dst = sa + (size_t)a * blk_bytes + (up ? HB * rbg : 0) + ch * HCH * rb;
                bulk_g2s_split(dst, src, HCH * rb, &bars[ci], pol, p.status);
            } else {  // down rows [rB0, rB0 + nrB) of selected expert k
                const int k = q - 2 * nchunk;
                const uint8_t *base = s_tab[3 * rids[k] + 2];
                bulk_g2s_split(sb + (size_t)k * (per + 16), base ? base + (size_t)rB0 * rbd : nullptr,
                               per, &bars[DBAR + k], pol, p.status);
            }
        }
    };
    // x of round r's phase-A block of this CTA (warps 1..15): its pair's token, from the
    // slot's q8_1 row (EP 2: tagged words in this rank's window; EP 1: the received bytes)
    auto stage_x = [&](int r) {
        const int KRr = min(K, npairs - r * K);
        const uint32_t BAr = (uint32_t)KRr * F / HB, b0r = BAr * c / G;
        if (BAr * (c + 1) / G == b0r) return;  // no phase-A block
        const int sl = s_pslot[r * K + (int)(b0r / (F / HB))];
        if constexpr (EP == 2) {
            ep2_stage_x(p, ep_e, H, sl, reinterpret_cast<uint32_t *>(act), xq, xd, xs32, xs16);
        } else {
            const uint8_t *row = ep_recv + (size_t)sl * p.ep_slot_bytes + p.ep_hdr_bytes;
            for (int g = warp - 1; g < H / 32; g += MOE_WARPS - 1) {
                const uint8_t *blk = row + 36 * g;
                const int qi = (int)__ldcg(reinterpret_cast<const signed char *>(blk) + 4 + lane);
                const int sum = __reduce_add_sync(KQ_FULL, qi);
                const int sum_lo = __reduce_add_sync(KQ_FULL, lane < 16 ? qi : 0);
                xq[32 * g + lane] = (int8_t)qi;
                if (lane == 0) {
                    xd[g] = h2f(__ldcg(reinterpret_cast<const unsigned short *>(blk)));
                    xs32[g] = sum;
                    xs16[2 * g] = sum_lo;
                    xs16[2 * g + 1] = sum - sum_lo;
                }
            }
        }
    };

    // EP 2: after the call's last grid barrier no CTA reads this rank's window of the call any
    // more; CTA 0 then writes this rank's done word into every rank's window (a rank with no
    // pairs passes one barrier for it)
    auto ep2_done = [&]() {
        if (EP == 2 && c == 0 && tid < p.ep_ranks)
            st_tagged(p.ep_peer_tdone[tid] + (size_t)(ep_e & 1u) * p.ep_ranks + p.ep_rank, 1u, ep_e);
    };
    if (EP == 2 && nrounds == 0) {
        grid_barrier(p, nbar, sbase);
        ep2_done();
    }
    // a slot of this rank whose token's experts are all here: its sum goes straight to y
    auto local_slot = [&](int sl) { return EP == 2 && sl / p.ep_tmax == p.ep_rank && s_nown[sl] == K; };

    for (int rd = 0; rd < nrounds; ++rd) {
    // pairs of this round: K (one token's experts), or expert-parallel pairs [rd K, rd K + KR)
    const int KR = EP ? min(K, npairs - rd * K) : K;
    const float *rw = EP ? s_pw + rd * K : s_w;  // the round's weights
    const int *rslot = s_pslot + rd * K;         // and slots (EP)
    if constexpr (EP) {
        if (rd > 0 && !pipe) {  // every wait of the previous round has returned: re-arm the barriers
            __syncthreads();
            if (tid == 32) {
                for (int i = 0; i < NBARS; ++i) {
                    mbar_inval(&bars[i]);
                    mbar_init(&bars[i], 1);
                }
                fence_mbar_init();
            }
            __syncthreads();
        }
    }
    const uint32_t BA = (uint32_t)KR * F / HB;  // phase-A blocks of this round
    const uint32_t b0 = BA * c / G, b1 = BA * (c + 1) / G;  // 32-bit: BA * G < 2^32
    const int nbA = (int)(b1 - b0);
    const uint32_t hb0 = EP ? (uint32_t)(rd * K) * (F / HB) : 0u;  // first h record of the round

    // ---- 2. request every expert byte this CTA needs; stage x ---------------------------
    if (!(pipe && rd > 0)) {  // (an overlapped round's bytes were requested in the previous one)
        if (warp == 0) {
            issue_round(rd, 3);
            trace(p, 3);
            if (!EP && !p.ids) {
                if (route_in_regs) route_weights_regs(p, lane, route_lv, s_ids, s_w);
                else route_weights<RT>(p, p.logits, nullptr, 0, lane, s_ids, s_w);
            }
        } else if (EP) {
            stage_x(rd);
        } else if (warp > 0) {
            for (int g = warp - 1; g < H / 32; g += MOE_WARPS - 1) {
                const float v = xf[xfi(32 * g + lane)];
                if (MODE == 0) {
                    quant_block_q8(v, lane, xq + 32 * g, xd + g, xs32 + g, xs16 + 2 * g, nullptr);
                } else {
                    const float s = warp_sum_f(v);
                    if (lane == 0) xfs[g] = s;
                }
            }
        }
        __syncthreads();
    }
    if (EP) trace(p, 21);

    // ---- 3. phase A: gate/up row pairs -> h = silu(g) * u, quantised per block --
    bool ok = true;
    const int nbh = H / 256;
    const ActQ8 ax{xq, xd, xs32, xs16, 0};
    Q4Act xr;
    if (MODE == 0 && nbh == 8 && nbA > 0) xr = load_q4act(ax, lane);  // this lane's unit of x
    for (int a = 0; a < nbA; ++a) {
        const uint8_t *base = sa + (size_t)a * blk_bytes;
        const int p0 = warp, p1 = warp + MOE_WARPS;  // two row pairs per warp, one per chunk
        const uint8_t *g0 = base + (size_t)p0 * rbg, *g1 = base + (size_t)p1 * rbg;
        const uint8_t *u0 = base + (size_t)HB * rbg + (size_t)p0 * rbu;
        const uint8_t *u1 = base + (size_t)HB * rbg + (size_t)p1 * rbu;
        double pg0, pu0, pg1, pu1;
        // pair p0 (first chunk) is computed while the second chunk is still arriving
        ok &= mbar_wait_warp(&bars[a * NCH + p0 / HCH], 0);
        if (a == 0) {
            trace(p, 4);
            if (EP && rd == 0) trace(p, 24);
        }
        if (MODE == 0 && nbh == 8) {
            pg0 = q4k_q8_unit_r(g0, lane, xr);
            pu0 = q4k_q8_unit_r(u0, lane, xr);
        } else if (MODE == 0) {
            pg0 = q4k_q8_partial(g0, nbh, ax, lane);
            pu0 = q4k_q8_partial(u0, nbh, ax, lane);
        } else {
            pg0 = q4k_f32_partial(g0, nbh, xf, xfs, lane, 1);
            pu0 = q4k_f32_partial(u0, nbh, xf, xfs, lane, 1);
        }
        ok &= mbar_wait_warp(&bars[a * NCH + p1 / HCH], 0);
        if (a == 0) trace(p, 12);
        if (MODE == 0 && nbh == 8) {
            pg1 = q4k_q8_unit_r(g1, lane, xr);
            pu1 = q4k_q8_unit_r(u1, lane, xr);
        } else if (MODE == 0) {
            pg1 = q4k_q8_partial(g1, nbh, ax, lane);
            pu1 = q4k_q8_partial(u1, nbh, ax, lane);
        } else {
            pg1 = q4k_f32_partial(g1, nbh, xf, xfs, lane, 1);
            pu1 = q4k_f32_partial(u1, nbh, xf, xfs, lane, 1);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            pg0 += __shfl_xor_sync(KQ_FULL, pg0, o);
            pu0 += __shfl_xor_sync(KQ_FULL, pu0, o);
            pg1 += __shfl_xor_sync(KQ_FULL, pg1, o);
            pu1 += __shfl_xor_sync(KQ_FULL, pu1, o);
        }
        if (lane == 0) {
            s_h[a * HB + p0] = __fmul_rn(kq_silu((float)pg0), (float)pu0);
            s_h[a * HB + p1] = __fmul_rn(kq_silu((float)pg1), (float)pu1);
        }
    }
    if (!ok && lane == 0) *p.status |= ERR_TIMEOUT_TMA;
    trace(p, 5);
    if (EP && rd == 0) trace(p, 25);
    __syncthreads();
    if (warp < nbA) {  // one warp per block: publish h as a q8_1 record (fp32 in mode 1)
        const int a = warp;
        const float v = s_h[a * HB + lane];
        const uint32_t blk = b0 + a;
        if (MODE == 0) {
            uint8_t *r = s_rec + a * REC_BYTES;
            float *md = reinterpret_cast<float *>(r + 32);
            int *ms = reinterpret_cast<int *>(r + 36);
            quant_block_q8(v, lane, reinterpret_cast<int8_t *>(r), md, ms, ms + 1, nullptr);
            __syncwarp();
            if (lane < 3)
                reinterpret_cast<uint4 *>(p.hbuf)[3 * (hb0 + blk) + lane] =
                    reinterpret_cast<const uint4 *>(r)[lane];
        } else {
            p.hbuf[HB * blk + lane] = v;
        }
    }

    // ---- 4. grid barrier: arrive, decode the down rows while waiting, then wait ----
    // The CTA barrier orders every thread's h stores before thread 0's release.
    __syncthreads();
    if (tid == 0) red_release_gpu_add(&p.sync[0], 1u);
    // Overlap: round rd + 1's gate/up rows into the phase-A staging (every read of it is done:
    // the decoded rows have their own area) and its x rows into the activation area.
    const bool pre = pipe && rd + 1 < nrounds;
    if (pre) {
        if (warp == 0) {
            if (lane == 0) {
                for (int i = 0; i < DBAR; ++i) {
                    mbar_inval(&bars[i]);
                    mbar_init(&bars[i], 1);
                }
                fence_mbar_init();
            }
            __syncwarp();
            issue_round(rd + 1, 1);
            trace(p, 23);
        } else {
            stage_x(rd + 1);
        }
    }
    const bool predecode = DT == T_Q6_K && p.dec_enabled && nrB != 0;
    // Phase B's expert-major path (F a power of two from 256 to 2048) reads h and the
    // decoded down rows in chunk-major order; the row-major path in element order.
    const bool xmaj = predecode && MODE == 0 && (F == 256 || F == 512 || F == 1024 || F == 2048);
    uint8_t *sdec = smem + p.dec_off;
    const uint32_t drb = p.dec_row_bytes;
    const uint32_t dstride = nrB * drb + 16;  // padded decoded expert stride
    if (predecode) {
        // Units in expert order; a thread waits for an expert's rows only when it
        // reaches that expert's units, so decoding overlaps the later arrivals.
        trace(p, 13);
        const int upr = F / 64;  // units per row
        const int per_k = (int)nrB * upr;
        const int total = KR * per_k;
        int kw = -1;  // the expert whose rows this thread has seen arrive
        for (int t = tid; t < total; t += MOE_THREADS) {
            const int kk = t / per_k, rem = t - kk * per_k, rr = rem / upr, u = rem - rr * upr;
            if (kk != kw) {
                if (!mbar_wait(&bars[DBAR + kk], 0)) {
                    *p.status |= ERR_TIMEOUT_TMA;
                    break;
                }
                kw = kk;
            }
            uint8_t *drow = sdec + (size_t)kk * dstride + (size_t)rr * drb;
            q6k_decode_unit(sb + (size_t)kk * (nrB * rbd + 16) + (size_t)rr * rbd, u,
                            reinterpret_cast<int8_t *>(drow),
                            reinterpret_cast<int8_t *>(drow + F),
                            reinterpret_cast<float *>(drow + F + F / 16), xmaj ? upr : 0);
        }
    }
    trace(p, 14);
    if constexpr (EP == 2) {
        // the round's weights (the sources store them after the ids), read while thread 0
        // waits at the barrier
        if (warp == 1 && lane < KR) {
            const int i = rd * K + lane, sl = s_pslot[i], k = __float_as_int(s_pw[i]);
            const uint64_t *wa = ep2_tslot(p, p.ep_rank, ep_e, sl / p.ep_tmax, sl % p.ep_tmax) + EPT_W + k;
            s_pw[i] = __uint_as_float(poll_tagged(wa, ep_e, p.status));
        }
    }
    if (tid == 0) grid_wait(p, sbase + (uint32_t)(nbar + 1) * G);
    ++nbar;
    __syncthreads();
    trace(p, 6);
    if (EP && rd == 0) trace(p, 26);
    if constexpr (EP == 2) {
        if (rd == nrounds - 1) ep2_done();
    }
    if (pre && warp == 0) {  // round rd + 1's down rows: every thread has decoded round rd's
        if (lane == 0) {
            for (int i = DBAR; i < NBARS; ++i) {
                mbar_inval(&bars[i]);
                mbar_init(&bars[i], 1);
            }
            fence_mbar_init();
        }
        __syncwarp();
        issue_round(rd + 1, 2);
    }

    // ---- 5. load h for phase B ------------------------------------------------
    int8_t *hq = reinterpret_cast<int8_t *>(hact);  // expert stride F + 16 (bank spread)
    float *hd = reinterpret_cast<float *>(hact + (size_t)K * (F + 16));
    int *hs32 = reinterpret_cast<int *>(hd + (size_t)K * F / 32);
    int *hs16 = hs32 + (size_t)K * F / 32;
    // fp32 mode: h bank-spread as x, each expert's part skewed by a further 4 floats per expert
    float *hf = reinterpret_cast<float *>(hact);
    float *hfs = hf + (size_t)K * F + (size_t)K * F / 16 + 4 * (size_t)K;
    auto hfi = [&](int e) { return fpos(1, e) + 4 * (e / F); };
    if (MODE == 0) {
        const int nrec = (int)BA;
        const int nun = F / 64;
        for (int t = tid; t < 3 * nrec; t += MOE_THREADS) {
            const int r = t / 3, part = t - 3 * r;
            const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(p.hbuf) + 3 * hb0 + t);
            if (part < 2) {  // elements [32 jb + 16 part, +16) of expert kk's h
                const int kk = r / (F / HB), jb = r - kk * (F / HB);
                const int off = xmaj ? 16 * ((2 * (jb & 1) + part) * nun + (jb >> 1))
                                     : HB * jb + 16 * part;
                *reinterpret_cast<uint4 *>(hq + (size_t)kk * (F + 16) + off) = v;
            } else {
                hd[r] = __uint_as_float(v.x);
                hs32[r] = (int)v.y;
                hs16[2 * r] = (int)v.z;
                hs16[2 * r + 1] = (int)v.w;
            }
        }
    } else {
        for (int t = tid; t < K * F / 4; t += MOE_THREADS)
            *reinterpret_cast<float4 *>(hf + hfi(4 * t)) = __ldcg(reinterpret_cast<const float4 *>(p.hbuf) + t);
        __syncthreads();
        for (int g = warp; g < K * F / 32; g += MOE_WARPS) {
            const float s = warp_sum_f(hf[hfi(32 * g + lane)]);
            if (lane == 0) hfs[g] = s;
        }
    }
    __syncthreads();

    // ---- 6. phase B: K down rows per output row, fixed-order weighted sum ------
    if (nrB) {
        bool down_in = true;  // the decode loop has already waited in predecode mode
        if (!predecode)
            for (int kk = 0; kk < KR; ++kk) down_in &= mbar_wait_warp(&bars[DBAR + kk], 0);
        if (!down_in) {
            if (lane == 0) *p.status |= ERR_TIMEOUT_TMA;
        } else if (xmaj) {
            trace(p, 7);
            if (EP && rd == 0) trace(p, 27);
            // Expert-major: warp -> (expert k, row subset); lane -> (row slot, 64-element
            // unit u). The lane keeps unit u of expert k's h in registers and dots it
            // with the same unit of several rows; dots meet in shared memory and the
            // weighted sum over experts runs in expert order.
            int kp2 = 1;
            while (kp2 < K) kp2 <<= 1;
            const int wpe = MOE_WARPS / kp2, k = warp / wpe, wsub = warp % wpe;  // k >= KR: idle
            const int nunits = F / 64, rpl = 32 / nunits;
            const int u = lane % nunits, rs = lane / nunits;
            float *s_dot = reinterpret_cast<float *>(smem + p.sdot_off);  // [K][nrB]
            if (k < KR) {
                const int8_t *hk = hq + (size_t)k * (F + 16) + 16 * u;  // chunk-major
                const uint4 a0 = *reinterpret_cast<const uint4 *>(hk);
                const uint4 a1 = *reinterpret_cast<const uint4 *>(hk + 16 * nunits);
                const uint4 a2 = *reinterpret_cast<const uint4 *>(hk + 32 * nunits);
                const uint4 a3 = *reinterpret_cast<const uint4 *>(hk + 48 * nunits);
                const double dx0 = (double)hd[(size_t)k * F / 32 + 2 * u];
                const double dx1 = (double)hd[(size_t)k * F / 32 + 2 * u + 1];
                const int4 x16 = reinterpret_cast<const int4 *>(hs16 + (size_t)k * F / 16)[u];
                const uint4 av[4] = {a0, a1, a2, a3};
                for (uint32_t r = wsub * rpl + rs; r < nrB + (uint32_t)rs; r += wpe * rpl) {
                    double part = 0.0;
                    const bool live = r < nrB;
                    if (live) {
                        const uint8_t *drow = sdec + (size_t)k * dstride + (size_t)r * drb;
                        const uint8_t *w = drow + 16 * u;  // chunk-major
                        int sg[4];
#pragma unroll
                        for (int gq = 0; gq < 4; ++gq) {
                            const uint4 wv = *reinterpret_cast<const uint4 *>(w + 16 * gq * nunits);
                            const uint4 xv = av[gq];
                            int acc = __dp4a((int)wv.x, (int)xv.x, 0);
                            acc = __dp4a((int)wv.y, (int)xv.y, acc);
                            acc = __dp4a((int)wv.z, (int)xv.z, acc);
                            sg[gq] = __dp4a((int)wv.w, (int)xv.w, acc);
                        }
                        const uint32_t scw = *reinterpret_cast<const uint32_t *>(drow + F + 4 * u);
                        const int sc0 = (int)(int8_t)(scw & 0xFF), sc1 = (int)(int8_t)((scw >> 8) & 0xFF);
                        const int sc2 = (int)(int8_t)((scw >> 16) & 0xFF), sc3 = (int)(int8_t)(scw >> 24);
                        const double d = (double)reinterpret_cast<const float *>(drow + F + F / 16)[u >> 2];
                        const int I0 = sc0 * (sg[0] - 32 * x16.x) + sc1 * (sg[1] - 32 * x16.y);
                        const int I1 = sc2 * (sg[2] - 32 * x16.z) + sc3 * (sg[3] - 32 * x16.w);
                        part = (d * dx0) * (double)I0 + (d * dx1) * (double)I1;
                    }
                    for (int o = 1; o < nunits; o <<= 1) part += __shfl_xor_sync(KQ_FULL, part, o);
                    if (live && u == 0) s_dot[(size_t)k * nrB + r] = (float)part;
                }
            }
            if (warp == 0) trace(p, 15);
            __syncthreads();
            for (uint32_t r = tid; r < nrB; r += MOE_THREADS) {
                if constexpr (EP) {
                    // runs of one slot's pairs, in k order; a run that began in the previous
                    // round continues from that round's sum (same thread, same row)
                    int cur = -1;
                    double acc = 0.0;
                    for (int kk = 0; kk < KR; ++kk) {
                        const int sl = rslot[kk];
                        if (sl != cur) {  // the previous slot's run ends here: its sum is final
                            if (cur >= 0) ep_store_t<EP>(p, ep_e, cur, H, rB0 + r, acc, true, local_slot(cur));
                            const bool cont = kk == 0 && rd > 0 && s_pslot[rd * K - 1] == sl;
                            acc = cont ? p.ep_ret[(size_t)sl * H + rB0 + r] : 0.0;
                            cur = sl;
                        }
                        acc += (double)rw[kk] * (double)s_dot[(size_t)kk * nrB + r];
                    }
                    // final unless the slot's run continues in the next round
                    const int nx = rd * K + KR;
                    if (cur >= 0)
                        ep_store_t<EP>(p, ep_e, cur, H, rB0 + r, acc, nx >= npairs || s_pslot[nx] != cur,
                                       local_slot(cur));
                } else {
                    double acc = 0.0;
                    for (int kk = 0; kk < K; ++kk) acc += (double)rw[kk] * (double)s_dot[(size_t)kk * nrB + r];
                    p.y[rB0 + r] = p.accum ? __fadd_rn(p.y[rB0 + r], (float)acc) : (float)acc;
                }
            }
        } else {
            trace(p, 7);
            if (EP && rd == 0) trace(p, 27);
            // lanes per expert: 32 / next_pow2(K); lane = (expert k, slot g)
            int kp2 = 1;
            while (kp2 < K) kp2 <<= 1;
            const int lpe = 32 / kp2, k = lane / lpe, g = lane % lpe;
            const int nunits = 4 * (F / 256);
            const uint32_t per = nrB * rbd;
            const ActQ8 ah{hq + (size_t)k * (F + 16), hd + (size_t)k * F / 32,
                           hs32 + (size_t)k * F / 32, hs16 + (size_t)k * F / 16, 0};
            const double wk = k < KR ? (double)rw[k] : 0.0;
            for (uint32_t rr = warp; rr < nrB; rr += MOE_WARPS) {
                double part = 0.0;
                if (k < K) {
                    if (predecode) {
                        const uint8_t *drow = sdec + (size_t)k * dstride + (size_t)rr * drb;
                        for (int i = g; i < nunits; i += lpe)
                            part += MODE == 0 ? dec_q8_unit(drow, F, i, ah)
                                              : dec_f32_unit(drow, F, f32_unit(i, nunits), hf + hfi(k * F));
                    } else {
                        const uint8_t *row = sb + (size_t)k * (per + 16) + (size_t)rr * rbd;
                        for (int u = g; u < nunits; u += lpe) {
                            if (MODE == 0) part += unit_q8<DT>(row, u, ah);
                            else part += unit_f32<DT>(row, f32_unit(u, nunits), hf + hfi(k * F),
                                                      hfs + (size_t)k * F / 32, 1);
                        }
                    }
                }
                if (rr == 0) trace(p, 15);
                for (int o = 1; o < lpe; o <<= 1) part += __shfl_xor_sync(KQ_FULL, part, o);
                double t = k < K ? wk * (double)(float)part : 0.0;
                for (int o = lpe; o < 32; o <<= 1) t += __shfl_xor_sync(KQ_FULL, t, o);
                if (!EP && lane == 0)
                    p.y[rB0 + rr] = p.accum ? __fadd_rn(p.y[rB0 + rr], (float)t) : (float)t;
            }
        }
    }
    if (EP && rd == 0) trace(p, 22);
    }  // rounds
    if constexpr (EP == 2) {
        trace(p, 18);
        ep2_combine(p, ep_e, H, s_own);
        trace(p, 19);
    }
    trace(p, 8);

    // ---- 7. CTA 0 leaves the barrier counter's value for the next launch; EP 2: it waits for
    // every rank's done word of this call (no rank reads its window of the call any more, so
    // call e + 2 may rewrite this parity) and advances the call number
    if (c == 0 && warp == 0) {
        if constexpr (EP == 2) {
            if (lane < p.ep_ranks)
                poll_tagged(p.ep_peer_tdone[p.ep_rank] + (size_t)(ep_e & 1u) * p.ep_ranks + lane, ep_e, p.status);
            __syncwarp();
            if (lane == 0) *p.ep_epoch = ep_e;
        }
        if (lane == 0 && nbar > 0)
            asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p.sync + 3), "r"(sbase + (uint32_t)nbar * G)
                         : "memory");
    }
}

static inline uint32_t al128(uint32_t v) { return (v + 127u) & ~127u; }

// Shared-memory plan for `grid` CTAs. Returns 0, or -1 when the layer does not
// fit (the caller reports KATALI_ERR_UNSUPPORTED_SHAPE).
int moe_plan(MoeParams &p, int grid, int max_smem) {
    if (p.gate_type != T_Q4_K || p.up_type != T_Q4_K) return -1;
    if (p.down_type != T_Q4_K && p.down_type != T_Q6_K) return -1;
    const uint32_t BA = (uint32_t)p.K * p.F / HB;
    const uint32_t maxA = (BA + grid - 1) / grid;
    if (maxA > (uint32_t)MAX_ABLK) return -1;
    p.sa_bytes = maxA * HB * (p.rbg + p.rbu);
    p.sb_off = al128(p.sa_bytes);
    uint32_t rg = 16;  // rows per phase-B group: 16 / gcd(rbd, 16)
    for (uint32_t v = p.rbd; v % 2 == 0 && rg > 1; v /= 2) rg /= 2;
    if (p.H % rg) return -1;
    p.rg = rg;
    const uint32_t Q = (uint32_t)p.H / rg;
    const uint32_t qpc = (Q + grid - 1) / grid;
    p.sb_bytes = (uint32_t)p.K * (rg * qpc * p.rbd + 16);
    p.act_off = al128(p.sb_off + p.sb_bytes);
    const uint32_t act = p.mode == 0 ? 5 * p.H + p.H / 32 * 16 : 4 * (p.H + p.H / 16) + p.H / 32 * 4;
    p.hact_off = al128(p.act_off + act);
    const uint32_t KF = (uint32_t)p.K * p.F;
    const uint32_t hact = p.mode == 0 ? KF + 16 * (uint32_t)p.K + KF / 32 * 16
                                      : 4 * (KF + KF / 16 + 4 * (uint32_t)p.K) + KF / 32 * 4;
    p.misc_off = al128(p.hact_off + hact);
    const uint32_t misc = 24 * (((uint32_t)p.n_experts + 1) & ~1u) + 8 * BAR_SLOTS +
                          8 * MOE_MAX_K + 4 * MAX_ABLK * HB + MAX_ABLK * REC_BYTES +
                          4 * (uint32_t)p.n_experts + 12 * MOE_EP_MAX_PAIRS + 16 + 8 * MOE_EP_MAX_SLOTS + 16;
    p.sdot_off = al128(p.misc_off + misc);
    p.smem_bytes = al128(p.sdot_off + 4 * (uint32_t)p.K * rg * qpc);
    // Decoded down rows (Q6_K, both activation modes): reuse the phase-A staging area
    // when it is large enough (phase A is finished by then), else append.
    p.dec_off = 0;
    p.dec_enabled = 0;
    p.dec_bytes = 0;
    p.dec_row_bytes = (uint32_t)((p.F + p.F / 16 + 4 * (p.F / 256) + 15) & ~15);
    if (p.down_type == T_Q6_K) {
        const uint32_t need = (uint32_t)p.K * (rg * qpc * p.dec_row_bytes + 16);
        p.dec_bytes = need;
        if (need <= p.sa_bytes) {
            p.dec_off = 0;  // the phase-A staging area
            p.dec_enabled = 1;
        } else if (al128(p.smem_bytes) + need <= (uint32_t)max_smem) {
            p.dec_off = al128(p.smem_bytes);
            p.smem_bytes = al128(p.dec_off + need);
            p.dec_enabled = 1;
        }
    }
    return p.smem_bytes <= (uint32_t)max_smem ? 0 : -1;
}

int moe_plan_dec_apart(MoeParams &p, int max_smem) {
    if (!p.dec_enabled || p.dec_off != 0) return p.dec_enabled && p.dec_off != 0;
    if (al128(p.smem_bytes) + p.dec_bytes > (uint32_t)max_smem) return 0;
    p.dec_off = al128(p.smem_bytes);
    p.smem_bytes = al128(p.dec_off + p.dec_bytes);
    return 1;
}

template <int MODE, uint32_t DT, int SHAPE, int EP = 0, int RT = 0>
static cudaError_t launch_t(MoeParams &p, int grid, cudaStream_t st) {
    // The shared-memory limit is raised once per device and size (an eager call precedes
    // any capture on that device).
    static size_t set_bytes[KQ_MAX_DEVICES];
    {
        cudaError_t e = ensure_smem_limit(moe_kernel<MODE, DT, SHAPE, EP, RT>, p.smem_bytes, set_bytes);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(MOE_THREADS);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = p.route_only ? 0 : 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    // A programmatic launch when asked for and accepted: the first such launch on a device
    // (always an eager one, before any graph capture) that the runtime refuses switches it
    // off for that device.
    static int pdl_refused[KQ_MAX_DEVICES];
    const int dev = current_device();
    const bool dev_ok = dev < 0 || dev >= KQ_MAX_DEVICES || !pdl_refused[dev];
    const bool pdl = p.pdl && dev_ok && !EP && !p.route_only;
    cfg.numAttrs = pdl ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, moe_kernel<MODE, DT, SHAPE, EP, RT>, p);
    if (pdl && (e == cudaErrorInvalidValue || e == cudaErrorNotSupported)) {
        cudaGetLastError();
        if (dev >= 0 && dev < KQ_MAX_DEVICES) pdl_refused[dev] = 1;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, moe_kernel<MODE, DT, SHAPE, EP, RT>, p);
    }
    return e;
}

cudaError_t launch_moe(MoeParams &p, int grid, cudaStream_t st) {
    const bool c2 = p.H == 2048 && p.F == 512 && p.K == 8 && p.gate_type == T_Q4_K &&
                    p.up_type == T_Q4_K && p.down_type == T_Q6_K;
    if (p.rt_w) {  // the router folded into the launch (a decoder's MoE block)
        if (p.mode == 0) {
            if (c2) return launch_t<0, T_Q6_K, 1, 0, 1>(p, grid, st);
            return p.down_type == T_Q6_K ? launch_t<0, T_Q6_K, 0, 0, 1>(p, grid, st)
                                         : launch_t<0, T_Q4_K, 0, 0, 1>(p, grid, st);
        }
        return p.down_type == T_Q6_K ? launch_t<1, T_Q6_K, 0, 0, 1>(p, grid, st)
                                     : launch_t<1, T_Q4_K, 0, 0, 1>(p, grid, st);
    }
    if (p.mode == 0) {
        if (c2) return launch_t<0, T_Q6_K, 1>(p, grid, st);
        return p.down_type == T_Q6_K ? launch_t<0, T_Q6_K, 0>(p, grid, st)
                                     : launch_t<0, T_Q4_K, 0>(p, grid, st);
    }
    return p.down_type == T_Q6_K ? launch_t<1, T_Q6_K, 0>(p, grid, st)
                                 : launch_t<1, T_Q4_K, 0>(p, grid, st);
}

cudaError_t launch_moe_ep(MoeParams &p, int grid, cudaStream_t st) {
    if (p.mode != 0 || p.down_type != T_Q6_K || !p.dec_enabled || p.ep_slots > MOE_EP_MAX_SLOTS)
        return cudaErrorInvalidValue;
    const bool c2 = p.H == 2048 && p.F == 512 && p.K == 8 && p.gate_type == T_Q4_K &&
                    p.up_type == T_Q4_K;
    return c2 ? launch_t<0, T_Q6_K, 1, 1>(p, grid, st) : launch_t<0, T_Q6_K, 0, 1>(p, grid, st);
}

cudaError_t launch_moe_ep_layer(MoeParams &p, int grid, cudaStream_t st) {
    if (p.mode != 0 || p.down_type != T_Q6_K || !p.dec_enabled ||
        p.ep_ranks * p.ep_tmax > MOE_EP_MAX_SLOTS || p.ep_tokens > p.ep_tmax)
        return cudaErrorInvalidValue;
    const bool c2 = p.H == 2048 && p.F == 512 && p.K == 8 && p.gate_type == T_Q4_K &&
                    p.up_type == T_Q4_K;
    return c2 ? launch_t<0, T_Q6_K, 1, 2>(p, grid, st) : launch_t<0, T_Q6_K, 0, 2>(p, grid, st);
}

}  // namespace kq
