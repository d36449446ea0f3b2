// kq_gemv.cu — dense quantized GEMV, activation quantiser and block encoders.
//
// GEMV (batch 1, HBM-bound): the matrix rows are streamed in their native GGUF
// layout into a ring of shared-memory stages by cp.async.bulk (TMA, no
// multicast) issued from one producer warp; consumer warps compute one row each
// (a lane owns a fixed 64-element chunk of a Q4_K block or a 16-element group of
// a Q6_K block) and reduce across the warp. Up to 8 projections that share x
// and cols are tiled into one launch (katali_cuda_matvec_multi).
#include "kq_device.cuh"
#include "kq_launch.h"

namespace kq {

// Consumer warps per CTA (+ one producer warp): 8 for launches that stream less than
// GEMV_BIG_BYTES of weights, 12 above (more rows in flight per SM for the long streams;
// the short ones run as programmatic dependents inside decode steps, where fewer, lighter
// CTAs overlap the previous kernel better).
constexpr int GEMV_CW_SMALL = 8, GEMV_CW_BIG = 12;
constexpr uint64_t GEMV_BIG_BYTES = 16ull << 20;

__device__ __forceinline__ void gemv_tile(const GemvParams &p, uint32_t t, int &job,
                                          uint64_t &r0, uint32_t &nrows) {
    job = 0;
    while (job + 1 < p.njobs && t >= p.job[job + 1].tile0) ++job;
    const GemvJob &J = p.job[job];
    r0 = (uint64_t)(t - J.tile0) * J.tr;
    const uint64_t rem = J.rows - r0;
    nrows = (uint32_t)(rem < J.tr ? rem : J.tr);
}

template <int MODE, int GEMV_CW>
__global__ void __launch_bounds__((GEMV_CW + 1) * 32)
    gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *stages = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.act_off - 16 * p.nstages);
    uint64_t *empty = full + p.nstages;
    const int cols = (int)p.cols;
    pdl_trigger();

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.nstages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GEMV_CW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == GEMV_CW) {
        // Producer: stream this CTA's tiles through the ring.
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            uint32_t i = 0;
            for (uint32_t t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++i) {
                const int s = (int)(i % p.nstages);
                if (i >= (uint32_t)p.nstages &&
                    !mbar_wait(&empty[s], ((i / p.nstages) - 1) & 1)) {
                    *p.status |= ERR_TIMEOUT_TMA;
                    break;
                }
                int job;
                uint64_t r0;
                uint32_t nrows;
                gemv_tile(p, t, job, r0, nrows);
                const GemvJob &J = p.job[job];
                const uint32_t bytes = nrows * J.rb;
                if (p.use_tma && (bytes & 15u) == 0) {
                    mbar_arrive_expect_tx(&full[s], bytes);
                    bulk_g2s_hint(stages + (size_t)s * p.stage_bytes, J.w + r0 * J.rb, bytes, &full[s], pol);
                } else {
                    mbar_arrive(&full[s]);  // consumers read this tile from global
                }
            }
        }
        return;
    }

    // Consumers: stage the activation vector once, bank-spread (16 bytes of padding
    // after every 64 elements) so the 32 lanes' units fall on distinct banks. Under a
    // programmatic launch the producer above streams weights (constant) while the
    // previous kernel finishes; x (and y, when accumulating) only after pdl_wait().
    pdl_wait();
    uint8_t *act = smem + p.act_off;
    ActQ8 a;
    const float *xf = nullptr, *xs = nullptr;
    const int nblk = cols / 32;
    float inv = 1.0f;
    if (MODE != 1 && p.norm_w) {  // RMSNorm prologue: every CTA computes the same sum
        double ss = 0.0;
        for (int i = threadIdx.x; i < cols; i += GEMV_CW * 32) ss += (double)p.x[i] * (double)p.x[i];
        ss = warp_sum_d(ss);
        double *red = reinterpret_cast<double *>(act);
        if (lane == 0) red[warp] = ss;
        asm volatile("bar.sync 1, %0;" ::"r"(GEMV_CW * 32));
        ss = 0.0;
        for (int w = 0; w < GEMV_CW; ++w) ss += red[w];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(ss / (double)cols), p.norm_eps)));
        asm volatile("bar.sync 1, %0;" ::"r"(GEMV_CW * 32));
    }
    auto xval = [&](int i, float v) {
        if (p.x_mul) v = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, kq_expf(-v))), p.x_mul[i]);
        if (p.norm_w) v = __fmul_rn(__fmul_rn(v, inv), p.norm_w[i]);
        return v;
    };
    const bool pro = p.x_mul || p.norm_w;
    if (MODE == 2) {
        float *sx = reinterpret_cast<float *>(act);  // cols + cols/16 floats
        float *sxs = sx + cols + cols / 16;
        for (int i = threadIdx.x; i < cols / 4; i += GEMV_CW * 32) {
            float4 v = reinterpret_cast<const float4 *>(p.x)[i];
            if (pro) {
                v.x = xval(4 * i, v.x);
                v.y = xval(4 * i + 1, v.y);
                v.z = xval(4 * i + 2, v.z);
                v.w = xval(4 * i + 3, v.w);
            }
            reinterpret_cast<float4 *>(sx + fpos(1, 4 * i))[0] = v;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(GEMV_CW * 32));
        for (int gb = warp; gb < nblk; gb += GEMV_CW) {
            const float v = warp_sum_f(sx[fpos(1, 32 * gb + lane)]);
            if (lane == 0) sxs[gb] = v;
        }
        xf = sx;
        xs = sxs;
    } else {
        int8_t *q = reinterpret_cast<int8_t *>(act);  // cols + cols/4 bytes
        float *d = reinterpret_cast<float *>(act + cols + cols / 4);
        int *s32 = reinterpret_cast<int *>(d + nblk);
        int *s16 = s32 + nblk;
        // Four independent blocks per warp per round so their reductions overlap.
        for (int g0 = warp; g0 < nblk; g0 += 4 * GEMV_CW) {
            float v[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int gb = g0 + t * GEMV_CW;
                v[t] = 0.0f;
                if (gb < nblk) {
                    if (MODE == 0) v[t] = pro ? xval(32 * gb + lane, p.x[32 * gb + lane]) : p.x[32 * gb + lane];
                    else v[t] = (float)(int8_t)p.xq[(size_t)Q81_BYTES * gb + 4 + lane];
                }
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int gb = g0 + t * GEMV_CW;
                if (gb >= nblk) break;
                int8_t *qb = q + 32 * gb + 16 * (gb >> 1);
                if (MODE == 0) {
                    quant_block_q8(v[t], lane, qb, d + gb, s32 + gb, s16 + 2 * gb, nullptr);
                } else {
                    const uint8_t *blk = p.xq + (size_t)Q81_BYTES * gb;
                    const int qi = (int)v[t];
                    qb[lane] = (int8_t)qi;
                    const int sum = __reduce_add_sync(KQ_FULL, qi);
                    const int lo = __reduce_add_sync(KQ_FULL, lane < 16 ? qi : 0);
                    if (lane == 0) {
                        d[gb] = h2f((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
                        s32[gb] = sum;
                        s16[2 * gb] = lo;
                        s16[2 * gb + 1] = sum - lo;
                    }
                }
            }
        }
        a = ActQ8{q, d, s32, s16, 1};
    }
    asm volatile("bar.sync 1, %0;" ::"r"(GEMV_CW * 32));

    uint32_t i = 0, g = 0;
    for (uint32_t t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++i) {
        const int s = (int)(i % p.nstages);
        if (!mbar_wait_warp(&full[s], (i / p.nstages) & 1)) {
            if (lane == 0) *p.status |= ERR_TIMEOUT_TMA;
            return;
        }
        int job;
        uint64_t r0;
        uint32_t nrows;
        gemv_tile(p, t, job, r0, nrows);
        const GemvJob &J = p.job[job];
        const bool in_smem = p.use_tma && ((nrows * J.rb) & 15u) == 0;
        const uint8_t *base = in_smem ? stages + (size_t)s * p.stage_bytes : J.w + r0 * J.rb;
        const int nb = cols / 256;
        for (uint32_t r = (uint32_t)((warp - (int)(g % GEMV_CW) + GEMV_CW) % GEMV_CW); r < nrows;
             r += GEMV_CW) {
            const uint8_t *row = base + (size_t)r * J.rb;
            double part;
            if (MODE == 2)
                part = J.type == T_Q4_K ? q4k_f32_partial(row, nb, xf, xs, lane, 1)
                                        : q6k_f32_partial(row, nb, xf, lane, 1);
            else
                part = J.type == T_Q4_K ? q4k_q8_partial(row, nb, a, lane)
                                        : q6k_q8_partial(row, nb, a, lane);
            part = warp_sum_d(part);
            if (lane == 0) J.y[r0 + r] = J.accum ? __fadd_rn(J.y[r0 + r], (float)part) : (float)part;
        }
        g += nrows;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}


// ---------------------------------------------------------------------------
// q8_1 quantiser: one warp per 32-element block.
// ---------------------------------------------------------------------------
__global__ void quantize_q8_1_kernel(const float *x, uint64_t nblocks, uint8_t *out) {
    const uint64_t wg = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wg >= nblocks) return;
    quant_block_q8(x[32 * wg + lane], lane, nullptr, nullptr, nullptr, nullptr,
                   out + Q81_BYTES * wg);
}

// ---------------------------------------------------------------------------
// Encoders (one thread per 256-element super-block). Same operations, in the
// same order, as kqo_quantize_q4_K / kqo_quantize_q6_K of the CPU restatement,
// so both produce identical bytes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__global__ void encode_q4k_kernel(const float *x, uint64_t nblk, uint8_t *out) {
    const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    const float *xb = x + b * 256;
    uint8_t *blk = out + b * Q4K_BYTES;
    float s[8], M[8], smax = 0.0f, Mmax = 0.0f;
    for (int j = 0; j < 8; j++) {
        float lo = xb[32 * j], hi = xb[32 * j];
        for (int i = 1; i < 32; i++) {
            const float v = xb[32 * j + i];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        M[j] = lo < 0.0f ? -lo : 0.0f;
        s[j] = __fdiv_rn(__fadd_rn(hi, M[j]), 15.0f);
        if (s[j] > smax) smax = s[j];
        if (M[j] > Mmax) Mmax = M[j];
    }
    const uint16_t dh = f2h(__fdiv_rn(smax, 63.0f));
    const uint16_t mh = f2h(__fdiv_rn(Mmax, 63.0f));
    const float d = h2f(dh), dmin = h2f(mh);
    int sc[8], mm[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = d > 0.0f ? clampi((int)roundf(__fdiv_rn(s[j], d)), 0, 63) : 0;
        mm[j] = dmin > 0.0f ? clampi((int)roundf(__fdiv_rn(M[j], dmin)), 0, 63) : 0;
    }
    uint8_t hdr[16];
    hdr[0] = (uint8_t)(dh & 0xFF);
    hdr[1] = (uint8_t)(dh >> 8);
    hdr[2] = (uint8_t)(mh & 0xFF);
    hdr[3] = (uint8_t)(mh >> 8);
    for (int j = 0; j < 4; j++) {
        hdr[4 + j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        hdr[8 + j] = (uint8_t)(mm[j] | ((mm[j + 4] >> 4) << 6));
        hdr[12 + j] = (uint8_t)((sc[j + 4] & 0x0F) | ((mm[j + 4] & 0x0F) << 4));
    }
    for (int i = 0; i < 16; i++) blk[i] = hdr[i];
    for (int c = 0; c < 4; c++) {
        const float ds0 = __fmul_rn(d, (float)sc[2 * c]), dm0 = __fmul_rn(dmin, (float)mm[2 * c]);
        const float ds1 = __fmul_rn(d, (float)sc[2 * c + 1]),
                    dm1 = __fmul_rn(dmin, (float)mm[2 * c + 1]);
        for (int i = 0; i < 32; i++) {
            int q0 = 0, q1 = 0;
            if (ds0 > 0.0f)
                q0 = clampi((int)roundf(__fdiv_rn(__fadd_rn(xb[64 * c + i], dm0), ds0)), 0, 15);
            if (ds1 > 0.0f)
                q1 = clampi((int)roundf(__fdiv_rn(__fadd_rn(xb[64 * c + 32 + i], dm1), ds1)), 0,
                            15);
            blk[16 + 32 * c + i] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

__global__ void encode_q6k_kernel(const float *x, uint64_t nblk, uint8_t *out) {
    const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    const float *xb = x + b * 256;
    uint8_t *blk = out + b * Q6K_BYTES;
    float s[16], smax = 0.0f;
    for (int k = 0; k < 16; k++) {
        float amax = 0.0f;
        for (int i = 0; i < 16; i++) {
            const float a = fabsf(xb[16 * k + i]);
            if (a > amax) amax = a;
        }
        s[k] = __fdiv_rn(amax, 31.0f);
        if (s[k] > smax) smax = s[k];
    }
    const uint16_t dh = f2h(__fdiv_rn(smax, 127.0f));
    const float d = h2f(dh);
    uint8_t ql[128], qh[64];
    for (int i = 0; i < 128; i++) ql[i] = 0;
    for (int i = 0; i < 64; i++) qh[i] = 0;
    for (int k = 0; k < 16; k++) {
        const int sc = d > 0.0f ? clampi((int)roundf(__fdiv_rn(s[k], d)), -128, 127) : 0;
        blk[192 + k] = (uint8_t)(int8_t)sc;
        const float ds = __fmul_rn(d, (float)sc);
        for (int i = 0; i < 16; i++) {
            const int e = 16 * k + i;
            int q = 32;
            if (ds != 0.0f) q = clampi((int)roundf(__fdiv_rn(xb[e], ds)), -32, 31) + 32;
            const int h = e >> 7, quarter = (e >> 5) & 3, l = e & 31;
            const int qi = 64 * h + 32 * (quarter & 1) + l;
            if (quarter >= 2) ql[qi] = (uint8_t)(ql[qi] | ((q & 0x0F) << 4));
            else ql[qi] = (uint8_t)(ql[qi] | (q & 0x0F));
            qh[32 * h + l] = (uint8_t)(qh[32 * h + l] | (((q >> 4) & 3) << (2 * quarter)));
        }
    }
    for (int i = 0; i < 128; i++) blk[i] = ql[i];
    for (int i = 0; i < 64; i++) blk[128 + i] = qh[i];
    blk[208] = (uint8_t)(dh & 0xFF);
    blk[209] = (uint8_t)(dh >> 8);
}

// ---------------------------------------------------------------------------
// Check kernel: integer in-block sums of every row (one warp per row, global
// loads, no staging). Lane mapping identical to the GEMV kernels.
// ---------------------------------------------------------------------------
__global__ void row_isums_kernel(uint32_t type, const uint8_t *w, uint64_t rows, int cols,
                                 uint32_t rb, const uint8_t *xq, int32_t *isum, int32_t *xsum) {
    const uint64_t r = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const uint8_t *row = w + r * rb;
    const int nb = cols / 256;
    if (type == T_Q4_K) {
        const int c = lane & 3;
        for (int b = lane >> 2; b < nb; b += 8) {
            const uint8_t *qs = row + Q4K_BYTES * b + 16 + 32 * c;
            for (int half = 0; half < 2; half++) {
                const int g = 8 * b + 2 * c + half;
                const int8_t *qx = reinterpret_cast<const int8_t *>(xq + (size_t)Q81_BYTES * g + 4);
                int s = 0, sx = 0;
                for (int i = 0; i < 32; i++) {
                    const int q = half ? (qs[i] >> 4) : (qs[i] & 15);
                    s += q * qx[i];
                    sx += qx[i];
                }
                isum[r * (cols / 32) + g] = s;
                if (xsum) xsum[r * (cols / 32) + g] = sx;
            }
        }
    } else {
        const int k = lane & 15, h = k >> 3, kk = k & 7, qq = kk >> 1, sub = kk & 1;
        for (int b = lane >> 4; b < nb; b += 2) {
            const uint8_t *blk = row + Q6K_BYTES * b;
            const int8_t *qx = reinterpret_cast<const int8_t *>(
                                   xq + (size_t)Q81_BYTES * (8 * b + (k >> 1)) + 4) +
                               16 * (k & 1);
            int s = 0, sx = 0;
            for (int i = 0; i < 16; i++) {
                const uint8_t l = blk[64 * h + 32 * (qq & 1) + 16 * sub + i];
                const uint8_t hb = blk[128 + 32 * h + 16 * sub + i];
                const int lo = qq >= 2 ? (l >> 4) : (l & 15);
                const int q = lo | (((hb >> (2 * qq)) & 3) << 4);
                s += (q - 32) * qx[i];
                sx += qx[i];
            }
            isum[r * (cols / 16) + 16 * b + k] = s;
            if (xsum) xsum[r * (cols / 16) + 16 * b + k] = sx;
        }
    }
}

}  // namespace kq

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
namespace kq {

static int num_sms() { return device_sms(); }

cudaError_t launch_gemv(GemvParams &p, int mode, cudaStream_t st) {
    // Rows per tile: ~16 KB stages, ~48 KB for launches that stream GEMV_BIG_BYTES or more
    // (every consumer warp passes through every tile of its CTA, so fewer, larger tiles cost
    // less per row: 2.9 -> 3.6 TB/s on a 113 MB Q4_K matrix with q8_1 activations); Q6_K
    // tiles in row multiples that keep every stage start 16-byte aligned.
    uint64_t bytes = 0;
    for (int j = 0; j < p.njobs; ++j) bytes += p.job[j].rows * p.job[j].rb;
    // A programmatic dependent inside a decode step with rows of 4096 columns or more streams
    // its tiles as a big launch from 8 MB (C4's q/k/v and output projections: +6 % tokens/s;
    // C5's 2048-column projections were 3 % slower that way).
    const bool big = bytes >= (p.pdl && p.cols >= 4096 ? (8ull << 20) : GEMV_BIG_BYTES);
    const uint32_t cols = p.cols;
    // activation area (bank-spread): fp32 x + per-32 sums, or q8 values + d + 32-sums + 16-sums
    const uint32_t act_bytes =
        mode == 2 ? (cols + cols / 16) * 4 + cols / 32 * 4 : cols + cols / 4 + cols / 32 * 16;
    // Big launches run two CTAs per SM with two-stage rings: the stages shrink for wide rows
    // (a long activation area) so that both CTAs still fit the SM's 228 KB.
    uint32_t tile_bytes = 16384u;
    if (big) {
        const uint32_t budget = 233472u / 2u - 1024u - act_bytes - 512u;  // per CTA
        tile_bytes = budget / 2u - 32u;
        if (tile_bytes > 49152u) tile_bytes = 49152u;
        if (tile_bytes < 16384u) tile_bytes = 16384u;
    }
    uint32_t stage = 0;
    uint32_t tiles = 0;
    for (int j = 0; j < p.njobs; ++j) {
        GemvJob &J = p.job[j];
        uint32_t m = 16;
        for (uint32_t g = J.rb; g % 2 == 0 && m > 1; g /= 2) m /= 2;  // 16 / gcd(rb, 16)
        uint32_t tr = J.rb >= tile_bytes ? 1 : tile_bytes / J.rb;
        tr = tr < m ? m : tr / m * m;
        J.tr = tr;
        J.tile0 = tiles;
        tiles += (uint32_t)((J.rows + tr - 1) / tr);
        const uint32_t sb = (tr * J.rb + 15u) & ~15u;
        if (sb > stage) stage = sb;
    }
    p.total_tiles = tiles;
    if (tiles == 0) return cudaSuccess;
    // A standalone small launch (not a programmatic dependent inside a decode step) runs up
    // to 3 CTAs per SM with 64 KB rings; the others 2 CTAs per SM with 96 KB rings.
    const bool three = !p.pdl && !big;
    p.stage_bytes = stage + 16;
    p.use_tma = 1;
    int ns = (int)((three ? 65536 : (big ? 2 * p.stage_bytes : 98304)) / p.stage_bytes);
    if (ns > 8) ns = 8;
    if (ns < 2) {
        ns = 2;
        if (2 * p.stage_bytes > 160 * 1024) {  // rows too long to stage: read from global
            p.use_tma = 0;
            p.stage_bytes = 16;
        }
    }
    p.nstages = ns;
    p.act_off = ((uint32_t)ns * p.stage_bytes + 16 * ns + 127u) & ~127u;
    const size_t smem = p.act_off + act_bytes;
    const int threads = ((big ? GEMV_CW_BIG : GEMV_CW_SMALL) + 1) * 32;
    void (*const fns[2][3])(GemvParams) = {
        {gemv_kernel<0, GEMV_CW_SMALL>, gemv_kernel<1, GEMV_CW_SMALL>, gemv_kernel<2, GEMV_CW_SMALL>},
        {gemv_kernel<0, GEMV_CW_BIG>, gemv_kernel<1, GEMV_CW_BIG>, gemv_kernel<2, GEMV_CW_BIG>}};
    void (*fn)(GemvParams) = fns[big][mode];
    static size_t set_bytes[2][3][KQ_MAX_DEVICES];
    {
        cudaError_t e = ensure_smem_limit(fn, smem, set_bytes[big][mode]);
        if (e != cudaSuccess) return e;
    }
    int per = 2;
    if (three && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, fn, threads, smem) != cudaSuccess)
        per = 2;
    if (per < 1) per = 1;
    if (per > 3) per = 3;
    int grid = per * num_sms();
    if ((uint32_t)grid > tiles) grid = (int)tiles;
    if (!p.pdl) {
        fn<<<grid, threads, smem, st>>>(p);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, p);
}

cudaError_t launch_quantize_q8_1(const float *x, uint64_t n, void *out, cudaStream_t st) {
    const uint64_t nb = n / 32;
    const int threads = 256;
    const uint64_t blocks = (nb * 32 + threads - 1) / threads;
    quantize_q8_1_kernel<<<(unsigned)blocks, threads, 0, st>>>(x, nb, (uint8_t *)out);
    return cudaGetLastError();
}

cudaError_t launch_encode(uint32_t type, const float *x, uint64_t n, void *out, cudaStream_t st) {
    if (type == T_Q8_1) return launch_quantize_q8_1(x, n, out, st);
    const uint64_t nblk = n / 256;
    const int threads = 128;
    const unsigned blocks = (unsigned)((nblk + threads - 1) / threads);
    if (type == T_Q4_K) encode_q4k_kernel<<<blocks, threads, 0, st>>>(x, nblk, (uint8_t *)out);
    else encode_q6k_kernel<<<blocks, threads, 0, st>>>(x, nblk, (uint8_t *)out);
    return cudaGetLastError();
}

cudaError_t launch_row_isums(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                             uint32_t rb, const void *xq, int32_t *isum, int32_t *xsum,
                             cudaStream_t st) {
    const int threads = 256;
    const unsigned blocks = (unsigned)((rows * 32 + threads - 1) / threads);
    row_isums_kernel<<<blocks, threads, 0, st>>>(type, (const uint8_t *)w, rows, (int)cols, rb,
                                                 (const uint8_t *)xq, isum, xsum);
    return cudaGetLastError();
}

}  // namespace kq
