// kq_moe_tc.cu — gate/up of the ragged-batch MoE on the 5th-generation tensor cores
// (tcgen05.mma kind::i8) for expert groups with many tokens.
//
// For one selected expert with n >= p.tc_min tokens, gate and up are dense
// [F x H] x [H x n] products of int4 weights (Q4_K nibbles 0..15) and int8
// activations (q8_1), with a scale per 32-element block on each side. Each
// 32-wide K chunk is exactly one Q4_K sub-block and one q8_1 block, so one
// M=128 x N=32 x K=32 MMA per chunk gives the exact integer block sums isum for
// 128 rows x 32 tokens; the CUDA cores then apply
//   acc += (d*sc) * dx * isum - (dmin*m) * (dx * xsum)
// in fp32 per block (the DP4A kernels use exact double terms; this path rounds
// each block term to fp32, within the layer tolerance).
//
// CTA = (group, 128-row tile), 4 warps; per token tile of 32 and per super-block
// of 256 columns: cp.async the 128 raw gate and up rows (144 B each) -> unpack to
// int8 in the canonical no-swizzle K-major layout (core matrices of 8 rows x
// 16 B: LBO 128 B between the two K halves, SBO 256 B between 8-row groups) with
// the per-row block scales -> stage the tokens' q8_1 values the same way ->
// thread 0 issues 16 MMAs (8 chunks x gate/up) into separate TMEM columns and
// commits to an mbarrier -> each warp reads its 32 TMEM lanes (= rows) and
// accumulates. TMEM: 16 chunks x 32 columns = 512 columns, allocated once per CTA.
#include <cuda_runtime.h>

#include "kq_device.cuh"
#include "kq_launch.h"

namespace kq {

namespace {

constexpr int TC_THREADS = 128;
constexpr int TC_NT = 32;  // tokens per tile (MMA N)
constexpr int TC_ROWS = 128;  // rows per tile (MMA M)
constexpr int TC_COLS = 512;  // TMEM columns: 2 matrices x 8 chunks x 32
constexpr uint32_t A_CHUNK = TC_ROWS * 32;  // 4096 B: one 128 x 32 int8 operand
constexpr uint32_t B_CHUNK = TC_NT * 32;    // 1024 B

// Shared-memory plan (bytes from the dynamic base, 1024-aligned).
constexpr uint32_t OFF_AG = 0;                        // 8 chunks of gate A
constexpr uint32_t OFF_AU = OFF_AG + 8 * A_CHUNK;     // 8 chunks of up A
constexpr uint32_t OFF_B = OFF_AU + 8 * A_CHUNK;      // 8 chunks of B
constexpr uint32_t OFF_RAW = OFF_B + 8 * B_CHUNK;     // raw rows: 128 gate + 128 up, 144 B each
constexpr uint32_t OFF_SC = OFF_RAW + 2 * TC_ROWS * 144;  // S_g, M_g, S_u, M_u: [8][128] floats each
constexpr uint32_t OFF_TOK = OFF_SC + 4 * 8 * TC_ROWS * 4;  // DX[32][8], XS[32][8] floats
constexpr uint32_t TC_SMEM = OFF_TOK + 2 * TC_NT * 8 * 4;

__device__ __forceinline__ uint64_t umma_sdesc(uint32_t saddr) {
    // start address >> 4, LBO 128 B, SBO 256 B, version 1, no swizzle
    return ((uint64_t)((saddr >> 4) & 0x3FFFu)) | ((uint64_t)(128u >> 4) << 16) |
           ((uint64_t)(256u >> 4) << 32) | (1ull << 46);
}
// kind::i8 instruction descriptor: s32 accumulator, signed A and B, K-major,
// N = TC_NT, M = TC_ROWS.
constexpr uint32_t TC_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_NT >> 3) << 17) |
                              ((uint32_t)(TC_ROWS >> 4) << 24);

__device__ __forceinline__ void umma_i8(uint32_t tmem, uint64_t da, uint64_t db) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
        "l"(da), "l"(db), "r"(TC_IDESC), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(addr));
}

// Canonical offset of the 16-byte piece (row r, K half h) inside one operand chunk.
__device__ __forceinline__ uint32_t canon(int r, int h) { return (r >> 3) * 256 + h * 128 + (r & 7) * 16; }

}  // namespace

__global__ void __launch_bounds__(TC_THREADS, 1) moe_batch_gateup_tc(MoeBatchParams p) {
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t taddr_s;
    const int ntile = p.F / TC_ROWS;
    const int g = blockIdx.x / ntile, rt = blockIdx.x % ntile;
    if (g >= *p.n_groups) return;
    const int p0 = p.grp_off[g], p1 = p.grp_off[g + 1];
    if (p1 - p0 < p.tc_min) return;  // small groups: the DP4A kernel
    const int e = p.grp_expert[g];
    const uint8_t *G = p.experts[3 * e], *U = p.experts[3 * e + 1];
    if (!G || !U) {
        if (threadIdx.x == 0 && p.status) atomicOr((uint32_t *)p.status, KQ_STATUS_NOT_RESIDENT);
        return;
    }
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = tid;  // the row this thread unpacks and accumulates (TMEM lane)
    const int j0 = rt * TC_ROWS, K = p.K, H = p.H, nb = H / 256;
    float *S_g = reinterpret_cast<float *>(sm + OFF_SC), *M_g = S_g + 8 * TC_ROWS;
    float *S_u = M_g + 8 * TC_ROWS, *M_u = S_u + 8 * TC_ROWS;
    float *DX = reinterpret_cast<float *>(sm + OFF_TOK), *XS = DX + TC_NT * 8;

    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&taddr_s)),
                     "r"(TC_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t taddr = taddr_s;
    uint32_t phase = 0;
    bool ok = true;

    for (int t0 = p0; t0 < p1; t0 += TC_NT) {
        const int nt = min(TC_NT, p1 - t0);
        float ag[TC_NT], au[TC_NT];
#pragma unroll
        for (int t = 0; t < TC_NT; ++t) ag[t] = au[t] = 0.0f;
        for (int b = 0; b < nb; ++b) {
            // raw rows of super-block b: 128 gate + 128 up rows x 144 B (9 x 16 B each)
            uint8_t *raw = sm + OFF_RAW;
            for (int i = tid; i < 2 * TC_ROWS * 9; i += TC_THREADS) {
                const int m = i / (TC_ROWS * 9), rr = (i / 9) % TC_ROWS, q = i % 9;
                const uint8_t *src = (m ? U + (size_t)(j0 + rr) * p.rbu : G + (size_t)(j0 + rr) * p.rbg) +
                                     (size_t)b * Q4K_BYTES + 16 * q;
                cp_async16(raw + (size_t)(m * TC_ROWS + rr) * 144 + 16 * q, src);
            }
            // B: the tile's tokens' q8_1 values of the 8 blocks of super-block b
            for (int i = tid; i < TC_NT * 8 * 2; i += TC_THREADS) {
                const int t = i / 16, c = (i / 2) % 8, h = i % 2;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (t < nt) {
                    const int tok = p.pair_src[t0 + t] / K;
                    v = *reinterpret_cast<const uint4 *>(p.xq + (size_t)tok * H + 256 * b + 32 * c + 16 * h);
                }
                *reinterpret_cast<uint4 *>(sm + OFF_B + c * B_CHUNK + canon(t, h)) = v;
            }
            for (int i = tid; i < TC_NT * 8; i += TC_THREADS) {
                const int t = i / 8, c = i % 8;
                float dx = 0.0f, xs = 0.0f;
                if (t < nt) {
                    const int tok = p.pair_src[t0 + t] / K, blk = 8 * b + c;
                    dx = p.xd[(size_t)tok * (H / 32) + blk];
                    xs = __fmul_rn(dx, (float)p.xs32[(size_t)tok * (H / 32) + blk]);
                }
                DX[t * 8 + c] = dx;
                XS[t * 8 + c] = xs;
            }
            cp_async_wait_all();
            __syncthreads();
            // unpack row r of gate and up: nibbles -> int8 chunks, block scales
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const uint8_t *blk = raw + (size_t)(m * TC_ROWS + r) * 144;
                const uint4 h = *reinterpret_cast<const uint4 *>(blk);
                uint8_t *A = sm + (m ? OFF_AU : OFF_AG);
                float *S = m ? S_u : S_g, *M = m ? M_u : M_g;
                const float d = h2f(h.x), dmin = h2f(h.x >> 16);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint4 w0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * c);
                    const uint4 w1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * c);
                    const uint32_t MK = 0x0F0F0F0Fu;
                    *reinterpret_cast<uint4 *>(A + (2 * c) * A_CHUNK + canon(r, 0)) =
                        make_uint4(w0.x & MK, w0.y & MK, w0.z & MK, w0.w & MK);
                    *reinterpret_cast<uint4 *>(A + (2 * c) * A_CHUNK + canon(r, 1)) =
                        make_uint4(w1.x & MK, w1.y & MK, w1.z & MK, w1.w & MK);
                    *reinterpret_cast<uint4 *>(A + (2 * c + 1) * A_CHUNK + canon(r, 0)) =
                        make_uint4((w0.x >> 4) & MK, (w0.y >> 4) & MK, (w0.z >> 4) & MK, (w0.w >> 4) & MK);
                    *reinterpret_cast<uint4 *>(A + (2 * c + 1) * A_CHUNK + canon(r, 1)) =
                        make_uint4((w1.x >> 4) & MK, (w1.y >> 4) & MK, (w1.z >> 4) & MK, (w1.w >> 4) & MK);
                    int sc0, m0, sc1, m1;
                    q4k_scales(h, c, sc0, m0, sc1, m1);
                    S[(2 * c) * TC_ROWS + r] = __fmul_rn(d, (float)sc0);
                    M[(2 * c) * TC_ROWS + r] = __fmul_rn(dmin, (float)m0);
                    S[(2 * c + 1) * TC_ROWS + r] = __fmul_rn(d, (float)sc1);
                    M[(2 * c + 1) * TC_ROWS + r] = __fmul_rn(dmin, (float)m1);
                }
            }
            // make the generic-proxy shared-memory writes visible to the tensor cores
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncthreads();
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (tid == 0) {
                const uint32_t sa_g = smem_u32(sm + OFF_AG), sa_u = smem_u32(sm + OFF_AU);
                const uint32_t sb = smem_u32(sm + OFF_B);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint64_t db = umma_sdesc(sb + c * B_CHUNK);
                    umma_i8(taddr + c * TC_NT, umma_sdesc(sa_g + c * A_CHUNK), db);
                    umma_i8(taddr + 256 + c * TC_NT, umma_sdesc(sa_u + c * A_CHUNK), db);
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&bar))
                             : "memory");
            }
            // bounded wait for this super-block's MMAs; the verdict is the CTA's, not a thread's
            uint32_t done = 0;
            for (uint32_t it = 0; it < SPIN_LIMIT && !done; ++it) {
                done = mbar_try_wait(&bar, phase) ? 1u : 0u;
                if (!done && it > 64) __nanosleep(64);
            }
            phase ^= 1u;
            if (!__syncthreads_and(done)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            // accumulate: this warp's 32 TMEM lanes are rows 32*warp .. +31
            const uint32_t lane_base = taddr + ((uint32_t)(32 * warp) << 16);
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                const float sg = S_g[c * TC_ROWS + r], mg = M_g[c * TC_ROWS + r];
                const float su = S_u[c * TC_ROWS + r], mu = M_u[c * TC_ROWS + r];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t vg[16], vu[16];
                    tmem_ld16(lane_base + c * TC_NT + 16 * half, vg);
                    tmem_ld16(lane_base + 256 + c * TC_NT + 16 * half, vu);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        const int t = 16 * half + q;
                        const float dx = DX[t * 8 + c], xs = XS[t * 8 + c];
                        ag[t] = fmaf(__fmul_rn(sg, dx), (float)(int)vg[q], fmaf(-mg, xs, ag[t]));
                        au[t] = fmaf(__fmul_rn(su, dx), (float)(int)vu[q], fmaf(-mu, xs, au[t]));
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncthreads();  // shared memory and TMEM are reused by the next super-block
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        }
        if (!ok) break;
#pragma unroll
        for (int t = 0; t < TC_NT; ++t)
            if (t < nt) p.h[(size_t)(t0 + t) * p.F + j0 + r] = __fmul_rn(kq_silu(ag[t]), au[t]);
    }
    if (!ok && tid == 0 && p.status) atomicOr((uint32_t *)p.status, 4u);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(TC_COLS));
}

void launch_gateup_tc(MoeBatchParams &p, int max_groups, cudaStream_t st) {
    static size_t set_bytes[KQ_MAX_DEVICES];
    ensure_smem_limit(moe_batch_gateup_tc, TC_SMEM, set_bytes);
    moe_batch_gateup_tc<<<max_groups * (p.F / TC_ROWS), TC_THREADS, TC_SMEM, st>>>(p);
}

}  // namespace kq
