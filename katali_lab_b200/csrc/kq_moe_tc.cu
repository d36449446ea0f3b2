// kq_moe_tc.cu — the ragged-batch MoE's expert groups with many tokens on the
// 5th-generation tensor cores (tcgen05.mma kind::i8): Q4_K gate/up and Q6_K down.
//
// For one selected expert with n >= p.tc_min tokens, gate and up are dense
// [F x H] x [H x n] products of int4 weights (Q4_K nibbles 0..15) and int8
// activations (q8_1), with a scale per 32-element block on each side. Each
// 32-wide K chunk is exactly one Q4_K sub-block and one q8_1 block, so one
// M=128 x N=32 x K=32 MMA per chunk gives the exact integer block sums isum for
// 128 rows x 32 tokens; the CUDA cores then apply
//   acc += (d*sc) * dx * isum - (dmin*m) * (dx * xsum)
// in fp32 per block (the DP4A kernels use exact double terms; this path rounds
// each block term to fp32, within the layer tolerance). The down projection
// (below moe_batch_gateup_tc) keeps exact terms in double.
//
// Gate/up items are (listed group, 128-row tile, matrix): the gate and the up rows
// of a tile are separate CTAs (8 warps, 256 TMEM columns, two CTAs per SM). Warp w
// serves TMEM lanes 32*(w%4)..+31 (the rows of its quadrant) for tokens 0..15 or
// 16..31 of the token tile (w/4). Per token tile of 32 and per super-block b of 256
// columns:
//   * the copies of super-block b+1 (raw rows, 144 B each; the tokens' q8_1 values
//     in the canonical no-swizzle K-major layout of the B operand; their block scales
//     and sums) go out with cp.async into the other half of a double buffer before b
//     is unpacked, so they land while b is computed;
//   * unpack row r (two of its four chunk pairs) to int8 in the canonical no-swizzle
//     K-major layout (core matrices of 8 rows x 16 B: LBO 128 B between the two K
//     halves, SBO 256 B between 8-row groups) with its block scales;
//   * thread 0 issues 8 MMAs (one per chunk) into separate TMEM columns and commits
//     to an mbarrier;
//   * each thread reads its row's 16 tokens (tcgen05.ld) and accumulates.
// The gate item writes its sums into h, the up item into hu; the h quantiser forms
// h = silu(g) * u for the pairs the group kernel flagged. Each token's arithmetic is
// the same sequence of fp32 operations for any warp split.
#include <cuda_runtime.h>

#include "kq_device.cuh"
#include "kq_launch.h"

namespace kq {

namespace {

constexpr int GU_THREADS = 256;    // gate/up kernel: 8 warps, two CTAs per SM
constexpr int TC_NT = 32;  // tokens per tile (MMA N)
constexpr int TC_ROWS = 128;  // rows per tile (MMA M)
constexpr int GU_COLS = 256;  // gate/up TMEM columns: 8 chunks x 32
constexpr uint32_t A_CHUNK = TC_ROWS * 32;  // 4096 B: one 128 x 32 int8 operand
constexpr uint32_t B_CHUNK = TC_NT * 32;    // 1024 B
constexpr uint32_t RAW_BYTES = TC_ROWS * 144;     // one super-block of 128 rows of one matrix
constexpr uint32_t XR_BYTES = 2 * TC_NT * 8 * 4;  // d [32][8] f32, then block sums [32][8] s32

// Gate/up shared-memory plan (bytes from the dynamic base, 1024-aligned).
constexpr uint32_t OFF_A = 0;                             // 8 chunks of A
constexpr uint32_t OFF_B = OFF_A + 8 * A_CHUNK;           // 2 buffers x 8 chunks of B
constexpr uint32_t OFF_RAW = OFF_B + 2 * 8 * B_CHUNK;     // 2 buffers of raw rows
constexpr uint32_t OFF_XR = OFF_RAW + 2 * RAW_BYTES;      // 2 buffers of token scales as copied
constexpr uint32_t OFF_SC = OFF_XR + 2 * XR_BYTES;        // S, M: [8][128] floats each
constexpr uint32_t OFF_DX = OFF_SC + 2 * 8 * TC_ROWS * 4;  // DX[8][32], XS[8][32] floats
constexpr uint32_t OFF_TOK = OFF_DX + 2 * 8 * TC_NT * 4;  // the tile's token indices
constexpr uint32_t TC_SMEM = OFF_TOK + TC_NT * 4;
static_assert(2 * (TC_SMEM + 2048) <= 228 * 1024, "two gate/up CTAs per SM");

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
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most N of this thread's committed cp.async groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_pending() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Canonical offset of the 16-byte piece (row r, K half h) inside one operand chunk.
__device__ __forceinline__ uint32_t canon(int r, int h) { return (r >> 3) * 256 + h * 128 + (r & 7) * 16; }

// 32 bytes of shared memory at a 2-byte aligned address as 8 words: nine aligned word
// loads, funnel-shifted into place.
__device__ __forceinline__ void ld32_unaligned(const uint8_t *src, uint32_t (&out)[8]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(src);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(a & 3) * 8;
    uint32_t x[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) x[i] = w[i];
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = __funnelshift_r(x[i], x[i + 1], sh);
}

// Down projection plan (bytes from the dynamic base): per half of a Q6_K super-block
// (4 chunks of 32), A holds two operands per chunk k: 2k with the chunk's first 16 values
// and zeros in its second K half, 2k + 1 with zeros in its first K half and the last 16
// values (each half has its own 16-element scale). The zero halves are written once per CTA.
constexpr int DN_THREADS = 256;                          // 8 warps
constexpr int DN_COLS = 256;                             // TMEM: 8 operands x 32 columns
constexpr uint32_t OFF_DA = 0;                           // 8 operands of 128 x 32 int8
constexpr uint32_t OFF_DB = OFF_DA + 8 * A_CHUNK;        // 2 buffers x 8 chunks of B
constexpr uint32_t OFF_DXR = OFF_DB + 2 * 8 * B_CHUNK;   // 2 buffers of h block scales [32][8]
constexpr uint32_t OFF_DDX = OFF_DXR + 2 * TC_NT * 8 * 4;  // DX [8][32] as doubles
constexpr uint32_t OFF_DRAW = OFF_DDX + 8 * TC_NT * 8;   // the raw 128-row tile (+16 B of slack)
constexpr uint32_t TC_DOWN_SMEM = OFF_DRAW + TC_DOWN_RAW_MAX + 16;
static_assert(TC_DOWN_SMEM <= 227 * 1024, "shared-memory plan");
static_assert(OFF_DRAW % 16 == 0, "bulk-copy destination");

}  // namespace

__global__ void __launch_bounds__(GU_THREADS, 2) moe_batch_gateup_tc(MoeBatchParams p) {
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t taddr_s;
    // Work items (listed group, 128-row tile, matrix): gate and up of one tile are items
    // 2i and 2i + 1; CTA j takes items j, j + gridDim.x, ...
    const int ntile = p.F / TC_ROWS, items = (int)p.work[2] * ntile * 2;
    if ((int)blockIdx.x >= items) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, th = warp >> 2;  // lane quadrant, token half
    const int r = 32 * quad + lane;  // the row this thread unpacks and accumulates (TMEM lane)
    const int K = p.K, H = p.H, nb = H / 256;
    float *S = reinterpret_cast<float *>(sm + OFF_SC), *M = S + 8 * TC_ROWS;  // [chunk][row]
    float *DX = reinterpret_cast<float *>(sm + OFF_DX), *XS = DX + 8 * TC_NT;  // [chunk][token]
    int *tok = reinterpret_cast<int *>(sm + OFF_TOK);

    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&taddr_s)),
                     "r"(GU_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t taddr = taddr_s;
    uint32_t phase = 0;
    bool ok = true;

    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const int m = it & 1, ti = it >> 1;  // m: 0 gate, 1 up
        const int g = p.tc_groups[ti / ntile], j0 = (ti % ntile) * TC_ROWS;
        const int p0 = p.grp_off[g], p1 = p.grp_off[g + 1];
        if (p.tc_min <= 0 || p1 - p0 < p.tc_min) continue;  // small groups: the DP4A kernel
        const uint8_t *W = p.experts[3 * p.grp_expert[g] + m];
        const size_t rb = m ? p.rbu : p.rbg;
        if (!W) {
            if (tid == 0 && p.status) atomicOr((uint32_t *)p.status, KQ_STATUS_NOT_RESIDENT);
            continue;
        }
        float *out = m ? p.hu : p.h;  // pre-activation sums; the h quantiser forms silu(g) * u
        for (int t0 = p0; t0 < p1 && ok; t0 += TC_NT) {
            const int nt = min(TC_NT, p1 - t0);
            if (tid < nt) tok[tid] = p.pair_src[t0 + tid] / K;
            __syncthreads();
            // The copies of super-block b into buffer buf: raw rows, the B operand (tokens
            // >= nt keep stale values; their columns are never read back) and the tokens'
            // block scales and sums of the 8 blocks.
            auto issue = [&](int b, int buf) {
                uint8_t *raw = sm + OFF_RAW + buf * RAW_BYTES;
                for (int i = tid; i < TC_ROWS * 9; i += GU_THREADS) {
                    const int rr = i / 9, q = i % 9;
                    cp_async16(raw + (size_t)rr * 144 + 16 * q, W + (size_t)(j0 + rr) * rb + (size_t)b * Q4K_BYTES + 16 * q);
                }
                uint8_t *B = sm + OFF_B + buf * 8 * B_CHUNK;
                for (int i = tid; i < nt * 16; i += GU_THREADS) {
                    const int t = i / 16, c = (i / 2) % 8, h = i % 2;
                    cp_async16(B + c * B_CHUNK + canon(t, h), p.xq + (size_t)tok[t] * H + 256 * b + 32 * c + 16 * h);
                }
                uint8_t *xr = sm + OFF_XR + buf * XR_BYTES;
                for (int i = tid; i < nt * 4; i += GU_THREADS) {
                    const int t = i / 4, k = i % 4;  // k 0, 1: halves of the 8 scales; 2, 3: of the 8 sums
                    const size_t at = (size_t)tok[t] * (H / 32) + 8 * b + 4 * (k & 1);
                    const void *src = k < 2 ? static_cast<const void *>(p.xd + at) : static_cast<const void *>(p.xs32 + at);
                    cp_async16(xr + (k >> 1) * (XR_BYTES / 2) + t * 32 + 16 * (k & 1), src);
                }
                cp_async_commit();
            };
            f32x2 acc[8];  // tokens 16*th + 2i, 16*th + 2i + 1
#pragma unroll
            for (int q = 0; q < 8; ++q) acc[q] = f2_pack(0.0f, 0.0f);
            issue(0, 0);
            for (int b = 0; b < nb; ++b) {
                const int buf = b & 1;
                if (b + 1 < nb) {
                    issue(b + 1, buf ^ 1);
                    cp_async_wait_pending<1>();
                } else {
                    cp_async_wait_pending<0>();
                }
                __syncthreads();  // super-block b's copies from every thread are in
                {  // token scales as [chunk][token]; xsum terms dx * s32
                    const int c = tid / TC_NT, t = tid % TC_NT;
                    const float *xd = reinterpret_cast<const float *>(sm + OFF_XR + buf * XR_BYTES);
                    const int *xs = reinterpret_cast<const int *>(sm + OFF_XR + buf * XR_BYTES + XR_BYTES / 2);
                    float dx = 0.0f, sx = 0.0f;
                    if (t < nt) {
                        dx = xd[t * 8 + c];
                        sx = __fmul_rn(dx, (float)xs[t * 8 + c]);
                    }
                    DX[c * TC_NT + t] = dx;
                    XS[c * TC_NT + t] = sx;
                }
                // unpack row r, chunk pairs 2*th and 2*th + 1: nibbles -> int8, block scales
                {
                    const uint8_t *blk = sm + OFF_RAW + buf * RAW_BYTES + (size_t)r * 144;
                    const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
                    uint8_t *A = sm + OFF_A;
                    const float d = h2f(hd.x), dmin = h2f(hd.x >> 16);
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const int c = 2 * th + cc;
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
                        q4k_scales(hd, c, sc0, m0, sc1, m1);
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
                    const uint32_t sa = smem_u32(sm + OFF_A), sb = smem_u32(sm + OFF_B + buf * 8 * B_CHUNK);
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        umma_i8(taddr + c * TC_NT, umma_sdesc(sa + c * A_CHUNK), umma_sdesc(sb + c * B_CHUNK));
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     smem_u32(&bar))
                                 : "memory");
                }
                // bounded wait for this super-block's MMAs; the verdict is the CTA's, not a thread's
                uint32_t done = 0;
                for (uint32_t sp = 0; sp < SPIN_LIMIT && !done; ++sp) {
                    done = mbar_try_wait(&bar, phase) ? 1u : 0u;
                    if (!done && sp > 64) __nanosleep(64);
                }
                phase ^= 1u;
                if (!__syncthreads_and(done)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                // accumulate tokens 16*th .. +15 for row r (TMEM lane r); token pairs in packed
                // f32x2 registers (each element the same fmaf / __fmul_rn sequence), the integer
                // sums (|isum| < 2^22) converted exactly by an integer add under the exponent of
                // 1.5 * 2^23 and one float subtraction
                {
                    const uint32_t col = taddr + ((uint32_t)(32 * quad) << 16) + 16 * th;
                    const f32x2 magic = f2_pack(12582912.0f, 12582912.0f);
#pragma unroll 1
                    for (int c = 0; c < 8; c += 2) {
                        uint32_t v0[16], v1[16];
                        tmem_ld16(col + c * TC_NT, v0);
                        tmem_ld16(col + (c + 1) * TC_NT, v1);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc) {
                            const float sc = S[(c + cc) * TC_ROWS + r], mn = M[(c + cc) * TC_ROWS + r];
                            const f32x2 sc2 = f2_pack(sc, sc), nm2 = f2_pack(-mn, -mn);
                            const float4 *dx4 = reinterpret_cast<const float4 *>(DX + (c + cc) * TC_NT + 16 * th);
                            const float4 *xs4 = reinterpret_cast<const float4 *>(XS + (c + cc) * TC_NT + 16 * th);
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const float4 dx = dx4[k], xs = xs4[k];
#pragma unroll
                                for (int hp = 0; hp < 2; ++hp) {
                                    const int i = 4 * k + 2 * hp;
                                    const uint32_t ia = cc ? v1[i] : v0[i], ib = cc ? v1[i + 1] : v0[i + 1];
                                    const f32x2 isf = f2_sub(f2_pack(__int_as_float((int)(ia + 0x4B400000u)),
                                                                     __int_as_float((int)(ib + 0x4B400000u))),
                                                             magic);
                                    const f32x2 d2 = hp ? f2_pack(dx.z, dx.w) : f2_pack(dx.x, dx.y);
                                    const f32x2 x2 = hp ? f2_pack(xs.z, xs.w) : f2_pack(xs.x, xs.y);
                                    acc[i / 2] = f2_fma(f2_mul(sc2, d2), isf, f2_fma(nm2, x2, acc[i / 2]));
                                }
                            }
                        }
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncthreads();  // A, the scales and TMEM are reused by the next super-block
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            }
            if (!ok) break;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float a[2];
                f2_unpack(acc[q], a[0], a[1]);
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const int t = 16 * th + 2 * q + k;
                    if (t < nt) out[(size_t)(t0 + t) * p.F + j0 + r] = a[k];
                }
            }
        }
    }
    cp_async_wait_all();  // a stopped CTA leaves no copy in flight
    if (!ok && tid == 0 && p.status) atomicOr((uint32_t *)p.status, 4u);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(GU_COLS));
}

// ---------------------------------------------------------------------------
// Down projection on the tensor cores: part[pair][row] for the pairs of groups with
// n >= p.tc_down_min tokens, Q6_K rows (values q - 32 in -32..31 are int8) against
// the pairs' q8_1 h. One q8_1 block (32 values) spans two Q6_K scale groups, so each
// chunk takes two M=128 x N=32 x K=32 MMAs over half-zeroed operands, giving the exact
// per-group sums I_lo, I_hi; the CUDA cores form I = sc_lo*I_lo + sc_hi*I_hi (exact:
// |I| < 2^24) and accumulate (d*dx) * I in double. Each term is exact there (d*dx, a
// product of two fp16, has 22 significant bits), the terms are added in the order of
// the reference's Q6_K x q8_1 dot (super-block, then block) and the row rounds once to
// fp32, so a row equals that dot for the same q8_1 h.
// CTA = (group, 128-row tile of H) items, 8 warps: warp w serves TMEM lanes
// 32*(w%4)..+31 for tokens 16*(w/4)..+15; each half of a super-block (4 chunks, 8 MMAs,
// 256 TMEM columns) is unpacked, multiplied and accumulated in turn, w unpacking chunks
// 2*(w/4) and 2*(w/4)+1 of the half. The raw 128-row tile arrives in one bulk copy and
// its size sets the shared memory (two CTAs per SM up to ~60 KB of tile); the B operand
// and h scales of super-block b+1 are copied (cp.async, double buffer) while b is computed.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(DN_THREADS, 2) moe_batch_down_tc(MoeBatchParams p) {
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ __align__(8) uint64_t bar, tbar;
    __shared__ uint32_t taddr_s;
    const int nrt = p.H / TC_ROWS, items = (int)p.work[2] * nrt;  // (listed group, 128-row tile)
    if ((int)blockIdx.x >= items) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, role = warp >> 2;
    const int r = 32 * quad + lane;
    const int F = p.F, nb = F / 256;
    const uint32_t rbd = p.rbd;
    uint8_t *raw = sm + OFF_DRAW;
    double *DX = reinterpret_cast<double *>(sm + OFF_DDX);  // [chunk][token]

    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&tbar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // the zero K halves of the 8 operands
    for (int i = tid; i < 4 * 2 * TC_ROWS; i += DN_THREADS) {
        const int k = i / (2 * TC_ROWS), hi = (i / TC_ROWS) & 1, rr = i % TC_ROWS;
        *reinterpret_cast<uint4 *>(sm + OFF_DA + (2 * k + hi) * A_CHUNK + canon(rr, hi ? 0 : 1)) =
            make_uint4(0, 0, 0, 0);
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&taddr_s)),
                     "r"(DN_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t taddr = taddr_s;
    uint32_t phase = 0, tphase = 0;
    bool ok = true;

    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const int g = p.tc_groups[it / nrt], j0 = (it % nrt) * TC_ROWS;
        const int p0 = p.grp_off[g], p1 = p.grp_off[g + 1];
        if (p.tc_down_min <= 0 || p1 - p0 < p.tc_down_min) continue;  // small groups: the DP4A kernel
        const uint8_t *D = p.experts[3 * p.grp_expert[g] + 2];
        if (!D) {
            if (tid == 0 && p.status) atomicOr((uint32_t *)p.status, KQ_STATUS_NOT_RESIDENT);
            continue;
        }
        __syncthreads();  // the previous item's raw tile is no longer read
        if (tid == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            const uint32_t bytes = TC_ROWS * rbd;
            mbar_arrive_expect_tx(&tbar, bytes);
            bulk_g2s_hint(raw, D + (size_t)j0 * rbd, bytes, &tbar, l2_evict_first_policy());
        }
        bool tile_in = false;
        for (int t0 = p0; t0 < p1 && ok; t0 += TC_NT) {
            const int nt = min(TC_NT, p1 - t0);
            auto issue = [&](int b, int buf) {
                uint8_t *B = sm + OFF_DB + buf * 8 * B_CHUNK;
                for (int i = tid; i < nt * 16; i += DN_THREADS) {
                    const int t = i / 16, c = (i / 2) % 8, h = i % 2;
                    cp_async16(B + c * B_CHUNK + canon(t, h), p.hq + (size_t)(t0 + t) * F + 256 * b + 32 * c + 16 * h);
                }
                uint8_t *xr = sm + OFF_DXR + buf * (TC_NT * 8 * 4);
                for (int i = tid; i < nt * 2; i += DN_THREADS) {
                    const int t = i / 2, k = i % 2;
                    cp_async16(xr + t * 32 + 16 * k, p.hd + (size_t)(t0 + t) * (F / 32) + 8 * b + 4 * k);
                }
                cp_async_commit();
            };
            double acc[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) acc[q] = 0.0;
            issue(0, 0);
            for (int b = 0; b < nb && ok; ++b) {
                const int buf = b & 1;
                if (b + 1 < nb) {
                    issue(b + 1, buf ^ 1);
                    cp_async_wait_pending<1>();
                } else {
                    cp_async_wait_pending<0>();
                }
                __syncthreads();  // super-block b's copies from every thread are in
                if (!tile_in) {
                    const bool in = mbar_wait(&tbar, tphase);
                    if (__syncthreads_or(!in)) {
                        ok = false;
                        break;
                    }
                    tphase ^= 1u;
                    tile_in = true;
                }
                {
                    const int c = tid / TC_NT, t = tid % TC_NT;
                    const float *xr = reinterpret_cast<const float *>(sm + OFF_DXR + buf * (TC_NT * 8 * 4));
                    DX[c * TC_NT + t] = t < nt ? (double)xr[t * 8 + c] : 0.0;
                }
                const uint8_t *blk = raw + (size_t)r * rbd + (size_t)b * Q6K_BYTES;
                for (int half = 0; half < 2; ++half) {
                    // unpack row r, chunks 4*half + 2*role + {0, 1}: 6-bit values - 32
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const int k = 2 * role + cc, c = 4 * half + k, n = c >> 2, j = c & 3;
                        uint32_t lo[8], hi[8], q[8];
                        ld32_unaligned(blk + 64 * n + 32 * (j & 1), lo);
                        ld32_unaligned(blk + 128 + 32 * n, hi);
                        const int ns = 4 * (j >> 1), hs = 2 * j;
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            q[i] = __vsub4(((lo[i] >> ns) & 0x0F0F0F0Fu) | (((hi[i] >> hs) & 0x03030303u) << 4),
                                           0x20202020u);
                        *reinterpret_cast<uint4 *>(sm + OFF_DA + (2 * k) * A_CHUNK + canon(r, 0)) =
                            make_uint4(q[0], q[1], q[2], q[3]);
                        *reinterpret_cast<uint4 *>(sm + OFF_DA + (2 * k + 1) * A_CHUNK + canon(r, 1)) =
                            make_uint4(q[4], q[5], q[6], q[7]);
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncthreads();
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    if (tid == 0) {
                        const uint32_t sa = smem_u32(sm + OFF_DA), sb = smem_u32(sm + OFF_DB + buf * 8 * B_CHUNK);
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint64_t db = umma_sdesc(sb + (4 * half + k) * B_CHUNK);
                            umma_i8(taddr + (2 * k) * TC_NT, umma_sdesc(sa + (2 * k) * A_CHUNK), db);
                            umma_i8(taddr + (2 * k + 1) * TC_NT, umma_sdesc(sa + (2 * k + 1) * A_CHUNK), db);
                        }
                        asm volatile(
                            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                smem_u32(&bar))
                            : "memory");
                    }
                    uint32_t done = 0;
                    for (uint32_t sp = 0; sp < SPIN_LIMIT && !done; ++sp) {
                        done = mbar_try_wait(&bar, phase) ? 1u : 0u;
                        if (!done && sp > 64) __nanosleep(64);
                    }
                    phase ^= 1u;
                    if (!__syncthreads_and(done)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    // accumulate tokens 16*role .. +15 of row r over the half's 4 chunks. I
                    // (|I| < 2^24) becomes a double exactly: the word pair {0x43380000,
                    // I ^ 2^31} is 1.5 * 2^52 + 2^31 + I.
                    {
                        const double dd = (double)h2f((uint32_t)blk[208] | ((uint32_t)blk[209] << 8));
                        const uint32_t col = taddr + ((uint32_t)(32 * quad) << 16) + 16 * role;
#pragma unroll 1
                        for (int k = 0; k < 4; ++k) {
                            const int c = 4 * half + k;
                            uint32_t lo[16], hi[16];
                            tmem_ld16(col + (2 * k) * TC_NT, lo);
                            tmem_ld16(col + (2 * k + 1) * TC_NT, hi);
                            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                            const int sl = (int)(int8_t)blk[192 + 2 * c], sh = (int)(int8_t)blk[193 + 2 * c];
                            const double2 *dx2 = reinterpret_cast<const double2 *>(DX + c * TC_NT + 16 * role);
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                const double2 dx = dx2[e];
#pragma unroll
                                for (int f = 0; f < 2; ++f) {
                                    const int q = 2 * e + f;
                                    const int I = sl * (int)lo[q] + sh * (int)hi[q];
                                    const double fI =
                                        __hiloint2double(0x43380000, I ^ (int)0x80000000) - 6755401588539392.0;
                                    acc[q] = fma(dd * (f ? dx.y : dx.x), fI, acc[q]);
                                }
                            }
                        }
                    }
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncthreads();  // A and TMEM are reused by the next half
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                }
            }
            if (!ok) break;
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const int t = 16 * role + q;
                if (t < nt) p.part[(size_t)(t0 + t) * p.H + j0 + r] = (float)acc[q];
            }
        }
    }
    cp_async_wait_all();  // a stopped CTA leaves no copy in flight
    if (!ok && tid == 0 && p.status) atomicOr((uint32_t *)p.status, 4u);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(DN_COLS));
}

// Persistent grids: the SM count at most, twice that where two CTAs fit an SM (each holds
// 256 TMEM columns), never more than the worst-case item count.
static int tc_grid(const MoeBatchParams &p, int max_items) {
    const int sms = p.sms > 0 ? p.sms : 1;
    return max_items < sms ? max_items : sms;
}

void launch_gateup_tc(MoeBatchParams &p, int max_groups, cudaStream_t st) {
    static size_t set_bytes[KQ_MAX_DEVICES];
    ensure_smem_limit(moe_batch_gateup_tc, TC_SMEM, set_bytes);
    const int max_items = 2 * max_groups * (p.F / TC_ROWS);
    const int grid = 2 * tc_grid(p, max_items) < max_items ? 2 * tc_grid(p, max_items) : max_items;
    if (grid > 0) moe_batch_gateup_tc<<<grid, GU_THREADS, TC_SMEM, st>>>(p);
}

void launch_down_tc(MoeBatchParams &p, int max_groups, cudaStream_t st) {
    static size_t set_bytes[KQ_MAX_DEVICES];
    ensure_smem_limit(moe_batch_down_tc, TC_DOWN_SMEM, set_bytes);
    const uint32_t smem = OFF_DRAW + TC_ROWS * p.rbd + 16;
    const int max_items = max_groups * (p.H / TC_ROWS), per_sm = 2 * (smem + 2048) <= 228 * 1024 ? 2 : 1;
    const int grid = per_sm * tc_grid(p, max_items) < max_items ? per_sm * tc_grid(p, max_items) : max_items;
    if (grid > 0) moe_batch_down_tc<<<grid, DN_THREADS, smem, st>>>(p);
}

}  // namespace kq
