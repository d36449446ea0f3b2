// kq_hybrid.cu — decode step of a hybrid MoE decoder (katali_cuda_hybrid_*): Gated DeltaNet
// (linear-attention) layers and gated full-attention layers, every layer followed by the fused
// MoE block, greedy argmax at the end, all on the device.
//
// The reference ships this model class (Qwen3.5/3.6-35B-A3B: 30 GDN + 10 full-attention
// layers, MoE every layer, README.md:15,19,322-336) only as binaries; its GDN and gated
// attention kernels have no source. The arithmetic here restates the published Gated DeltaNet
// decode rule (Yang, Kautz, Hatamizadeh, "Gated Delta Networks", ICLR 2025) in the layout of
// the Qwen3-Next / Qwen3.5 layers:
//   conv   : depthwise causal conv (kernel conv_k) over the q|k|v channels, then SiLU
//   norm   : q, k L2-normalised per head (eps 1e-6); q scaled by 1/sqrt(dk)
//   gates  : beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias), decay = exp(g)
//   step   : S <- decay * S;  kv = S^T k;  S <- S + k (beta (v - kv))^T;  o = S^T q
//   output : RMSNorm(o) * w * silu(z) per value head, then the out projection (+ residual)
// Gated attention: q and its gate come from one projection (per head: q rows, then gate
// rows); q/k RMSNorm per head, RoPE on the first rope_dim dimensions (pairs i, i + rope_dim/2
// as V/src/gguf_kernels.c:45-61), GQA decode attention as the dense decoder (kq_dense.cu), the
// head output multiplied by sigmoid(gate).
// MoE block: RMSNorm (ffn_norm), fp32 router GEMV (double accumulation, as the reference's
// F32 dot, V/src/gguf_dtype.c:640-644) and the fused MoE kernel (kq_moe.cu) adding its output
// into the residual stream. On one GPU the RMSNorm and the router run inside the MoE launch
// (MoeParams.rt_w); under expert parallelism k_router below runs before the MoE launch.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "kq_device.cuh"
#include "kq_launch.h"

namespace cg = cooperative_groups;

namespace kq {

namespace {

constexpr int DT = 256;           // threads of the attention kernel (head_dim <= 256)
constexpr int GD = 128;           // GDN head dimension (dk = dv)
constexpr int GDN_CPH = 4;        // CTAs (one cluster) per GDN value head
constexpr int GDN_THREADS = 256;  // 8 warps x 4 state columns per CTA
constexpr int RW = 4;             // router: warps per CTA, one expert row each

__device__ __forceinline__ double block_sum_d(double v, double *sh) {
    v = warp_sum_d(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0)
        for (int i = 0; i < nw; ++i) t += sh[i];
    __syncthreads();
    if (threadIdx.x == 0) sh[0] = t;
    __syncthreads();
    t = sh[0];
    __syncthreads();
    return t;
}

__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, kq_expf(-x))); }
__device__ __forceinline__ float sigmoid_f(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, kq_expf(-x)));
}

// One Gated DeltaNet decode step for value head h = blockIdx.x / GDN_CPH, split over a cluster
// of GDN_CPH CTAs: CTA rank r owns state columns [r 32, r 32 + 32) of the head (8 warps x 4
// columns, four dk values per lane). Every CTA computes the head's conv + SiLU for q and k (the
// q/k channels shared by `ratio` value heads are written back to the ring by rank 0 of the first
// of them) and for its own 32 v channels, the L2 norms and gates; after the delta-rule update the
// gated RMSNorm needs the sum of squares over all 128 outputs: each CTA publishes its partial in
// shared memory and, after a cluster barrier, reads the others' through distributed shared
// memory in rank order (the same double sum on every CTA).
__global__ void __launch_bounds__(GDN_THREADS) k_gdn(HybridParams p, HybridLayer L) {
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ __align__(16) float sq[GD];
    __shared__ __align__(16) float sk[GD];
    __shared__ float sv[GD / GDN_CPH], so[GD / GDN_CPH];
    __shared__ double sh[32];
    __shared__ double s_part;
    __shared__ float s_par[2];
    const int rank = (int)cluster.block_rank();
    const int vh = blockIdx.x / GDN_CPH, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ratio = p.nv / p.nk, kh = vh / ratio;
    const int C = 2 * p.nk * GD + p.nv * GD, K = p.conv_k;
    constexpr int CW = GD / GDN_CPH;          // columns of this CTA
    constexpr int CPW = CW / (GDN_THREADS / 32);  // columns per warp
    const int j0 = rank * CW;
    // The state columns are loaded before pdl_wait(): this layer's state was last written by
    // this kernel in the previous decode step, a separate graph launch (or eager launch
    // sequence) whose every kernel completed before this step's first launch started.
    float *S = L.state + (size_t)vh * GD * GD;
    float4 s[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c)
        s[c] = __ldcs(reinterpret_cast<const float4 *>(S + (size_t)(j0 + warp + 8 * c) * GD) + lane);
    // Also before pdl_wait(): the position (advanced by the previous step), each channel's
    // conv over its older inputs (ring slots written by earlier steps; this step writes slot
    // pos % K, which is not among them) and the gate constants. The new input, b and a come
    // from the in-projection GEMV: after the wait.
    constexpr int NCH = (2 * GD + CW + GDN_THREADS - 1) / GDN_THREADS;  // channels per thread
    const int pos = *p.d.pos;
    int chs[NCH];
    float pre[NCH], wl[NCH];
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
        const int t = tid + q * GDN_THREADS;
        chs[q] = -1;
        if (t >= 2 * GD + CW) continue;
        const int which = t < GD ? 0 : t < 2 * GD ? 1 : 2, c = which < 2 ? t % GD : t - 2 * GD;
        const int ch = which == 0   ? kh * GD + c
                       : which == 1 ? p.nk * GD + kh * GD + c
                                    : 2 * p.nk * GD + vh * GD + j0 + c;
        const float *w = L.conv_w + (size_t)ch * K;
        float acc = 0.0f;
        for (int j = 0; j < K - 1; ++j) {
            const int tp = pos - (K - 1) + j;  // input position; slots of tp < 0 hold zeros
            const int slot = ((tp % K) + K) % K;
            acc = __fadd_rn(acc, __fmul_rn(w[j], L.ring[(size_t)slot * C + ch]));
        }
        chs[q] = ch;
        pre[q] = acc;
        wl[q] = w[K - 1];
    }
    const float ea = L.a_neg ? -L.a_neg[vh] : kq_expf(L.a_log[vh]), dtb = L.dt_bias[vh];
    pdl_trigger();
    pdl_wait();
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
        if (chs[q] < 0) continue;
        const int t = tid + q * GDN_THREADS;
        const int which = t < GD ? 0 : t < 2 * GD ? 1 : 2, c = which < 2 ? t % GD : t - 2 * GD;
        const int ch = chs[q];
        const float cur = p.qkv[ch];
        const float acc = __fadd_rn(pre[q], __fmul_rn(wl[q], cur));
        if (which == 2 || (vh % ratio == 0 && rank == 0)) L.ring[(size_t)(pos % K) * C + ch] = cur;
        const float act = silu_f(acc);
        if (which == 0) sq[c] = act;
        else if (which == 1) sk[c] = act;
        else sv[c] = act;
    }
    if (tid == 0) {
        const float b = p.ba[vh], a = p.ba[p.nv + vh];
        const float xa = __fadd_rn(a, dtb);
        const float sp = xa > 20.0f ? xa : log1pf(kq_expf(xa));  // softplus
        const float g = -__fmul_rn(ea, sp);
        s_par[0] = sigmoid_f(b);
        s_par[1] = kq_expf(g);
    }
    __syncthreads();
    const double nq = block_sum_d(tid < GD ? (double)sq[tid] * (double)sq[tid] : 0.0, sh);
    const double nk2 = block_sum_d(tid < GD ? (double)sk[tid] * (double)sk[tid] : 0.0, sh);
    if (tid < GD) {
        const float iq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)nq, 1e-6f)));
        const float ik = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)nk2, 1e-6f)));
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)GD));
        sq[tid] = __fmul_rn(__fmul_rn(sq[tid], iq), scale);
        sk[tid] = __fmul_rn(sk[tid], ik);
    }
    __syncthreads();

    const float beta = s_par[0], decay = s_par[1];
    const float4 kk = reinterpret_cast<const float4 *>(sk)[lane];
    const float4 qq = reinterpret_cast<const float4 *>(sq)[lane];
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
        const int jl = warp + 8 * c, j = j0 + jl;
        float4 v = s[c];
        v.x = __fmul_rn(v.x, decay);
        v.y = __fmul_rn(v.y, decay);
        v.z = __fmul_rn(v.z, decay);
        v.w = __fmul_rn(v.w, decay);
        double kv = (double)v.x * kk.x;
        kv += (double)v.y * kk.y;
        kv += (double)v.z * kk.z;
        kv += (double)v.w * kk.w;
        kv = warp_sum_d(kv);
        const float delta = __fmul_rn(__fsub_rn(sv[jl], (float)kv), beta);
        v.x = __fadd_rn(v.x, __fmul_rn(kk.x, delta));
        v.y = __fadd_rn(v.y, __fmul_rn(kk.y, delta));
        v.z = __fadd_rn(v.z, __fmul_rn(kk.z, delta));
        v.w = __fadd_rn(v.w, __fmul_rn(kk.w, delta));
        double o = (double)v.x * qq.x;
        o += (double)v.y * qq.y;
        o += (double)v.z * qq.z;
        o += (double)v.w * qq.w;
        o = warp_sum_d(o);
        __stcs(reinterpret_cast<float4 *>(S + (size_t)j * GD) + lane, v);
        if (lane == 0) so[jl] = (float)o;
    }
    __syncthreads();
    const double part = block_sum_d(tid < CW ? (double)so[tid] * (double)so[tid] : 0.0, sh);
    if (tid == 0) s_part = part;
    cluster.sync();  // every CTA's partial is published
    double no = 0.0;
    for (int r = 0; r < GDN_CPH; ++r) no += *cluster.map_shared_rank(&s_part, r);
    if (tid < CW) {
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(no / (double)GD), p.d.eps)));
        const float zz = p.z[(size_t)vh * GD + j0 + tid];
        p.go[(size_t)vh * GD + j0 + tid] =
            __fmul_rn(__fmul_rn(__fmul_rn(so[tid], inv), L.ssm_norm[j0 + tid]), silu_f(zz));
    }
    cluster.sync();  // no CTA leaves while another still reads its partial
}

// One head of q or k: RMSNorm over head_dim (when nw), then RoPE on the first 2 * rope_half
// dimensions with the table row of position pos, into dst (shared memory).
__device__ __forceinline__ void norm_rope_head(const DenseParams &p, const float *src, const float *nw,
                                               int pos, float *tmp, float *dst, double *sh) {
    const int HD = p.HD, rh = p.rope_half, i = threadIdx.x;
    float val = i < HD ? src[i] : 0.0f;
    if (nw) {
        const double s = block_sum_d(i < HD ? (double)val * (double)val : 0.0, sh);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(s / (double)HD), p.eps)));
        if (i < HD) val = __fmul_rn(__fmul_rn(val, inv), nw[i]);
    }
    if (i < HD) tmp[i] = val;
    __syncthreads();
    if (i < HD) {
        float out = val;
        if (i < rh) {
            const float c = p.rope_cos[(size_t)pos * rh + i], s = p.rope_sin[(size_t)pos * rh + i];
            out = __fsub_rn(__fmul_rn(val, c), __fmul_rn(tmp[i + rh], s));
        } else if (i < 2 * rh) {
            const int j = i - rh;
            const float c = p.rope_cos[(size_t)pos * rh + j], s = p.rope_sin[(size_t)pos * rh + j];
            out = __fadd_rn(__fmul_rn(val, c), __fmul_rn(tmp[j], s));
        }
        dst[i] = out;
    }
    __syncthreads();
}

// Gated GQA decode attention, one CTA per query head over kv_len = pos + 1: q of head h is
// q[h * 2 HD .. + HD), its gate the next HD values; out = attention(q, K, V) * sigmoid(gate).
__global__ void __launch_bounds__(DT) k_attn_gated(HybridParams hp, HybridLayer L) {
    const DenseParams &p = hp.d;
    extern __shared__ float scores[];  // kv_cap floats
    __shared__ double sh[32];
    __shared__ float red[32];
    __shared__ float sq[DT], sk[DT], sv[DT], tmp[DT];
    pdl_trigger();
    pdl_wait();
    const int HD = p.HD, hq = blockIdx.x, reps = p.NH / p.NKV;
    const int hk = hq / reps, pos = *p.pos, kv_len = pos + 1;
    const float *qh = p.q + (size_t)hq * 2 * HD;
    norm_rope_head(p, qh, L.q_norm, pos, tmp, sq, sh);
    norm_rope_head(p, p.k + (size_t)hk * HD, L.k_norm, pos, tmp, sk, sh);
    float *K = L.kv_k + (size_t)hk * p.kv_cap * HD;
    float *V = L.kv_v + (size_t)hk * p.kv_cap * HD;
    if (threadIdx.x < HD) {
        sv[threadIdx.x] = p.v[(size_t)hk * HD + threadIdx.x];
        if (hq % reps == 0) {
            const size_t o = (size_t)pos * HD + threadIdx.x;
            K[o] = sk[threadIdx.x];
            V[o] = sv[threadIdx.x];
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int t = warp; t < kv_len; t += DT / 32) {
        const float *kt = t == pos ? sk : K + (size_t)t * HD;
        double acc = 0.0;
        for (int d = lane; d < HD; d += 32) acc += (double)sq[d] * (double)kt[d];
        acc = warp_sum_d(acc);
        if (lane == 0) scores[t] = __fmul_rn((float)acc, p.attn_scale);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int t = threadIdx.x; t < kv_len; t += DT) m = fmaxf(m, scores[t]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(KQ_FULL, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int i = 1; i < DT / 32; ++i) m = fmaxf(m, red[i]);
    double s = 0.0;
    for (int t = threadIdx.x; t < kv_len; t += DT) {
        const float e = kq_expf(__fsub_rn(scores[t], m));
        scores[t] = e;
        s += (double)e;
    }
    s = block_sum_d(s, sh);
    const float inv = (float)(1.0 / s);
    for (int t = threadIdx.x; t < kv_len; t += DT) scores[t] = __fmul_rn(scores[t], inv);
    __syncthreads();
    for (int d = threadIdx.x; d < HD; d += DT) {
        float o = 0.0f;
        for (int t = 0; t < pos; ++t) o = __fadd_rn(o, __fmul_rn(scores[t], V[(size_t)t * HD + d]));
        o = __fadd_rn(o, __fmul_rn(scores[pos], sv[d]));
        p.attn[(size_t)hq * HD + d] = __fmul_rn(o, sigmoid_f(qh[HD + d]));
    }
}

// MoE block input: xb = RMSNorm(x) * ffn_norm (written by CTA 0; every CTA recomputes it in
// shared memory), router logits = R xb with fp32 rows and double accumulation. One warp per
// expert row; the row (NV float4 per lane, H = 128 NV) is loaded into registers before
// pdl_wait(), so under a programmatic launch the 2 MB of router weights stream while the
// previous kernel finishes. NV = 0: any H, loads in the dot loop.
template <int NV>
__global__ void __launch_bounds__(RW * 32) k_router(HybridParams hp, HybridLayer L) {
    extern __shared__ __align__(16) float xn[];  // H floats
    __shared__ double sh[32];
    const DenseParams &p = hp.d;
    const int H = p.H, tid = threadIdx.x, lane = tid & 31;
    const int r = blockIdx.x * RW + (tid >> 5);
    const bool live = r < hp.n_experts;
    const float4 *w = reinterpret_cast<const float4 *>(L.router + (size_t)(live ? r : 0) * H);
    float4 wr[NV > 0 ? NV : 1];
    if constexpr (NV > 0) {
#pragma unroll
        for (int i = 0; i < NV; ++i) wr[i] = __ldcs(w + lane + 32 * i);
    }
    pdl_trigger();
    pdl_wait();
    double ss = 0.0;
    for (int i = tid; i < H; i += RW * 32) ss += (double)p.x[i] * (double)p.x[i];
    ss = block_sum_d(ss, sh);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(ss / (double)H), p.eps)));
    for (int i = tid; i < H; i += RW * 32) {
        const float v = __fmul_rn(__fmul_rn(p.x[i], inv), L.ffn_norm[i]);
        xn[i] = v;
        if (blockIdx.x == 0) p.xb[i] = v;
    }
    __syncthreads();
    if (!live) return;
    const float4 *xv = reinterpret_cast<const float4 *>(xn);
    double acc = 0.0;
    auto dot4 = [&](const float4 a, const float4 b) {
        acc += (double)a.x * (double)b.x;
        acc += (double)a.y * (double)b.y;
        acc += (double)a.z * (double)b.z;
        acc += (double)a.w * (double)b.w;
    };
    if constexpr (NV > 0) {
#pragma unroll
        for (int i = 0; i < NV; ++i) dot4(wr[i], xv[lane + 32 * i]);
    } else {
        for (int i = lane; i < H / 4; i += 32) dot4(__ldcs(w + i), xv[i]);
    }
    acc = warp_sum_d(acc);
    if (lane == 0) hp.rlogits[r] = (float)acc;
}

// k_gdn: clusters of GDN_CPH CTAs, programmatic dependent of the in-projection GEMV.
cudaError_t launch_gdn(HybridParams &p, const HybridLayer &L, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(p.nv * GDN_CPH));
    cfg.blockDim = dim3(GDN_THREADS);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = GDN_CPH;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, k_gdn, p, L);
}

}  // namespace

cudaError_t launch_hybrid_step(HybridParams &p, const HybridLayer *L, GemvParams *g,
                               MoeParams *moe, const int *moe_grid, cudaStream_t st,
                               HybridHook before_moe, void *ctx, int *hook_status) {
    // Every launch but the first (the embedding) and the cooperative MoE kernels is a
    // programmatic dependent of the one before it (the GEMVs carry it in GemvParams.pdl).
    cudaError_t e = launch_dense_embed(p.d, st);
    if (e != cudaSuccess) return e;
    const int mode = p.d.gemv_mode;
    const size_t att_smem = (size_t)p.d.kv_cap * sizeof(float);
    const size_t rt_smem = (size_t)p.d.H * sizeof(float);
    void (*router)(HybridParams, HybridLayer) = p.d.H == 2048   ? k_router<16>
                                                : p.d.H == 1024 ? k_router<8>
                                                : p.d.H == 4096 ? k_router<32>
                                                                : k_router<0>;
    const dim3 rgrid((p.n_experts + RW - 1) / RW);
    for (int l = 0; l < p.d.NL; ++l) {
        if ((e = launch_gemv(g[2 * l], mode, st)) != cudaSuccess) return e;
        if (L[l].kind == 0) e = launch_gdn(p, L[l], st);
        else e = launch_k(k_attn_gated, dim3(p.d.NH), dim3(DT), att_smem, st, 1, p, L[l]);
        if (e != cudaSuccess) return e;
        if ((e = launch_gemv(g[2 * l + 1], mode, st)) != cudaSuccess) return e;
        if ((p.moe_ep || !moe[l].rt_w) &&  // else the router runs inside the MoE launch
            (e = launch_k(router, rgrid, dim3(RW * 32), rt_smem, st, 1, p, L[l])) != cudaSuccess)
            return e;
        if (before_moe) {
            const int hs = before_moe(ctx, l);
            if (hs) {
                if (hook_status) *hook_status = hs;
                return cudaSuccess;
            }
        }
        e = p.moe_ep ? launch_moe_ep_layer(moe[l], moe_grid[l], st) : launch_moe(moe[l], moe_grid[l], st);
        if (e != cudaSuccess) return e;
    }
    if ((e = launch_gemv(g[2 * p.d.NL], mode, st)) != cudaSuccess) return e;
    return launch_dense_argmax(p.d, st, 1);
}

cudaError_t hybrid_set_attention_smem(int kv_cap) {
    return cudaFuncSetAttribute(k_attn_gated, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kv_cap * (int)sizeof(float));
}

}  // namespace kq
