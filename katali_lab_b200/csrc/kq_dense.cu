// kq_dense.cu — dense Qwen3-style decoder decode step fully on the device
// (katali_cuda_dense_*).
//
// The reference runs this loop on the CPU and crosses to the GPU once per
// projection (V/src/gguf_model.c:570-703, each matvec_t through
// katali_dense_cuda_matvec with an upload and a download, README.md:164-171).
// Here the whole step — embedding row, RMSNorm, q/k/v, per-head q/k RMSNorm,
// RoPE, KV append, grouped-query attention, o projection + residual, RMSNorm,
// gate/up, SiLU * up, down + residual, final RMSNorm, LM head and the greedy
// argmax — is a fixed sequence of launches on one stream that reads the token
// and the position from device memory, so one captured CUDA graph serves every
// step and generation never returns to the host between tokens.
//
// RMSNorm runs inside the GEMVs' activation staging (kq_gemv.cu), the per-head q/k
// RMSNorm and RoPE inside attention, so a layer is six launches.
// Arithmetic follows the reference's kernels (V/src/gguf_kernels.c):
//   rmsnorm      :13-25   double sum of squares, inv = 1/sqrtf(mean + eps) in
//                         float, out = x * inv * w (two float products)
//   rope_apply   :45-61   v[i] = x1*c - x2*s, v[i+half] = x2*c + x1*s; the
//                         cos/sin table is computed on the host with the same
//                         libm calls as rope_prepare (V/src/gguf_model.c:466-475)
//   attention    :103-160 per query head: scores = (float)(double dot) * scale,
//                         softmax with max subtraction and a double sum, then
//                         out[d] += p_t * v_t[d] in t order
//   silu * up    V/src/gguf_simd_x86.c:763-773 (scalar tail form)
//   argmax       V/src/gguf_sampler.c:62-66 (first index of the strict maximum)
#include <cuda_runtime.h>

#include "kq_device.cuh"
#include "kq_launch.h"

namespace kq {

namespace {

constexpr int DT = 256;  // threads per CTA for the element-wise kernels

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

// One element of a GGUF row (dequantisation as kqo_dequant / the reference's
// katali_ggml_dequant_ref, V/src/gguf_dtype.c:429-452, :487-512).
__device__ __forceinline__ float dequant_elem(uint32_t type, const uint8_t *row, int i) {
    if (type == T_Q4_K) {
        const uint8_t *blk = row + (size_t)(i >> 8) * Q4K_BYTES;
        const int e = i & 255, j = e >> 5, l = e & 31;
        const uint4 h = *reinterpret_cast<const uint4 *>(blk);
        int sc0, m0, sc1, m1;
        q4k_scales(h, j >> 1, sc0, m0, sc1, m1);
        const int sc = (j & 1) ? sc1 : sc0, m = (j & 1) ? m1 : m0;
        const float d = h2f(h.x), mn = h2f(h.x >> 16);
        const uint8_t b = blk[16 + 32 * (j >> 1) + l];
        const int q = (j & 1) ? (b >> 4) : (b & 15);
        return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(mn, (float)m));
    }
    const uint8_t *blk = row + (size_t)(i >> 8) * Q6K_BYTES;
    const int e = i & 255, h = e >> 7, quarter = (e >> 5) & 3, l = e & 31;
    const uint8_t ql = blk[64 * h + 32 * (quarter & 1) + l];
    const uint8_t qh = blk[128 + 32 * h + l];
    const int lo = quarter >= 2 ? (ql >> 4) : (ql & 15);
    const int q = lo | (((qh >> (2 * quarter)) & 3) << 4);
    const float d = h2f(ld_u16(blk + 208));
    const int sc = (int)(int8_t)blk[192 + e / 16];
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)(q - 32));
}

__global__ void k_embed(DenseParams p) {
    pdl_trigger();
    pdl_wait();
    const int tok = *p.tok;
    const uint8_t *row = p.embed + (size_t)tok * p.embed_rb;
    for (int i = blockIdx.x * DT + threadIdx.x; i < p.H; i += gridDim.x * DT)
        p.x[i] = dequant_elem(p.embed_type, row, i);
}

// One head of q or k: RMSNorm over head_dim (when nw), then RoPE with the table
// row of position pos, written to dst (shared memory). All threads of the CTA call it.
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
        float out = val;  // pairs (i, i + rh) for i < rh, rh = rope_dim / 2
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

// Grouped-query decode attention, one CTA per query head over kv_len = pos + 1. The
// CTA first applies the per-head q/k RMSNorm and RoPE (gguf_forward_token's order:
// q norm, q rope, k norm, k rope); the first CTA of each kv group appends k and v to
// the layer's cache, and every CTA uses its own copy of the new k and v for t = pos.
__global__ void __launch_bounds__(DT) k_attention(DenseParams p, int layer) {
    extern __shared__ float scores[];  // kv_cap floats
    __shared__ double sh[32];
    __shared__ float red[32];
    __shared__ float sq[512], sk[512], sv[512], tmp[512];
    pdl_trigger();
    pdl_wait();
    const int HD = p.HD, hq = blockIdx.x, reps = p.NH / p.NKV;
    const int hk = hq / reps, pos = *p.pos, kv_len = pos + 1;
    norm_rope_head(p, p.q + (size_t)hq * HD, p.q_norm_dev[layer], pos, tmp, sq, sh);
    norm_rope_head(p, p.k + (size_t)hk * HD, p.k_norm_dev[layer], pos, tmp, sk, sh);
    const float *K = p.kv_k + ((size_t)layer * p.NKV + hk) * p.kv_cap * HD;
    const float *V = p.kv_v + ((size_t)layer * p.NKV + hk) * p.kv_cap * HD;
    if (threadIdx.x < HD) {
        sv[threadIdx.x] = p.v[(size_t)hk * HD + threadIdx.x];
        if (hq % reps == 0) {
            const size_t o = (size_t)pos * HD + threadIdx.x;
            const_cast<float *>(K)[o] = sk[threadIdx.x];
            const_cast<float *>(V)[o] = sv[threadIdx.x];
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // scores: one warp per key row, lanes over head dims, double accumulation
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
        p.attn[(size_t)hq * HD + d] = o;
    }
}

__global__ void k_silu_mul(float *g, const float *u, int n) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * DT + threadIdx.x;
    if (i < n) {
        const float x = g[i];
        g[i] = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, kq_expf(-x))), u[i]);
    }
}

// Greedy argmax, first index of the strict maximum: per-CTA (value, index)
// candidates, then one CTA folds them in index order and advances the step.
__device__ __forceinline__ void better(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi) || (bi < 0)) {
        bv = v;
        bi = i;
    }
}
__global__ void k_argmax_part(DenseParams p) {
    __shared__ float sv[32];
    __shared__ int si[32];
    pdl_trigger();
    pdl_wait();
    float bv = -INFINITY;
    int bi = -1;
    for (int i = blockIdx.x * DT + threadIdx.x; i < p.vocab; i += gridDim.x * DT)
        if (!(p.logits[i] != p.logits[i])) better(bv, bi, p.logits[i], i);  // NaN never wins
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(KQ_FULL, bv, o);
        const int oi = __shfl_xor_sync(KQ_FULL, bi, o);
        if (oi >= 0) better(bv, bi, ov, oi);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < DT / 32; ++w)
            if (si[w] >= 0) better(bv, bi, sv[w], si[w]);
        p.arg_v[blockIdx.x] = bv;
        p.arg_i[blockIdx.x] = bi;
    }
}
__global__ void k_argmax_final(DenseParams p, int nparts) {
    pdl_trigger();
    pdl_wait();
    float bv = -INFINITY;
    int bi = -1;
    for (int b = threadIdx.x; b < nparts; b += 32)
        if (p.arg_i[b] >= 0) better(bv, bi, p.arg_v[b], p.arg_i[b]);
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(KQ_FULL, bv, o);
        const int oi = __shfl_xor_sync(KQ_FULL, bi, o);
        if (oi >= 0) better(bv, bi, ov, oi);
    }
    if (threadIdx.x != 0) return;
    const int step = *p.step;
    if (step < p.out_cap) p.out_tokens[step] = bi < 0 ? 0 : bi;
    // the next step's input: the forced prompt token while prefilling, else this argmax
    *p.tok = step + 1 < *p.n_forced ? p.forced[step + 1] : (bi < 0 ? 0 : bi);
    *p.pos = *p.pos + 1;
    *p.step = step + 1;
}

}  // namespace

cudaError_t launch_dense_step(DenseParams &p, GemvParams *g, cudaStream_t st) {
    // g[4 l + 0..3]: qkv (attn RMSNorm in the staging), o (+ residual), gate/up (ffn
    // RMSNorm in the staging), down (+ residual) after SiLU * up; g[4 NL]: the LM head
    // (final RMSNorm in the staging). Every launch after the embedding is a programmatic
    // dependent of the one before it (GEMV weights stream while the previous kernel ends).
    k_embed<<<(p.H + DT - 1) / DT, DT, 0, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    for (int l = 0; l < p.NL; ++l) {
        if ((e = launch_gemv(g[4 * l + 0], p.gemv_mode, st)) != cudaSuccess) return e;
        e = launch_k(k_attention, dim3(p.NH), dim3(DT), (size_t)p.kv_cap * sizeof(float), st, 1, p, l);
        if (e != cudaSuccess) return e;
        if ((e = launch_gemv(g[4 * l + 1], p.gemv_mode, st)) != cudaSuccess) return e;
        if ((e = launch_gemv(g[4 * l + 2], p.gemv_mode, st)) != cudaSuccess) return e;
        e = launch_k(k_silu_mul, dim3((p.F + DT - 1) / DT), dim3(DT), 0, st, 1, p.gate,
                     (const float *)p.up, p.F);
        if (e != cudaSuccess) return e;
        if ((e = launch_gemv(g[4 * l + 3], p.gemv_mode, st)) != cudaSuccess) return e;
    }
    if ((e = launch_gemv(g[4 * p.NL], p.gemv_mode, st)) != cudaSuccess) return e;
    return launch_dense_argmax(p, st, 1);
}

cudaError_t launch_dense_embed(DenseParams &p, cudaStream_t st) {
    k_embed<<<(p.H + DT - 1) / DT, DT, 0, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_dense_argmax(DenseParams &p, cudaStream_t st, int pdl) {
    const int nparts = 148;
    cudaError_t e = launch_k(k_argmax_part, dim3(nparts), dim3(DT), 0, st, pdl, p);
    if (e == cudaSuccess) e = launch_k(k_argmax_final, dim3(1), dim3(32), 0, st, pdl, p, nparts);
    return e;
}

cudaError_t dense_set_attention_smem(int kv_cap) {
    return cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kv_cap * (int)sizeof(float));
}

}  // namespace kq
