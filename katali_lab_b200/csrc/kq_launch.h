// kq_launch.h — kernel parameter blocks and host launchers (internal to the plugin).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace kq {

// Status bits the kernels set in the mapped status word (1, 2, 4: a bounded
// wait gave up).
constexpr uint32_t KQ_STATUS_NOT_RESIDENT = 8u;  // a selected expert has no device copy


struct GemvJob {
    const uint8_t *w;  // device matrix, native GGUF rows, 16-byte aligned
    float *y;
    uint64_t rows;
    uint32_t type;
    uint32_t rb;     // bytes per row
    uint32_t tr;     // rows per tile (set by the launcher)
    uint32_t tile0;  // first global tile of this job (set by the launcher)
    uint32_t accum;  // 1: y[r] += W x (the residual add of a decoder layer), else y[r] = W x
};

struct GemvParams {
    GemvJob job[8];
    int njobs;
    uint32_t total_tiles;
    uint32_t cols;
    uint32_t stage_bytes;
    int nstages;
    uint32_t act_off;
    int use_tma;
    const float *x;     // fp32 activations (modes 0 and 2)
    const uint8_t *xq;  // q8_1 blocks (mode 1)
    volatile uint32_t *status;
    // Optional prologue applied to x while it is staged (modes 0 and 2):
    //   x_mul  : x_i <- silu(x_i) * x_mul_i            (the SwiGLU product)
    //   norm_w : x_i <- (x_i * inv) * norm_w_i, inv = 1 / sqrt(mean(x^2) + norm_eps)
    const float *x_mul;
    const float *norm_w;
    float norm_eps;
    int pdl;  // 1: launched as a programmatic dependent of the previous kernel on the stream
};

// Kernel attributes such as the dynamic shared-memory limit belong to a device, so what a
// launcher remembers about them is kept per device. Devices with an id of KQ_MAX_DEVICES or
// more are not cached: their attribute is set on every launch.
constexpr int KQ_MAX_DEVICES = 64;
inline int current_device() {
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess) d = -1;
    return d;
}
// Raises k's dynamic shared-memory limit on the current device to at least `bytes`;
// per_device[d] holds the limit already set on device d.
template <typename KernelT>
inline cudaError_t ensure_smem_limit(KernelT k, size_t bytes, size_t *per_device) {
    const int d = current_device();
    const bool cached = d >= 0 && d < KQ_MAX_DEVICES;
    if (cached && per_device[d] >= bytes) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess && cached) per_device[d] = bytes;
    return e;
}
// SM count of the current device (cached per device).
inline int device_sms() {
    static int sms[KQ_MAX_DEVICES];
    const int d = current_device();
    if (d >= 0 && d < KQ_MAX_DEVICES && sms[d] > 0) return sms[d];
    int n = 0;
    if (d < 0 || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0)
        n = 148;
    if (d >= 0 && d < KQ_MAX_DEVICES) sms[d] = n;
    return n;
}

// Launch of kernel k, as a programmatic dependent of the previous kernel on st when pdl
// (the kernel then follows the pdl_wait() rule of kq_device.cuh).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            int pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

// mode 0: q8_1 activations quantised in-kernel from fp32 x; 1: from q8_1 blocks;
// 2: fp32 activations.
cudaError_t launch_gemv(GemvParams &p, int mode, cudaStream_t st);
cudaError_t launch_quantize_q8_1(const float *x, uint64_t n, void *out, cudaStream_t st);
cudaError_t launch_encode(uint32_t type, const float *x, uint64_t n, void *out, cudaStream_t st);
cudaError_t launch_row_isums(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                             uint32_t rb, const void *xq, int32_t *isum, int32_t *xsum,
                             cudaStream_t st);

constexpr int MOE_MAX_K = 16;
// Expert-parallel experts stage in the fused kernel: at most this many received slots
// (pairs processed in rounds of K), else the ragged-batch pipeline.
constexpr int MOE_EP_MAX_SLOTS = 16;
constexpr int MOE_EP_MAX_PAIRS = MOE_EP_MAX_SLOTS * MOE_MAX_K;
constexpr int MOE_MAX_CHUNKS = 64;
constexpr int MOE_RT_ROWS = 4;   // router rows per CTA when the router is folded into the launch
// Per CTA when tracing: %globaltimer slots 0-15 and 18-31, clock64 at start and end in 16, 17.
constexpr int TRACE_SLOTS = 32;

struct MoeParams {
    const uint8_t *const *experts;  // device table: gate_e, up_e, down_e per expert
    const float *x;
    const float *logits;   // router logits (NULL when ids/w are given)
    const int32_t *ids;    // routed variant
    const float *w;
    float *y;
    float *hbuf;           // scratch: top_k * ffn floats
    uint32_t *sync;        // scratch: grid-barrier arrive / done counters (zero between calls)
    volatile uint32_t *status;
    int32_t *dbg_ids;      // optional: routing decision (written by CTA 0)
    float *dbg_w;
    uint64_t *trace;       // optional: TRACE_SLOTS timestamps per CTA
    int n_experts, H, F, K, norm, mode;
    uint32_t gate_type, up_type, down_type;
    uint32_t rbg, rbu, rbd;
    uint32_t rg;           // phase-B rows per aligned group (set by moe_plan)
    int route_only;        // 1: routing decision only (check entry point)
    int accum;             // 1: y[r] += layer output (a decoder's residual add), 0: y[r] = output
    int pdl;               // 1: programmatic dependent of the previous kernel (not EP, not route_only)
    // Router folded into the launch (a decoder's MoE block, not EP): x is the residual stream,
    // the kernel forms RMSNorm(x) * rt_norm itself and the logits R xb (fp32 rows rt_w, double
    // sums) into the scratch p.logits before routing. Needs H <= 4 * MOE_THREADS and at most
    // MOE_RT_ROWS router rows per CTA.
    const float *rt_w;
    const float *rt_norm;
    float rt_eps;
    // shared-memory plan (bytes), identical for every CTA
    uint32_t chunk_units;  // max row pairs per phase-A chunk
    uint32_t sa_bytes;     // phase-A staging capacity
    uint32_t sb_off, sb_bytes;
    uint32_t act_off, hact_off, misc_off, smem_bytes;
    uint32_t dec_off, dec_row_bytes;  // decoded 6-bit down rows (Q6_K), read by phase B
    uint32_t dec_bytes;               // their area (dec_off == 0: inside the phase-A staging)
    uint32_t sdot_off;                // phase-B per-expert row dots [K][rows]
    int dec_enabled;
    // Expert-parallel experts stage (launch_moe_ep): the received slots in (the slot
    // layout of katali_cuda_moe_ep_dispatch), per-slot weighted sums out (doubles).
    // hbuf then holds ep_slots * K * F / 32 q8_1 records of h.
    const uint8_t *ep_recv;
    double *ep_ret;
    uint32_t ep_slots, ep_slot_bytes, ep_hdr_bytes;
    // The whole expert-parallel layer over peer memory in one launch (launch_moe_ep_layer):
    // this rank's ep_tokens (<= ep_tmax) tokens in x / logits, out in y; ep_recv and
    // ep_slots are then derived on the device (this rank's window of the call's parity)
    // and ep_ret is local scratch for the per-slot sums. Windows as in EpPeer.
    int ep_rank, ep_ranks, ep_tmax, ep_tokens;
    uint64_t *ep_route_rec;  // [tmax][K] this rank's routing, tagged words (read by the combine)
    uint8_t *const *ep_peer_recv;
    double *const *ep_peer_back;
    uint32_t *const *ep_peer_flags;
    uint32_t *ep_epoch, *ep_done;
    // tagged regions of the peer windows (EpPeer)
    uint64_t *const *ep_peer_trecv;
    uint64_t *const *ep_peer_tback;
    uint64_t *const *ep_peer_tdone;
    uint32_t ep_tslot_words;
};

cudaError_t launch_moe(MoeParams &p, int grid, cudaStream_t st);
// Move the decoded down rows out of the phase-A staging area when shared memory allows, so
// that the expert-parallel kernel can request a round's gate/up rows while the previous
// round still decodes and sums (its rounds then overlap). Returns 1 when moved.
int moe_plan_dec_apart(MoeParams &p, int max_smem);
// The experts stage of an expert-parallel layer for at most MOE_EP_MAX_SLOTS received
// slots (q8_1, Q6_K down, F a power of two in [256, 2048], K * F / 32 <= grid).
cudaError_t launch_moe_ep(MoeParams &p, int grid, cudaStream_t st);
// The whole expert-parallel layer (dispatch, experts, return, combine) over NVLink peer
// memory in one cooperative launch per rank; same conditions as launch_moe_ep, with
// ep_ranks * ep_tmax <= MOE_EP_MAX_SLOTS.
cudaError_t launch_moe_ep_layer(MoeParams &p, int grid, cudaStream_t st);

// Ragged multi-token MoE layer (q8_1 activations); scratch owned by the layer object.
struct MoeBatchParams {
    const uint8_t *const *experts;
    const float *X, *logits;
    float *Y;
    int T, n_experts, H, F, K, norm;
    uint32_t gate_type, up_type, down_type, rbg, rbu, rbd;
    int32_t *ids;
    float *w;
    int8_t *xq;
    float *xd;
    int *xs32, *xs16;
    int *grp_expert, *grp_off, *n_groups, *pair_src, *pos_of;
    uint32_t *work;  // item counters of the gate/up and down kernels, zeroed by the group kernel;
                     // work[2]: the number of listed tensor-core groups
    float *h;
    int8_t *hq;
    float *hd;
    int *hs32, *hs16;
    float *part;
    // expert parallelism (slot exchange between ranks)
    int ep_ranks, ep_tmax, ep_tokens;
    uint32_t ep_slot_bytes, ep_hdr_bytes;
    uint8_t *ep_send;
    const uint8_t *ep_recv;
    double *ep_ret;
    const double *ep_back;
    int32_t *ep_src_ids;
    volatile uint32_t *status;  // device-side timeout bits (mapped host word)
    int gu_rows, dn_rows;       // row-tile heights, set by the launcher
    int sms;                    // SM count (persistent grids)
    // expert parallelism over peer memory (ep_p2p = 1): every rank's window holds
    // recv [2][G][Tmax][slot], back [2][G][Tmax][H] doubles and flags [2][2][G]
    // (recv flags, then back flags, per parity); entry d of each array is rank d's
    // window as mapped in this process (this rank's own entry is local memory).
    int ep_p2p, ep_rank;
    uint8_t *const *ep_peer_recv;
    double *const *ep_peer_back;
    uint32_t *const *ep_peer_flags;
    uint32_t *ep_epoch;  // calls completed by this rank (the next call is *ep_epoch + 1)
    uint32_t *ep_done;   // last-CTA counters of the three peer kernels
    int tc_min;          // groups with >= tc_min tokens: gate/up on the tensor cores (0: never)
    int tc_down_min;     // groups with >= tc_down_min tokens: down on the tensor cores (0: never)
    int *tc_groups;      // indices of the groups with >= min(positive tc thresholds) tokens; count in work[2]
    float *hu;           // up sums of the pairs whose gate/up ran on the tensor cores (their gate sums in h)
    uint8_t *pair_tc;    // per grouped pair: 1 when its gate/up ran on the tensor cores
    const int32_t *ids_in;  // routing given (ids / weights [T][K]) instead of logits
    const float *w_in;
};
// The peer-memory exchange of an expert-parallel communicator (device arrays of
// n_ranks window pointers; see MoeBatchParams).
struct EpPeer {
    int rank;
    uint8_t *const *recv;
    double *const *back;
    uint32_t *const *flags;
    uint32_t *epoch, *done;
    // Tagged regions of the windows for the single-launch layer (NULL when the exchange is too
    // large for it): 8-byte words {32-bit payload, 32-bit call number}, so a receiver polls the
    // data itself and no flag or system-scope fence is needed. trecv [2][G src][tmax][tslot_words]
    // slots, tback [2][G owner][tmax][H][2] per-row sums (hi, lo words of the double), tdone
    // [2][G] "finished reading this call's window" words.
    uint64_t *const *trecv;
    uint64_t *const *tback;
    uint64_t *const *tdone;
    uint32_t tslot_words;
};
// Word offsets in a tagged slot: n_owned, ids[MOE_MAX_K], weights[MOE_MAX_K], then the q8_1
// row (9 words per 32-element block).
constexpr int EPT_IDS = 1;
constexpr int EPT_W = 1 + MOE_MAX_K;
constexpr int EPT_ROW = 1 + 2 * MOE_MAX_K;
inline uint32_t ep_tslot_words(uint32_t H) { return EPT_ROW + H / 32 * 9; }
cudaError_t launch_moe_batch(MoeBatchParams &p, cudaStream_t st);
void launch_gateup_tc(MoeBatchParams &p, int max_groups, cudaStream_t st);
void launch_down_tc(MoeBatchParams &p, int max_groups, cudaStream_t st);
// Largest raw row tile (128 rows of the down matrix) the tensor-core down kernel stages.
constexpr uint32_t TC_DOWN_RAW_MAX = 96 * 1024;
cudaError_t launch_moe_ep_dispatch(MoeBatchParams &p, cudaStream_t st);
cudaError_t launch_moe_ep_experts(MoeBatchParams &p, cudaStream_t st);
cudaError_t launch_moe_ep_combine(MoeBatchParams &p, cudaStream_t st);
int moe_plan(MoeParams &p, int grid, int max_smem);

// Dense decoder decode step (kq_dense.cu).
struct DenseLayer {  // host-side view for the launcher
    const float *attn_norm, *ffn_norm;
};
struct DenseParams {
    int H, F, NH, NKV, HD, NL, vocab, kv_cap, rope_half;
    float eps, attn_scale;
    const uint8_t *embed;
    uint32_t embed_type, embed_rb;
    const float *out_norm;
    const DenseLayer *L;              // host array, n_layers
    const float *const *q_norm_dev;   // device arrays of n_layers pointers (entries may be NULL)
    const float *const *k_norm_dev;
    float *x, *xb, *q, *k, *v, *attn, *gate, *up, *logits;
    float *kv_k, *kv_v;               // [NL][NKV][kv_cap][HD]
    const float *rope_cos, *rope_sin; // [kv_cap][rope_half]
    int *tok, *pos, *step, *n_forced; // device control words
    const int *forced;                // prompt tokens (forced inputs)
    int *out_tokens;                  // argmax of every step of a call
    int out_cap;
    float *arg_v;
    int *arg_i;
    int gemv_mode;                    // 2: fp32 activations, 0: q8_1 (quantised in the GEMV)
};
cudaError_t launch_dense_step(DenseParams &p, GemvParams *g, cudaStream_t st);
cudaError_t dense_set_attention_smem(int kv_cap);
// Pieces of the dense step shared with the hybrid decoder: the embedding row of *p.tok
// into p.x, and the greedy argmax of p.logits (advances tok / pos / step).
cudaError_t launch_dense_embed(DenseParams &p, cudaStream_t st);
cudaError_t launch_dense_argmax(DenseParams &p, cudaStream_t st, int pdl = 0);

// Hybrid decoder (kq_hybrid.cu): Gated DeltaNet and gated-attention layers, each followed
// by a fused MoE block. Per-layer device pointers, passed by value to that layer's launches.
struct HybridLayer {
    int kind;                        // 0: Gated DeltaNet, 1: gated full attention
    const float *conv_w;             // GDN: [C][conv_k] depthwise causal conv, C = 2 nk dk + nv dv
    const float *a_log, *dt_bias;    // GDN: [nv]
    const float *a_neg;              // GDN, optional: [nv] A = -exp(A_log), used instead of a_log
    const float *ssm_norm;           // GDN: [dv] weight of the gated RMSNorm
    float *ring;                     // GDN: [conv_k][C] last conv_k inputs (slot pos % conv_k)
    float *state;                    // GDN: [nv][dv][dk] recurrent state, column j of head h contiguous
    const float *q_norm, *k_norm;    // attention: [HD]
    float *kv_k, *kv_v;              // attention: [NKV][kv_cap][HD] of this layer
    const float *ffn_norm;           // [H]
    const float *router;             // fp32 [n_experts][H]
};
struct HybridParams {
    DenseParams d;                   // x, xb, q (q and gate per head), k, v, attn, logits, KV, RoPE,
                                     // control words, argmax scratch
    int nk, nv, dk, dv, conv_k, n_experts;
    float *qkv;                      // GDN in-projection: [q nk*dk][k nk*dk][v nv*dv]
    float *z;                        // [nv*dv] output gate
    float *ba;                       // [nv] beta logits, then [nv] decay inputs
    float *go;                       // [nv*dv] gated-norm output of the recurrence
    float *rlogits;                  // [n_experts] router logits
    int moe_ep;                      // 1: the MoE blocks run expert-parallel over peer memory
};
// One decode step: g[2 l], g[2 l + 1] are layer l's input and output projections, g[2 NL]
// the LM head; moe[l] / moe_grid[l] the layer's fused MoE launch (x = xb, y = x, accum).
// before_moe (optional): called after layer l's router launch and before its MoE launch
// (the residency mode binds the layer's selected experts there); nonzero stops the step.
typedef int (*HybridHook)(void *ctx, int layer);
cudaError_t launch_hybrid_step(HybridParams &p, const HybridLayer *L, GemvParams *g,
                               MoeParams *moe, const int *moe_grid, cudaStream_t st,
                               HybridHook before_moe = nullptr, void *ctx = nullptr,
                               int *hook_status = nullptr);
cudaError_t hybrid_set_attention_smem(int kv_cap);

}  // namespace kq
