/* katali_cuda.h — C ABI of the B200 (sm_100a) katali_cuda plugin.
 *
 * libkatali_cuda.so is a drop-in for the reference's runtime-loaded CUDA plugin
 * (katali_cuda.dll, loaded with LoadLibrary, README.md:11,313-320). The
 * reference checkout has neither the plugin source nor this header
 * (build-qwen3.bat:5 names the missing src/katali_cuda.c); the entry points in
 * section 1 are reconstructed from their call sites in
 * vendor/katali_gguf_dense/src/katali_dense_cuda.c (abbreviated KDC below),
 * with the same names, argument order and meaning. Sections 2-5 are new.
 *
 * Conventions
 *  - Every int-returning call returns KATALI_OK (0) or a KataliStatus code.
 *    The plugin never falls back to the CPU; the caller decides (KDC:46-55).
 *  - Pointers named *_dev / w / x / y / xq are DEVICE pointers unless the
 *    comment says host. Weights stay in native GGUF block layout.
 *  - Calls are not re-entrant (KDC:8-12 keeps plugin state in globals). They
 *    run on the plugin stream (katali_cuda_set_stream). In the default
 *    synchronous mode each compute call returns after the GPU finished, like
 *    the reference's upload -> matvec -> download sequence; after
 *    katali_cuda_set_async(1) compute calls only enqueue and katali_cuda_sync()
 *    reports errors raised on the device (KATALI_ERR_TIMEOUT).
 */
#ifndef KATALI_CUDA_H
#define KATALI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum KataliStatus {
    KATALI_OK = 0,                    /* success value tested at KDC:27-28,41,52-54 */
    KATALI_ERR_NO_DEVICE = 1,         /* no driver / no sm_100 device */
    KATALI_ERR_OOM = 2,
    KATALI_ERR_BAD_ARG = 3,
    KATALI_ERR_UNSUPPORTED_TYPE = 4,
    KATALI_ERR_UNSUPPORTED_SHAPE = 5,
    KATALI_ERR_TIMEOUT = 6,           /* a bounded device-side wait gave up */
    KATALI_ERR_CUDA = 7,
    KATALI_ERR_NCCL = 8,
    KATALI_ERR_NOT_RESIDENT = 9  /* a call selected an expert with no device copy */
} KataliStatus;

/* GGUF tensor type ids used here (V/include/katali_gguf_dtype.h:20-41). */
#define KATALI_TYPE_Q8_1 9u
#define KATALI_TYPE_Q4_K 12u
#define KATALI_TYPE_Q6_K 14u

/* ------------------------------------------------------------------------ */
/* 1. Entry points the reference already calls (KDC = katali_dense_cuda.c)    */
/* ------------------------------------------------------------------------ */
/* Nonzero when a usable sm_100 device and driver are present (KDC:19). */
int katali_cuda_probe(void);
/* Human-readable reason for the probe result; never NULL (KDC:19). */
const char *katali_cuda_status(void);
/* Device allocation owned by the caller (KDC:27-28,40). 256-byte aligned. */
int katali_cuda_malloc(void **ptr, size_t bytes);
/* Frees a katali_cuda_malloc pointer; NULL is a no-op (KDC:25-26,41,76-78). */
int katali_cuda_free(void *ptr);
/* Host -> device copy of `bytes` (KDC:41,52,65). Synchronous. */
int katali_cuda_upload(void *dev, const void *host, size_t bytes);
/* Device -> host copy of `bytes` (KDC:54,69). Synchronous. */
int katali_cuda_download(void *host, const void *dev, size_t bytes);
/* Nonzero when katali_cuda_matvec accepts this GGUF type (KDC:48,67). */
int katali_cuda_supports_type(uint32_t ggml_type);
/* y[rows] = W x with fp32 activations; W is a GGUF matrix, dims[0] = cols
 * contiguous, dims[1] = rows (KDC:49-53). Q4_K and Q6_K. */
int katali_cuda_matvec(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                       const float *x, float *y);

/* ------------------------------------------------------------------------ */
/* 2. Streams, modes, errors                                                 */
/* ------------------------------------------------------------------------ */
/* Run subsequent work on `stream` (a cudaStream_t); NULL selects the plugin's
 * own non-blocking stream, which is not ordered with the legacy default
 * stream: to share the legacy default stream pass cudaStreamLegacy. */
int katali_cuda_set_stream(void *stream);
/* 0 (default): compute calls synchronise before returning. 1: enqueue only. */
int katali_cuda_set_async(int on);
/* Wait for the plugin stream; returns and clears any device-side error. */
int katali_cuda_sync(void);
/* Name of a status code. */
const char *katali_cuda_strerror(int status);

/* ------------------------------------------------------------------------ */
/* 3. Dense GEMV family                                                      */
/* ------------------------------------------------------------------------ */
/* n (<= 8) projections sharing one x and cols, in ONE launch; replaces the
 * per-projection loop of katali_dense_cuda_matvec_multi (KDC:58-73) and mirrors
 * the CPU katali_ggml_matvec_fused (V/src/gguf_dtype.c:925-985). */
int katali_cuda_matvec_multi(int n, const uint32_t *types, const void *const *w,
                             const uint64_t *rows, uint64_t cols, const float *x,
                             float *const *y);
/* Quantise n fp32 values (n % 32 == 0) to GGUF q8_1 blocks (36 B per 32);
 * xq 4-byte aligned. */
int katali_cuda_quantize_q8_1(const float *x, uint64_t n, void *xq);
/* y = W xq with q8_1 activations (the DP4A path, README.md:17). */
int katali_cuda_matvec_q8_1(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                            const void *xq, float *y);
/* Encode rows x cols fp32 (device) into GGUF blocks of `type` (Q4_K, Q6_K,
 * Q8_1) at dst. Byte-identical to the CPU encoder of the test oracle. */
int katali_cuda_quantize_rows(uint32_t type, const float *src, uint64_t rows,
                              uint64_t cols, void *dst);

/* ------------------------------------------------------------------------ */
/* 4. Fused MoE layer ("one GPU call per MoE layer", README.md:13,17)         */
/* ------------------------------------------------------------------------ */
typedef struct KataliMoe KataliMoe;

/* Activation modes. */
#define KATALI_MOE_Q8_1 0u   /* x and h quantised to q8_1, integer block dots */
#define KATALI_MOE_F32  1u   /* fp32 activations (parity with the CPU kernels) */
/* Descriptor flags. */
#define KATALI_MOE_NORM_TOPK 1u  /* renormalise the top-k softmax weights */

typedef struct KataliMoeDesc {
    uint32_t n_experts;   /* <= 1024 */
    uint32_t hidden;      /* H: gate/up cols, down rows; multiple of 256 */
    uint32_t ffn;         /* F: gate/up rows, down cols; multiple of 256 */
    uint32_t top_k;       /* 1..16 */
    uint32_t gate_type, up_type, down_type;  /* Q4_K, Q4_K, Q6_K */
    uint32_t flags;       /* KATALI_MOE_NORM_TOPK */
    /* HOST array of 3*n_experts device pointers: gate_e, up_e, down_e for each
     * expert e (16-byte aligned). NULL leaves every expert unset. A NULL entry
     * is an expert that is not resident: a call that selects it returns
     * KATALI_ERR_NOT_RESIDENT (checked on the device; nothing is read). */
    const void *const *experts;
} KataliMoeDesc;

int katali_cuda_moe_create(const KataliMoeDesc *desc, KataliMoe **out);
/* Point expert e at resident device copies (used by the residency tier). */
int katali_cuda_moe_set_expert(KataliMoe *m, uint32_t e, const void *gate,
                               const void *up, const void *down);
int katali_cuda_moe_destroy(KataliMoe *m);
/* One token: y[H] = sum_k w_k * down_ek(silu(gate_ek x) * up_ek x), with
 * (e_k, w_k) the top-k of softmax(router_logits[n_experts]). One launch. A layer
 * shape whose single-launch plan does not fit shared memory (e.g. FFN 768) runs
 * the ragged-batch pipeline with one token instead (q8_1 mode; in fp32 mode such
 * shapes return KATALI_ERR_UNSUPPORTED_SHAPE). */
int katali_cuda_moe_layer(KataliMoe *m, const float *x, const float *router_logits,
                          float *y, uint32_t mode);
/* Same with routing given: ids[top_k] (int32), w[top_k] (fp32). */
int katali_cuda_moe_layer_routed(KataliMoe *m, const float *x, const int32_t *ids,
                                 const float *w, float *y, uint32_t mode);
/* A ragged continuous batch (the step of a server whose live sequence count
 * changes every step; the reference engine's per-token calls, README.md:13,17,
 * batched): x[n_tokens][H], router_logits[n_tokens][n_experts],
 * y[n_tokens][H], row-major device buffers. Each token is routed as in
 * katali_cuda_moe_layer; the (token, expert) pairs are grouped by expert so
 * every selected expert's rows are read once per call. Row t of y equals
 * katali_cuda_moe_layer on row t up to the order of double additions. Experts
 * with many of the batch's pairs run on the tensor cores: from 8 pairs the Q6_K
 * down projection (exact integer block sums accumulated in double, each row
 * equal to the reference's Q6_K x q8_1 dot), from 16 pairs also the Q4_K
 * gate/up (fp32 block terms: the layer output then within a relative L2 of 5e-4).
 * The environment variable KATALI_CUDA_NO_TC=1 keeps every expert on the
 * other kernels.
 * mode: KATALI_MOE_Q8_1 only (else KATALI_ERR_UNSUPPORTED_TYPE). Scratch is
 * allocated on the layer object on first use and grown when n_tokens grows. */
#define KATALI_MOE_BATCH_MAX_TOKENS 4096
int katali_cuda_moe_batch(KataliMoe *m, uint32_t n_tokens, const float *x,
                          const float *router_logits, float *y, uint32_t mode);

/* No-allocation variant of katali_cuda_moe_layer. No counterpart in the
 * reference. For callers that cannot allocate device memory when a layer runs
 * (device memory owned by another allocator, a host that forbids allocations
 * after start-up, or a fixed memory budget): nothing is allocated; the expert
 * table (copied from desc->experts, a HOST array of 3*n_experts device
 * pointers), the h records and the barrier counters live in a file-scope device
 * array of about 89 KB that every GPU loading the library keeps until exit.
 * Limits: n_experts <= KATALI_MOE_STATIC_MAX_EXPERTS and
 * top_k * ffn <= KATALI_MOE_STATIC_MAX_TOPK_FFN, else
 * KATALI_ERR_UNSUPPORTED_SHAPE (katali_cuda_status() says which). Runs on
 * `stream` (a cudaStream_t, NULL = default stream) and is synchronous: it
 * returns after the layer finished, with the kernel's status read back. The first call on a device looks the array up for that device:
 * make it before any stream capture. All calls share the array, so calls that
 * overlap on the GPU race; serialise them. */
#define KATALI_MOE_STATIC_MAX_EXPERTS 1024
#define KATALI_MOE_STATIC_MAX_TOPK_FFN 16384
int katali_cuda_moe_layer_static(const KataliMoeDesc *desc, const float *x,
                                 const float *router_logits, float *y, uint32_t mode,
                                 void *stream);

/* ------------------------------------------------------------------------ */
/* 6. Expert parallelism: experts split over n_ranks GPUs, one process each   */
/* ------------------------------------------------------------------------ */
/* Rank r holds experts [r*E/n_ranks, (r+1)*E/n_ranks) of a layer (the other
 * entries of its KataliMoe table may stay NULL); every rank calls with its own
 * tokens (at most max_tokens, the same max_tokens on every rank). The call is
 * three stages around two all-to-all exchanges of fixed-size slots:
 *   dispatch: route + q8_1 + one slot per (destination rank, token) -> send
 *   exchange: recv[d] = what rank d sent to this rank (n_ranks*max_tokens slots)
 *   experts : every received slot's pairs on this rank's experts -> ret
 *             (per slot: sum over its owned experts, in top-k order, of
 *             w_k * down_k(silu(gate_k x) * up_k x), as H doubles)
 *   exchange: back[d] = what rank d returned for this rank's tokens
 *   combine : y[t] = sum over ranks (rank order) of back[d][t], to fp32.
 * Buffers are device memory, 16-byte aligned: send/recv n_ranks*max_tokens*
 * slot_bytes, ret/back n_ranks*max_tokens*ret_slot_bytes. Slot (d, t) is at
 * (d*max_tokens + t)*slot_bytes. combine must follow the dispatch of the same
 * tokens on the same KataliMoe. Row t of y equals katali_cuda_moe_batch's up
 * to the order of double additions. No counterpart in the reference (its
 * engine runs on one GPU); the expert-parallel step is an extension. */
int katali_cuda_moe_ep_slot_bytes(KataliMoe *m, uint64_t *slot_bytes,
                                  uint64_t *ret_slot_bytes);
int katali_cuda_moe_ep_dispatch(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens,
                                uint32_t n_tokens, const float *x,
                                const float *router_logits, void *send);
int katali_cuda_moe_ep_experts(KataliMoe *m, uint32_t n_ranks, uint32_t rank,
                               uint32_t max_tokens, const void *recv, void *ret);
int katali_cuda_moe_ep_combine(KataliMoe *m, uint32_t n_ranks, uint32_t max_tokens,
                               uint32_t n_tokens, const void *back, float *y);

/* The same step with both exchanges done by NCCL inside the plugin (grouped
 * ncclSend/ncclRecv on the plugin stream; libnccl.so.2 is opened at run time).
 * Rank 0 makes a 128-byte id with katali_cuda_ep_unique_id and hands it to every
 * rank by its own means; every rank then calls katali_cuda_ep_create on its
 * GPU. A failed NCCL call returns KATALI_ERR_NCCL. */
typedef struct KataliEp KataliEp;
int katali_cuda_ep_unique_id(void *id128);
int katali_cuda_ep_create(uint32_t n_ranks, uint32_t rank, const void *id128, KataliEp **out);
int katali_cuda_ep_destroy(KataliEp *ep);
int katali_cuda_moe_ep_layer(KataliMoe *m, KataliEp *ep, uint32_t max_tokens,
                             uint32_t n_tokens, const float *x, const float *router_logits,
                             float *y);
/* on != 0: later katali_cuda_moe_ep_layer calls exchange over NVLink peer memory
 * instead of NCCL: the dispatch kernel stores each slot straight into the owner
 * rank's receive window and the experts kernel stores each partial sum straight
 * into the source rank's window, each signalled by a flag the reader polls with
 * a bounded wait (a wait that runs out returns KATALI_ERR_TIMEOUT). The windows
 * are allocated and mapped between the ranks (CUDA IPC) by the first such call,
 * collectively, for that call's layer shape and max_tokens. */
int katali_cuda_ep_use_peer_memory(KataliEp *ep, int on);

/* ------------------------------------------------------------------------ */
/* 7. Expert residency tier (the reference's expert cache, README.md:13,21,   */
/*    329-333; its API is binary-only, these entry points are new)           */
/* ------------------------------------------------------------------------ */
/* n_slots device slots of slot_bytes each; one slot holds one expert's gate,
 * up and down matrices (native GGUF bytes, each 16-byte aligned in the slot).
 * Uploads run on the cache's own stream; the compute stream waits on events. */
typedef struct KataliExpertCache KataliExpertCache;
int katali_cuda_expert_cache_create(uint64_t slot_bytes, uint32_t n_slots,
                                    KataliExpertCache **out);
/* Layers still bound to the cache see their bound experts as not resident. */
int katali_cuda_expert_cache_destroy(KataliExpertCache *c);
/* Registers expert `key` (any caller id, e.g. layer * n_experts + e) with its
 * borrowed HOST matrices (e.g. inside an mmap'd GGUF file; they must stay
 * valid). The ranges are page-locked when possible so uploads are async. */
int katali_cuda_expert_register(KataliExpertCache *c, uint64_t key, const void *gate,
                                uint64_t gate_bytes, const void *up, uint64_t up_bytes,
                                const void *down, uint64_t down_bytes);
/* Starts the upload of `key` into a free or least-recently-used slot and
 * returns at once (a resident key is only marked used). A refilled slot's
 * upload waits for every compute call enqueued before it. */
int katali_cuda_expert_prefetch_async(KataliExpertCache *c, uint64_t key);
/* Makes expert e of layer m use the device copy of `key` (uploading it if
 * needed): compute calls enqueued after this wait for the upload. When the
 * slot is later refilled or evicted, the entry becomes NULL (not resident). */
int katali_cuda_expert_bind(KataliExpertCache *c, uint64_t key, KataliMoe *m, uint32_t e);
/* Drops `key` from the device; its bindings become NULL. */
int katali_cuda_expert_evict(KataliExpertCache *c, uint64_t key);
/* *resident = 1 when `key` is on the device (its slot's pointers returned in
 * gate/up/down, each may be NULL), else 0. */
int katali_cuda_expert_lookup(KataliExpertCache *c, uint64_t key, int *resident, void **gate,
                              void **up, void **down);
/* Waits for every upload started so far. */
int katali_cuda_expert_sync(KataliExpertCache *c);

/* ------------------------------------------------------------------------ */
/* 8. Dense decoder decode on the device (the reference's dense CPU forward,  */
/*    V/src/gguf_model.c:570-703, with its per-projection GPU crossings       */
/*    removed; README.md:164-171). Qwen3 layout: RMSNorm, q/k/v, per-head q/k  */
/*    RMSNorm, RoPE, GQA with an fp32 KV cache, o + residual, RMSNorm,         */
/*    gate/up, SiLU * up, down + residual, final RMSNorm, LM head, greedy.     */
/* ------------------------------------------------------------------------ */
typedef struct KataliDenseLayerW {
    const float *attn_norm, *ffn_norm;  /* device fp32, hidden entries */
    const float *q_norm, *k_norm;       /* device fp32, head_dim entries, or NULL */
    const void *wq, *wk, *wv, *wo, *gate, *up, *down;  /* device GGUF matrices */
    uint32_t wq_type, wk_type, wv_type, wo_type, gate_type, up_type, down_type;
} KataliDenseLayerW;

typedef struct KataliDenseDesc {
    uint32_t n_layers, hidden, ffn, n_heads, n_kv_heads, head_dim, vocab;
    uint32_t kv_cap;    /* positions in the KV cache (<= 51200) */
    uint32_t rope_dim;  /* 0 = head_dim */
    float rms_eps, rope_theta;
    const void *embed;  /* device, vocab rows of `hidden` (embed_type) */
    uint32_t embed_type;
    const float *out_norm;  /* device fp32, hidden entries */
    const void *lm_head;    /* device, vocab rows of `hidden` (lm_head_type) */
    uint32_t lm_head_type;
    const KataliDenseLayerW *layers;  /* HOST array of n_layers (copied) */
    uint32_t flags;  /* KATALI_DENSE_Q8_1: projections with q8_1 activations (DP4A) */
} KataliDenseDesc;
/* Projections quantise their fp32 input to q8_1 on the device and use integer
 * block dots (the reference's KATALI_CUDA_DP4A mode, README.md:17); default:
 * fp32 activations, the parity mode against the CPU path. */
#define KATALI_DENSE_Q8_1 1u

typedef struct KataliDense KataliDense;
int katali_cuda_dense_create(const KataliDenseDesc *desc, KataliDense **out);
int katali_cuda_dense_destroy(KataliDense *m);
/* Empties the KV cache (next position 0). */
int katali_cuda_dense_reset(KataliDense *m);
/* Greedy decode continuing at the current position: feeds prompt[0..n_prompt)
 * (HOST ints), then feeds back each argmax; out_tokens (HOST) receives the
 * n_gen generated tokens (the argmax after the last prompt token first). The
 * whole loop stays on the device (one graph replay per step). */
int katali_cuda_dense_generate(KataliDense *m, const int32_t *prompt, uint32_t n_prompt,
                               uint32_t n_gen, int32_t *out_tokens);
/* Device pointer to the logits of the last step (vocab floats) and the next
 * position. */
int katali_cuda_dense_logits(KataliDense *m, const float **logits_dev, int32_t *position);

/* ------------------------------------------------------------------------ */
/* 9. Hybrid MoE decoder decode on the device: Gated DeltaNet (linear        */
/*    attention) and gated full-attention layers, each followed by the fused  */
/*    MoE block — the Qwen3.5/3.6-35B-A3B layer family the reference runs     */
/*    with KATALI_CUDA_MOE=1 / KATALI_CUDA_GDN=1 (README.md:15,19,322-336;    */
/*    binary-only there, so these entry points are new). Per layer: RMSNorm,  */
/*    the mixer (GDN or gated attention) + residual, RMSNorm, fp32 router,    */
/*    top-k MoE + residual; then final RMSNorm, LM head, greedy argmax.       */
/* ------------------------------------------------------------------------ */
#define KATALI_HYBRID_GDN 0u   /* Gated DeltaNet layer */
#define KATALI_HYBRID_ATTN 1u  /* gated full-attention layer */

typedef struct KataliHybridLayerW {
    uint32_t kind;                 /* KATALI_HYBRID_GDN or KATALI_HYBRID_ATTN */
    const float *attn_norm;        /* device fp32 [hidden]: RMSNorm before the mixer */
    const float *ffn_norm;         /* device fp32 [hidden]: RMSNorm before the MoE block */
    const float *router;           /* device fp32 [n_experts][hidden] router rows */
    KataliMoe *moe;                /* the layer's experts (katali_cuda_moe_create) */
    /* GDN: in-projections (cols hidden) q|k|v (rows 2 nk dk + nv dv), z (nv dv),
     * b (nv), a (nv); out projection (rows hidden, cols nv dv) */
    const void *ssm_qkv, *ssm_z, *ssm_b, *ssm_a, *ssm_out;
    uint32_t ssm_qkv_type, ssm_z_type, ssm_b_type, ssm_a_type, ssm_out_type;
    const float *ssm_conv;         /* device fp32 [2 nk dk + nv dv][ssm_conv] */
    const float *ssm_a_log;        /* device fp32 [nv] */
    const float *ssm_dt_bias;      /* device fp32 [nv] */
    const float *ssm_norm;         /* device fp32 [dv]: gated RMSNorm weight */
    /* attention: wq rows n_heads * 2 head_dim (per head: q rows, then gate rows),
     * wk / wv rows n_kv_heads * head_dim, wo rows hidden (cols n_heads * head_dim) */
    const void *wq, *wk, *wv, *wo;
    uint32_t wq_type, wk_type, wv_type, wo_type;
    const float *q_norm, *k_norm;  /* device fp32 [head_dim], or NULL */
    /* GDN, optional: device fp32 [nv] decay rates A = -exp(A_log) as GGUF files store them
     * (tensor ssm_a); when set the recurrence uses -A in place of exp(ssm_a_log), which
     * may then be NULL. */
    const float *ssm_decay;
} KataliHybridLayerW;

typedef struct KataliHybridDesc {
    uint32_t n_layers, hidden, vocab;
    uint32_t kv_cap;               /* positions of the attention layers' KV cache */
    uint32_t n_heads, n_kv_heads, head_dim, rope_dim;  /* rope_dim 0 = head_dim */
    float rms_eps, rope_theta;
    uint32_t ssm_k_heads, ssm_v_heads, ssm_head_dim, ssm_conv;  /* dk = dv = ssm_head_dim */
    const void *embed;             /* device, vocab rows of `hidden` (embed_type) */
    uint32_t embed_type;
    const float *out_norm;         /* device fp32 [hidden] */
    const void *lm_head;           /* device, vocab rows of `hidden` (lm_head_type) */
    uint32_t lm_head_type;
    const KataliHybridLayerW *layers;  /* HOST array of n_layers (copied) */
    uint32_t flags;                /* KATALI_DENSE_Q8_1: q8_1 activations in the projections
                                      and the MoE block (DP4A); default fp32 (parity mode) */
} KataliHybridDesc;
/* Supported: ssm_head_dim 128, ssm_v_heads a multiple of ssm_k_heads, ssm_conv
 * 2..8, head_dim <= 256 and a multiple of 32, hidden <= 8192 (multiple of 256),
 * every layer's MoE with the decoder's hidden size and a fused single-launch
 * plan; else KATALI_ERR_UNSUPPORTED_SHAPE. The MoE objects stay owned by the
 * caller and must outlive the decoder. */
typedef struct KataliHybrid KataliHybrid;
int katali_cuda_hybrid_create(const KataliHybridDesc *desc, KataliHybrid **out);
int katali_cuda_hybrid_destroy(KataliHybrid *m);
/* Empties the KV cache and zeroes the recurrent (GDN) and conv states. */
int katali_cuda_hybrid_reset(KataliHybrid *m);
/* Greedy decode as katali_cuda_dense_generate (one graph replay per step). A decoder whose
 * experts are fed by a residency cache (katali_cuda_hybrid_create_from_gguf with a cache)
 * runs each step layer by layer instead: after a layer's router the routing decision is read
 * back, the selected experts are bound through the cache (uploading the ones not on the
 * device from the file's mapping on the cache's stream), then the MoE block runs. */
int katali_cuda_hybrid_generate(KataliHybrid *m, const int32_t *prompt, uint32_t n_prompt,
                                uint32_t n_gen, int32_t *out_tokens);
int katali_cuda_hybrid_logits(KataliHybrid *m, const float **logits_dev, int32_t *position);
/* Expert parallelism for the MoE blocks (collective: every rank of ep calls it, then
 * every rank runs the same sequence of generate calls, each with its own sequence).
 * Rank r's KataliMoe tables hold experts [r E/G, (r+1) E/G) of every layer (others
 * NULL); each layer's MoE block then runs as the single-launch expert-parallel layer
 * over NVLink peer memory (ep in peer-memory mode, katali_cuda_ep_use_peer_memory):
 * the token's slot goes to the owners of its top-k experts, which return per-slot
 * partial sums. Needs KATALI_DENSE_Q8_1. ep NULL: back to the local MoE launches. */
int katali_cuda_hybrid_set_ep(KataliHybrid *m, KataliEp *ep);

/* ------------------------------------------------------------------------ */
/* 10. GGUF container: parse a model file and upload tensors to the device in */
/*     their native block layout (the reference's reader, katali_gguf_open /  */
/*     katali_gguf_find_tensor / katali_gguf_get_*, V/include/katali_gguf.h:  */
/*     117-152, V/src/gguf_reader.c:351-545, feeding its backends as           */
/*     V/src/gguf_model.c:187-227 does). GGUF v2 and v3.                        */
/* ------------------------------------------------------------------------ */
typedef struct KataliGguf KataliGguf;
typedef struct KataliGgufTensorInfo {
    const char *name;   /* NUL-terminated, owned by the reader until close */
    uint32_t type;      /* ggml type id */
    uint32_t n_dims;    /* 1..4 */
    uint64_t dims[4];   /* dims[0] contiguous; unused dims are 1 */
    uint64_t offset;    /* absolute file offset of the tensor's bytes */
    uint64_t nbytes;    /* 0 for a type the reader does not size (not uploadable) */
} KataliGgufTensorInfo;
/* Maps the file read-only and parses its directory. A malformed file (bad magic
 * or version, truncation, nested arrays, misaligned or out-of-range tensor data)
 * returns KATALI_ERR_BAD_ARG and katali_cuda_status() says why. No GPU needed. */
int katali_cuda_gguf_open(const char *path, KataliGguf **out);
int katali_cuda_gguf_close(KataliGguf *g);
int katali_cuda_gguf_counts(const KataliGguf *g, uint64_t *n_tensors, uint64_t *n_kv,
                            uint32_t *version);
int katali_cuda_gguf_tensor(const KataliGguf *g, uint64_t index, KataliGgufTensorInfo *info);
/* KATALI_ERR_BAD_ARG when no tensor has that name. */
int katali_cuda_gguf_find(const KataliGguf *g, const char *name, uint64_t *index);
/* Metadata. get_int: integer and bool scalars; get_float: any numeric scalar;
 * get_str: string value, not NUL-terminated (len bytes, points into the mapping);
 * array: element type and count; array_int: element i of an integer array.
 * A missing key or a type mismatch returns KATALI_ERR_BAD_ARG. */
int katali_cuda_gguf_get_int(const KataliGguf *g, const char *key, int64_t *value);
int katali_cuda_gguf_get_float(const KataliGguf *g, const char *key, double *value);
int katali_cuda_gguf_get_str(const KataliGguf *g, const char *key, const char **value,
                             uint64_t *len);
int katali_cuda_gguf_array(const KataliGguf *g, const char *key, uint32_t *elem_type,
                           uint64_t *count);
int katali_cuda_gguf_array_int(const KataliGguf *g, const char *key, uint64_t i, int64_t *value);
/* Copies tensor `index`'s nbytes, unchanged, to device memory dev (e.g. from
 * katali_cuda_malloc) on the plugin stream through pinned staging buffers;
 * returns after the copy has finished. */
int katali_cuda_gguf_upload(KataliGguf *g, uint64_t index, void *dev);
/* The on-device dense decoder (section 8) of a qwen3-architecture file: dimensions from
 * the metadata (qwen3.block_count, embedding_length, feed_forward_length,
 * attention.head_count[_kv], attention.key_length, rope.freq_base,
 * attention.layer_norm_rms_epsilon, rope.dimension_count), tensors by their llama.cpp
 * names (token_embd, output_norm, output — the embedding when absent —, blk.N.attn_norm,
 * attn_q, attn_k, attn_v, attn_output, attn_q_norm, attn_k_norm, ffn_norm, ffn_gate,
 * ffn_up, ffn_down), uploaded unchanged into one device allocation that the decoder owns
 * (freed by katali_cuda_dense_destroy). The file may be closed afterwards. A missing
 * tensor or metadata key, or an fp32 norm of the wrong size, returns KATALI_ERR_BAD_ARG;
 * another architecture KATALI_ERR_UNSUPPORTED_SHAPE; matrices of other types
 * KATALI_ERR_UNSUPPORTED_TYPE. flags as KataliDenseDesc.flags. */
int katali_cuda_dense_create_from_gguf(KataliGguf *g, uint32_t kv_cap, uint32_t flags,
                                       KataliDense **out);
/* The on-device hybrid MoE decoder (section 9) of a qwen35moe-architecture file (Gated
 * DeltaNet and gated-attention layers, each followed by a routed-expert block; the names
 * and layout of llama.cpp's conversion of that family). Metadata (prefix qwen35moe.):
 * block_count, embedding_length, attention.head_count[_kv], attention.key_length,
 * rope.dimension_count, rope.freq_base, attention.layer_norm_rms_epsilon, expert_count,
 * expert_used_count, expert_feed_forward_length, ssm.conv_kernel, ssm.state_size,
 * ssm.group_count, ssm.time_step_rank, ssm.inner_size, expert_weights_norm (default 1).
 * Tensors: token_embd, output_norm, output (the embedding when absent); per layer
 * blk.N.attn_norm, post_attention_norm, ffn_gate_inp (fp32 router, [hidden, experts]),
 * the stacked experts ffn_gate_exps / ffn_up_exps ([hidden, ffn, experts]) and
 * ffn_down_exps ([ffn, hidden, experts]); a GDN layer attn_qkv, attn_gate (z),
 * ssm_beta, ssm_alpha, ssm_out, ssm_conv1d (fp32 [conv, channels]), ssm_a (fp32 A =
 * -exp(A_log)), ssm_dt.bias, ssm_norm; an attention layer attn_q (query and gate rows per
 * head), attn_k, attn_v, attn_output, attn_q_norm, attn_k_norm. Shared-expert tensors
 * (ffn_*_shexp) are not supported (KATALI_ERR_UNSUPPORTED_SHAPE).
 * cache NULL: every tensor, experts included, is uploaded unchanged into device memory the
 * decoder owns. cache non-NULL: the experts stay in the file's read-only mapping, registered
 * with the cache under key = layer * expert_count + e (slot_bytes must hold one expert), and
 * are uploaded on demand by katali_cuda_hybrid_generate; the file and the cache must outlive
 * the decoder. The decoder owns the MoE objects it creates (freed by
 * katali_cuda_hybrid_destroy). Errors as katali_cuda_dense_create_from_gguf. */
int katali_cuda_hybrid_create_from_gguf(KataliGguf *g, uint32_t kv_cap, uint32_t flags,
                                        KataliExpertCache *cache, KataliHybrid **out);

/* ------------------------------------------------------------------------ */
/* 5. Checks (the cuda-check / cuda-dp4a-selftest family, README.md:99-102)  */
/* ------------------------------------------------------------------------ */
/* Integer in-block sums of every row against q8_1 xq. Q4_K: per 32-group
 * isum and xsum (rows x cols/32 each); Q6_K: per 16-group isum
 * (rows x cols/16), xsum may be NULL. */
int katali_cuda_debug_row_isums(uint32_t type, const void *w, uint64_t rows,
                                uint64_t cols, const void *xq, int32_t *isum,
                                int32_t *xsum);
/* Phase timeline of subsequent katali_cuda_moe_layer calls: when trace is a
 * device buffer of (*grid) * 32 uint64, every CTA writes %globaltimer (ns) at
 * start, routed, x staged, loads issued, first gate/up chunk landed, gate/up
 * done, barrier passed, down rows landed, end (slots 0-8), phase details in
 * slots 9-15 and 18-31 (the expert-parallel layer's exchange steps and its
 * first round), and the SM cycle counter at start and end (slots 16, 17).
 * NULL switches tracing off. *grid receives the launch's CTA count. */
int katali_cuda_debug_moe_trace(KataliMoe *m, uint64_t *trace, int *grid);
/* The MoE kernel's routing decision for router_logits: ids/w of top_k. */
int katali_cuda_debug_route(KataliMoe *m, const float *router_logits, int32_t *ids,
                            float *w);

#ifdef __cplusplus
}
#endif
#endif /* KATALI_CUDA_H */
