/* kq_oracle — CPU restatement of the quantized expert hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker the parity tests, the
 * smoke test and the bench's CPU-baseline leg compare the CUDA plugin against.
 * The plugin never links, loads or calls it.
 *
 * What it restates, and from where (paths inside the reference checkout,
 * vendor/katali_gguf_dense/ abbreviated V/):
 *   - GGUF block layouts and decode: Q4_K V/src/gguf_dtype.c:429-452 with the
 *     6-bit scale/min unpacking of :350-358, Q6_K :487-512, Q8_1 :328-335;
 *     block sizes from the type table :158-180.
 *   - fp16 <-> fp32: the decode direction follows V/include/katali_gguf_fp.h:14-36.
 *     The encode direction here is IEEE round-to-nearest-even (the reference's
 *     katali_f32_to_f16 rounds ties away, :38-57); every encoder in this project
 *     and the plugin use RNE, so both sides produce the same bytes.
 *   - fp32-activation row dot: V/src/gguf_dtype.c:594-624 (per-group sums,
 *     double accumulation across groups).
 *   - SiLU: V/src/gguf_kernels.c:323; softmax: :63-72; greedy argmax
 *     V/src/gguf_sampler.c:62-66 (first strict maximum).
 *
 * What is NOT in the reference checkout and is specified here instead (the
 * reference's MoE engine and CUDA plugin are binary-only, README.md:13,17):
 *   - Q4_K / Q6_K encoders (the checkout has no quantiser): per-group min/scale
 *     fit, 6-bit / 8-bit sub-scales, RNE fp16 super-scales.
 *   - q8_1 activation quantiser: d = amax/127 (fp32), q = roundf(x/d), d and
 *     s = d*sum(q) stored as RNE fp16.
 *   - Integer block dots of Q4_K and Q6_K against q8_1, and their float combine
 *     (exact per-group double terms, double accumulation, one final rounding).
 *   - kq_expf: Cody-Waite reduction by ln2 plus a degree-7 Taylor polynomial,
 *     evaluated with fmaf, so the device and the oracle agree bit for bit.
 *   - Routing: top-k on the raw logits (ties -> lower expert id), weights from
 *     the softmax, optionally renormalised over the selected k.
 *   - The fused MoE layer: route -> q8_1(x) -> gate/up -> silu(g)*u -> q8_1(h)
 *     -> down -> sum_k w_k * down_k, in that order.
 * Parity of these pieces against the reference is "unpinned": the reference
 * ships them only inside katali_cuda.dll / katali-lab.exe.
 */
#ifndef KQ_ORACLE_H
#define KQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { KQO_Q8_1 = 9, KQO_Q4_K = 12, KQO_Q6_K = 14 };

#define KQO_QK_K 256
#define KQO_Q4_K_BYTES 144
#define KQO_Q6_K_BYTES 210
#define KQO_Q8_1_BYTES 36

uint16_t kqo_f32_to_f16(float f);
float    kqo_f16_to_f32(uint16_t h);
float    kqo_expf(float x);
float    kqo_silu(float x);

uint64_t kqo_row_bytes(uint32_t type, uint64_t cols);

/* Decode n elements (multiple of the block size). Returns 0, or -1 on a bad type. */
int kqo_dequant(uint32_t type, const void *src, uint64_t n, float *out);

/* Encoders: n a multiple of 256 (K-quants) or 32 (q8_1). Return 0 or -1. */
int kqo_quantize_q4_K(const float *x, uint64_t n, void *out);
int kqo_quantize_q6_K(const float *x, uint64_t n, void *out);
int kqo_quantize_q8_1(const float *x, uint64_t n, void *out);
int kqo_quantize(uint32_t type, const float *x, uint64_t n, void *out);

/* Integer in-block sums of one weight row against a q8_1 activation row.
 * Q4_K: isum[g] = sum_i q4 * qx and xsum[g] = sum_i qx per 32-element group g
 *       (cols/32 entries each).
 * Q6_K: isum[g] = sum_i (q6-32) * qx per 16-element group (cols/16 entries);
 *       xsum may be NULL. */
int kqo_row_isums(uint32_t type, const void *row, const void *xq, uint64_t cols,
                  int32_t *isum, int32_t *xsum);

/* Row dot against q8_1 activations: exact per-q8-block double terms, double
 * accumulation, rounded once to float. */
float kqo_dot_q8(uint32_t type, const void *row, const void *xq, uint64_t cols);
int   kqo_matvec_q8(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                    const void *xq, float *y);

/* Row dot against fp32 activations (restates V/src/gguf_dtype.c:594-624). */
float kqo_dot_f32(uint32_t type, const void *row, const float *x, uint64_t cols);
int   kqo_matvec_f32(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                     const float *x, float *y);

/* Routing: top-k of n logits. ids[k] in descending-logit order (ties -> lower
 * id), w[k] from the softmax over all n, renormalised over the k when norm. */
int kqo_route_topk(const float *logits, int n, int k, int norm,
                   int32_t *ids, float *w);

/* One MoE layer for one token. Expert e's matrices are at
 *   gate[e] : ffn rows x hidden cols, gate_type
 *   up[e]   : ffn rows x hidden cols, up_type
 *   down[e] : hidden rows x ffn cols, down_type
 * mode 0 = q8_1 activations (the DP4A path), 1 = fp32 activations.
 * ids/w may be NULL; when non-NULL they receive the routing decision.
 * h_out (k*ffn floats) may be NULL; it receives silu(g)*u per selected expert. */
typedef struct KqoMoe {
    int n_experts, hidden, ffn, top_k, norm_topk;
    uint32_t gate_type, up_type, down_type;
    const void *const *gate;
    const void *const *up;
    const void *const *down;
} KqoMoe;

int kqo_moe_layer(const KqoMoe *m, const float *x, const float *logits,
                  float *y, int mode, int32_t *ids, float *w, float *h_out);

/* Same with a given routing (ids/w of length top_k), no softmax/top-k. */
int kqo_moe_layer_routed(const KqoMoe *m, const float *x, const int32_t *ids,
                         const float *w, float *y, int mode, float *h_out);

/* Expert-parallel slot protocol (no counterpart in the reference, whose engine
 * runs on one GPU). Experts split over n_ranks ranks in contiguous blocks of
 * n_experts/n_ranks. A send buffer holds n_ranks*max_tokens slots of
 * kqo_ep_slot_bytes: slot (d, t) at (d*max_tokens + t)*slot_bytes =
 *   int32 n_owned, int32 t, int32 0, int32 0, int32 ids[K], float w[K], padding
 *   to 16 bytes, then the token's q8_1 row (H/32 blocks of 36 B) when n_owned > 0;
 * ids[k] is the global expert id if rank d owns it, else -1. A return buffer
 * holds per slot H doubles: sum over the slot's owned k (in k order) of
 * (double)w_k * (double)down_k(q8(silu(gate_k x) * up_k x)). */
uint32_t kqo_ep_slot_bytes(int hidden, int top_k);
/* Routes and packs this rank's n_tokens tokens; src_ids receives top_k ids per token. */
int kqo_ep_dispatch(const KqoMoe *m, int n_ranks, int max_tokens, int n_tokens,
                    const float *x, const float *logits, uint8_t *send, int32_t *src_ids);
/* Computes every received slot that owns a pair; untouched slots keep ret's contents. */
int kqo_ep_experts(const KqoMoe *m, int n_ranks, int rank, int max_tokens,
                   const uint8_t *recv, double *ret);
/* y[t] = sum over ranks d owning one of t's experts (rank order) of back[d][t]. */
int kqo_ep_combine(const KqoMoe *m, int n_ranks, int max_tokens, int n_tokens,
                   const int32_t *src_ids, const double *back, float *y);

/* Greedy argmax: first index of the strict maximum (V/src/gguf_sampler.c:62-66). */
int kqo_argmax(const float *x, int n);

#ifdef __cplusplus
}
#endif
#endif
