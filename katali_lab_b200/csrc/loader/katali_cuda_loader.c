/* katali_cuda_loader.c — runtime discovery of the CUDA plugin (Linux).
 *
 * The reference engine links no CUDA library; its loader (src/katali_cuda.c,
 * named by build-qwen3.bat:5 but absent from the checkout) finds
 * katali_cuda.dll with LoadLibrary at run time, honours KATALI_CUDA_DLL and
 * KATALI_CUDA=0, and reports why the GPU is unavailable instead of failing
 * (README.md:11,296-303,320). This is the same contract with dlopen/dlsym:
 * link this file (or libkatali_cuda_loader.so) into the engine and every
 * katali_cuda_* call forwards to libkatali_cuda.so when it can be loaded;
 * otherwise katali_cuda_probe() returns 0, katali_cuda_status() says why and
 * every other call returns KATALI_ERR_NO_DEVICE, so the caller stays on its
 * CPU path (vendor/katali_gguf_dense/src/katali_dense_cuda.c:14-22,46-55).
 *
 * Search order: $KATALI_CUDA_DLL, then libkatali_cuda.so beside this loader,
 * then the dynamic linker's default path.
 */
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include <dlfcn.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "katali_cuda.h"

#define KATALI_FN_LIST(X)                                                                     \
    X(int, katali_cuda_probe, (void), ())                                                     \
    X(const char *, katali_cuda_status, (void), ())                                           \
    X(int, katali_cuda_malloc, (void **p, size_t n), (p, n))                                  \
    X(int, katali_cuda_free, (void *p), (p))                                                  \
    X(int, katali_cuda_upload, (void *d, const void *h, size_t n), (d, h, n))                 \
    X(int, katali_cuda_download, (void *h, const void *d, size_t n), (h, d, n))               \
    X(int, katali_cuda_supports_type, (uint32_t t), (t))                                      \
    X(int, katali_cuda_matvec,                                                                \
      (uint32_t t, const void *w, uint64_t r, uint64_t c, const float *x, float *y),          \
      (t, w, r, c, x, y))                                                                     \
    X(int, katali_cuda_set_stream, (void *s), (s))                                            \
    X(int, katali_cuda_set_async, (int on), (on))                                             \
    X(int, katali_cuda_sync, (void), ())                                                      \
    X(const char *, katali_cuda_strerror, (int s), (s))                                       \
    X(int, katali_cuda_matvec_multi,                                                          \
      (int n, const uint32_t *t, const void *const *w, const uint64_t *r, uint64_t c,         \
       const float *x, float *const *y),                                                      \
      (n, t, w, r, c, x, y))                                                                  \
    X(int, katali_cuda_quantize_q8_1, (const float *x, uint64_t n, void *q), (x, n, q))       \
    X(int, katali_cuda_matvec_q8_1,                                                           \
      (uint32_t t, const void *w, uint64_t r, uint64_t c, const void *q, float *y),           \
      (t, w, r, c, q, y))                                                                     \
    X(int, katali_cuda_quantize_rows,                                                         \
      (uint32_t t, const float *s, uint64_t r, uint64_t c, void *d), (t, s, r, c, d))         \
    X(int, katali_cuda_moe_create, (const KataliMoeDesc *d, KataliMoe **o), (d, o))           \
    X(int, katali_cuda_moe_set_expert,                                                        \
      (KataliMoe * m, uint32_t e, const void *g, const void *u, const void *d),               \
      (m, e, g, u, d))                                                                        \
    X(int, katali_cuda_moe_destroy, (KataliMoe * m), (m))                                     \
    X(int, katali_cuda_moe_layer,                                                             \
      (KataliMoe * m, const float *x, const float *l, float *y, uint32_t mo),                 \
      (m, x, l, y, mo))                                                                       \
    X(int, katali_cuda_moe_layer_routed,                                                      \
      (KataliMoe * m, const float *x, const int32_t *i, const float *w, float *y,             \
       uint32_t mo),                                                                          \
      (m, x, i, w, y, mo))                                                                    \
    X(int, katali_cuda_moe_batch,                                                             \
      (KataliMoe * m, uint32_t n, const float *x, const float *l, float *y, uint32_t mo),     \
      (m, n, x, l, y, mo))                                                                    \
    X(int, katali_cuda_moe_ep_slot_bytes, (KataliMoe * m, uint64_t *s, uint64_t *r),          \
      (m, s, r))                                                                              \
    X(int, katali_cuda_moe_ep_dispatch,                                                       \
      (KataliMoe * m, uint32_t g, uint32_t tm, uint32_t n, const float *x, const float *l,    \
       void *s),                                                                              \
      (m, g, tm, n, x, l, s))                                                                 \
    X(int, katali_cuda_moe_ep_experts,                                                        \
      (KataliMoe * m, uint32_t g, uint32_t r, uint32_t tm, const void *i, void *o),           \
      (m, g, r, tm, i, o))                                                                    \
    X(int, katali_cuda_moe_ep_combine,                                                        \
      (KataliMoe * m, uint32_t g, uint32_t tm, uint32_t n, const void *b, float *y),          \
      (m, g, tm, n, b, y))                                                                    \
    X(int, katali_cuda_expert_cache_create, (uint64_t b, uint32_t n, KataliExpertCache **o),  \
      (b, n, o))                                                                              \
    X(int, katali_cuda_expert_cache_destroy, (KataliExpertCache * c), (c))                    \
    X(int, katali_cuda_expert_register,                                                       \
      (KataliExpertCache * c, uint64_t k, const void *g, uint64_t gb, const void *u,          \
       uint64_t ub, const void *d, uint64_t db),                                              \
      (c, k, g, gb, u, ub, d, db))                                                            \
    X(int, katali_cuda_expert_prefetch_async, (KataliExpertCache * c, uint64_t k), (c, k))    \
    X(int, katali_cuda_expert_bind, (KataliExpertCache * c, uint64_t k, KataliMoe * m,        \
                                     uint32_t e),                                             \
      (c, k, m, e))                                                                           \
    X(int, katali_cuda_expert_evict, (KataliExpertCache * c, uint64_t k), (c, k))             \
    X(int, katali_cuda_expert_lookup,                                                         \
      (KataliExpertCache * c, uint64_t k, int *r, void **g, void **u, void **d),              \
      (c, k, r, g, u, d))                                                                     \
    X(int, katali_cuda_expert_sync, (KataliExpertCache * c), (c))                             \
    X(int, katali_cuda_dense_create, (const KataliDenseDesc *d, KataliDense **o), (d, o))     \
    X(int, katali_cuda_dense_destroy, (KataliDense * m), (m))                                 \
    X(int, katali_cuda_dense_reset, (KataliDense * m), (m))                                   \
    X(int, katali_cuda_dense_generate,                                                        \
      (KataliDense * m, const int32_t *p, uint32_t np, uint32_t ng, int32_t *o),              \
      (m, p, np, ng, o))                                                                      \
    X(int, katali_cuda_dense_logits, (KataliDense * m, const float **l, int32_t *p),          \
      (m, l, p))                                                                              \
    X(int, katali_cuda_hybrid_create, (const KataliHybridDesc *d, KataliHybrid **o), (d, o))  \
    X(int, katali_cuda_hybrid_destroy, (KataliHybrid * m), (m))                               \
    X(int, katali_cuda_hybrid_reset, (KataliHybrid * m), (m))                                 \
    X(int, katali_cuda_hybrid_generate,                                                       \
      (KataliHybrid * m, const int32_t *p, uint32_t np, uint32_t ng, int32_t *o),             \
      (m, p, np, ng, o))                                                                      \
    X(int, katali_cuda_hybrid_logits, (KataliHybrid * m, const float **l, int32_t *p),        \
      (m, l, p))                                                                              \
    X(int, katali_cuda_hybrid_set_ep, (KataliHybrid * m, KataliEp * e), (m, e))               \
    X(int, katali_cuda_gguf_open, (const char *p, KataliGguf **o), (p, o))                    \
    X(int, katali_cuda_gguf_close, (KataliGguf * g), (g))                                     \
    X(int, katali_cuda_gguf_counts, (const KataliGguf *g, uint64_t *t, uint64_t *k,          \
                                     uint32_t *v),                                            \
      (g, t, k, v))                                                                           \
    X(int, katali_cuda_gguf_tensor, (const KataliGguf *g, uint64_t i, KataliGgufTensorInfo *o), \
      (g, i, o))                                                                              \
    X(int, katali_cuda_gguf_find, (const KataliGguf *g, const char *n, uint64_t *i), (g, n, i)) \
    X(int, katali_cuda_gguf_get_int, (const KataliGguf *g, const char *k, int64_t *v), (g, k, v)) \
    X(int, katali_cuda_gguf_get_float, (const KataliGguf *g, const char *k, double *v),      \
      (g, k, v))                                                                              \
    X(int, katali_cuda_gguf_get_str,                                                          \
      (const KataliGguf *g, const char *k, const char **v, uint64_t *n), (g, k, v, n))        \
    X(int, katali_cuda_gguf_array, (const KataliGguf *g, const char *k, uint32_t *t,         \
                                    uint64_t *n),                                             \
      (g, k, t, n))                                                                           \
    X(int, katali_cuda_gguf_array_int,                                                        \
      (const KataliGguf *g, const char *k, uint64_t i, int64_t *v), (g, k, i, v))             \
    X(int, katali_cuda_gguf_upload, (KataliGguf * g, uint64_t i, void *d), (g, i, d))        \
    X(int, katali_cuda_dense_create_from_gguf,                                                \
      (KataliGguf * g, uint32_t c, uint32_t f, KataliDense **o), (g, c, f, o))                \
    X(int, katali_cuda_hybrid_create_from_gguf,                                               \
      (KataliGguf * g, uint32_t c, uint32_t f, KataliExpertCache *x, KataliHybrid **o),       \
      (g, c, f, x, o))                                                                        \
    X(int, katali_cuda_ep_unique_id, (void *id), (id))                                        \
    X(int, katali_cuda_ep_create, (uint32_t g, uint32_t r, const void *id, KataliEp **o),     \
      (g, r, id, o))                                                                          \
    X(int, katali_cuda_ep_destroy, (KataliEp * e), (e))                                       \
    X(int, katali_cuda_ep_use_peer_memory, (KataliEp * e, int on), (e, on))                   \
    X(int, katali_cuda_moe_ep_layer,                                                          \
      (KataliMoe * m, KataliEp * e, uint32_t tm, uint32_t n, const float *x, const float *l,  \
       float *y),                                                                             \
      (m, e, tm, n, x, l, y))                                                                 \
    X(int, katali_cuda_debug_row_isums,                                                       \
      (uint32_t t, const void *w, uint64_t r, uint64_t c, const void *q, int32_t *is,         \
       int32_t *xs),                                                                          \
      (t, w, r, c, q, is, xs))                                                                \
    X(int, katali_cuda_debug_route, (KataliMoe * m, const float *l, int32_t *i, float *w),    \
      (m, l, i, w))                                                                           \
    X(int, katali_cuda_debug_moe_trace, (KataliMoe * m, uint64_t *t, int *g), (m, t, g))     \
    X(int, katali_cuda_moe_layer_static,                                                      \
      (const KataliMoeDesc *d, const float *x, const float *l, float *y, uint32_t mo,         \
       void *s),                                                                              \
      (d, x, l, y, mo, s))

#define DECLARE_PTR(ret, name, params, args) static ret(*p_##name) params;
KATALI_FN_LIST(DECLARE_PTR)

static int g_state = -1; /* -1 unresolved, 0 unavailable, 1 loaded */
static void *g_handle;
static char g_why[512] = "not loaded";

/* Path of libkatali_cuda.so beside the library that contains this function. */
static int sibling_path(char *out, size_t cap) {
    Dl_info info;
    if (!dladdr((void *)&sibling_path, &info) || !info.dli_fname) return -1;
    const char *slash = strrchr(info.dli_fname, '/');
    if (!slash) return -1;
    size_t dir = (size_t)(slash - info.dli_fname) + 1;
    if (dir + strlen("libkatali_cuda.so") + 1 > cap) return -1;
    memcpy(out, info.dli_fname, dir);
    strcpy(out + dir, "libkatali_cuda.so");
    return 0;
}

static int resolve(void) {
    if (g_state >= 0) return g_state;
    g_state = 0;
    const char *off = getenv("KATALI_CUDA");
    if (off && off[0] == '0') {
        snprintf(g_why, sizeof g_why, "disabled by KATALI_CUDA=0");
        return 0;
    }
    const char *cands[3] = {getenv("KATALI_CUDA_DLL"), NULL, "libkatali_cuda.so"};
    char sib[4096];
    if (sibling_path(sib, sizeof sib) == 0) cands[1] = sib;
    for (int i = 0; i < 3 && !g_handle; i++) {
        if (!cands[i] || !cands[i][0]) continue;
        g_handle = dlopen(cands[i], RTLD_NOW | RTLD_LOCAL);
        if (!g_handle) snprintf(g_why, sizeof g_why, "cannot load %s: %s", cands[i], dlerror());
        if (i == 0 && !g_handle) return 0; /* an explicit path that fails is final */
    }
    if (!g_handle) return 0;
#define RESOLVE(ret, name, params, args)                                              \
    p_##name = (ret(*) params)dlsym(g_handle, #name);                                 \
    if (!p_##name) {                                                                  \
        snprintf(g_why, sizeof g_why, "plugin lacks symbol %s", #name);               \
        dlclose(g_handle);                                                            \
        g_handle = NULL;                                                              \
        return 0;                                                                     \
    }
    KATALI_FN_LIST(RESOLVE)
    g_state = 1;
    return 1;
}

int katali_cuda_probe(void) { return resolve() ? p_katali_cuda_probe() : 0; }
const char *katali_cuda_status(void) { return resolve() ? p_katali_cuda_status() : g_why; }
const char *katali_cuda_strerror(int s) {
    return resolve() ? p_katali_cuda_strerror(s) : "plugin not loaded";
}

#define FORWARD(ret, name, params, args) \
    ret name params { return resolve() ? p_##name args : KATALI_ERR_NO_DEVICE; }
#define KATALI_INT_FN_LIST(X)                                                                 \
    X(int, katali_cuda_malloc, (void **p, size_t n), (p, n))                                  \
    X(int, katali_cuda_free, (void *p), (p))                                                  \
    X(int, katali_cuda_upload, (void *d, const void *h, size_t n), (d, h, n))                 \
    X(int, katali_cuda_download, (void *h, const void *d, size_t n), (h, d, n))               \
    X(int, katali_cuda_matvec,                                                                \
      (uint32_t t, const void *w, uint64_t r, uint64_t c, const float *x, float *y),          \
      (t, w, r, c, x, y))                                                                     \
    X(int, katali_cuda_set_stream, (void *s), (s))                                            \
    X(int, katali_cuda_set_async, (int on), (on))                                             \
    X(int, katali_cuda_sync, (void), ())                                                      \
    X(int, katali_cuda_matvec_multi,                                                          \
      (int n, const uint32_t *t, const void *const *w, const uint64_t *r, uint64_t c,         \
       const float *x, float *const *y),                                                      \
      (n, t, w, r, c, x, y))                                                                  \
    X(int, katali_cuda_quantize_q8_1, (const float *x, uint64_t n, void *q), (x, n, q))       \
    X(int, katali_cuda_matvec_q8_1,                                                           \
      (uint32_t t, const void *w, uint64_t r, uint64_t c, const void *q, float *y),           \
      (t, w, r, c, q, y))                                                                     \
    X(int, katali_cuda_quantize_rows,                                                         \
      (uint32_t t, const float *s, uint64_t r, uint64_t c, void *d), (t, s, r, c, d))         \
    X(int, katali_cuda_moe_create, (const KataliMoeDesc *d, KataliMoe **o), (d, o))           \
    X(int, katali_cuda_moe_set_expert,                                                        \
      (KataliMoe * m, uint32_t e, const void *g, const void *u, const void *d),               \
      (m, e, g, u, d))                                                                        \
    X(int, katali_cuda_moe_destroy, (KataliMoe * m), (m))                                     \
    X(int, katali_cuda_moe_layer,                                                             \
      (KataliMoe * m, const float *x, const float *l, float *y, uint32_t mo),                 \
      (m, x, l, y, mo))                                                                       \
    X(int, katali_cuda_moe_layer_routed,                                                      \
      (KataliMoe * m, const float *x, const int32_t *i, const float *w, float *y,             \
       uint32_t mo),                                                                          \
      (m, x, i, w, y, mo))                                                                    \
    X(int, katali_cuda_moe_batch,                                                             \
      (KataliMoe * m, uint32_t n, const float *x, const float *l, float *y, uint32_t mo),     \
      (m, n, x, l, y, mo))                                                                    \
    X(int, katali_cuda_moe_ep_slot_bytes, (KataliMoe * m, uint64_t *s, uint64_t *r),          \
      (m, s, r))                                                                              \
    X(int, katali_cuda_moe_ep_dispatch,                                                       \
      (KataliMoe * m, uint32_t g, uint32_t tm, uint32_t n, const float *x, const float *l,    \
       void *s),                                                                              \
      (m, g, tm, n, x, l, s))                                                                 \
    X(int, katali_cuda_moe_ep_experts,                                                        \
      (KataliMoe * m, uint32_t g, uint32_t r, uint32_t tm, const void *i, void *o),           \
      (m, g, r, tm, i, o))                                                                    \
    X(int, katali_cuda_moe_ep_combine,                                                        \
      (KataliMoe * m, uint32_t g, uint32_t tm, uint32_t n, const void *b, float *y),          \
      (m, g, tm, n, b, y))                                                                    \
    X(int, katali_cuda_expert_cache_create, (uint64_t b, uint32_t n, KataliExpertCache **o),  \
      (b, n, o))                                                                              \
    X(int, katali_cuda_expert_cache_destroy, (KataliExpertCache * c), (c))                    \
    X(int, katali_cuda_expert_register,                                                       \
      (KataliExpertCache * c, uint64_t k, const void *g, uint64_t gb, const void *u,          \
       uint64_t ub, const void *d, uint64_t db),                                              \
      (c, k, g, gb, u, ub, d, db))                                                            \
    X(int, katali_cuda_expert_prefetch_async, (KataliExpertCache * c, uint64_t k), (c, k))    \
    X(int, katali_cuda_expert_bind, (KataliExpertCache * c, uint64_t k, KataliMoe * m,        \
                                     uint32_t e),                                             \
      (c, k, m, e))                                                                           \
    X(int, katali_cuda_expert_evict, (KataliExpertCache * c, uint64_t k), (c, k))             \
    X(int, katali_cuda_expert_lookup,                                                         \
      (KataliExpertCache * c, uint64_t k, int *r, void **g, void **u, void **d),              \
      (c, k, r, g, u, d))                                                                     \
    X(int, katali_cuda_expert_sync, (KataliExpertCache * c), (c))                             \
    X(int, katali_cuda_dense_create, (const KataliDenseDesc *d, KataliDense **o), (d, o))     \
    X(int, katali_cuda_dense_destroy, (KataliDense * m), (m))                                 \
    X(int, katali_cuda_dense_reset, (KataliDense * m), (m))                                   \
    X(int, katali_cuda_dense_generate,                                                        \
      (KataliDense * m, const int32_t *p, uint32_t np, uint32_t ng, int32_t *o),              \
      (m, p, np, ng, o))                                                                      \
    X(int, katali_cuda_dense_logits, (KataliDense * m, const float **l, int32_t *p),          \
      (m, l, p))                                                                              \
    X(int, katali_cuda_hybrid_create, (const KataliHybridDesc *d, KataliHybrid **o), (d, o))  \
    X(int, katali_cuda_hybrid_destroy, (KataliHybrid * m), (m))                               \
    X(int, katali_cuda_hybrid_reset, (KataliHybrid * m), (m))                                 \
    X(int, katali_cuda_hybrid_generate,                                                       \
      (KataliHybrid * m, const int32_t *p, uint32_t np, uint32_t ng, int32_t *o),             \
      (m, p, np, ng, o))                                                                      \
    X(int, katali_cuda_hybrid_logits, (KataliHybrid * m, const float **l, int32_t *p),        \
      (m, l, p))                                                                              \
    X(int, katali_cuda_hybrid_set_ep, (KataliHybrid * m, KataliEp * e), (m, e))               \
    X(int, katali_cuda_gguf_open, (const char *p, KataliGguf **o), (p, o))                    \
    X(int, katali_cuda_gguf_close, (KataliGguf * g), (g))                                     \
    X(int, katali_cuda_gguf_counts, (const KataliGguf *g, uint64_t *t, uint64_t *k,          \
                                     uint32_t *v),                                            \
      (g, t, k, v))                                                                           \
    X(int, katali_cuda_gguf_tensor, (const KataliGguf *g, uint64_t i, KataliGgufTensorInfo *o), \
      (g, i, o))                                                                              \
    X(int, katali_cuda_gguf_find, (const KataliGguf *g, const char *n, uint64_t *i), (g, n, i)) \
    X(int, katali_cuda_gguf_get_int, (const KataliGguf *g, const char *k, int64_t *v), (g, k, v)) \
    X(int, katali_cuda_gguf_get_float, (const KataliGguf *g, const char *k, double *v),      \
      (g, k, v))                                                                              \
    X(int, katali_cuda_gguf_get_str,                                                          \
      (const KataliGguf *g, const char *k, const char **v, uint64_t *n), (g, k, v, n))        \
    X(int, katali_cuda_gguf_array, (const KataliGguf *g, const char *k, uint32_t *t,         \
                                    uint64_t *n),                                             \
      (g, k, t, n))                                                                           \
    X(int, katali_cuda_gguf_array_int,                                                        \
      (const KataliGguf *g, const char *k, uint64_t i, int64_t *v), (g, k, i, v))             \
    X(int, katali_cuda_gguf_upload, (KataliGguf * g, uint64_t i, void *d), (g, i, d))        \
    X(int, katali_cuda_dense_create_from_gguf,                                                \
      (KataliGguf * g, uint32_t c, uint32_t f, KataliDense **o), (g, c, f, o))                \
    X(int, katali_cuda_hybrid_create_from_gguf,                                               \
      (KataliGguf * g, uint32_t c, uint32_t f, KataliExpertCache *x, KataliHybrid **o),       \
      (g, c, f, x, o))                                                                        \
    X(int, katali_cuda_ep_unique_id, (void *id), (id))                                        \
    X(int, katali_cuda_ep_create, (uint32_t g, uint32_t r, const void *id, KataliEp **o),     \
      (g, r, id, o))                                                                          \
    X(int, katali_cuda_ep_destroy, (KataliEp * e), (e))                                       \
    X(int, katali_cuda_ep_use_peer_memory, (KataliEp * e, int on), (e, on))                   \
    X(int, katali_cuda_moe_ep_layer,                                                          \
      (KataliMoe * m, KataliEp * e, uint32_t tm, uint32_t n, const float *x, const float *l,  \
       float *y),                                                                             \
      (m, e, tm, n, x, l, y))                                                                 \
    X(int, katali_cuda_debug_row_isums,                                                       \
      (uint32_t t, const void *w, uint64_t r, uint64_t c, const void *q, int32_t *is,         \
       int32_t *xs),                                                                          \
      (t, w, r, c, q, is, xs))                                                                \
    X(int, katali_cuda_debug_route, (KataliMoe * m, const float *l, int32_t *i, float *w),    \
      (m, l, i, w))                                                                           \
    X(int, katali_cuda_debug_moe_trace, (KataliMoe * m, uint64_t *t, int *g), (m, t, g))     \
    X(int, katali_cuda_moe_layer_static,                                                      \
      (const KataliMoeDesc *d, const float *x, const float *l, float *y, uint32_t mo,         \
       void *s),                                                                              \
      (d, x, l, y, mo, s))
KATALI_INT_FN_LIST(FORWARD)

int katali_cuda_supports_type(uint32_t t) { return resolve() ? p_katali_cuda_supports_type(t) : 0; }

/* Loader-only: which plugin file was loaded (NULL when none). */
const char *katali_cuda_loader_path(void) {
    if (!resolve()) return NULL;
    Dl_info info;
    if (p_katali_cuda_probe && dladdr((void *)p_katali_cuda_probe, &info)) return info.dli_fname;
    return NULL;
}
