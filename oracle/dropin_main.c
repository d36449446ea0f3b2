/* dropin_main.c — test infrastructure: runs the reference's own dense backend
 * (vendor/katali_gguf_dense: gguf_model.c, katali_dense_cuda.c and the rest, compiled
 * unchanged from the reference checkout) with this repository's katali_cuda.h and dlopen
 * loader in place of the reference's missing src/katali_cuda.c (build-qwen3.bat:5).
 *
 *   katali_dropin <model.gguf> <max_tokens> <prompt> <out_prefix>
 *
 * Greedy generation through katali_gguf_model_generate (V/src/gguf_model.c:985-1101).
 * For every generated token the per-token observer (katali_gguf_model_set_token_callback)
 * stores the logits the sampler saw (m->logits) to <out_prefix>.logits (float32,
 * max_tokens x vocab) and the chosen id (first maximum, V/src/gguf_sampler.c:62-66) to
 * <out_prefix>.ids (int32). The calls the reference code makes into the plugin are counted
 * with the linker's --wrap of katali_cuda_matvec, so nothing in the reference sources is
 * edited. One JSON line on stdout: tokens generated, vocab, whether the reference switched
 * its CUDA path on (katali_dense_cuda_enabled, V/src/katali_dense_cuda.c:14-22) and the
 * plugin matvec calls that returned KATALI_OK.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "katali_cuda.h"
#include "katali_dense_cuda.h"
#include "katali_gguf_model.h"

static long g_matvec_calls, g_matvec_ok;

int __real_katali_cuda_matvec(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                              const float *x, float *y);
int __wrap_katali_cuda_matvec(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                              const float *x, float *y) {
    const int rc = __real_katali_cuda_matvec(type, w, rows, cols, x, y);
    ++g_matvec_calls;
    if (rc == KATALI_OK) ++g_matvec_ok;
    return rc;
}

typedef struct {
    KataliGgufModel *m;
    FILE *logits, *ids;
    int n;
} Observer;

static int on_token(const char *bytes, size_t len, void *user) {
    (void)bytes;
    (void)len;
    Observer *o = (Observer *)user;
    const float *lg = o->m->logits;
    int best = 0;
    for (int i = 1; i < o->m->vocab; ++i)
        if (lg[i] > lg[best]) best = i;  // first maximum, as the greedy sampler
    fwrite(lg, sizeof(float), (size_t)o->m->vocab, o->logits);
    fwrite(&best, sizeof(int), 1, o->ids);
    ++o->n;
    return 0;
}

int main(int argc, char **argv) {
    if (argc != 5) {
        fprintf(stderr, "usage: %s <model.gguf> <max_tokens> <prompt> <out_prefix>\n", argv[0]);
        return 2;
    }
    KataliBackendOptions opts;
    memset(&opts, 0, sizeof opts);
    opts.model_path = argv[1];
    opts.max_tokens = atoi(argv[2]);
    opts.use_mmap = 1;  /* greedy: temperature 0 */
    static KataliGgufModel m;
    char err[512] = {0};
    if (katali_gguf_model_open(&m, &opts, err, sizeof err) != 0) {
        fprintf(stderr, "open failed: %s\n", err);
        return 3;
    }
    char path[4096];
    snprintf(path, sizeof path, "%s.logits", argv[4]);
    FILE *fl = fopen(path, "wb");
    snprintf(path, sizeof path, "%s.ids", argv[4]);
    FILE *fi = fopen(path, "wb");
    if (!fl || !fi) {
        fprintf(stderr, "cannot write %s\n", argv[4]);
        return 4;
    }
    Observer o = {&m, fl, fi, 0};
    katali_gguf_model_set_token_callback(&m, on_token, &o);
    static char out[1 << 16];
    const int gen = katali_gguf_model_generate(&m, argv[3], out, sizeof out);
    fclose(fl);
    fclose(fi);
    printf("{\"generated\": %d, \"observed\": %d, \"vocab\": %d, \"cuda_enabled\": %d, "
           "\"plugin_matvec_calls\": %ld, \"plugin_matvec_ok\": %ld, \"status\": \"%s\"}\n",
           gen, o.n, m.vocab, katali_dense_cuda_enabled(), g_matvec_calls, g_matvec_ok,
           katali_cuda_status());
    katali_dense_cuda_shutdown();
    katali_gguf_model_close(&m);
    return gen < 0 ? 5 : 0;
}
