/* katali_cuda_check — command-line checks of the plugin through the loader, the
 * host-side equivalents of the reference engine's `cuda-info`, `cuda-check`,
 * `cuda-check-moe` and `cuda-bench` commands (README.md:17,21,99-102,149-152).
 * Everything runs through the C ABI with host buffers, as the engine would.
 *
 *   katali_cuda_check info       probe result and device
 *   katali_cuda_check check      Q4_K / Q6_K GEMV: fp32 activations vs q8_1 (DP4A)
 *   katali_cuda_check check-moe  fused MoE layer: device routing vs given routing
 *                                (bit-identical) and fp32 vs q8_1 activations
 *   katali_cuda_check bench      matvec 6144 x 2048 Q4_K with upload + download per call
 *
 * Exit status: 0 pass, 1 a check failed, 2 no usable device or plugin.
 * Weights are synthetic (a fixed-seed generator), encoded by the plugin itself.
 */
#define _GNU_SOURCE
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "katali_cuda.h"

static uint64_t g_rng = 0x9E3779B97F4A7C15ull;
static double urand(void) { /* xorshift64*, uniform in (0, 1) */
    g_rng ^= g_rng >> 12;
    g_rng ^= g_rng << 25;
    g_rng ^= g_rng >> 27;
    return ((g_rng * 2685821657736338717ull) >> 11) * (1.0 / 9007199254740992.0) + 1e-300;
}
static float nrand(void) { return (float)(sqrt(-2.0 * log(urand())) * cos(6.283185307179586 * urand())); }

static int fail(const char *what, int rc) {
    fprintf(stderr, "%s: %s (%s)\n", what, katali_cuda_strerror(rc), katali_cuda_status());
    return 1;
}

/* Device matrix of rows x cols from N(0, std) encoded to `type` by the plugin. */
static void *make_matrix(uint32_t type, uint64_t rows, uint64_t cols, float std, int *rc) {
    const uint64_t rb = cols / 256 * (type == KATALI_TYPE_Q4_K ? 144 : 210);
    float *h = (float *)malloc(rows * cols * sizeof(float));
    void *src = NULL, *dst = NULL;
    for (uint64_t i = 0; i < rows * cols; i++) h[i] = std * nrand();
    *rc = katali_cuda_malloc(&src, rows * cols * sizeof(float));
    if (!*rc) *rc = katali_cuda_malloc(&dst, rows * rb);
    if (!*rc) *rc = katali_cuda_upload(src, h, rows * cols * sizeof(float));
    if (!*rc) *rc = katali_cuda_quantize_rows(type, (const float *)src, rows, cols, dst);
    katali_cuda_free(src);
    free(h);
    return dst;
}

static double rel_l2(const float *a, const float *b, size_t n) {
    double num = 0, den = 0;
    for (size_t i = 0; i < n; i++) {
        num += ((double)a[i] - b[i]) * ((double)a[i] - b[i]);
        den += (double)b[i] * b[i];
    }
    return den > 0 ? sqrt(num / den) : sqrt(num);
}

static int cmd_info(void) {
    const int ok = katali_cuda_probe();
    printf("katali_cuda: %s\n", katali_cuda_status());
    return ok ? 0 : 2;
}

static int cmd_check(void) {
    const uint32_t types[2] = {KATALI_TYPE_Q4_K, KATALI_TYPE_Q6_K};
    const uint64_t rows = 4096, cols = 2048;
    int bad = 0;
    for (int t = 0; t < 2; t++) {
        int rc;
        void *w = make_matrix(types[t], rows, cols, 0.02f, &rc);
        if (rc) return fail("encode", rc);
        float *x = (float *)malloc(cols * 4), *y32 = (float *)malloc(rows * 4), *y8 = (float *)malloc(rows * 4);
        for (uint64_t i = 0; i < cols; i++) x[i] = nrand();
        void *xd, *yd, *xq;
        rc = katali_cuda_malloc(&xd, cols * 4);
        if (!rc) rc = katali_cuda_malloc(&yd, rows * 4);
        if (!rc) rc = katali_cuda_malloc(&xq, cols / 32 * 36);
        if (!rc) rc = katali_cuda_upload(xd, x, cols * 4);
        if (!rc) rc = katali_cuda_matvec(types[t], w, rows, cols, (const float *)xd, (float *)yd);
        if (!rc) rc = katali_cuda_download(y32, yd, rows * 4);
        if (!rc) rc = katali_cuda_quantize_q8_1((const float *)xd, cols, xq);
        if (!rc) rc = katali_cuda_matvec_q8_1(types[t], w, rows, cols, xq, (float *)yd);
        if (!rc) rc = katali_cuda_download(y8, yd, rows * 4);
        if (rc) return fail("matvec", rc);
        const double e = rel_l2(y8, y32, rows);
        const int ok = e < 3e-2;  /* q8_1 activation rounding */
        printf("%s %llux%llu: fp32 vs q8_1 rel_L2 %.3e %s\n", t ? "Q6_K" : "Q4_K",
               (unsigned long long)rows, (unsigned long long)cols, e, ok ? "ok" : "FAIL");
        bad |= !ok;
        katali_cuda_free(w);
        katali_cuda_free(xd);
        katali_cuda_free(yd);
        katali_cuda_free(xq);
        free(x);
        free(y32);
        free(y8);
    }
    return bad;
}

static int cmd_check_moe(void) {
    const uint32_t E = 64, H = 2048, F = 512, K = 8;
    int rc;
    void *gate = make_matrix(KATALI_TYPE_Q4_K, (uint64_t)E * F, H, 0.02f, &rc);
    void *up = rc ? NULL : make_matrix(KATALI_TYPE_Q4_K, (uint64_t)E * F, H, 0.02f, &rc);
    void *down = rc ? NULL : make_matrix(KATALI_TYPE_Q6_K, (uint64_t)E * H, F, 0.02f, &rc);
    if (rc) return fail("encode", rc);
    const void **ptrs = (const void **)malloc(3 * E * sizeof(void *));
    for (uint32_t e = 0; e < E; e++) {
        ptrs[3 * e] = (const uint8_t *)gate + (size_t)e * F * (H / 256 * 144);
        ptrs[3 * e + 1] = (const uint8_t *)up + (size_t)e * F * (H / 256 * 144);
        ptrs[3 * e + 2] = (const uint8_t *)down + (size_t)e * H * (F / 256 * 210);
    }
    KataliMoeDesc d = {E, H, F, K, KATALI_TYPE_Q4_K, KATALI_TYPE_Q4_K, KATALI_TYPE_Q6_K,
                       KATALI_MOE_NORM_TOPK, ptrs};
    KataliMoe *m;
    if ((rc = katali_cuda_moe_create(&d, &m))) return fail("moe_create", rc);
    float *x = (float *)malloc(H * 4), *lg = (float *)malloc(E * 4);
    float *y1 = (float *)malloc(H * 4), *y2 = (float *)malloc(H * 4), *y3 = (float *)malloc(H * 4);
    void *xd, *ld, *yd, *idd, *wd;
    rc = katali_cuda_malloc(&xd, H * 4);
    if (!rc) rc = katali_cuda_malloc(&ld, E * 4);
    if (!rc) rc = katali_cuda_malloc(&yd, H * 4);
    if (!rc) rc = katali_cuda_malloc(&idd, K * 4);
    if (!rc) rc = katali_cuda_malloc(&wd, K * 4);
    int bad = 0;
    for (int it = 0; it < 4 && !rc; it++) {
        for (uint32_t i = 0; i < H; i++) x[i] = nrand();
        for (uint32_t i = 0; i < E; i++) lg[i] = nrand();
        rc = katali_cuda_upload(xd, x, H * 4);
        if (!rc) rc = katali_cuda_upload(ld, lg, E * 4);
        if (!rc) rc = katali_cuda_moe_layer(m, (const float *)xd, (const float *)ld, (float *)yd, KATALI_MOE_Q8_1);
        if (!rc) rc = katali_cuda_download(y1, yd, H * 4);
        if (!rc) rc = katali_cuda_debug_route(m, (const float *)ld, (int32_t *)idd, (float *)wd);
        if (!rc) rc = katali_cuda_moe_layer_routed(m, (const float *)xd, (const int32_t *)idd,
                                                   (const float *)wd, (float *)yd, KATALI_MOE_Q8_1);
        if (!rc) rc = katali_cuda_download(y2, yd, H * 4);
        if (!rc) rc = katali_cuda_moe_layer(m, (const float *)xd, (const float *)ld, (float *)yd, KATALI_MOE_F32);
        if (!rc) rc = katali_cuda_download(y3, yd, H * 4);
        if (rc) break;
        const int same = memcmp(y1, y2, H * 4) == 0;
        const double e = rel_l2(y1, y3, H);
        printf("layer %d: routed == device-routed %s, q8_1 vs fp32 rel_L2 %.3e %s\n", it,
               same ? "yes" : "NO", e, e < 3e-2 ? "ok" : "FAIL");
        bad |= !same || !(e < 3e-2);
    }
    katali_cuda_moe_destroy(m);
    katali_cuda_free(gate);
    katali_cuda_free(up);
    katali_cuda_free(down);
    katali_cuda_free(xd);
    katali_cuda_free(ld);
    katali_cuda_free(yd);
    katali_cuda_free(idd);
    katali_cuda_free(wd);
    free(ptrs);
    free(x);
    free(lg);
    free(y1);
    free(y2);
    free(y3);
    if (rc) return fail("moe layer", rc);
    return bad;
}

static double now_s(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + 1e-9 * t.tv_nsec;
}

static int cmd_bench(void) {
    const uint64_t rows = 6144, cols = 2048, bytes = rows * (cols / 256 * 144);
    int rc;
    void *w = make_matrix(KATALI_TYPE_Q4_K, rows, cols, 0.02f, &rc);
    if (rc) return fail("encode", rc);
    float *x = (float *)malloc(cols * 4), *y = (float *)malloc(rows * 4);
    for (uint64_t i = 0; i < cols; i++) x[i] = nrand();
    void *xd, *yd;
    rc = katali_cuda_malloc(&xd, cols * 4);
    if (!rc) rc = katali_cuda_malloc(&yd, rows * 4);
    const int n = 200;
    double t0 = 0;
    for (int i = 0; i < n + 20 && !rc; i++) {
        if (i == 20) t0 = now_s();
        rc = katali_cuda_upload(xd, x, cols * 4);
        if (!rc) rc = katali_cuda_matvec(KATALI_TYPE_Q4_K, w, rows, cols, (const float *)xd, (float *)yd);
        if (!rc) rc = katali_cuda_download(y, yd, rows * 4);
    }
    if (rc) return fail("bench", rc);
    const double us = (now_s() - t0) / n * 1e6;
    printf("matvec Q4_K %llux%llu with upload + download: %.1f us per call, %.1f GB/s of weights\n",
           (unsigned long long)rows, (unsigned long long)cols, us, bytes / us * 1e-3);
    katali_cuda_free(w);
    katali_cuda_free(xd);
    katali_cuda_free(yd);
    free(x);
    free(y);
    return 0;
}

int main(int argc, char **argv) {
    const char *cmd = argc > 1 ? argv[1] : "info";
    if (strcmp(cmd, "info") == 0) return cmd_info();
    if (!katali_cuda_probe()) {
        fprintf(stderr, "katali_cuda: %s\n", katali_cuda_status());
        return 2;
    }
    if (strcmp(cmd, "check") == 0) return cmd_check();
    if (strcmp(cmd, "check-moe") == 0) return cmd_check_moe();
    if (strcmp(cmd, "bench") == 0) return cmd_bench();
    fprintf(stderr, "usage: %s info|check|check-moe|bench\n", argv[0]);
    return 2;
}
