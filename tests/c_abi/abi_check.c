/*
 * abi_check.c -- the qdc_b200 C ABI used from plain C, as a foreign-language
 * binding would use it: include/qdc_b200.h and libqdc_b200.so only, no
 * Python, no torch.
 *
 *   abi_check          host-only checks (no GPU needed): ABI version, status
 *                      strings, RoPE tables, context-free argument errors
 *   abi_check --gpu    also a post-attention residual RMSNorm on cuda:0 through
 *                      qdc_init / qdc_residual_rms / qdc_sync, against a double
 *                      precision restatement of src/backbone_cpu.jl:321-350
 *
 * Built and run by tests/test_c_abi.py; exit status 0 = pass.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qdc_b200.h"

#ifdef QDC_CHECK_GPU
#include <cuda_runtime.h>
#endif

static int failures = 0;
#define EXPECT(cond, what)                                   \
    do {                                                     \
        if (!(cond)) {                                       \
            fprintf(stderr, "FAIL: %s (line %d)\n", what, __LINE__); \
            ++failures;                                      \
        }                                                    \
    } while (0)

static void host_checks(void) {
    EXPECT(qdc_abi_version() == QDC_B200_ABI_VERSION, "ABI version");
    EXPECT(strcmp(qdc_status_string(QDC_OK), "ok") == 0, "status string ok");
    EXPECT(strcmp(qdc_status_string(QDC_EINVAL), "invalid argument") == 0, "status string EINVAL");

    /* RoPE tables, src/backbone_cpu.jl:90-105: position 0 is (cos, sin) = (1, 0) */
    float c[3 * 2], s[3 * 2];
    EXPECT(qdc_rope_table(10000.0f, 4, 3, c, s) == QDC_OK, "rope table");
    EXPECT(c[0] == 1.0f && c[1] == 1.0f && s[0] == 0.0f && s[1] == 0.0f, "rope position 0");
    /* position 1, frequency 0: angle 1 rad */
    EXPECT(fabs(c[2] - cos(1.0)) < 1e-7 && fabs(s[2] - sin(1.0)) < 1e-7, "rope position 1");
    EXPECT(qdc_rope_table(10000.0f, 3, 3, c, s) == QDC_EINVAL, "odd rotary refused");

    /* every compute entry point checks its context before anything else */
    EXPECT(qdc_residual_rms(NULL, NULL, NULL, NULL, NULL, NULL, 1e-6f, 1, 1, 8, 8, 8, 8, 8, QDC_F32,
                            NULL) == QDC_EINVAL, "NULL context");
    EXPECT(strstr(qdc_last_error(NULL), "NULL") != NULL, "last error text");
}

#ifdef QDC_CHECK_GPU
static int gpu_checks(void) {
    enum { ROWS = 37, W = 1024 };
    const float eps = 1e-6f;
    size_t bytes = sizeof(float) * ROWS * W;
    float *hx = malloc(bytes), *hm = malloc(bytes), *hr = malloc(bytes), *hy = malloc(bytes);
    float hg[W];
    unsigned s = 12345u;
    for (int i = 0; i < ROWS * W; ++i) {
        s = s * 1664525u + 1013904223u;
        hx[i] = (float)((int)(s >> 9) % 2001 - 1000) / 500.0f;
        s = s * 1664525u + 1013904223u;
        hm[i] = (float)((int)(s >> 9) % 2001 - 1000) / 700.0f;
    }
    for (int i = 0; i < W; ++i) hg[i] = 0.01f * (float)((i % 13) - 6);

    float *dx, *dm, *dr, *dy, *dg;
    if (cudaMalloc((void **)&dx, bytes) || cudaMalloc((void **)&dm, bytes) || cudaMalloc((void **)&dr, bytes) ||
        cudaMalloc((void **)&dy, bytes) || cudaMalloc((void **)&dg, sizeof hg)) {
        fprintf(stderr, "FAIL: cudaMalloc\n");
        return 1;
    }
    cudaMemcpy(dx, hx, bytes, cudaMemcpyHostToDevice);
    cudaMemcpy(dm, hm, bytes, cudaMemcpyHostToDevice);
    cudaMemcpy(dg, hg, sizeof hg, cudaMemcpyHostToDevice);

    qdc_ctx *ctx = NULL;
    EXPECT(qdc_init(0, &ctx) == QDC_OK && ctx != NULL, "qdc_init");
    EXPECT(qdc_residual_rms(ctx, dr, dy, dx, dm, dg, eps, 1, ROWS, W, W, W, W, W, QDC_F32, NULL) == QDC_OK,
           "qdc_residual_rms");
    EXPECT(qdc_sync(ctx, NULL) == QDC_OK, "qdc_sync");
    /* a width the library cannot take: leading dimension below the width */
    EXPECT(qdc_residual_rms(ctx, dr, dy, dx, dm, dg, eps, 1, ROWS, W, W - 1, W, W, W, QDC_F32, NULL) ==
               QDC_EINVAL, "bad leading dimension refused");
    cudaMemcpy(hr, dr, bytes, cudaMemcpyDeviceToHost);
    cudaMemcpy(hy, dy, bytes, cudaMemcpyDeviceToHost);

    double worst = 0.0;
    for (int t = 0; t < ROWS; ++t) {
        double ss = 0.0;
        for (int i = 0; i < W; ++i) {
            float r = hx[t * W + i] + hm[t * W + i];  /* Float32 add, stored exactly */
            EXPECT(hr[t * W + i] == r, "residual bit-exact");
            ss += (double)r * r;
        }
        float scale = (float)(1.0 / sqrt(ss / W + eps));
        for (int i = 0; i < W; ++i) {
            double e = (double)((hx[t * W + i] + hm[t * W + i]) * scale) * (1.0f + hg[i]);
            double v = fabs(hy[t * W + i] - e) / (1e-6 + 1e-5 * fabs(e));
            if (v > worst) worst = v;
        }
    }
    EXPECT(worst <= 1.0, "normalized rows within 1e-6 + 1e-5|b|");
    EXPECT(qdc_destroy(ctx) == QDC_OK, "qdc_destroy");
    cudaFree(dx); cudaFree(dm); cudaFree(dr); cudaFree(dy); cudaFree(dg);
    free(hx); free(hm); free(hr); free(hy);
    printf("gpu: worst %.3f of the tolerance\n", worst);
    return 0;
}
#endif

int main(int argc, char **argv) {
    host_checks();
#ifdef QDC_CHECK_GPU
    if (argc > 1 && strcmp(argv[1], "--gpu") == 0 && gpu_checks()) ++failures;
#else
    (void)argc;
    (void)argv;
#endif
    if (failures) {
        fprintf(stderr, "%d check(s) failed\n", failures);
        return 1;
    }
    printf("abi_check: ok\n");
    return 0;
}
