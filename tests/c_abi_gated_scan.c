/* A C caller of the library, with no Python in the loop: the prefill gated
 * scan (B=2, T=300, C=256 bf16, packed-segment resets, h0, fp32 final state)
 * through need_gated_scan, against the C oracle (decay = sigmoid(z), update =
 * (1 - decay) * (sigmoid(g) * x) in bf16, the chunked fp32 scan, the output
 * rounded to bf16).  Built and run by tests/test_c_abi_gpu.py; prints
 * "C-ABI-OK" and exits 0 when the outputs agree within the bf16 budget
 * (max |diff| <= 2e-2 * max |ref|, at least 99% bit-identical) and the final
 * state within 1e-5 relative. */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "need_scan.h"

/* the oracle's entry points (oracle/need_scan_oracle.c) */
void ora_gated_prep(const float* x, const float* z, const float* g, const uint8_t* seg, float* a, float* b,
                    int64_t N, int64_t T, int64_t C, int mode, int nthreads);
void ora_affine_scan(const float* a, const float* b, const float* h0, float* h, float* h_final, int64_t N,
                     int64_t T, int64_t C, int64_t chunk, int nthreads);
void ora_round(float* x, int64_t n, int mode);

static uint64_t rng = 0x9e3779b97f4a7c15ull;
static double uniform(void) {
    rng = rng * 6364136223846793005ull + 1442695040888963407ull;
    return ((rng >> 11) + 0.5) / 9007199254740992.0;
}
static float normal(void) { /* Box-Muller */
    const double u = uniform(), v = uniform();
    return (float)(sqrt(-2.0 * log(u)) * cos(6.283185307179586 * v));
}
static uint16_t to_bf16(float f) { /* round to nearest even */
    uint32_t u;
    memcpy(&u, &f, 4);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
static float from_bf16(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

#define CHECK_CUDA(x)                                                                  \
    do {                                                                               \
        cudaError_t e_ = (x);                                                          \
        if (e_ != cudaSuccess) {                                                       \
            fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));                   \
            return 1;                                                                  \
        }                                                                              \
    } while (0)

int main(void) {
    const int64_t B = 2, T = 300, C = 256, n = B * T * C;
    uint16_t *hx = malloc(n * 2), *hz = malloc(n * 2), *hg = malloc(n * 2), *hout = malloc(n * 2);
    float *fx = malloc(n * 4), *fz = malloc(n * 4), *fg = malloc(n * 4), *fa = malloc(n * 4), *fb = malloc(n * 4);
    float *want = malloc(n * 4), *h0 = malloc(B * C * 4), *hf = malloc(B * C * 4), *want_hf = malloc(B * C * 4);
    uint8_t* seg = calloc(B * T, 1);
    for (int64_t i = 0; i < n; ++i) {
        hx[i] = to_bf16(normal());
        hz[i] = to_bf16(normal() + 4.0f);
        hg[i] = to_bf16(normal());
        fx[i] = from_bf16(hx[i]);
        fz[i] = from_bf16(hz[i]);
        fg[i] = from_bf16(hg[i]);
    }
    for (int64_t i = 0; i < B * C; ++i) h0[i] = normal();
    for (int64_t b = 0; b < B; ++b) /* segments of 16..96 tokens */
        for (int64_t t = 0; t < T; t += 16 + (int64_t)(uniform() * 81)) seg[b * T + t] = 1;

    /* device buffers and the workspace (zeroed once) */
    void *dx, *dz, *dg, *dout, *dws;
    float *dh0, *dhf;
    uint8_t* dseg;
    const size_t ws = need_scan_workspace_size(NEED_FORM_GATED, NEED_BF16, NEED_BF16, 0, B, 1, T, C);
    CHECK_CUDA(cudaMalloc(&dx, n * 2));
    CHECK_CUDA(cudaMalloc(&dz, n * 2));
    CHECK_CUDA(cudaMalloc(&dg, n * 2));
    CHECK_CUDA(cudaMalloc(&dout, n * 2));
    CHECK_CUDA(cudaMalloc((void**)&dh0, B * C * 4));
    CHECK_CUDA(cudaMalloc((void**)&dhf, B * C * 4));
    CHECK_CUDA(cudaMalloc((void**)&dseg, B * T));
    CHECK_CUDA(cudaMalloc(&dws, ws));
    CHECK_CUDA(cudaMemset(dws, 0, ws));
    CHECK_CUDA(cudaMemcpy(dx, hx, n * 2, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dz, hz, n * 2, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dg, hg, n * 2, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dh0, h0, B * C * 4, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dseg, seg, B * T, cudaMemcpyHostToDevice));

    need_scan_args a;
    memset(&a, 0, sizeof a);
    a.form = NEED_FORM_GATED;
    a.dtype = a.decay_dtype = NEED_BF16;
    a.nb = B, a.nh = 1, a.T = T, a.C = C;
    const void* ins[3] = {dz, dg, dx}; /* in[0] = decay logit z, in[1] = gate logit g, in[2] = x */
    for (int k = 0; k < 3; ++k) {
        a.in[k].ptr = ins[k];
        a.in[k].stride_b = T * C;
        a.in[k].stride_h = 0;
        a.in[k].stride_t = C;
    }
    a.out = dout;
    a.out_stride_b = T * C, a.out_stride_h = 0, a.out_stride_t = C;
    a.h0 = dh0;
    a.h_final = dhf;
    a.seg_start = dseg;
    a.seg_stride_b = T, a.seg_stride_t = 1;
    a.workspace = dws;
    a.workspace_bytes = ws;
    cudaStream_t stream;
    CHECK_CUDA(cudaStreamCreate(&stream));
    int rc = need_gated_scan(&a, stream);
    if (rc != NEED_OK) {
        fprintf(stderr, "need_gated_scan: %d %s\n", rc, need_last_error());
        return 1;
    }
    uint32_t err = 0;
    rc = need_workspace_error(dws, &err, stream); /* synchronises the stream */
    if (rc != NEED_OK || err != 0) {
        fprintf(stderr, "workspace error word %u (rc %d)\n", err, rc);
        return 1;
    }
    CHECK_CUDA(cudaMemcpy(hout, dout, n * 2, cudaMemcpyDeviceToHost));
    CHECK_CUDA(cudaMemcpy(hf, dhf, B * C * 4, cudaMemcpyDeviceToHost));

    /* the oracle */
    ora_gated_prep(fx, fz, fg, seg, fa, fb, B, T, C, 1, 1);
    ora_affine_scan(fa, fb, h0, want, want_hf, B, T, C, 64, 1);
    ora_round(want, n, 1);

    double maxd = 0, maxr = 0, maxdf = 0, maxrf = 0;
    int64_t equal = 0;
    for (int64_t i = 0; i < n; ++i) {
        const float got = from_bf16(hout[i]);
        maxd = fmax(maxd, fabs((double)got - want[i]));
        maxr = fmax(maxr, fabs((double)want[i]));
        equal += got == want[i];
    }
    for (int64_t i = 0; i < B * C; ++i) {
        maxdf = fmax(maxdf, fabs((double)hf[i] - want_hf[i]));
        maxrf = fmax(maxrf, fabs((double)want_hf[i]));
    }
    printf("max rel %.3e, bit-identical %.4f, final state max rel %.3e\n", maxd / maxr, (double)equal / n,
           maxdf / maxrf);
    if (maxd > 2e-2 * maxr || equal < 0.99 * n || maxdf > 1e-5 * maxrf) return 1;
    printf("C-ABI-OK\n");
    cudaFree(dx), cudaFree(dz), cudaFree(dg), cudaFree(dout), cudaFree(dh0), cudaFree(dhf), cudaFree(dseg);
    cudaFree(dws);
    cudaStreamDestroy(stream);
    return 0;
}
