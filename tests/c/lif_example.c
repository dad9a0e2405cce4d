/* cc -std=c11 -I include -I $CUDA_HOME/include tests/c/lif_example.c -L hard_resets_compose_b200/lib -llifb -lcudart */
#include <stdio.h>
#include <stdlib.h>
#include <cuda_runtime.h>
#include "lifscan_b200.h"

static int fail(const char *what, int st)
{
    fprintf(stderr, "%s: %s (%s)\n", what, lifb_status_string(st), lifb_last_error());
    return 1;
}

int main(void)
{
    const int64_t T = 1024, N = 4096;
    const int C = 64, K = 16;
    const float beta = 0.9f, theta = 1.0f, u_r = 0.0f, alpha = 4.0f;
    const size_t bytes = (size_t)T * N * sizeof(float);
    float *h = malloc(bytes), *I, *U, *S, *GS, *Lam, *u0;
    for (int64_t i = 0; i < T * N; i++) h[i] = 0.1f + 0.3f * ((float)rand() / RAND_MAX - 0.5f);
    cudaMalloc((void **)&I, bytes); cudaMalloc((void **)&U, bytes); cudaMalloc((void **)&S, bytes);
    cudaMalloc((void **)&GS, bytes); cudaMalloc((void **)&Lam, bytes);
    cudaMalloc((void **)&u0, N * sizeof(float));
    cudaMemcpy(I, h, bytes, cudaMemcpyHostToDevice);
    cudaMemset(u0, 0, N * sizeof(float));
    cudaMemcpy(GS, h, bytes, cudaMemcpyHostToDevice);          /* any upstream gradient on S */
    cudaStream_t s;
    cudaStreamCreate(&s);

    /* forward: the caller owns the scratch (query, allocate once, reuse) */
    size_t fw = lifb_scan_fwd_v3_workspace_bytes(T, N, C, K), bw = lifb_scan_bwd_workspace_bytes(T, N, C);
    void *ws;
    cudaMalloc(&ws, fw > bw ? fw : bw);                          /* cudaMalloc: 256-byte aligned */
    int st = lifb_scan_fwd_v3(I, u0, U, S, T, N, beta, theta, u_r, C, K, -1, ws, fw, NULL, s);
    if (st) return fail("lifb_scan_fwd_v3", st);
    /* adjoint (detached reset, no gradient on U): S may be NULL, it is recomputed from U and I */
    st = lifb_scan_bwd(I, u0, U, NULL, GS, NULL, Lam, T, N, beta, theta, u_r, alpha, 1, C, ws, bw, s);
    if (st) return fail("lifb_scan_bwd", st);
    cudaMemcpyAsync(h, S, bytes, cudaMemcpyDeviceToHost, s);
    if (cudaStreamSynchronize(s) != cudaSuccess || lifb_device_status(1)) return 1;
    double spikes = 0;
    for (int64_t i = 0; i < T * N; i++) spikes += h[i];
    printf("spike rate %.4f\n", spikes / (double)(T * N));
    return 0;
}
