// Leaky (non-spiking) integrator over time, the readout of config 3's network:
// forward y_t = beta * y_{t-1} + z_t (y_{-1} = 0) and its adjoint
// lam_t = g_t + beta * lam_{t+1} (lam_T = 0), over [T, M] row-major.
//
// Both are linear recurrences, so time splits into chunks of kLkChunk rows:
// one CTA owns 32 columns (one per lane) and all T rows, one warp per chunk.
// A warp runs its chunk's recurrence from 0 in registers, publishes the
// chunk's last value, takes its carry-in from the earlier chunks' ends in order
// (a sequential fold over at most 31 values, each warp on its own) and adds
// carry * beta^k to its rows.  One launch, one read and one write of the data.
// The result equals the sequential recurrence up to fp32 rounding (the carry
// enters as one scaled add instead of row by row).
#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace lifb {

namespace {
constexpr int kLkChunk = 32;   // rows per warp
constexpr int kLkMaxWarps = 32;  // T <= 1024 in one launch (the chunk lives in registers)
}  // namespace

// REV = false: the forward (chunks in time order, carry from the chunks before);
// REV = true: the adjoint (each chunk swept backwards, carry from the chunks after).
template <bool REV>
__global__ void __launch_bounds__(32 * kLkMaxWarps) k_leaky(const float *__restrict__ in, float *__restrict__ out,
                                                            int64_t T, int64_t M, float beta)
{
    __shared__ float s_end[kLkMaxWarps][32];
    __shared__ float s_pow[kLkMaxWarps];  // beta^(rows of chunk w)
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = blockDim.x >> 5;
    const int64_t col = (int64_t)blockIdx.x * 32 + lane;
    const bool act = col < M;
    const int64_t t0 = (int64_t)w * kLkChunk;
    const int rows = (int)(T - t0 < kLkChunk ? (T - t0 > 0 ? T - t0 : 0) : kLkChunk);

    float loc[kLkChunk];
#pragma unroll
    for (int r = 0; r < kLkChunk; r++) {
        const int rr = REV ? kLkChunk - 1 - r : r;  // the order the recurrence visits the rows
        loc[rr] = (act && rr < rows) ? __ldg(in + (t0 + rr) * M + col) : 0.0f;
    }
    float y = 0.0f;
#pragma unroll
    for (int r = 0; r < kLkChunk; r++) {
        const int rr = REV ? kLkChunk - 1 - r : r;
        if (rr < rows) {
            y = __fadd_rn(__fmul_rn(beta, y), loc[rr]);
            loc[rr] = y;
        }
    }
    s_end[w][lane] = y;  // the chunk's value at its last visited row
    if (lane == 0) {
        float p = 1.0f;
        for (int r = 0; r < rows; r++) p = __fmul_rn(p, beta);
        s_pow[w] = p;
    }
    __syncthreads();
    // carry into this chunk: the chunks visited before it, folded in visiting order
    float cin = 0.0f;
    if (!REV) {
        for (int v = 0; v < w; v++) cin = __fadd_rn(__fmul_rn(s_pow[v], cin), s_end[v][lane]);
    } else {
        for (int v = nw - 1; v > w; v--) cin = __fadd_rn(__fmul_rn(s_pow[v], cin), s_end[v][lane]);
    }
    float p = beta;  // beta^(rows visited since the carry entered, + 1)
#pragma unroll
    for (int r = 0; r < kLkChunk; r++) {
        const int rr = REV ? kLkChunk - 1 - r : r;
        if (rr < rows) {
            const float v = __fadd_rn(loc[rr], __fmul_rn(p, cin));
            if (act) out[(t0 + rr) * M + col] = v;
            p = __fmul_rn(p, beta);
        }
    }
}

// False when T is past the one-launch form (32 chunks of 32 rows).
bool leaky(const float *in, float *out, int64_t T, int64_t M, float beta, bool rev, cudaStream_t s)
{
    if (T <= 0 || M <= 0) return true;
    const int64_t nw = (T + kLkChunk - 1) / kLkChunk;
    if (nw > kLkMaxWarps || (M + 31) / 32 > INT32_MAX) return false;
    const unsigned grid = (unsigned)((M + 31) / 32);
    count_launches(1);
    if (rev) k_leaky<true><<<grid, (unsigned)(32 * nw), 0, s>>>(in, out, T, M, beta);
    else k_leaky<false><<<grid, (unsigned)(32 * nw), 0, s>>>(in, out, T, M, beta);
    return true;
}

}  // namespace lifb

extern "C" int lifb_leaky_fwd(const float *Z, float *Y, int64_t T, int64_t M, float beta, void *stream)
{
    LIFB_RANGE("lifb_leaky_fwd");
    if (T < 0 || M < 0) {
        lifb::set_last_error("lifb_leaky_fwd: negative shape");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (T == 0 || M == 0) return LIFB_OK;
    if (!Z || !Y) {
        lifb::set_last_error("lifb_leaky_fwd: null tensor pointer");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (!lifb::leaky(Z, Y, T, M, beta, false, (cudaStream_t)stream)) {
        lifb::set_last_error("lifb_leaky_fwd: needs T <= 1024");
        return LIFB_ERR_UNSUPPORTED;
    }
    if (cudaGetLastError() != cudaSuccess) {
        lifb::set_last_error("lifb_leaky_fwd: launch failed");
        return LIFB_ERR_CUDA;
    }
    lifb::set_last_error("");
    return LIFB_OK;
}

extern "C" int lifb_leaky_bwd(const float *GY, float *GZ, int64_t T, int64_t M, float beta, void *stream)
{
    LIFB_RANGE("lifb_leaky_bwd");
    if (T < 0 || M < 0) {
        lifb::set_last_error("lifb_leaky_bwd: negative shape");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (T == 0 || M == 0) return LIFB_OK;
    if (!GY || !GZ) {
        lifb::set_last_error("lifb_leaky_bwd: null tensor pointer");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (!lifb::leaky(GY, GZ, T, M, beta, true, (cudaStream_t)stream)) {
        lifb::set_last_error("lifb_leaky_bwd: needs T <= 1024");
        return LIFB_ERR_UNSUPPORTED;
    }
    if (cudaGetLastError() != cudaSuccess) {
        lifb::set_last_error("lifb_leaky_bwd: launch failed");
        return LIFB_ERR_CUDA;
    }
    lifb::set_last_error("");
    return LIFB_OK;
}
