// Fused spike-input Linear -> hard-reset LIF forward (the producer of I for a
// layer of a spiking network such as the 700-256-256-20 net of
// lifscan/shdnet.py:30-66).
//
// A layer computes I[t, b, :] = X[t, b, :] W^T + bias and then the LIF
// recurrence over t for every (b, j).  In a spiking network X is itself a
// spike raster (0/1, a few percent active), so each I row is a sparse sum of
// weight columns.  cuBLAS's fp32 GEMM on such an input sums the active terms
// in input order and adds the bias last (measured bit for bit on B200 for
// both layer shapes of the network); this kernel forms each I element the
// same way, acc = fma(x_c, W[j, c], acc) over the nonzero x_c in increasing c
// from acc = 0, then fl(acc + bias[j]), so I, and with it every spike of the
// layer, equals the unfused Linear -> lif_tuned bit for bit.  I never goes to
// memory: it is formed in shared memory tile by tile and consumed there by
// the recurrence, which writes V (the pre-reset potential the V-path adjoint
// reads) and S.
//
// CTA = one batch element b x 32 outputs j (one per lane), the weight slice
// W[j0:j0+32, :] transposed into shared memory ([Din][32], read conflict-free).
// For each tile of R = 64 rows, the CTA's 8 warps form I for 8 rows each
// (row (t, b) of X read with coalesced loads, a ballot per 32 columns, the
// active columns taken in order), then warp 0 steps the recurrence over the
// tile (state in registers across tiles) and writes the 128-byte V and S rows.
// The tile's I buffer is double-buffered so warps 1-7 form the next tile while
// warp 0 steps this one.
#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace lifb {

namespace {
constexpr int kSLWarps = 8;
constexpr int kSLRows = 64;                  // rows per tile
constexpr int kSLRowsPerWarp = kSLRows / kSLWarps;
constexpr int kSLMaxChunks = 32;             // Din <= 1024

size_t spike_linear_smem(int64_t Din) { return (size_t)Din * 32 * 4 + 2 * (size_t)kSLRows * 32 * 4; }
}  // namespace

template <int NCH>
__global__ void __launch_bounds__(32 * kSLWarps) k_spike_linear_lif(
    const float *__restrict__ X, const float *__restrict__ W, const float *__restrict__ bias,
    const float *__restrict__ u0, float *__restrict__ V, float *__restrict__ S, int64_t T, int64_t B, int Din,
    int Dout, float beta, float theta, float u_r)
{
    extern __shared__ __align__(16) float sl_smem[];
    float *Ws = sl_smem;                          // [Din][32]
    float *Itile = sl_smem + (size_t)Din * 32;    // [2][kSLRows][32]
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int jg = blockIdx.x % (Dout / 32);
    const int64_t b = blockIdx.x / (Dout / 32);
    const int j = jg * 32 + lane;
    const unsigned full = 0xffffffffu;

    // the weight slice, transposed: Ws[c][l] = W[jg*32 + l, c]
    for (int64_t e = threadIdx.x; e < (int64_t)Din * 32; e += blockDim.x) {
        const int l = (int)(e / Din), c = (int)(e % Din);
        Ws[c * 32 + l] = W[(int64_t)(jg * 32 + l) * Din + c];
    }
    const float bj = bias ? bias[j] : 0.0f;
    const int64_t N = B * Dout;
    const int64_t n = b * Dout + j;
    float u = u0 ? u0[n] : 0.0f;
    __syncthreads();

    // I of row t for this lane's output: the active columns in input order
    auto form_row = [&](int64_t t) -> float {
        const float *xr = X + (t * B + b) * Din;
        float xv[NCH];
#pragma unroll
        for (int k = 0; k < NCH; k++) {
            const int c = k * 32 + lane;
            xv[k] = c < Din ? __ldg(xr + c) : 0.0f;
        }
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < NCH; k++) {
            unsigned m = __ballot_sync(full, xv[k] != 0.0f);
            while (m) {
                const int q = __ffs(m) - 1;
                m &= m - 1;
                const float xc = __shfl_sync(full, xv[k], q);
                acc = fmaf(xc, Ws[(k * 32 + q) * 32 + lane], acc);
            }
        }
        return __fadd_rn(acc, bj);
    };

    const int64_t ntiles = (T + kSLRows - 1) / kSLRows;
    // tile 0 by every warp
    for (int r = w * kSLRowsPerWarp; r < (w + 1) * kSLRowsPerWarp; r++)
        if (r < T) Itile[r * 32 + lane] = form_row(r);
    __syncthreads();
    for (int64_t k = 0; k < ntiles; k++) {
        const float *cur = Itile + (k & 1) * kSLRows * 32;
        float *nxt = Itile + ((k + 1) & 1) * kSLRows * 32;
        const int64_t t0 = k * kSLRows;
        if (w == 0) {
            // the recurrence over this tile
            const int rows = (int)(T - t0 < kSLRows ? T - t0 : kSLRows);
            for (int r = 0; r < rows; r++) {
                const float v = __fadd_rn(__fmul_rn(beta, u), cur[r * 32 + lane]);
                const bool f = v >= theta;
                u = f ? u_r : v;
                const int64_t o = (t0 + r) * N + n;
                V[o] = v;
                S[o] = f ? 1.0f : 0.0f;
            }
        } else if (k + 1 < ntiles) {
            // warps 1..7 form the next tile meanwhile (its 64 rows over 7 warps)
            const int64_t t1 = t0 + kSLRows;
            for (int r = w - 1; r < kSLRows; r += kSLWarps - 1)
                if (t1 + r < T) nxt[r * 32 + lane] = form_row(t1 + r);
        }
        __syncthreads();
    }
}

bool spike_linear_lif_fwd(const float *X, const float *W, const float *bias, const float *u0, float *V, float *S,
                          int64_t T, int64_t B, int64_t Din, int64_t Dout, float beta, float theta, float u_r,
                          cudaStream_t s)
{
    if (Din <= 0 || Din > 32 * kSLMaxChunks || Dout <= 0 || Dout % 32) return false;
    const size_t smem = spike_linear_smem(Din);
    int dev = 0, lim = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&lim, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        smem > (size_t)lim)
        return false;
    const int64_t grid = B * (Dout / 32);
    if (grid <= 0 || grid > INT32_MAX) return false;
    const int nch = (int)((Din + 31) / 32);
    auto go = [&](auto kern) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        count_launches(1);
        kern<<<(unsigned)grid, 32 * kSLWarps, smem, s>>>(X, W, bias, u0, V, S, T, B, (int)Din, (int)Dout, beta, theta,
                                                         u_r);
    };
    if (nch <= 8) go(k_spike_linear_lif<8>);
    else if (nch <= 24) go(k_spike_linear_lif<24>);
    else go(k_spike_linear_lif<32>);
    return true;
}

}  // namespace lifb

extern "C" int lifb_spike_linear_lif_fwd(const float *X, const float *W, const float *bias, const float *u0, float *V,
                                         float *S, int64_t T, int64_t B, int64_t Din, int64_t Dout, float beta,
                                         float theta, float u_r, void *stream)
{
    LIFB_RANGE("lifb_spike_linear_lif_fwd");
    if (T < 0 || B < 0 || Din <= 0 || Dout <= 0) {
        lifb::set_last_error("lifb_spike_linear_lif_fwd: negative shape or empty Din/Dout");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (T == 0 || B == 0) return LIFB_OK;
    if (!X || !W || !V || !S) {
        lifb::set_last_error("lifb_spike_linear_lif_fwd: null tensor pointer");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (!lifb::spike_linear_lif_fwd(X, W, bias, u0, V, S, T, B, Din, Dout, beta, theta, u_r, (cudaStream_t)stream)) {
        lifb::set_last_error("lifb_spike_linear_lif_fwd: needs Dout a multiple of 32 and Din <= 1024 (the weight "
                             "slice in shared memory)");
        return LIFB_ERR_UNSUPPORTED;
    }
    if (cudaGetLastError() != cudaSuccess) {
        lifb::set_last_error("lifb_spike_linear_lif_fwd: launch failed");
        return LIFB_ERR_CUDA;
    }
    lifb::set_last_error("");
    return LIFB_OK;
}
