// Spike-input Linear layers of a spiking network (the 700-256-256-20 net of
// lifscan/shdnet.py:30-66): the bitmask spike format, the fused
// Linear -> hard-reset LIF forward, and the sparse weight gradient.
//
// Spike mask.  A [R, D] fp32 tensor whose rows are mostly zeros (a spike
// raster, R = T*B rows (t, b)) is described by mask words [R, NWp], NWp =
// round_up(ceil(D/32) + 1, 4): word k of a row holds bit q set when element
// 32k + q is nonzero (NaN counts as nonzero, -0 as zero), word ceil(D/32)
// has bit 0 set when some nonzero element of the row is not exactly 1.0 (an
// "odd" row: its consumers read the values from the dense tensor), the rest
// is padding so that a row is a whole number of 16-byte TMA units.  88-96
// bytes describe a 700-input row of 2800 bytes.  k_spike_mask writes it from
// the dense tensor; the fused forward writes the mask of its own spikes for
// the next layer, so only the network input is ever scanned.
//
// Fused forward (k_spike_linear_lif).  I[t, b, j] = X[t, b, :] W[j, :]^T +
// bias[j], then the LIF recurrence over t for every (b, j), writing V (the
// pre-reset potentials the V-path adjoint reads), S and the mask of S.
// cuBLAS's fp32 GEMM on such an input sums x_c * W[j, c] with fused
// multiply-adds in input order from 0 and adds the bias last (measured bit
// for bit on B200 for both layer shapes of the network); terms with x_c = 0
// leave the sum unchanged, so summing only the active inputs in increasing c
// gives the same bits, and so do the spikes.  One CTA owns 32*JW outputs j
// (JW = 1, 2 or 4 per lane: the widest whose slice fits) and `bpc` batch elements: the weight slice sits transposed in
// shared memory ([Din][32] JW-vectors, a conflict-free broadcast read per
// active input), the mask rows of each 16-step tile arrive by one 3-D TMA
// load (four stages in flight, bounded mbarrier waits), and the warps take the
// tile's rows from a shared counter, expand each row's mask into a list of
// active inputs (a warp prefix sum of the words' popcounts) and sum the listed
// weight vectors in order; one warp per batch element first steps the
// recurrence over the previous tile from shared memory.  I never reaches global memory.  Weights that are not finite make
// the GEMM's zero terms NaN (0 * inf): the lanes of such outputs take the
// dense sum over every input instead, so the bits still match.
//
// Weight gradient (k_spike_wgrad).  gW[j, c] = sum_r dI[r, j] X[r, c] and
// gb[j] = sum_r dI[r, j] touch only the active (r, c): per 32-row block a
// producer warp stages the dI tile of the CTA's outputs and the block's mask
// rows by TMA into a 4-stage ring (full/empty mbarriers, so consumer warps
// drift apart instead of meeting at a barrier per block);
// each warp owns 8 input columns and 32*JJ outputs (JJ per lane, up to 8: an
// accumulator per column and output in registers), turns the block's mask
// bits into per-column row sets with ballots (only for columns active in the
// block) and adds the listed dI rows in row order.  Each CTA covers a chunk of
// rows whose size follows from the shape alone; a second pass adds the
// chunks in a fixed order (eight contiguous groups in chunk order, then the
// groups in order), so the result is deterministic and the same on every GPU.
#include "lifb_common.cuh"
#include "lifb_internal.h"
#include "tma.cuh"

#include <algorithm>
#include <string>

namespace lifb {

namespace {
constexpr unsigned kFull = 0xffffffffu;
constexpr int kMaskWarps = 8;    // rows (one per warp) in flight per mask CTA
constexpr int kSLTile = 16;      // time steps per producer tile
constexpr int kSLStages = 4;     // mask tiles in flight
constexpr int kSLWarps = 16;     // producer CTA: every warp forms rows; bpc of them also step the LIF
constexpr int kWgWarps = 16;     // weight-gradient CTA: 16 consumer warps x 8 columns, plus a producer warp
constexpr int kWgCols = 8;
constexpr int kWgTargetCtas = 148;  // row chunks sized for about this many CTAs (from the shape alone)
constexpr int kWgStages = 4;        // dI and mask tiles in flight per CTA
}  // namespace

int64_t spike_mask_stride(int64_t D) { return ((D + 31) / 32 + 1 + 3) / 4 * 4; }

template <int NCH>
__global__ void __launch_bounds__(32 * kMaskWarps) k_spike_mask(const float *__restrict__ X, uint32_t *__restrict__ M,
                                                               int64_t R, int D, int NWp)
{
    const int lane = threadIdx.x & 31;
    const int NW = (D + 31) >> 5;
    const int64_t nwarps = (int64_t)gridDim.x * kMaskWarps;
    for (int64_t row = (int64_t)blockIdx.x * kMaskWarps + (threadIdx.x >> 5); row < R; row += nwarps) {
        const float *xr = X + row * D;
        float xv[NCH];
#pragma unroll
        for (int k = 0; k < NCH; k++) {
            const int c = k * 32 + lane;
            xv[k] = c < D ? __ldcs(xr + c) : 0.0f;
        }
        uint32_t mine = 0;
        bool odd = false;
#pragma unroll
        for (int k = 0; k < NCH; k++) {
            const uint32_t b = __ballot_sync(kFull, xv[k] != 0.0f);
            mine = lane == k ? b : mine;
            odd |= xv[k] != 0.0f && xv[k] != 1.0f;
        }
        const bool any_odd = __any_sync(kFull, odd);
        uint32_t *mr = M + row * NWp;
        for (int i = lane; i < NWp; i += 32) mr[i] = i < NW ? mine : (i == NW && any_odd ? 1u : 0u);
    }
}

bool spike_mask(const float *X, uint32_t *M, int64_t R, int64_t D, cudaStream_t s)
{
    if (D <= 0 || D > 1024 || ((uintptr_t)M & 15)) return false;
    int dev = 0, nsm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev))
        return false;
    const int NWp = (int)spike_mask_stride(D);
    const int64_t want = (R + kMaskWarps - 1) / kMaskWarps;
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)nsm * 8));
    const int nch = (int)((D + 31) / 32);
    count_launches(1);
    if (nch <= 8) k_spike_mask<8><<<grid, 32 * kMaskWarps, 0, s>>>(X, M, R, (int)D, NWp);
    else if (nch <= 16) k_spike_mask<16><<<grid, 32 * kMaskWarps, 0, s>>>(X, M, R, (int)D, NWp);
    else if (nch <= 24) k_spike_mask<24><<<grid, 32 * kMaskWarps, 0, s>>>(X, M, R, (int)D, NWp);
    else k_spike_mask<32><<<grid, 32 * kMaskWarps, 0, s>>>(X, M, R, (int)D, NWp);
    return true;
}

// ---------------------------------------------------------------------------
// fused forward

namespace {
struct SLSmem {
    size_t it, mk, lst, total;
};
__host__ __device__ inline SLSmem sl_layout(int Din, int JW, int bpc, int NWp)
{
    SLSmem L;
    L.it = (size_t)Din * 32 * JW * 4;                                    // weight slice at 0
    L.mk = (L.it + (size_t)2 * bpc * kSLTile * 32 * JW * 4 + 127) / 128 * 128;  // I tiles, then mask tiles
    L.lst = L.mk + (size_t)kSLStages * kSLTile * bpc * NWp * 4;
    L.total = L.lst + (size_t)kSLWarps * 32 * 4;
    return L;
}
}  // namespace

// Shared-memory loads at 32-bit shared addresses: JW consecutive floats, and
// four ints (a broadcast read of four list entries).
template <int JW>
__device__ __forceinline__ void lds_f32(uint32_t a, float (&w)[JW])
{
    if constexpr (JW == 4)
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(w[0]), "=f"(w[1]), "=f"(w[2]), "=f"(w[3]) : "r"(a));
    else if constexpr (JW == 2)
        asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(w[0]), "=f"(w[1]) : "r"(a));
    else
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(w[0]) : "r"(a));
}

__device__ __forceinline__ int4 lds_s32x4(uint32_t a)
{
    int4 v;
    asm volatile("ld.shared.v4.s32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(a)
                 : "memory");
    return v;
}

template <int JW>
__global__ void __launch_bounds__(32 * kSLWarps, 1) k_spike_linear_lif(
    const __grid_constant__ CUtensorMap tm, const float *__restrict__ X, const float *__restrict__ W,
    const float *__restrict__ bias, const float *__restrict__ u0, float *__restrict__ V, float *__restrict__ S,
    uint32_t *__restrict__ Sm, int64_t T, int64_t B, int Din, int Dout, int bpc, int NWp, int NWop, float beta,
    float theta, float u_r, int *status)
{
    constexpr int OG = 32 * JW;
    extern __shared__ __align__(128) unsigned char sl_raw[];
    const SLSmem L = sl_layout(Din, JW, bpc, NWp);
    float *Ws = reinterpret_cast<float *>(sl_raw);
    float *It = reinterpret_cast<float *>(sl_raw + L.it);
    uint32_t *Mk = reinterpret_cast<uint32_t *>(sl_raw + L.mk);
    __shared__ uint64_t bar[kSLStages];
    __shared__ int s_bad[OG];
    __shared__ int s_err;
    __shared__ int s_next[2];

    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ngroups = Dout / OG;
    const int jg = (int)(blockIdx.x % ngroups);
    const int64_t b0 = (int64_t)(blockIdx.x / ngroups) * bpc;
    const int nb = (int)(B - b0 < bpc ? B - b0 : bpc);
    const int j0 = jg * OG;
    const int NW = (Din + 31) >> 5;
    const int NWo = Dout >> 5;
    const int64_t ntiles = (T + kSLTile - 1) / kSLTile;
    const size_t mtile = (size_t)kSLTile * bpc * NWp;  // words per mask tile
    const uint32_t tile_bytes = (uint32_t)(mtile * 4);
    int *lst = reinterpret_cast<int *>(sl_raw + L.lst) + w * 32;
    constexpr int kWRow = 128 * JW;  // bytes per input row of the weight slice
    const uint32_t wbase = smem_u32(Ws) + 4u * JW * lane;
    const uint32_t lst_s = smem_u32(lst);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kSLStages; i++) mbar_init(&bar[i], 1);
        fence_barrier_init();
        s_err = 0;
        s_next[0] = 0;
    }
    for (int i = threadIdx.x; i < OG; i += blockDim.x) s_bad[i] = 0;
    __syncthreads();
    int64_t last[kSLStages];  // (thread 0) the last tile issued into each buffer
    for (int i = 0; i < kSLStages; i++) last[i] = -1;
    if (threadIdx.x == 0) {
        for (int k = 0; k < kSLStages && k < ntiles; k++) {
            mbar_arrive_expect_tx(&bar[k], tile_bytes);
            tma_load_3d(Mk + k * mtile, &tm, 0, (int)b0, k * kSLTile, &bar[k]);
            last[k] = k;
        }
    }
    // the weight slice, transposed: Ws[(c * 32 + l) * JW + e] = W[j0 + e * 32 + l, c]; a lane
    // reads 16 contiguous bytes of one output's row (whole rows aligned to 16 bytes), else 4
    if (Din % 4 == 0 && ((uintptr_t)W & 15) == 0) {
        const int nq = Din / 4;
#pragma unroll 4
        for (int e = threadIdx.x; e < OG * nq; e += blockDim.x) {
            const int o = e % OG, q = e / OG;
            const float4 v = __ldg(reinterpret_cast<const float4 *>(W + (int64_t)(j0 + o) * Din) + q);
            float *wd = Ws + ((size_t)(4 * q) * 32 + (o & 31)) * JW + (o >> 5);
            wd[0] = v.x;
            wd[32 * JW] = v.y;
            wd[64 * JW] = v.z;
            wd[96 * JW] = v.w;
            if (!(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w))) s_bad[o] = 1;
        }
    } else {
#pragma unroll 8
        for (int64_t e = threadIdx.x; e < (int64_t)Din * OG; e += blockDim.x) {
            const int o = (int)(e % OG), c = (int)(e / OG);
            const float wv = __ldg(W + (int64_t)(j0 + o) * Din + c);
            Ws[((size_t)c * 32 + (o & 31)) * JW + (o >> 5)] = wv;
            if (!isfinite(wv)) s_bad[o] = 1;
        }
    }
    __syncthreads();
    float bj[JW];
    bool bad[JW];
    bool any_bad = false;
#pragma unroll
    for (int e = 0; e < JW; e++) {
        bj[e] = bias ? __ldg(bias + j0 + e * 32 + lane) : 0.0f;
        bad[e] = s_bad[e * 32 + lane] != 0;
        any_bad |= bad[e];
    }
    const bool warp_bad = __any_sync(kFull, any_bad);

    // I of one row for this lane's outputs: the active inputs, in order
    auto form = [&](const uint32_t *mr, int64_t row, float *dst) {
        uint32_t m = lane < NW ? mr[lane] : 0u;
        if (lane == NW - 1 && (Din & 31)) m &= (1u << (Din & 31)) - 1u;  // bits past Din are not inputs
        const bool odd = (mr[NW] & 1u) != 0;
        const float *xr = X + row * Din;
        float a[JW];
#pragma unroll
        for (int e = 0; e < JW; e++) a[e] = 0.0f;
        const int cnt = __popc(m);
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += y;
        }
        const int total = __shfl_sync(kFull, incl, 31);
        uint32_t mm = m;
        int p = incl - cnt;  // list position of this lane's next active input
        for (int base = 0; base < total; base += 32) {
            // the list holds the active inputs' byte offsets into the weight slice
            while (mm && p < base + 32) {
                const int q = __ffs(mm) - 1;
                mm &= mm - 1;
                lst[p - base] = (lane * 32 + q) * kWRow;
                p++;
            }
            __syncwarp();
            const int n = total - base < 32 ? total - base : 32;
            int i = 0;
            if (!odd) {
                for (; i + 4 <= n; i += 4) {
                    const int4 o = lds_s32x4(lst_s + 4 * i);
                    float w0[JW], w1[JW], w2[JW], w3[JW];
                    lds_f32<JW>(wbase + o.x, w0);
                    lds_f32<JW>(wbase + o.y, w1);
                    lds_f32<JW>(wbase + o.z, w2);
                    lds_f32<JW>(wbase + o.w, w3);
#pragma unroll
                    for (int e = 0; e < JW; e++)
                        a[e] = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(a[e], w0[e]), w1[e]), w2[e]), w3[e]);
                }
                for (; i < n; i++) {
                    float w0[JW];
                    lds_f32<JW>(wbase + lst[i], w0);
#pragma unroll
                    for (int e = 0; e < JW; e++) a[e] = __fadd_rn(a[e], w0[e]);
                }
            } else {
                for (; i < n; i++) {
                    const int o = lst[i];
                    const float x = __ldg(xr + o / kWRow);
                    float w0[JW];
                    lds_f32<JW>(wbase + o, w0);
#pragma unroll
                    for (int e = 0; e < JW; e++) a[e] = fmaf(x, w0[e], a[e]);
                }
            }
            __syncwarp();  // the next batch rewrites the list
        }
        if (warp_bad) {  // non-finite weights: every term, zeros included
            float d[JW];
#pragma unroll
            for (int e = 0; e < JW; e++) d[e] = 0.0f;
            for (int c = 0; c < Din; c++) {
                const float x = __ldg(xr + c);
#pragma unroll
                for (int e = 0; e < JW; e++) d[e] = fmaf(x, Ws[((size_t)c * 32 + lane) * JW + e], d[e]);
            }
#pragma unroll
            for (int e = 0; e < JW; e++) a[e] = bad[e] ? d[e] : a[e];
        }
#pragma unroll
        for (int e = 0; e < JW; e++) dst[e * 32 + lane] = __fadd_rn(a[e], bj[e]);
    };

    float u[JW];
#pragma unroll
    for (int e = 0; e < JW; e++) u[e] = (w < nb && u0) ? u0[(b0 + w) * Dout + j0 + e * 32 + lane] : 0.0f;
    const int slots = nb * kSLTile;
    for (int64_t k = 0; k <= ntiles; k++) {
        if (threadIdx.x == 0) s_next[(k + 1) & 1] = 0;  // the row counter of the next tile
        if (w < nb && k >= 1) {  // the recurrence over tile k - 1
            const int64_t t0 = (k - 1) * kSLTile;
            const float *cur = It + ((size_t)((k - 1) & 1) * bpc + w) * kSLTile * OG;
            const int rows = (int)(T - t0 < kSLTile ? T - t0 : kSLTile);
            auto step_row = [&](int r) {
                const int64_t row = (t0 + r) * B + b0 + w;
                float *vo = V + row * Dout + j0;
                float *so = S + row * Dout + j0;
                uint32_t mw[JW];
#pragma unroll
                for (int e = 0; e < JW; e++) {
                    const float v = __fadd_rn(__fmul_rn(beta, u[e]), cur[r * OG + e * 32 + lane]);
                    const bool f = v >= theta;
                    u[e] = f ? u_r : v;
                    vo[e * 32 + lane] = v;
                    so[e * 32 + lane] = f ? 1.0f : 0.0f;
                    mw[e] = __ballot_sync(kFull, f);
                }
                if (Sm) {
                    uint32_t *mo = Sm + row * NWop;
                    uint32_t mine = mw[0];
#pragma unroll
                    for (int e = 1; e < JW; e++) mine = lane == e ? mw[e] : mine;
                    if (lane < JW) mo[jg * JW + lane] = mine;
                    if (jg == 0 && NWo + lane < NWop) mo[NWo + lane] = 0u;  // spikes are 0/1: not odd
                }
            };
            if (rows == kSLTile) {  // unrolled: the tile's I loads go ahead of the chain through u
#pragma unroll
                for (int r = 0; r < kSLTile; r++) step_row(r);
            } else {
                for (int r = 0; r < rows; r++) step_row(r);
            }
        }
        if (k < ntiles) {  // form tile k: every warp takes rows from a shared counter until none are left
            const int st = (int)(k % kSLStages);
            if (!s_err && !mbar_wait(&bar[st], (uint32_t)((k / kSLStages) & 1)) && lane == 0) atomicExch(&s_err, 1);
            const uint32_t *mt = Mk + st * mtile;
            float *nxt = It + (size_t)(k & 1) * bpc * kSLTile * OG;
            const int64_t t0 = k * kSLTile;
            for (;;) {
                int f = 0;
                if (lane == 0) f = atomicAdd(&s_next[k & 1], 1);
                f = __shfl_sync(kFull, f, 0);
                if (f >= slots) break;
                const int bi = f / kSLTile, r = f % kSLTile;
                if (t0 + r < T)
                    form(mt + ((size_t)r * bpc + bi) * NWp, (t0 + r) * B + b0 + bi,
                         nxt + ((size_t)bi * kSLTile + r) * OG);
            }
        }
        __syncthreads();
        if (threadIdx.x == 0 && k < ntiles && k + kSLStages < ntiles && !s_err) {  // stage k is free again
            const int st = (int)(k % kSLStages);
            mbar_arrive_expect_tx(&bar[st], tile_bytes);
            tma_load_3d(Mk + st * mtile, &tm, 0, (int)b0, (int)((k + kSLStages) * kSLTile), &bar[st]);
            last[st] = k + kSLStages;
        }
    }
    if (threadIdx.x == 0 && s_err) {
        // let copies still in flight land before the CTA's shared memory goes away
        for (int i = 0; i < kSLStages; i++)
            if (last[i] >= 0) mbar_wait(&bar[i], (uint32_t)((last[i] / kSLStages) & 1));
        if (status) atomicCAS(status, 0, (int)kStatusTmaWaitTimeout);
    }
}

bool spike_linear_lif_fwd(const float *X, const uint32_t *Xm, const float *W, const float *bias, const float *u0,
                          float *V, float *S, uint32_t *Sm, int64_t T, int64_t B, int64_t Din, int64_t Dout,
                          float beta, float theta, float u_r, cudaStream_t s)
{
    if (Din <= 0 || Din > 1024 || Dout <= 0 || Dout % 32 || T >= INT32_MAX || B >= INT32_MAX) return false;
    if (((uintptr_t)Xm & 15) || (Sm && ((uintptr_t)Sm & 15))) return false;
    const int NWp = (int)spike_mask_stride(Din), NWop = (int)spike_mask_stride(Dout);
    int dev = 0, nsm = 0, lim = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) ||
        cudaDeviceGetAttribute(&lim, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev))
        return false;
    int JW = 1;  // outputs per lane: the widest whose weight slice fits in shared memory
    for (int cand = 4; cand >= 2; cand /= 2)
        if (JW == 1 && Dout % (32 * cand) == 0 && sl_layout((int)Din, cand, 1, NWp).total <= (size_t)lim) JW = cand;
    if (sl_layout((int)Din, JW, 1, NWp).total > (size_t)lim) return false;
    const int64_t groups = Dout / (32 * JW);
    auto go = [&](auto kern) -> bool {
        // batch elements per CTA: the fewest that put every CTA on the GPU at once
        int bpc = 1;
        for (int cand = 1; cand <= 4; cand++) {
            const size_t sm = sl_layout((int)Din, JW, cand, NWp).total;
            if (sm > (size_t)lim) break;
            int occ = 0;
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 32 * kSLWarps, sm) != cudaSuccess || occ < 1)
                break;
            bpc = cand;
            if (groups * ((B + cand - 1) / cand) <= (int64_t)nsm * occ) break;
        }
        const size_t smem = sl_layout((int)Din, JW, bpc, NWp).total;
        CUtensorMap tm;
        if (!make_tmap_3d_u32(&tm, Xm, NWp, B, T, NWp, bpc, kSLTile)) return false;
        const int64_t grid = groups * ((B + bpc - 1) / bpc);
        if (grid > INT32_MAX) return false;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        count_launches(1);
        kern<<<(unsigned)grid, 32 * kSLWarps, smem, s>>>(tm, X, W, bias, u0, V, S, Sm, T, B, (int)Din, (int)Dout,
                                                          bpc, NWp, NWop, beta, theta, u_r, device_status_ptr());
        return true;
    };
    return JW == 4 ? go(k_spike_linear_lif<4>) : JW == 2 ? go(k_spike_linear_lif<2>) : go(k_spike_linear_lif<1>);
}

// ---------------------------------------------------------------------------
// weight gradient

namespace {
// A lane's JJ outputs: groups of 4 consecutive outputs, 128 apart (JJ >= 4),
// or JJ consecutive ones; either way a lane's shared-memory reads are
// conflict-free 16-, 8- or 4-byte vectors.
template <int JJ>
__device__ __forceinline__ int wg_out(int lane, int e)
{
    return JJ >= 4 ? (e >> 2) * 128 + 4 * lane + (e & 3) : JJ * lane + e;
}

template <int JJ>
__device__ __forceinline__ void wg_load(const float *row, int lane, float (&d)[JJ])
{
    if constexpr (JJ >= 4) {
#pragma unroll
        for (int g = 0; g < JJ / 4; g++) {
            const float4 v = *reinterpret_cast<const float4 *>(row + g * 128 + 4 * lane);
            d[4 * g] = v.x;
            d[4 * g + 1] = v.y;
            d[4 * g + 2] = v.z;
            d[4 * g + 3] = v.w;
        }
    } else if constexpr (JJ == 2) {
        const float2 v = *reinterpret_cast<const float2 *>(row + 2 * lane);
        d[0] = v.x;
        d[1] = v.y;
    } else {
        d[0] = row[lane];
    }
}

struct WgPlan {
    int JJ;
    int64_t nsg, njs, chunk, nck, Dp;
};

// Work split of the weight gradient: 32*JJ outputs per warp, kWgCols columns
// per warp, kWgWarps warps per CTA, and the rows in chunks sized so that
// about kWgTargetCtas CTAs cover the job.  It depends on the shape only, so
// the summation order (and the result) is the same on every GPU.
WgPlan wg_plan(int64_t R, int64_t Din, int64_t Dout)
{
    WgPlan p;
    p.JJ = Dout % 256 == 0 ? 8 : Dout % 128 == 0 ? 4 : Dout % 64 == 0 ? 2 : 1;
    p.Dp = (Din + kWgCols - 1) / kWgCols * kWgCols;
    p.nsg = (p.Dp / kWgCols + kWgWarps - 1) / kWgWarps;
    p.njs = (Dout + 32 * p.JJ - 1) / (32 * p.JJ);  // the last slice may be partial (JJ = 1)
    const int64_t want = std::max<int64_t>(1, kWgTargetCtas / (p.nsg * p.njs));
    p.chunk = std::max<int64_t>(32, ((R + want - 1) / want + 31) / 32 * 32);
    p.nck = (R + p.chunk - 1) / p.chunk;
    return p;
}

size_t wg_smem(int JJ, int NWp) { return (size_t)kWgStages * 32 * 32 * JJ * 4 + (size_t)kWgStages * 32 * NWp * 4; }
}  // namespace

template <int JJ>
__global__ void __launch_bounds__(32 * (kWgWarps + 1), 1) k_spike_wgrad(const __grid_constant__ CUtensorMap tdi,
                                                                       const __grid_constant__ CUtensorMap tmk,
                                                                       const float *__restrict__ X,
                                                                       float *__restrict__ Pw, float *__restrict__ Pb,
                                                                       int64_t R, int Din, int Dout, int NWp, int Dp,
                                                                       int64_t chunk, int *status)
{
    constexpr int JS = 32 * JJ;
    extern __shared__ __align__(128) unsigned char wg_raw[];
    float *s_d = reinterpret_cast<float *>(wg_raw);                                         // [stages][32][JS]
    uint32_t *s_m = reinterpret_cast<uint32_t *>(wg_raw + (size_t)kWgStages * 32 * JS * 4);  // [stages][32][NWp]
    __shared__ uint64_t full[kWgStages], empty[kWgStages];
    __shared__ int s_err;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int js = blockIdx.y;
    const int64_t ck = blockIdx.z;
    const int64_t r0 = ck * chunk;
    const int64_t rend = R < r0 + chunk ? R : r0 + chunk;
    const int nblk = (int)((rend - r0 + 31) / 32);
    const bool do_bias = Pb && blockIdx.x == 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kWgStages; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kWgWarps);
        }
        fence_barrier_init();
        s_err = 0;
    }
    __syncthreads();

    if (w == kWgWarps) {
        // producer warp: one lane streams the dI and mask tiles of the chunk's
        // blocks, refilling a stage once every consumer warp has released it
        if (lane == 0) {
            const uint32_t bytes = (uint32_t)(32 * JS * 4 + 32 * NWp * 4);
            int last[kWgStages];
            for (int i = 0; i < kWgStages; i++) last[i] = -1;
            for (int b = 0; b < nblk && !s_err; b++) {
                const int st = b % kWgStages;
                if (b >= kWgStages && !mbar_wait(&empty[st], (uint32_t)((b / kWgStages - 1) & 1))) {
                    atomicExch(&s_err, 1);
                    break;
                }
                mbar_arrive_expect_tx(&full[st], bytes);
                tma_load_2d(s_d + st * 32 * JS, &tdi, js * JS, (int)(r0 + 32 * b), &full[st]);
                tma_load_2d(s_m + st * 32 * NWp, &tmk, 0, (int)(r0 + 32 * b), &full[st]);
                last[st] = b;
            }
            if (s_err) {  // let copies in flight land before the CTA's shared memory goes away
                for (int i = 0; i < kWgStages; i++)
                    if (last[i] >= 0) mbar_wait(&full[i], (uint32_t)((last[i] / kWgStages) & 1));
                if (status) atomicCAS(status, 0, (int)kStatusTmaWaitTimeout);
            }
        }
        __syncthreads();  // the consumers' closing barrier
        return;
    }

    const int c0 = (blockIdx.x * kWgWarps + w) * kWgCols;
    const int NW = (Din + 31) >> 5;
    const bool has_cols = c0 < Din;
    float acc[kWgCols][JJ];
    float accb[JJ];
#pragma unroll
    for (int q = 0; q < kWgCols; q++)
#pragma unroll
        for (int e = 0; e < JJ; e++) acc[q][e] = 0.0f;
#pragma unroll
    for (int e = 0; e < JJ; e++) accb[e] = 0.0f;

    for (int b = 0; b < nblk; b++) {
        const int st = b % kWgStages;
        if (s_err) break;
        if (!mbar_wait(&full[st], (uint32_t)((b / kWgStages) & 1))) {
            if (lane == 0) atomicExch(&s_err, 1);
            break;
        }
        const float *dt = s_d + st * 32 * JS;
        const uint32_t *mt = s_m + st * 32 * NWp;
        if (has_cols) {
            uint32_t wd = (mt[lane * NWp + (c0 >> 5)] >> (c0 & 31)) & ((1u << kWgCols) - 1u);
            if (Din - c0 < kWgCols) wd &= (1u << (Din - c0)) - 1u;  // bits past Din are not inputs
            const bool od = (mt[lane * NWp + NW] & 1u) != 0;
            const uint32_t odd_rows = __ballot_sync(kFull, od && wd != 0);
            const uint32_t colany = __reduce_or_sync(kFull, wd);
            const int64_t rb = r0 + 32 * b;
#pragma unroll
            for (int q = 0; q < kWgCols; q++) {
                if (!((colany >> q) & 1u)) continue;
                uint32_t cw = __ballot_sync(kFull, (wd >> q) & 1u);
                if (!(cw & odd_rows)) {
                    // rows in increasing order, two loads in flight
                    while (cw) {
                        const int r1 = __ffs(cw) - 1;
                        cw &= cw - 1;
                        float d1[JJ];
                        wg_load<JJ>(dt + r1 * JS, lane, d1);
                        if (cw) {
                            const int r2 = __ffs(cw) - 1;
                            cw &= cw - 1;
                            float d2[JJ];
                            wg_load<JJ>(dt + r2 * JS, lane, d2);
#pragma unroll
                            for (int e = 0; e < JJ; e++) acc[q][e] = __fadd_rn(__fadd_rn(acc[q][e], d1[e]), d2[e]);
                        } else {
#pragma unroll
                            for (int e = 0; e < JJ; e++) acc[q][e] = __fadd_rn(acc[q][e], d1[e]);
                        }
                    }
                } else {
                    while (cw) {
                        const int r = __ffs(cw) - 1;
                        cw &= cw - 1;
                        const float x = ((odd_rows >> r) & 1u) ? __ldg(X + (rb + r) * Din + c0 + q) : 1.0f;
                        float d[JJ];
                        wg_load<JJ>(dt + r * JS, lane, d);
#pragma unroll
                        for (int e = 0; e < JJ; e++) acc[q][e] = fmaf(x, d[e], acc[q][e]);
                    }
                }
            }
        }
        if (do_bias) {  // this warp's share of the block's rows
#pragma unroll
            for (int r = (32 / kWgWarps) * w; r < (32 / kWgWarps) * (w + 1); r++) {
                float d[JJ];
                wg_load<JJ>(dt + r * JS, lane, d);
#pragma unroll
                for (int e = 0; e < JJ; e++) accb[e] = __fadd_rn(accb[e], d[e]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
    }
    if (has_cols) {
#pragma unroll
        for (int e = 0; e < JJ; e++) {
            const int j = js * JS + wg_out<JJ>(lane, e);
            if (j >= Dout) continue;
            float4 *o = reinterpret_cast<float4 *>(Pw + ((size_t)ck * Dout + j) * Dp + c0);
#pragma unroll
            for (int q = 0; q < kWgCols; q += 4)
                o[q / 4] = make_float4(acc[q][e], acc[q + 1][e], acc[q + 2][e], acc[q + 3][e]);
        }
    }
    __syncthreads();  // every consumer is past its last stage (the producer warp joins here)
    if (do_bias) {  // the warps' bias sums, added in warp order: one partial per chunk
        float *s_b = s_d;  // the tiles are no longer read
#pragma unroll
        for (int e = 0; e < JJ; e++) s_b[w * JS + wg_out<JJ>(lane, e)] = accb[e];
        asm volatile("bar.sync 1, %0;" ::"r"(32 * kWgWarps) : "memory");  // the consumer warps only
        for (int j = threadIdx.x; j < JS; j += 32 * kWgWarps) {
            float acc = 0.0f;
            for (int v = 0; v < kWgWarps; v++) acc = __fadd_rn(acc, s_b[v * JS + j]);
            if (js * JS + j < Dout) Pb[(size_t)ck * Dout + js * JS + j] = acc;
        }
    }
}

// The chunks' partial sums.  A block takes 32 outputs (one per lane) and G
// warps (G = blockDim.x / 32, at most kWgRedGroups): warp g adds the chunks of
// its contiguous range [g*nck/G, (g+1)*nck/G) in chunk order (the 32 lanes
// read 32 consecutive floats), then lane l of warp 0 adds the G group sums in
// group order.  G follows from the shape alone (wg_red_groups), and so does
// the order: the result is deterministic and the same on every GPU.  Blocks
// past the weight's go to the bias.
constexpr int kWgRedGroups = 8;

// The fewest groups that leave at most 16 chunks to each thread.
static int wg_red_groups(int64_t nck)
{
    int G = 1;
    while (G < kWgRedGroups && (nck + G - 1) / G > 16) G *= 2;
    return G;
}

__global__ void __launch_bounds__(32 * kWgRedGroups) k_spike_wgrad_reduce(const float *__restrict__ Pw,
                                                                          const float *__restrict__ Pb,
                                                                          float *__restrict__ gW,
                                                                          float *__restrict__ gb, int64_t nck, int Din,
                                                                          int Dout, int Dp)
{
    __shared__ float part[kWgRedGroups][32];
    const int lane = threadIdx.x & 31, g = threadIdx.x >> 5, G = blockDim.x >> 5;
    const int64_t nW = (int64_t)Dout * Din, nWb = (nW + 31) / 32;
    const int64_t k0 = nck * g / G, k1 = nck * (g + 1) / G;
    const float *p = nullptr;
    float *out = nullptr;
    int64_t stride = 0;
    if ((int64_t)blockIdx.x < nWb) {
        const int64_t i = (int64_t)blockIdx.x * 32 + lane;
        if (i < nW) {
            p = Pw + (i / Din) * Dp + i % Din;
            stride = (int64_t)Dout * Dp;
            out = gW + i;
        }
    } else {
        const int64_t j = ((int64_t)blockIdx.x - nWb) * 32 + lane;
        if (gb && j < Dout) {
            p = Pb + j;
            stride = Dout;
            out = gb + j;
        }
    }
    float acc = 0.0f;
    if (p) {
        int64_t k = k0;
        for (; k + 8 <= k1; k += 8) {  // eight loads in flight
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = p[(k + u) * stride];
#pragma unroll
            for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, v[u]);
        }
        for (; k < k1; k++) acc = __fadd_rn(acc, p[k * stride]);
    }
    part[g][lane] = acc;
    __syncthreads();
    if (g == 0 && out) {
        float t = part[0][lane];
        for (int q = 1; q < G; q++) t = __fadd_rn(t, part[q][lane]);
        *out = t;
    }
}

size_t spike_wgrad_workspace_bytes(int64_t R, int64_t Din, int64_t Dout)
{
    const WgPlan p = wg_plan(R, Din, Dout);
    return (size_t)(p.nck * Dout * p.Dp + p.nck * Dout) * 4;
}

bool spike_wgrad(const float *dI, const float *X, const uint32_t *Xm, float *gW, float *gb, int64_t R, int64_t Din,
                 int64_t Dout, void *ws, size_t ws_bytes, cudaStream_t s)
{
    if (Din <= 0 || Din > 1024 || Dout <= 0 || Dout % 4 || R >= INT32_MAX) return false;
    if (((uintptr_t)dI & 15) || ((uintptr_t)Xm & 15) || ((uintptr_t)ws & 15)) return false;
    if (!ws || ws_bytes < spike_wgrad_workspace_bytes(R, Din, Dout)) return false;
    const int NWp = (int)spike_mask_stride(Din);
    const WgPlan p = wg_plan(R, Din, Dout);
    if (p.nck > 65535 || p.njs > 65535) return false;
    float *Pw = static_cast<float *>(ws);
    float *Pb = Pw + p.nck * Dout * p.Dp;
    CUtensorMap tdi, tmk;
    if (!make_tmap_2d(&tdi, dI, Dout, R, 32 * p.JJ, 32) || !make_tmap_2d_typed(&tmk, Xm, true, NWp, R, NWp, 32))
        return false;
    const dim3 grid((unsigned)p.nsg, (unsigned)p.njs, (unsigned)p.nck);
    const size_t smem = wg_smem(p.JJ, NWp);
    float *pb = gb ? Pb : nullptr;
    int *st = device_status_ptr();
    auto go = [&](auto kern) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<grid, 32 * (kWgWarps + 1), smem, s>>>(tdi, tmk, X, Pw, pb, R, (int)Din, (int)Dout, NWp, (int)p.Dp,
                                                      p.chunk, st);
    };
    count_launches(2);
    if (p.JJ == 8) go(k_spike_wgrad<8>);
    else if (p.JJ == 4) go(k_spike_wgrad<4>);
    else if (p.JJ == 2) go(k_spike_wgrad<2>);
    else go(k_spike_wgrad<1>);
    const int64_t nWb = (Dout * Din + 31) / 32, nbb = gb ? (Dout + 31) / 32 : 0;
    k_spike_wgrad_reduce<<<(unsigned)(nWb + nbb), 32 * wg_red_groups(p.nck), 0, s>>>(Pw, pb, gW, gb, p.nck,
                                                                                    (int)Din, (int)Dout, (int)p.Dp);
    return true;
}

}  // namespace lifb

namespace {
int sl_fail(const char *msg, int code)
{
    lifb::set_last_error(msg);
    return code;
}
int sl_done(const char *what)
{
    if (cudaGetLastError() != cudaSuccess) {
        lifb::set_last_error((std::string(what) + ": launch failed").c_str());
        return LIFB_ERR_CUDA;
    }
    lifb::set_last_error("");
    return LIFB_OK;
}
}  // namespace

extern "C" int64_t lifb_spike_mask_stride(int64_t D) { return D > 0 ? lifb::spike_mask_stride(D) : 0; }

extern "C" int lifb_spike_mask(const float *X, uint32_t *mask, int64_t R, int64_t D, void *stream)
{
    LIFB_RANGE("lifb_spike_mask");
    if (R < 0 || D <= 0) return sl_fail("lifb_spike_mask: negative R or empty D", LIFB_ERR_INVALID_ARGUMENT);
    if (R == 0) return LIFB_OK;
    if (!X || !mask) return sl_fail("lifb_spike_mask: null tensor pointer", LIFB_ERR_INVALID_ARGUMENT);
    if (!lifb::spike_mask(X, mask, R, D, (cudaStream_t)stream))
        return sl_fail("lifb_spike_mask: needs D <= 1024 and a 16-byte aligned mask", LIFB_ERR_UNSUPPORTED);
    return sl_done("lifb_spike_mask");
}

extern "C" int lifb_spike_linear_lif_fwd(const float *X, const uint32_t *Xmask, const float *W, const float *bias,
                                         const float *u0, float *V, float *S, uint32_t *Smask, int64_t T, int64_t B,
                                         int64_t Din, int64_t Dout, float beta, float theta, float u_r, void *stream)
{
    LIFB_RANGE("lifb_spike_linear_lif_fwd");
    if (T < 0 || B < 0 || Din <= 0 || Dout <= 0)
        return sl_fail("lifb_spike_linear_lif_fwd: negative shape or empty Din/Dout", LIFB_ERR_INVALID_ARGUMENT);
    if (T == 0 || B == 0) return LIFB_OK;
    if (!X || !Xmask || !W || !V || !S)
        return sl_fail("lifb_spike_linear_lif_fwd: null tensor pointer", LIFB_ERR_INVALID_ARGUMENT);
    if (!lifb::spike_linear_lif_fwd(X, Xmask, W, bias, u0, V, S, Smask, T, B, Din, Dout, beta, theta, u_r,
                                    (cudaStream_t)stream))
        return sl_fail("lifb_spike_linear_lif_fwd: needs Dout a multiple of 32, Din <= 1024 (the weight slice in "
                       "shared memory) and 16-byte aligned masks",
                       LIFB_ERR_UNSUPPORTED);
    return sl_done("lifb_spike_linear_lif_fwd");
}

extern "C" size_t lifb_spike_linear_wgrad_workspace_bytes(int64_t R, int64_t Din, int64_t Dout)
{
    if (R <= 0 || Din <= 0 || Dout <= 0) return 0;
    return lifb::spike_wgrad_workspace_bytes(R, Din, Dout);
}

extern "C" int lifb_spike_linear_wgrad(const float *dI, const float *X, const uint32_t *Xmask, float *gW, float *gb,
                                       int64_t R, int64_t Din, int64_t Dout, void *workspace, size_t workspace_bytes,
                                       void *stream)
{
    LIFB_RANGE("lifb_spike_linear_wgrad");
    if (R < 0 || Din <= 0 || Dout <= 0)
        return sl_fail("lifb_spike_linear_wgrad: negative R or empty Din/Dout", LIFB_ERR_INVALID_ARGUMENT);
    if (!dI || !X || !Xmask || !gW)
        return sl_fail("lifb_spike_linear_wgrad: null tensor pointer", LIFB_ERR_INVALID_ARGUMENT);
    if (R == 0) {
        if (cudaMemsetAsync(gW, 0, (size_t)(Din * Dout) * 4, (cudaStream_t)stream) != cudaSuccess ||
            (gb && cudaMemsetAsync(gb, 0, (size_t)Dout * 4, (cudaStream_t)stream) != cudaSuccess))
            return sl_fail("lifb_spike_linear_wgrad: memset failed", LIFB_ERR_CUDA);
        return LIFB_OK;
    }
    if (!workspace || workspace_bytes < lifb::spike_wgrad_workspace_bytes(R, Din, Dout))
        return sl_fail("lifb_spike_linear_wgrad: workspace missing or smaller than "
                       "lifb_spike_linear_wgrad_workspace_bytes",
                       LIFB_ERR_INVALID_ARGUMENT);
    if (!lifb::spike_wgrad(dI, X, Xmask, gW, gb, R, Din, Dout, workspace, workspace_bytes, (cudaStream_t)stream))
        return sl_fail("lifb_spike_linear_wgrad: needs Dout a multiple of 4, Din <= 1024 and 16-byte aligned dI, "
                       "mask and workspace",
                       LIFB_ERR_UNSUPPORTED);
    return sl_done("lifb_spike_linear_wgrad");
}
