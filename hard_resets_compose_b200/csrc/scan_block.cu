// Block-level fused scan forward: one CTA owns a slab of 32 neurons for all T
// rows, staged once in shared memory by TMA, and runs every phase of the
// two-level scan on chip, writing U and S once.
//
// Layout: lane = neuron (the slab's 32 neurons, 128-byte rows of [T, N]),
// warp = chunk (M = T / C warps, warp w owns rows [w*C, (w+1)*C)).  The slab
// [T][32] fp32 arrives as M TMA box loads (32 x C, no multicast), one
// mbarrier per chunk, so a warp starts as soon as its own rows have landed.
//
// MAPS (the map-space scan of lifscan/triton_lif.py:782-817, on chip):
//   1. envelope   each warp folds its chunk into the envelope map
//                 l -> min(c, a*l + b)                    (env_chunk_kernel :698-719)
//   2. prefix     warp w folds the maps of chunks < w into its entry bound
//                 Lo[w] = l - 1e-5 (|l| + 1)              (env_carry_kernel :722-733)
//   3. build      warp w builds its pruned capacity-K chunk map in registers
//                 (A, B, descending breakpoints xd, constants cd, count,
//                 overflow flag) with the reference's rounding, and leaves it
//                 in shared memory                        (build3_kernel :736-779)
//   4. carry      one warp evaluates the maps in chunk order from u0; an
//                 overflowed map whose stored breakpoints do not cover the
//                 state falls back to the serial recurrence over the chunk's
//                 rows, read from shared memory           (carry2_kernel :578-606)
//   5. replay     every warp replays its chunk from its carried start,
//                 writing U and S rows (128-byte coalesced stores)
//                                                         (fwd_tiled_kernel :353-379)
//   6. fix-up     in rounds, every warp whose start differs bit for bit from
//                 the previous chunk's current end replays its chunk from that
//                 end, beside the old trajectory, until the two states are
//                 bit-identical (or the chunk ends, moving its end); rounds
//                 stop when no end moved: the reference's repair loop
//                 (:805-811) on chip, replaying only until rows rejoin
// !MAPS (speculation): steps 1-4 are replaced by a lead-in: warp w runs the W
// rows before its chunk from u_r (from u0 when they reach row 0), and its
// replay follows at once; the fix-up is the same.
//
// U and S equal the serial fp32 recurrence (lifscan/fast.py:69-81) bit for
// bit whatever the carried or guessed starts were: every row written is the
// exact step of lif_step()'s arithmetic from an exact state, once the fix-up
// has run.  Maps only decide how much the fix-up replays.
#include "lifb_common.cuh"
#include "lifb_internal.h"
#include "tma.cuh"

namespace lifb {

namespace {

constexpr int kSlab = 32;          // neurons per CTA (one per lane)
constexpr int kMaxChunksMaps = 16;  // warps per CTA with maps (registers: <= 128 per thread)
constexpr int kMaxChunksSpec = 32;
constexpr float kEnvMargin = 1e-5f;

struct BlockSmem {
    // byte offsets into the dynamic shared memory
    size_t xs, ec, eb, mb, mn, mx, mc, st, en, ob, bar, total;
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// RT > 0: every warp also owns two output tiles of RT rows x 32 neurons for
// U and for S (double-buffered, written out by TMA stores).
__host__ __device__ inline BlockSmem block_smem(int T, int M, int KM, bool maps, int RT)
{
    BlockSmem s{};
    size_t o = 0;
    const size_t row = kSlab * 4;  // bytes per [M][32] array row
    s.xs = o;
    o += (size_t)T * row;
    if (maps) {
        s.ec = o; o += (size_t)M * row;
        s.eb = o; o += (size_t)M * row;
        s.mb = o; o += (size_t)M * row;
        s.mn = o; o += (size_t)M * row;
        s.mx = o; o += (size_t)M * KM * row;
        s.mc = o; o += (size_t)M * KM * row;
    }
    s.st = o; o += (size_t)M * row;
    s.en = o; o += (size_t)M * row;
    o = align_up(o, 128);
    s.ob = o; o += (size_t)M * 4 * RT * row;
    o = align_up(o, 8);
    s.bar = o; o += (size_t)M * 8;
    s.total = align_up(o, 128);
    return s;
}

__device__ __forceinline__ bool same_bits(float a, float b) { return __float_as_uint(a) == __float_as_uint(b); }

// u after `len` steps over the rows xr[0], xr[kSlab], ... (shared memory):
// the rows are loaded eight at a time ahead of their steps, so a load's
// latency is paid once per eight dependent steps.
__device__ __forceinline__ float run_rows(float u, const float *xr, int len, float beta, float theta, float u_r)
{
    int j = 0;
    for (; j + 8 <= len; j += 8) {
        float xb[8];
#pragma unroll
        for (int q = 0; q < 8; q++) xb[q] = xr[(j + q) * kSlab];
#pragma unroll
        for (int q = 0; q < 8; q++) u = lif_step_u(u, xb[q], beta, theta, u_r);
    }
    for (; j < len; j++) u = lif_step_u(u, xr[j * kSlab], beta, theta, u_r);
    return u;
}

__device__ __forceinline__ void block_stats(lifb_stats *st, int cnt, int ovf, bool act)
{
    const unsigned full = 0xffffffffu;
    const unsigned c = act ? (unsigned)cnt : 0u, o = act ? (unsigned)ovf : 0u, a = act ? 1u : 0u;
    const unsigned sc = __reduce_add_sync(full, c), so = __reduce_add_sync(full, o), sa = __reduce_add_sync(full, a);
    const unsigned mc = __reduce_max_sync(full, c);
    if ((threadIdx.x & 31) == 0 && sa) {
        atomicAdd((unsigned long long *)&st->sum_cnt, (unsigned long long)sc);
        atomicAdd((unsigned long long *)&st->n_overflow, (unsigned long long)so);
        atomicAdd((unsigned long long *)&st->n_maps, (unsigned long long)sa);
        atomicMax(&st->max_cnt, (int)mc);
    }
}

}  // namespace

// z = num / den as the reference rounds it (lifscan/triton_lif.py:760-761):
// +-inf on a zero denominator.
__device__ __forceinline__ float breakpoint_div(float num, float den)
{
    return den == 0.0f ? (num > 0.0f ? kInf : -kInf) : __fdiv_rn(num, den);
}

template <int KM, bool MAPS, int RT>
__global__ void __launch_bounds__(MAPS ? 32 * kMaxChunksMaps : 32 * kMaxChunksSpec, 1)
    k_scan_block(const __grid_constant__ CUtensorMap tI, const __grid_constant__ CUtensorMap tU,
                 const __grid_constant__ CUtensorMap tS, const float *__restrict__ u0, float *__restrict__ U,
                 float *__restrict__ S, int64_t N, int T, int C, int K, int W, float beta, float theta, float u_r,
                 lifb_stats *stats, int *status)
{
    extern __shared__ __align__(128) unsigned char smem[];
    const int M = blockDim.x >> 5;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const BlockSmem L = block_smem(T, M, KM, MAPS, RT);
    float *xs = reinterpret_cast<float *>(smem + L.xs);
    float *sts = reinterpret_cast<float *>(smem + L.st);
    float *ens = reinterpret_cast<float *>(smem + L.en);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L.bar);
    __shared__ int s_err;
    __shared__ int s_moved[2];  // per round parity: some chunk's end moved
    const unsigned full = 0xffffffffu;

    const int64_t n0 = (int64_t)blockIdx.x * kSlab;
    const int64_t n = n0 + lane;
    const bool act = n < N;
    const float u0n = act ? u0[n] : 0.0f;

    if (threadIdx.x == 0) {
        s_err = 0;
        prefetch_tmap(&tI);
        if (RT > 0) {
            prefetch_tmap(&tU);
            prefetch_tmap(&tS);
        }
        for (int m = 0; m < M; m++) mbar_init(&bar[m], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t bytes = (uint32_t)C * kSlab * 4;
        for (int m = 0; m < M; m++) {
            mbar_arrive_expect_tx(&bar[m], bytes);
            tma_load_2d(xs + (size_t)m * C * kSlab, &tI, (int)n0, m * C, &bar[m]);
        }
    }
    // every chunk barrier completes once (phase 0); waiting on a completed
    // phase returns at once
    auto wait_rows = [&](int m) -> bool {
        if (mbar_wait(&bar[m], 0)) return true;
        if (lane == 0) atomicExch(&s_err, 1);
        return false;
    };
    const float *xw = xs + (size_t)w * C * kSlab + lane;  // this warp's chunk, this lane's neuron

    if constexpr (MAPS) {
        float *ec = reinterpret_cast<float *>(smem + L.ec);
        float *eb = reinterpret_cast<float *>(smem + L.eb);
        float *mb = reinterpret_cast<float *>(smem + L.mb);
        int *mn = reinterpret_cast<int *>(smem + L.mn);
        float *mx = reinterpret_cast<float *>(smem + L.mx);
        float *mc = reinterpret_cast<float *>(smem + L.mc);
        // the last chunk's map is never evaluated by the carry: without stats
        // neither it nor its envelope is built
        const int Mb = stats ? M : M - 1;
        float a = 1.0f;  // beta^C, the same for every chunk and neuron
        for (int j = 0; j < C; j++) a = __fmul_rn(beta, a);

        // 1. envelope of the warp's chunk
        if (w < Mb && wait_rows(w)) {
            float c = kInf, b = 0.0f;
#pragma unroll 8
            for (int j = 0; j < C; j++) {
                const float x = xw[j * kSlab];
                const float cc = mul_add_rn(beta, c, x);
                c = u_r < cc ? u_r : cc;
                b = mul_add_rn(beta, b, x);
            }
            ec[w * kSlab + lane] = c;
            eb[w * kSlab + lane] = b;
        }
        __syncthreads();
        if (s_err) goto done;
        if (w < Mb) {
            // 2. entry bound of chunk w from the envelopes of chunks < w
            float l = u0n;
            for (int m = 0; m < w; m++) {
                const float lin = mul_add_rn(a, l, eb[m * kSlab + lane]);
                const float cm = ec[m * kSlab + lane];
                l = cm < lin ? cm : lin;
            }
            const float lo = __fsub_rn(l, __fmul_rn(kEnvMargin, __fadd_rn(fabsf(l), 1.0f)));
            // 3. pruned capacity-K map of chunk w
            const float hi = fmaxf(u0n, fmaxf(theta, u_r));
            float A = 1.0f, B = 0.0f, xmin = kInf;
            int cnt = 0, ovf = 0;
            float xd[KM], cd[KM];
#pragma unroll
            for (int i = 0; i < KM; i++) { xd[i] = kInf; cd[i] = 0.0f; }
            // a breakpoint is kept only if z < min(xmin, hi^+): a cheap
            // quotient first, the correctly rounded one only near the bound
            float xnext = xw[0];
            for (int j = 0; j < C; j++) {
                const float x = xnext;
                if (j + 1 < C) xnext = xw[(j + 1) * kSlab];  // next row's load overlaps this step
                const int cmax = (int)__reduce_max_sync(full, (unsigned)cnt);
                // slots in groups of four (one uniform branch per group);
                // stepping a slot above cnt is harmless: insertion resets it
#pragma unroll
                for (int g = 0; g < KM; g += 4) {
                    if (g >= cmax) break;
#pragma unroll
                    for (int i = g; i < g + 4; i++) cd[i] = lif_step_u(cd[i], x, beta, theta, u_r);
                }
                bool cand = xmin > lo;
                float num = 0.0f, den = 1.0f;
                if (cand) {
                    num = __fsub_rn(__fsub_rn(theta, x), __fmul_rn(beta, B));
                    den = __fmul_rn(beta, A);
                    // fast reject: num/den clearly above both xmin and hi
                    const float bound = fminf(xmin, hi);
                    if (den > 1e-30f && bound < 1e30f) {
                        const float q = __fdividef(num, den);
                        cand = !(q > bound + fabsf(bound) * 1e-5f + 1e-30f);
                    }
                }
                if (__any_sync(full, cand) && cand) {
                    const float z = breakpoint_div(num, den);
                    if (z < xmin && z <= hi) {
                        if (cnt >= K) {
                            ovf = 1;
                        } else {
#pragma unroll
                            for (int i = 0; i < KM; i++)
                                if (i == cnt) { xd[i] = z; cd[i] = u_r; }
                            cnt++;
                            xmin = z;
                        }
                    }
                }
                A = __fmul_rn(beta, A);
                B = mul_add_rn(beta, B, x);
            }
            mb[w * kSlab + lane] = B;
            mn[w * kSlab + lane] = cnt | (ovf << 16);
#pragma unroll
            for (int i = 0; i < KM; i++)
                if (i < cnt) {
                    mx[(w * KM + i) * kSlab + lane] = xd[i];
                    mc[(w * KM + i) * kSlab + lane] = cd[i];
                }
            if (stats) block_stats(stats, cnt, ovf, act);
        }
        __syncthreads();
        // 4. carry: chunk starts in order (warp 0)
        if (w == 0) {
            float u = u0n;
            sts[lane] = u;
            for (int m = 0; m + 1 < M; m++) {
                const int v = mn[m * kSlab + lane];
                const int cnt = v & 0xffff, ovf = v >> 16;
                const float *X = mx + (size_t)m * KM * kSlab + lane;
                float xv[KM];
#pragma unroll
                for (int i = 0; i < KM; i++) xv[i] = i < cnt ? X[i * kSlab] : -kInf;
                int k = 0;  // breakpoints strictly descending: k = #{i < cnt : xd[i] > u}
#pragma unroll
                for (int i = 0; i < KM; i++) k += xv[i] > u ? 1 : 0;
                float nu;
                if (k < cnt) {
                    nu = mc[((size_t)m * KM + k) * kSlab + lane];
                } else if (!ovf) {
                    nu = mul_add_rn(a, u, mb[m * kSlab + lane]);
                } else {
                    // overflow below the stored breakpoints: the serial recurrence
                    nu = run_rows(u, xs + (size_t)m * C * kSlab + lane, C, beta, theta, u_r);
                }
                u = nu;
                sts[(m + 1) * kSlab + lane] = u;
            }
        }
        __syncthreads();
    } else {
        // lead-in: chunk w's start guessed from the W rows before it
        float u = u0n;
        if (w > 0) {
            int t0 = w * C - W;
            u = u_r;
            if (t0 <= 0) {
                t0 = 0;
                u = u0n;
            }
            // chunk by chunk, each as soon as its rows have landed: the
            // lead-in overlaps the loads of the later chunks
            for (int m = t0 / C; m < w; m++) {
                if (!wait_rows(m)) break;
                const int r0 = m * C > t0 ? m * C : t0;
                u = run_rows(u, xs + (size_t)r0 * kSlab + lane, (m + 1) * C - r0, beta, theta, u_r);
            }
        }
        sts[w * kSlab + lane] = u;
    }
    // 5. replay of chunk w from its start
    if (!s_err && wait_rows(w)) {
        float u = sts[w * kSlab + lane];
        if constexpr (RT > 0) {
            // rows go to a shared-memory tile that one TMA store per tile
            // writes out (the hardware clips neurons beyond N), two tiles in
            // flight per warp; no global store sits on the recurrence
            float *ob = reinterpret_cast<float *>(smem + L.ob) + (size_t)w * 4 * RT * kSlab;
            const int nt = C / RT;
            for (int k = 0; k < nt; k++) {
                float *ou = ob + (k & 1) * 2 * RT * kSlab;
                float *os = ou + RT * kSlab;
                if (k >= 2) {  // the store issued two tiles ago must have read this buffer
                    if (lane == 0) bulk_wait_read<1>();
                    __syncwarp();
                }
                float xb[RT];  // loaded before the tile's stores: no load waits behind a store
#pragma unroll
                for (int r = 0; r < RT; r++) xb[r] = xw[(k * RT + r) * kSlab];
#pragma unroll
                for (int r = 0; r < RT; r++) {
                    const float v = __fadd_rn(__fmul_rn(beta, u), xb[r]);
                    const bool f = v >= theta;
                    u = f ? u_r : v;
                    ou[r * kSlab + lane] = u;
                    os[r * kSlab + lane] = f ? 1.0f : 0.0f;
                }
                fence_proxy_async_shared();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tU, (int)n0, w * C + k * RT, ou);
                    tma_store_2d(&tS, (int)n0, w * C + k * RT, os);
                    bulk_commit();
                }
            }
            // the fix-up may rewrite these rows with plain stores: the TMA
            // stores must have completed first
            if (lane == 0) {
                bulk_wait_all();
                asm volatile("fence.proxy.async.global;" ::: "memory");
            }
        } else {
            float *Uo = U + (int64_t)w * C * N + n;
            float *So = S + (int64_t)w * C * N + n;
#pragma unroll 4
            for (int j = 0; j < C; j++) {
                const float v = __fadd_rn(__fmul_rn(beta, u), xw[j * kSlab]);
                const bool f = v >= theta;
                u = f ? u_r : v;
                if (act) {
                    Uo[(int64_t)j * N] = u;
                    So[(int64_t)j * N] = f ? 1.0f : 0.0f;
                }
            }
        }
        ens[w * kSlab + lane] = u;
    }
    if (threadIdx.x == 0) s_moved[0] = 0;
    __syncthreads();
    if (s_err) goto done;
    // 6. fix-up in rounds (the reference's repair loop, on chip): in each
    // round every warp whose start differs bit for bit from the previous
    // chunk's current end replays its chunk from that end beside the old
    // trajectory until the two states are equal (the rest of the chunk is
    // then unchanged); a chunk that never rejoins moves its end, and the next
    // chunk is looked at again in the next round.  Chunk 0 starts exact, so
    // after round r chunks 0..r+1 are exact: at most M - 1 rounds.
    for (int r = 0; r + 1 < M; r++) {
        float ep = 0.0f, s0 = 0.0f;
        bool live = false;
        if (w > 0) {
            ep = ens[(w - 1) * kSlab + lane];
            s0 = sts[w * kSlab + lane];
            live = !same_bits(ep, s0);
        }
        __syncthreads();  // every read of this round's ends precedes any write
        // every thread has read the previous round's flag: clear the next one
        if (threadIdx.x == 0) s_moved[(r + 1) & 1] = 0;
        if (__any_sync(full, live)) {
            const bool need = live;
            float un = ep, uo = s0;
            float *Uo = U + (int64_t)w * C * N + n;
            float *So = S + (int64_t)w * C * N + n;
            for (int j = 0; j < C && __any_sync(full, live); j++) {
                if (live) {
                    const float x = xw[j * kSlab];
                    const float v = __fadd_rn(__fmul_rn(beta, un), x);
                    const bool f = v >= theta;
                    un = f ? u_r : v;
                    uo = lif_step_u(uo, x, beta, theta, u_r);
                    if (act) {
                        Uo[(int64_t)j * N] = un;
                        So[(int64_t)j * N] = f ? 1.0f : 0.0f;
                    }
                    live = !same_bits(un, uo);
                }
            }
            if (need) sts[w * kSlab + lane] = ep;
            if (live) {  // never rejoined: this chunk's end moved
                ens[w * kSlab + lane] = un;
                s_moved[r & 1] = 1;
            }
        }
        __syncthreads();
        if (!s_moved[r & 1]) break;
    }
done:
    if (threadIdx.x == 0 && s_err && status) atomicCAS(status, 0, (int)kStatusTmaWaitTimeout);
}

namespace {

template <int KM, bool MAPS, int RT>
bool launch_block(const CUtensorMap &tm, const CUtensorMap &tu, const CUtensorMap &ts, const float *u0, float *U,
                  float *S, int64_t N, int T, int C, int K, int W, float beta, float theta, float u_r,
                  lifb_stats *st, cudaStream_t s)
{
    const int M = T / C;
    const BlockSmem L = block_smem(T, M, KM, MAPS, RT);
    auto kern = k_scan_block<KM, MAPS, RT>;
    // a per-device attribute: set on every call (a host-side call, no launch)
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total) != cudaSuccess)
        return false;
    count_launches(1);
    kern<<<(unsigned)((N + kSlab - 1) / kSlab), (unsigned)(M * 32), L.total, s>>>(
        tm, tu, ts, u0, U, S, N, T, C, K, W, beta, theta, u_r, st, device_status_ptr());
    return true;
}

// Output tile height: the tallest of 8, 4 and 2 rows dividing C whose tiles
// fit beside the slab (and maps), else 0 (plain stores).
int pick_rt(int64_t T, int64_t M, int64_t C, int KM, bool maps, int limit)
{
    for (int rt : {8, 4, 2})
        if (C % rt == 0 && (int64_t)block_smem((int)T, (int)M, KM, maps, rt).total <= limit) return rt;
    return 0;
}

template <int KM, bool MAPS>
bool launch_rt(int rt, const CUtensorMap &tm, const CUtensorMap &tu, const CUtensorMap &ts, const float *u0,
               float *U, float *S, int64_t N, int T, int C, int K, int W, float beta, float theta, float u_r,
               lifb_stats *st, cudaStream_t s)
{
    switch (rt) {
    case 8: return launch_block<KM, MAPS, 8>(tm, tu, ts, u0, U, S, N, T, C, K, W, beta, theta, u_r, st, s);
    case 4: return launch_block<KM, MAPS, 4>(tm, tu, ts, u0, U, S, N, T, C, K, W, beta, theta, u_r, st, s);
    case 2: return launch_block<KM, MAPS, 2>(tm, tu, ts, u0, U, S, N, T, C, K, W, beta, theta, u_r, st, s);
    default: return launch_block<KM, MAPS, 0>(tm, tu, ts, u0, U, S, N, T, C, K, W, beta, theta, u_r, st, s);
    }
}

int smem_limit()
{
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
        return 0;
    return v;
}

}  // namespace

bool scan_block_applies(int64_t T, int64_t N, int C, int K, bool maps)
{
    if (T <= 0 || N <= 0 || C <= 0 || T % C || C > 256 || N % 4) return false;
    const int64_t M = T / C;
    if (M < 2 || M > (maps ? kMaxChunksMaps : kMaxChunksSpec)) return false;
    if (maps && (K < 1 || K > 16)) return false;
    const int KM = !maps ? 1 : K <= 4 ? 4 : K <= 8 ? 8 : 16;
    return (int64_t)block_smem((int)T, (int)M, KM, maps, 0).total <= smem_limit();
}

bool scan_block(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, int C, int K, bool maps,
                int64_t W, float beta, float theta, float u_r, lifb_stats *st, cudaStream_t s)
{
    if (!scan_block_applies(T, N, C, K, maps)) return false;
    const void *ptrs[] = {I, U, S};
    if (!tma_ok(ptrs, 3, N)) return false;
    const int KM = !maps ? 1 : K <= 4 ? 4 : K <= 8 ? 8 : 16;
    const int rt = pick_rt(T, T / C, C, KM, maps, smem_limit());
    CUtensorMap tm, tu, ts;
    if (!make_tmap_2d(&tm, I, N, T, kSlab, C)) return false;
    if (rt > 0 && (!make_tmap_2d(&tu, U, N, T, kSlab, rt) || !make_tmap_2d(&ts, S, N, T, kSlab, rt))) return false;
    if (rt == 0) tu = ts = tm;  // unused
    const int Wl = (int)(W < 0 ? 0 : W > T ? T : W);
    if (!maps) return launch_rt<1, false>(rt, tm, tu, ts, u0, U, S, N, (int)T, C, 0, Wl, beta, theta, u_r, nullptr, s);
    if (K <= 4) return launch_rt<4, true>(rt, tm, tu, ts, u0, U, S, N, (int)T, C, K, 0, beta, theta, u_r, st, s);
    if (K <= 8) return launch_rt<8, true>(rt, tm, tu, ts, u0, U, S, N, (int)T, C, K, 0, beta, theta, u_r, st, s);
    return launch_rt<16, true>(rt, tm, tu, ts, u0, U, S, N, (int)T, C, K, 0, beta, theta, u_r, st, s);
}

}  // namespace lifb
