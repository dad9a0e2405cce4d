// Adaptive-threshold LIF (ALIF) neurons: the state is (u, w), the threshold
// theta0 + w rises by q at every spike and decays by rho per step
// (lifscan/triton_alif.py:25-31 _alif_step):
//     v = fl(fl(beta*u) + x);  s = v >= fl(theta0 + w);
//     u' = s ? u_r : v;        w' = s ? fl(fl(rho*w) + q) : fl(rho*w)
//
//   forward        one streaming pass (TMA ring for I, TMA stores of U, W, S)
//                  or, for long sequences, speculative segments: each segment
//                  of L rows starts from a lead-in over the W rows before it
//                  (from (u_r, w guess), or (u0, w0) when it reaches row 0),
//                  all segments replay at once, and a fix-up makes the result
//                  exact (a segment is redone from the previous one's true end
//                  until its (u, w, s) rows match the stored ones bit for bit).
//                  The reference instead builds box-restricted chunk maps
//                  (triton_alif.py:95-253); its result is the same serial
//                  recurrence, which this path reproduces for any prediction.
//   warm predict   alif_warm_predict (triton_alif.py:74-92, 276-285)
//   backward       the detached-reset adjoint of triton_alif.py:359-364: with
//                  sg_t = alpha sig (1 - sig) at v_t - theta0 - w_{t-1} and
//                  d_t = gS_t + q lw_t,
//                      lv_t = (1 - s_t) beta lv_{t+1} + sg_t d_t,
//                      lw_{t-1} = rho lw_t - sg_t d_t
//                  in one reverse sweep per neuron (LW[t] = lw_t, LV[t] = lv_t),
//                  optionally with ALIFFn's parameter sums (triton_alif.py:
//                  542-554) in fp64: dbeta = sum lv_t u_{t-1}, drho = sum lw_t
//                  w_{t-1}, dq = sum lw_t s_t, dtheta0 = -sum sg_t d_t, and
//                  dw0 = lw_{-1}.
#include <cstdio>

#include "lifb_common.cuh"
#include "lifb_internal.h"
#include "tma.cuh"
#include "vec.cuh"

namespace lifb {

struct AlifP {
    float beta, rho, q, theta0, u_r;
};

__device__ __forceinline__ void alif_step(float &u, float &w, float x, const AlifP &p, bool &s)
{
    const float v = __fadd_rn(__fmul_rn(p.beta, u), x);
    s = v >= __fadd_rn(p.theta0, w);
    const float rw = __fmul_rn(p.rho, w);
    u = s ? p.u_r : v;
    w = s ? __fadd_rn(rw, p.q) : rw;
}

__device__ __forceinline__ bool same_bits2(float a, float b) { return __float_as_uint(a) == __float_as_uint(b); }

// ------------------------------------------------------------------ forward (TMA)
constexpr int kAlifFwd4R = 16, kAlifFwd4S = 6;  // NPL = 4: rows per tile, ring stages
constexpr int kAlifFwd1R = 32, kAlifFwd1S = 4;  // NPL = 1

// Chunk m of C rows starts from (SU, SW)[m] (NULL: (u0, w0) for every chunk,
// used with M = 1).  lead > 0 (a multiple of R, C a multiple of R): chunk
// m >= 1 first runs the `lead` rows before it without stores, from (u_r,
// Wpred[row / Cpred] or 0), or from (u0, w0) when they reach row 0, and
// records that start in (LU, LW)[m].  (EU, EW)[m] (optional) receive the
// chunk's final state.
template <int NPL, int R, int S>
__global__ void __launch_bounds__(32) k_alif_fwd_tma(
    const __grid_constant__ CUtensorMap tI, const __grid_constant__ CUtensorMap tU,
    const __grid_constant__ CUtensorMap tW, const __grid_constant__ CUtensorMap tS, const float *__restrict__ u0,
    const float *__restrict__ w0, const float *__restrict__ SU, const float *__restrict__ SW, float *__restrict__ U,
    float *__restrict__ W, float *__restrict__ Sout, float *__restrict__ EU, float *__restrict__ EW, int64_t N,
    int64_t C, AlifP p, int64_t lead, float *__restrict__ LU, float *__restrict__ LW, const float *__restrict__ Wpred,
    int64_t Cpred, int *status)
{
    constexpr int NB = 32 * NPL;
    constexpr int kTile = R * NB;
    constexpr uint32_t kStageBytes = kTile * 4;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    float *ring = reinterpret_cast<float *>(smem_raw);  // S input tiles
    float *obuf = ring + S * kTile;                      // 2 x (U, W, S tiles)
    __shared__ __align__(8) uint64_t full[S];
    const int lane = threadIdx.x;
    const int64_t n0 = (int64_t)blockIdx.x * NB;
    const int64_t m = blockIdx.y;
    const int64_t row0 = m * C;
    const int64_t nfull = C / R;
    const int rem = (int)(C - nfull * R);
    const int64_t ntiles = nfull + (rem ? 1 : 0);
    const bool leading = lead > 0 && m > 0;
    const int64_t lrow0 = leading ? (row0 > lead ? row0 - lead : 0) : row0;
    const int64_t nlead = (row0 - lrow0) / R;
    const int64_t ntot = nlead + ntiles;
    auto tile_row = [&](int64_t k) { return k < nlead ? lrow0 + k * R : row0 + (k - nlead) * R; };

    if (lane == 0) {
        prefetch_tmap(&tI);
        prefetch_tmap(&tU);
        prefetch_tmap(&tW);
        prefetch_tmap(&tS);
        for (int s = 0; s < S; s++) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncwarp();
    if (lane == 0) {
        for (int s = 0; s < S && s < ntot; s++) {
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            tma_load_2d(ring + s * kTile, &tI, (int)n0, (int)tile_row(s), &full[s]);
        }
    }
    const int64_t nl = n0 + NPL * lane;
    const bool act = nl < N;
    Vec<NPL> u, w;
#pragma unroll
    for (int i = 0; i < NPL; i++) { u.v[i] = 0.f; w.v[i] = 0.f; }
    if (act) {
        if (leading) {
            if (lrow0 == 0) {
                u = ld_vec<NPL>(u0 + nl);
                w = ld_vec<NPL>(w0 + nl);
            } else {
#pragma unroll
                for (int i = 0; i < NPL; i++) u.v[i] = p.u_r;
                if (Wpred) w = ld_vec<NPL>(Wpred + (lrow0 / Cpred) * N + nl);
            }
        } else if (SU) {
            u = ld_vec<NPL>(SU + m * N + nl);
            w = ld_vec<NPL>(SW + m * N + nl);
        } else {
            u = ld_vec<NPL>(u0 + nl);
            w = ld_vec<NPL>(w0 + nl);
        }
    }
    bool ok = true;

    for (int64_t k = 0; k < nlead; k++) {  // lead-in: states only
        const int s = (int)(k % S);
        if (!mbar_wait(&full[s], (uint32_t)((k / S) & 1))) { ok = false; break; }
        const float *in = ring + s * kTile + NPL * lane;
        Vec<NPL> x[R];
#pragma unroll
        for (int r = 0; r < R; r++) x[r] = ld_vec<NPL>(in + r * NB);
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int i = 0; i < NPL; i++) {
                bool f;
                alif_step(u.v[i], w.v[i], x[r].v[i], p, f);
            }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0 && k + S < ntot) {
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            tma_load_2d(ring + s * kTile, &tI, (int)n0, (int)tile_row(k + S), &full[s]);
        }
    }
    if (leading && ok && LU && act) {
        st_vec<NPL>(LU + m * N + nl, u);
        st_vec<NPL>(LW + m * N + nl, w);
    }

    for (int64_t kk = 0; kk < nfull && ok; kk++) {
        const int64_t k = nlead + kk;
        const int s = (int)(k % S);
        if (!mbar_wait(&full[s], (uint32_t)((k / S) & 1))) { ok = false; break; }
        const float *in = ring + s * kTile + NPL * lane;
        Vec<NPL> x[R];
#pragma unroll
        for (int r = 0; r < R; r++) x[r] = ld_vec<NPL>(in + r * NB);
        float *ou = obuf + (int)(kk & 1) * 3 * kTile;
        float *ow = ou + kTile;
        float *os = ow + kTile;
        if (kk >= 2) {  // the stores issued two tiles ago must have read this buffer
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
            Vec<NPL> sp;
#pragma unroll
            for (int i = 0; i < NPL; i++) {
                bool f;
                alif_step(u.v[i], w.v[i], x[r].v[i], p, f);
                sp.v[i] = f ? 1.0f : 0.0f;
            }
            st_vec<NPL>(ou + r * NB + NPL * lane, u);
            st_vec<NPL>(ow + r * NB + NPL * lane, w);
            st_vec<NPL>(os + r * NB + NPL * lane, sp);
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
            const int row = (int)(row0 + kk * R);
            tma_store_2d(&tU, (int)n0, row, ou);
            tma_store_2d(&tW, (int)n0, row, ow);
            tma_store_2d(&tS, (int)n0, row, os);
            bulk_commit();
            if (k + S < ntot) {
                mbar_arrive_expect_tx(&full[s], kStageBytes);
                tma_load_2d(ring + s * kTile, &tI, (int)n0, (int)tile_row(k + S), &full[s]);
            }
        }
    }
    if (ok && rem) {  // ragged last tile: checked rows, direct stores
        const int64_t k = nlead + nfull;
        const int s = (int)(k % S);
        if (!mbar_wait(&full[s], (uint32_t)((k / S) & 1))) {
            ok = false;
        } else {
            const float *in = ring + s * kTile + NPL * lane;
            for (int r = 0; r < rem; r++) {
                const Vec<NPL> x = ld_vec<NPL>(in + r * NB);
                Vec<NPL> sp;
#pragma unroll
                for (int i = 0; i < NPL; i++) {
                    bool f;
                    alif_step(u.v[i], w.v[i], x.v[i], p, f);
                    sp.v[i] = f ? 1.0f : 0.0f;
                }
                if (act) {
                    const int64_t o = (row0 + nfull * R + r) * N + nl;
                    st_vec<NPL>(U + o, u);
                    st_vec<NPL>(W + o, w);
                    st_vec<NPL>(Sout + o, sp);
                }
            }
        }
    }
    if (!ok && status) atomicCAS(status, 0, (int)kStatusTmaWaitTimeout);
    if (ok && EU && act) {
        st_vec<NPL>(EU + m * N + nl, u);
        st_vec<NPL>(EW + m * N + nl, w);
    }
    if (lane == 0) bulk_wait_all();
}

template <int NPL>
static void launch_alif_fwd(const CUtensorMap *maps, const float *u0, const float *w0, const float *SU,
                            const float *SW, float *U, float *W, float *S, float *EU, float *EW, int64_t N, int64_t M,
                            int64_t C, const AlifP &p, int64_t lead, float *LU, float *LW, const float *Wpred,
                            int64_t Cpred, int *status, cudaStream_t s)
{
    constexpr int NB = 32 * NPL;
    constexpr int R = NPL == 4 ? kAlifFwd4R : kAlifFwd1R;
    constexpr int ST = NPL == 4 ? kAlifFwd4S : kAlifFwd1S;
    const size_t smem = (size_t)(ST + 6) * R * NB * 4;
    auto kern = k_alif_fwd_tma<NPL, R, ST>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 g((unsigned)((N + NB - 1) / NB), (unsigned)M);
    count_launches(1);
    kern<<<g, 32, smem, s>>>(maps[0], maps[1], maps[2], maps[3], u0, w0, SU, SW, U, W, S, EU, EW, N, C, p, lead, LU,
                             LW, Wpred, Cpred, status);
}

// False when the TMA path does not apply (nothing launched).
static bool alif_fwd_tma(const float *I, const float *u0, const float *w0, const float *SU, const float *SW, float *U,
                         float *W, float *S, float *EU, float *EW, int64_t T, int64_t N, int64_t C, const AlifP &p,
                         int64_t lead, float *LU, float *LW, const float *Wpred, int64_t Cpred, cudaStream_t s)
{
    const void *ptrs[] = {I, u0, w0, SU, SW, U, W, S, EU, EW, LU, LW, Wpred};
    if (!tma_ok(ptrs, 13, N) || C <= 0 || T % C) return false;
    const int64_t M = T / C;
    if (M > 65535) return false;
    const int npl = pick_npl(N, M, 2);
    const int R = npl == 4 ? kAlifFwd4R : kAlifFwd1R;
    if (lead > 0) {
        if (C % R) return false;
        lead = (lead + R - 1) / R * R;
    }
    CUtensorMap maps[4];
    const float *arrs[4] = {I, U, W, S};
    for (int i = 0; i < 4; i++)
        if (!make_tmap_2d(&maps[i], arrs[i], N, T, 32 * npl, R)) return false;
    int *status = device_status_ptr();
    if (npl == 4)
        launch_alif_fwd<4>(maps, u0, w0, SU, SW, U, W, S, EU, EW, N, M, C, p, lead, LU, LW, Wpred, Cpred, status, s);
    else
        launch_alif_fwd<1>(maps, u0, w0, SU, SW, U, W, S, EU, EW, N, M, C, p, lead, LU, LW, Wpred, Cpred, status, s);
    return true;
}

// ------------------------------------------------------------------ forward (plain)
constexpr int kAlifBlock = 128;

// One neuron per thread, rows of the next batch loaded while this one steps.
template <int D>
__global__ void __launch_bounds__(kAlifBlock) k_alif_fwd_plain(const float *__restrict__ I, const float *__restrict__ u0,
                                                               const float *__restrict__ w0, float *__restrict__ U,
                                                               float *__restrict__ W, float *__restrict__ S, int64_t T,
                                                               int64_t N, AlifP p)
{
    const int64_t n = (int64_t)blockIdx.x * kAlifBlock + threadIdx.x;
    if (n >= N) return;
    float u = u0[n], w = w0[n];
    float cur[D], nxt[D];
#pragma unroll
    for (int d = 0; d < D; d++) cur[d] = d < T ? __ldg(I + d * N + n) : 0.0f;
    for (int64_t t0 = 0; t0 < T; t0 += D) {
#pragma unroll
        for (int d = 0; d < D; d++) nxt[d] = t0 + D + d < T ? __ldg(I + (t0 + D + d) * N + n) : 0.0f;
#pragma unroll
        for (int d = 0; d < D; d++) {
            if (t0 + d < T) {
                bool s;
                alif_step(u, w, cur[d], p, s);
                const int64_t o = (t0 + d) * N + n;
                U[o] = u;
                W[o] = w;
                S[o] = s ? 1.0f : 0.0f;
            }
        }
#pragma unroll
        for (int d = 0; d < D; d++) cur[d] = nxt[d];
    }
}

static void alif_serial(const float *I, const float *u0, const float *w0, float *U, float *W, float *S, int64_t T,
                        int64_t N, const AlifP &p, cudaStream_t s)
{
    if (alif_fwd_tma(I, u0, w0, nullptr, nullptr, U, W, S, nullptr, nullptr, T, N, T, p, 0, nullptr, nullptr, nullptr,
                     1, s))
        return;
    count_launches(1);
    k_alif_fwd_plain<16><<<(unsigned)((N + kAlifBlock - 1) / kAlifBlock), kAlifBlock, 0, s>>>(I, u0, w0, U, W, S, T,
                                                                                               N, p);
}

// ------------------------------------------------------------------ fix-up
// Replays rows [r0, r0 + L) of one neuron per lane from (u, w) (active lanes
// only), comparing (u, w, s) with the stored rows: a lane stops at the first
// row that matches (every later row is then already right) and otherwise
// rewrites the row.  True for lanes that resynchronised.
template <int kB>
__device__ __forceinline__ bool alif_replay_until_sync(const float *__restrict__ I, float *__restrict__ U,
                                                       float *__restrict__ W, float *__restrict__ S, int64_t N,
                                                       int64_t n, bool act, int64_t r0, int64_t L, float &u, float &w,
                                                       bool active, const AlifP &p)
{
    const unsigned full = 0xffffffffu;
    bool synced = !active;
    if (!__any_sync(full, active)) return synced;
    float x[kB], uo[kB], wo[kB], so[kB];
#pragma unroll
    for (int q = 0; q < kB; q++) {
        if (act && q < L) {
            const int64_t o = (r0 + q) * N + n;
            x[q] = __ldg(I + o);
            uo[q] = U[o];
            wo[q] = W[o];
            so[q] = S[o];
        }
    }
    for (int64_t b = 0; b < L; b += kB) {
        if (!__any_sync(full, active)) break;
        float xn[kB], un_[kB], wn_[kB], sn[kB];
#pragma unroll
        for (int q = 0; q < kB; q++) {
            if (act && b + kB + q < L) {
                const int64_t o = (r0 + b + kB + q) * N + n;
                xn[q] = __ldg(I + o);
                un_[q] = U[o];
                wn_[q] = W[o];
                sn[q] = S[o];
            }
        }
#pragma unroll
        for (int q = 0; q < kB; q++) {
            if (active && b + q < L) {
                bool f;
                alif_step(u, w, x[q], p, f);
                const float fs = f ? 1.0f : 0.0f;
                if (same_bits2(u, uo[q]) && same_bits2(w, wo[q]) && fs == so[q]) {
                    active = false;
                    synced = true;
                } else {
                    const int64_t o = (r0 + b + q) * N + n;
                    U[o] = u;
                    W[o] = w;
                    S[o] = fs;
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kB; q++) {
            x[q] = xn[q];
            uo[q] = un_[q];
            wo[q] = wn_[q];
            so[q] = sn[q];
        }
    }
    return synced;
}

constexpr int kAlifFixBlock = 128;

// Parallel pass (blockIdx.y = segment sg >= 1): assumes segment sg-1's end
// (EU, EW) is exact and fixes segment sg from it; segments that never
// resynchronise get a new end (EUn, EWn) and a flag.
__global__ void __launch_bounds__(kAlifFixBlock) k_alif_fixup_par(
    const float *__restrict__ I, const float *__restrict__ SU, const float *__restrict__ SW, float *__restrict__ U,
    float *__restrict__ W, float *__restrict__ S, const float *__restrict__ EU, const float *__restrict__ EW,
    float *__restrict__ EUn, float *__restrict__ EWn, int32_t *__restrict__ Changed, int64_t N, int64_t L, AlifP p)
{
    const int64_t n = (int64_t)blockIdx.x * kAlifFixBlock + threadIdx.x;
    const int64_t sg = (int64_t)blockIdx.y + 1;
    const bool act = n < N;
    const float pu = act ? EU[(sg - 1) * N + n] : 0.0f, pw = act ? EW[(sg - 1) * N + n] : 0.0f;
    const bool need = act && !(same_bits2(pu, SU[sg * N + n]) && same_bits2(pw, SW[sg * N + n]));
    if (!__any_sync(0xffffffffu, need)) {
        if (act) Changed[sg * N + n] = 0;
        return;
    }
    float u = pu, w = pw;
    const bool synced = alif_replay_until_sync<16>(I, U, W, S, N, n, act, sg * L, L, u, w, need, p);
    if (act) {
        Changed[sg * N + n] = synced ? 0 : 1;
        if (!synced) {
            EUn[sg * N + n] = u;
            EWn[sg * N + n] = w;
        }
    }
}

// Sequential pass per neuron: a segment whose fix did not resynchronise has a
// new end, so the next segment is redone from it (and so on).
__global__ void __launch_bounds__(kAlifFixBlock) k_alif_fixup_seq(
    const float *__restrict__ I, float *__restrict__ U, float *__restrict__ W, float *__restrict__ S,
    float *__restrict__ EU, float *__restrict__ EW, const float *__restrict__ EUn, const float *__restrict__ EWn,
    const int32_t *__restrict__ Changed, int64_t N, int64_t NS, int64_t L, AlifP p)
{
    const int64_t n = (int64_t)blockIdx.x * kAlifFixBlock + threadIdx.x;
    const bool act = n < N;
    bool any_ch = false;
    for (int64_t s0 = 1; s0 < NS && !__any_sync(0xffffffffu, any_ch); s0 += 16) {
#pragma unroll
        for (int q = 0; q < 16; q++)
            if (act && s0 + q < NS) any_ch |= Changed[(s0 + q) * N + n] != 0;
    }
    if (!__any_sync(0xffffffffu, any_ch)) return;
    bool carry = false;
    float eu = 0.0f, ew = 0.0f;
    for (int64_t sg = 1; sg < NS; sg++) {
        bool ch = act && Changed[sg * N + n] != 0;
        float cu = ch ? EUn[sg * N + n] : (act ? EU[sg * N + n] : 0.0f);
        float cw = ch ? EWn[sg * N + n] : (act ? EW[sg * N + n] : 0.0f);
        if (__any_sync(0xffffffffu, carry)) {
            float u = eu, w = ew;
            const bool synced = alif_replay_until_sync<16>(I, U, W, S, N, n, act, sg * L, L, u, w, carry, p);
            if (carry && !synced) {
                ch = true;
                cu = u;
                cw = w;
            }
        }
        if (ch && act) {
            EU[sg * N + n] = cu;
            EW[sg * N + n] = cw;
        }
        carry = ch;
        eu = cu;
        ew = cw;
    }
}

// ------------------------------------------------------------------ warm predict
// WP[m] = w after simulating the Wn chunks before chunk m from (u_init,
// w_init), or from (UI, WI)[s0] when given; from (u0, w0) when the warm-up
// reaches row 0 (triton_alif.py:74-92).
__global__ void __launch_bounds__(kAlifBlock) k_alif_warm(const float *__restrict__ I, const float *__restrict__ u0,
                                                          const float *__restrict__ w0, float *__restrict__ WP,
                                                          const float *__restrict__ UI, const float *__restrict__ WI,
                                                          int64_t N, int64_t C, int64_t Wn, float u_init, float w_init,
                                                          AlifP p)
{
    const int64_t n = (int64_t)blockIdx.x * kAlifBlock + threadIdx.x;
    const int64_t m = blockIdx.y;
    if (n >= N) return;
    const int64_t s0 = m - Wn > 0 ? m - Wn : 0;
    float u, w;
    if (s0 == 0) {
        u = u0[n];
        w = w0[n];
    } else if (UI) {
        u = UI[s0 * N + n];
        w = WI[s0 * N + n];
    } else {
        u = u_init;
        w = w_init;
    }
    constexpr int kB = 8;
    for (int64_t t = s0 * C; t < m * C; t += kB) {
        float x[kB];
#pragma unroll
        for (int q = 0; q < kB; q++) x[q] = t + q < m * C ? __ldg(I + (t + q) * N + n) : 0.0f;
#pragma unroll
        for (int q = 0; q < kB; q++)
            if (t + q < m * C) {
                bool f;
                alif_step(u, w, x[q], p, f);
            }
    }
    WP[m * N + n] = w;
}

// ------------------------------------------------------------------ backward
// One reverse sweep per neuron (triton_alif.py:359-364, 443-487): LV[t] =
// lv_t, LW[t] = lw_t (optional); s_t from S or recomputed as
// [v_t >= theta0 + w_{t-1}] bit for bit; lwm1 [N] (optional) = lw_{-1};
// PG [4][N] fp64 (optional) = (dbeta, drho, dq, dtheta0) per neuron.
template <int D>
__global__ void __launch_bounds__(kAlifBlock) k_alif_bwd(
    const float *__restrict__ I, const float *__restrict__ u0, const float *__restrict__ w0,
    const float *__restrict__ U, const float *__restrict__ W, const float *__restrict__ S,
    const float *__restrict__ GS, float *__restrict__ LV, float *__restrict__ LW, float *__restrict__ lwm1,
    double *__restrict__ PG, int64_t pg_stride, int64_t T, int64_t N, AlifP p, float alpha)
{
    const int64_t n = (int64_t)blockIdx.x * kAlifBlock + threadIdx.x;
    if (n >= N) return;
    const float u00 = u0[n], w00 = w0[n];
    const float k2 = alpha * 1.4426950408889634f;  // exp(x) = 2^(x log2 e)
    float lv = 0.0f, lw = 0.0f;
    double db = 0.0, dr = 0.0, dq = 0.0, dt = 0.0;
    float x[D] = {}, up[D] = {}, wp[D] = {}, gs[D] = {}, sv[D] = {};
    float xn[D] = {}, upn[D] = {}, wpn[D] = {}, gsn[D] = {}, svn[D] = {};
    auto load = [&](int64_t t0, int cnt, float *xa, float *ua, float *wa, float *ga, float *sa) {
#pragma unroll
        for (int d = 0; d < D; d++) {
            if (d < cnt) {
                const int64_t t = t0 + d, o = t * N + n;
                xa[d] = __ldg(I + o);
                ua[d] = t > 0 ? __ldg(U + o - N) : u00;
                wa[d] = t > 0 ? __ldg(W + o - N) : w00;
                ga[d] = __ldg(GS + o);
                sa[d] = S ? __ldg(S + o) : 0.0f;
            }
        }
    };
    int64_t tend = T;
    int64_t t0 = tend - D > 0 ? tend - D : 0;
    int cnt = (int)(tend - t0);
    load(t0, cnt, x, up, wp, gs, sv);
    while (tend > 0) {
        const int64_t ntend = t0;
        const int64_t nt0 = ntend - D > 0 ? ntend - D : 0;
        const int ncnt = (int)(ntend - nt0);
        if (ntend > 0) load(nt0, ncnt, xn, upn, wpn, gsn, svn);
#pragma unroll
        for (int dd = D - 1; dd >= 0; dd--) {
            if (dd < cnt) {
                const float v = __fadd_rn(__fmul_rn(p.beta, up[dd]), x[dd]);
                const float thr = __fadd_rn(p.theta0, wp[dd]);
                const float s = S ? sv[dd] : (v >= thr ? 1.0f : 0.0f);
                const float a = (v - p.theta0) - wp[dd];
                const float e = ex2_approx(-k2 * a);
                const float sig = rcp_approx(1.0f + e);
                const float sg = alpha * sig * (1.0f - sig);
                const float d = gs[dd] + p.q * lw;
                lv = (1.0f - s) * p.beta * lv + sg * d;
                const int64_t o = (t0 + dd) * N + n;
                if (LW) LW[o] = lw;
                LV[o] = lv;
                if (PG) {
                    db = fma((double)lv, (double)up[dd], db);
                    dr = fma((double)lw, (double)wp[dd], dr);
                    dq = fma((double)lw, (double)s, dq);
                    dt = fma((double)sg, (double)d, dt);
                }
                lw = p.rho * lw - sg * d;
            }
        }
#pragma unroll
        for (int d = 0; d < D; d++) {
            x[d] = xn[d];
            up[d] = upn[d];
            wp[d] = wpn[d];
            gs[d] = gsn[d];
            sv[d] = svn[d];
        }
        tend = ntend;
        t0 = nt0;
        cnt = ncnt;
    }
    if (lwm1) lwm1[n] = lw;
    if (PG) {
        PG[n] = db;
        PG[pg_stride + n] = dr;
        PG[2 * pg_stride + n] = dq;
        PG[3 * pg_stride + n] = -dt;
    }
}

// ------------------------------------------------------------------ backward (TMA)
constexpr int kAlifBwdR = 16, kAlifBwdS = 4;  // rows per tile, ring stages (one neuron per lane)
constexpr int kAlifReplay = 0, kAlifCompose = 1;

// The reverse sweep over chunk m = blockIdx.y (rows [m*C, (m+1)*C)) with
// I[t], U[t-1], W[t-1], GS[t] (and S[t]) streamed through a TMA ring of R-row
// tiles from the chunk's last row up.  One step is affine in (lv, lw):
//     lv' = c lv + sg q lw + sg g,   lw' = (rho - sg q) lw - sg g,   c = (1 - s) beta
// kAlifReplay: starts from (LVE, LWE)[m] (NULL: 0), writes LV (and LW) by TMA
// stores, and per (chunk, neuron) the parameter sums PG[4][M][N] and, for
// chunk 0, dL/dw0.  kAlifCompose: writes the chunk's map (m11, m12, m22, b1,
// b2) into Map[j * mst + m * N + n], j = 0..4: (lv, lw) at the chunk's first row = [[m11, m12],
// [0, m22]] (lv, lw entering) + (b1, b2).  Full tiles above row 0 take the
// fast path; the tile holding row 0 (u_{-1}, w_{-1} = u0, w0) and a ragged
// first tile take checked rows with direct stores.
template <int R, int S, int MODE, bool READ_S, bool PGF, bool WRITE_LW>
__global__ void __launch_bounds__(32) k_alif_bwd_tma(
    const __grid_constant__ CUtensorMap tI, const __grid_constant__ CUtensorMap tU,
    const __grid_constant__ CUtensorMap tW, const __grid_constant__ CUtensorMap tGS,
    const __grid_constant__ CUtensorMap tS, const __grid_constant__ CUtensorMap tLV,
    const __grid_constant__ CUtensorMap tLW, const float *__restrict__ u0, const float *__restrict__ w0,
    float *__restrict__ LV, float *__restrict__ LW, float *__restrict__ lwm1, double *__restrict__ PG,
    const float *__restrict__ LVE, const float *__restrict__ LWE, float *__restrict__ Map, int64_t mst, int64_t N,
    int64_t C, AlifP p, float alpha, int *status)
{
    constexpr int NB = 32;
    constexpr int NT = READ_S ? 5 : 4;  // I, U, W, GS (, S)
    constexpr int kTile = R * NB;
    constexpr uint32_t kStageBytes = NT * kTile * 4;
    constexpr int NO = WRITE_LW ? 2 : 1;  // LV (, LW) output tiles
    constexpr bool kOut = MODE == kAlifReplay;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    float *ring = reinterpret_cast<float *>(smem_raw);
    float *obuf = ring + (size_t)S * NT * kTile;  // 2 x NO tiles (replay)
    __shared__ __align__(8) uint64_t full[S];
    const int lane = threadIdx.x;
    const int64_t n0 = (int64_t)blockIdx.x * NB;
    const int64_t m = blockIdx.y, M = gridDim.y;
    const int64_t cstart = m * C, cend = cstart + C;
    const int64_t nfull = C / R;
    const int64_t ntiles = nfull + (C % R ? 1 : 0);

    auto issue = [&](int s, int64_t k) {
        const int row = (int)(cend - (k + 1) * R);  // may be negative: zero-filled
        float *b = ring + (size_t)s * NT * kTile;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        tma_load_2d(b, &tI, (int)n0, row, &full[s]);
        tma_load_2d(b + kTile, &tU, (int)n0, row - 1, &full[s]);
        tma_load_2d(b + 2 * kTile, &tW, (int)n0, row - 1, &full[s]);
        tma_load_2d(b + 3 * kTile, &tGS, (int)n0, row, &full[s]);
        if (READ_S) tma_load_2d(b + 4 * kTile, &tS, (int)n0, row, &full[s]);
    };
    if (lane == 0) {
        prefetch_tmap(&tI);
        prefetch_tmap(&tU);
        prefetch_tmap(&tW);
        prefetch_tmap(&tGS);
        if (READ_S) prefetch_tmap(&tS);
        if (kOut) prefetch_tmap(&tLV);
        if (kOut && WRITE_LW) prefetch_tmap(&tLW);
        for (int s = 0; s < S; s++) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncwarp();
    if (lane == 0)
        for (int s = 0; s < S && s < ntiles; s++) issue(s, s);

    const int64_t n = n0 + lane;
    const bool act = n < N;
    const float u00 = act ? u0[n] : 0.0f, w00 = act ? w0[n] : 0.0f;
    const float k2 = alpha * 1.4426950408889634f;  // exp(x) = 2^(x log2 e)
    float lv = 0.0f, lw = 0.0f;
    if (kOut && act && LVE) {
        lv = LVE[m * N + n];
        lw = LWE[m * N + n];
    }
    float m11 = 1.0f, m12 = 0.0f, m22 = 1.0f;  // kAlifCompose: the chunk map's matrix
    // parameter sums: each tile's rows in fp32 (tb, tr, tq, tt), folded into
    // the fp64 totals once per tile
    double db = 0.0, dr = 0.0, dq = 0.0, dt = 0.0;
    float tb = 0.0f, tr = 0.0f, tq = 0.0f, tt = 0.0f;
    bool ok = true;
    auto fold = [&]() {
        db += (double)tb;
        dr += (double)tr;
        dq += (double)tq;
        dt += (double)tt;
        tb = tr = tq = tt = 0.0f;
    };
    // the coefficients of row t, which do not depend on (lv, lw): the spike s,
    // the surrogate sg and c = (1 - s) beta
    auto coef = [&](float x, float up, float wp, float sread, float &s, float &sg, float &c) {
        const float v = __fadd_rn(__fmul_rn(p.beta, up), x);
        s = READ_S ? sread : (v >= __fadd_rn(p.theta0, wp) ? 1.0f : 0.0f);
        const float a = (v - p.theta0) - wp;
        const float sig = rcp_approx(1.0f + ex2_approx(-k2 * a));
        sg = alpha * sig * (1.0f - sig);
        c = (1.0f - s) * p.beta;
    };
    // one reverse step at row t from its coefficients; returns (lv_t, lw_t)
    auto chain = [&](float s, float sg, float c, float up, float wp, float gs, float &out_lv, float &out_lw) {
        if (MODE == kAlifCompose) {
            const float sgq = sg * p.q;
            m12 = c * m12 + sgq * m22;
            m11 = c * m11;
            m22 = (p.rho - sgq) * m22;
        }
        const float d = gs + p.q * lw;
        lv = c * lv + sg * d;
        out_lv = lv;
        out_lw = lw;
        if (PGF) {
            tb = fmaf(lv, up, tb);
            tr = fmaf(lw, wp, tr);
            tq = fmaf(lw, s, tq);
            tt = fmaf(sg, d, tt);
        }
        lw = p.rho * lw - sg * d;
    };

    for (int64_t k = 0; k < ntiles; k++) {
        const int s = (int)(k % S);
        if (!mbar_wait(&full[s], (uint32_t)((k / S) & 1))) { ok = false; break; }
        const float *b = ring + (size_t)s * NT * kTile + lane;
        const int64_t rbase = cend - (k + 1) * R;  // global row of in-tile row 0
        const bool fast = k < nfull && rbase > 0;
        if (fast) {
            float *ov = obuf + (int)(k & 1) * NO * kTile;
            float *ow = ov + kTile;
            // the whole tile's coefficients first: their exponentials and
            // reciprocals overlap instead of each sitting in the (lv, lw) chain
            // behind the previous row's stores
            float sv[R], sgv[R], cv[R], upv[R], wpv[R], gsv[R];
#pragma unroll
            for (int rr = 0; rr < R; rr++) {
                const int o = rr * NB;
                upv[rr] = b[kTile + o];
                wpv[rr] = b[2 * kTile + o];
                gsv[rr] = b[3 * kTile + o];
                coef(b[o], upv[rr], wpv[rr], READ_S ? b[4 * kTile + o] : 0.0f, sv[rr], sgv[rr], cv[rr]);
            }
            if (kOut && k >= 2) {  // the stores issued two tiles ago must have read this buffer
                if (lane == 0) bulk_wait_read<1>();
                __syncwarp();
            }
#pragma unroll
            for (int rr = R - 1; rr >= 0; rr--) {
                const int o = rr * NB;
                float a, c;
                chain(sv[rr], sgv[rr], cv[rr], upv[rr], wpv[rr], gsv[rr], a, c);
                if (kOut) {
                    ov[o + lane] = a;
                    if (WRITE_LW) ow[o + lane] = c;
                }
            }
            if (kOut) {
                fence_proxy_async_shared();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tLV, (int)n0, (int)rbase, ov);
                    if (WRITE_LW) tma_store_2d(&tLW, (int)n0, (int)rbase, ow);
                    bulk_commit();
                }
            }
        } else {
            for (int rr = R - 1; rr >= 0; rr--) {
                const int64_t t = rbase + rr;
                if (t < cstart) break;
                const int o = rr * NB;
                const float up = t == 0 ? u00 : b[kTile + o];
                const float wp = t == 0 ? w00 : b[2 * kTile + o];
                float a, c, sp, sg, cf;
                coef(b[o], up, wp, READ_S ? b[4 * kTile + o] : 0.0f, sp, sg, cf);
                chain(sp, sg, cf, up, wp, b[3 * kTile + o], a, c);
                if (kOut && act) {
                    LV[t * N + n] = a;
                    if (WRITE_LW) LW[t * N + n] = c;
                }
            }
        }
        if (PGF) fold();
        // every lane has consumed the stage: order those reads before the refill
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0 && k + S < ntiles) issue(s, k + S);
    }
    if (!ok && status) atomicCAS(status, 0, (int)kStatusTmaWaitTimeout);
    if (ok && act) {
        if (MODE == kAlifCompose) {
            const int64_t o = m * N + n;
            Map[o] = m11;
            Map[mst + o] = m12;
            Map[2 * mst + o] = m22;
            Map[3 * mst + o] = lv;
            Map[4 * mst + o] = lw;
        } else {
            if (lwm1 && m == 0) lwm1[n] = lw;
            if (PGF) {
                const int64_t o = m * N + n, st = M * N;
                PG[o] = db;
                PG[st + o] = dr;
                PG[2 * st + o] = dq;
                PG[3 * st + o] = -dt;
            }
        }
    }
    if (kOut && lane == 0) bulk_wait_all();
}

// Entering (lv, lw) of every chunk from the chunk maps, last chunk first
// (entering 0): chunk m-1 enters with chunk m's map applied to chunk m's entry.
__global__ void __launch_bounds__(kAlifBlock) k_alif_bwd_carry(const float *__restrict__ Map, int64_t st,
                                                               float *__restrict__ LVE, float *__restrict__ LWE,
                                                               int64_t N, int64_t M)
{
    const int64_t n = (int64_t)blockIdx.x * kAlifBlock + threadIdx.x;
    if (n >= N) return;
    float e1 = 0.0f, e2 = 0.0f;
    LVE[(M - 1) * N + n] = 0.0f;
    LWE[(M - 1) * N + n] = 0.0f;
    for (int64_t m = M - 1; m >= 1; m--) {
        const int64_t o = m * N + n;
        const float a11 = Map[o], a12 = Map[st + o], a22 = Map[2 * st + o], b1 = Map[3 * st + o],
                    b2 = Map[4 * st + o];
        const float n1 = a11 * e1 + a12 * e2 + b1;
        const float n2 = a22 * e2 + b2;
        e1 = n1;
        e2 = n2;
        LVE[(m - 1) * N + n] = e1;
        LWE[(m - 1) * N + n] = e2;
    }
}

template <int MODE, bool READ_S, bool PGF, bool WRITE_LW>
static void launch_alif_bwd(const CUtensorMap *maps, const float *u0, const float *w0, float *LV, float *LW,
                            float *lwm1, double *PG, const float *LVE, const float *LWE, float *Map, int64_t mst,
                            int64_t N, int64_t M, int64_t C, const AlifP &p, float alpha, int *status, cudaStream_t s)
{
    constexpr int R = kAlifBwdR, ST = kAlifBwdS, NT = READ_S ? 5 : 4, NO = WRITE_LW ? 2 : 1;
    const size_t smem = ((size_t)ST * NT + (MODE == kAlifReplay ? 2 * NO : 0)) * R * 32 * 4;
    auto kern = k_alif_bwd_tma<R, ST, MODE, READ_S, PGF, WRITE_LW>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    count_launches(1);
    kern<<<dim3((unsigned)((N + 31) / 32), (unsigned)M), 32, smem, s>>>(
        maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], maps[6], u0, w0, LV, LW, lwm1, PG, LVE, LWE, Map, mst, N,
        C, p, alpha, status);
}

// The adjoint over M = T/C chunks (M = 1: one sweep).  M > 1 needs the
// chunk maps Map (5 arrays of [M][N], mst floats apart) and LVE, LWE [M][N].
// PG is [4][M][N].  False when the TMA path does not apply (nothing launched).
static bool alif_bwd_tma(const float *I, const float *u0, const float *w0, const float *U, const float *W,
                         const float *S, const float *GS, float *LV, float *LW, float *lwm1, double *PG, int64_t T,
                         int64_t N, int64_t C, float *Map, int64_t mst, float *LVE, float *LWE, const AlifP &p,
                         float alpha, cudaStream_t s)
{
    const void *ptrs[] = {I, U, W, S, GS, LV, LW};
    if (!tma_ok(ptrs, 7, N) || T <= 0 || T > (1LL << 31) - 64 || ((uintptr_t)PG & 7) || C <= 0 || T % C) return false;
    const int64_t M = T / C;
    if (M > 65535) return false;
    constexpr int R = kAlifBwdR;
    CUtensorMap maps[7];
    if (!make_tmap_2d(&maps[0], I, N, T, 32, R) || !make_tmap_2d(&maps[1], U, N, T, 32, R) ||
        !make_tmap_2d(&maps[2], W, N, T, 32, R) || !make_tmap_2d(&maps[3], GS, N, T, 32, R) ||
        !make_tmap_2d(&maps[5], LV, N, T, 32, R))
        return false;
    maps[4] = maps[0];
    maps[6] = maps[5];
    if (S && !make_tmap_2d(&maps[4], S, N, T, 32, R)) return false;
    if (LW && !make_tmap_2d(&maps[6], LW, N, T, 32, R)) return false;
    int *status = device_status_ptr();
    const bool rs = S != nullptr, pg = PG != nullptr, wl = LW != nullptr;
    const float *le = nullptr, *we = nullptr;
    if (M > 1) {
        if (rs) launch_alif_bwd<kAlifCompose, true, false, false>(maps, u0, w0, LV, LW, lwm1, PG, nullptr, nullptr, Map, mst, N, M, C, p, alpha, status, s);
        else launch_alif_bwd<kAlifCompose, false, false, false>(maps, u0, w0, LV, LW, lwm1, PG, nullptr, nullptr, Map, mst, N, M, C, p, alpha, status, s);
        count_launches(1);
        k_alif_bwd_carry<<<(unsigned)((N + kAlifBlock - 1) / kAlifBlock), kAlifBlock, 0, s>>>(Map, mst, LVE, LWE, N, M);
        le = LVE;
        we = LWE;
    }
    // the combinations the library uses: (S, LW) for alif_backward, neither
    // with the parameter sums for the layer; the rest for completeness
#define LIFB_ALIF_GO(RS, PGF, WL) \
    launch_alif_bwd<kAlifReplay, RS, PGF, WL>(maps, u0, w0, LV, LW, lwm1, PG, le, we, Map, mst, N, M, C, p, alpha, status, s)
    if (rs && wl && !pg) LIFB_ALIF_GO(true, false, true);
    else if (!rs && wl && !pg) LIFB_ALIF_GO(false, false, true);
    else if (!rs && !wl && pg) LIFB_ALIF_GO(false, true, false);
    else if (rs && wl && pg) LIFB_ALIF_GO(true, true, true);
    else if (!rs && wl && pg) LIFB_ALIF_GO(false, true, true);
    else if (rs && !wl && pg) LIFB_ALIF_GO(true, true, false);
    else if (rs && !wl && !pg) LIFB_ALIF_GO(true, false, false);
    else LIFB_ALIF_GO(false, false, false);
#undef LIFB_ALIF_GO
    return true;
}

}  // namespace lifb

namespace {
int fail(int st, const char *msg)
{
    lifb::set_last_error(msg);
    return st;
}

int done(const char *who)
{
    if (cudaGetLastError() != cudaSuccess) {
        char msg[128];
        snprintf(msg, sizeof msg, "%s: launch failed", who);
        return fail(LIFB_ERR_CUDA, msg);
    }
    lifb::set_last_error("");
    return LIFB_OK;
}

size_t al256(size_t b) { return (b + 255) / 256 * 256; }
}  // namespace

extern "C" {

int lifb_alif_serial_fwd(const float *I, const float *u0, const float *w0, float *U, float *W, float *S, int64_t T,
                         int64_t N, float beta, float rho, float q, float theta0, float u_r, void *stream)
{
    LIFB_RANGE("lifb_alif_serial_fwd");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_alif_serial_fwd: negative size");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !w0 || !U || !W || !S) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_alif_serial_fwd: null pointer");
    lifb::alif_serial(I, u0, w0, U, W, S, T, N, lifb::AlifP{beta, rho, q, theta0, u_r}, (cudaStream_t)stream);
    return done("lifb_alif_serial_fwd");
}

size_t lifb_alif_scan_fwd_workspace_bytes(int64_t T, int64_t N, int64_t L)
{
    if (T <= 0 || N <= 0 || L <= 0 || T % L) return 0;
    return 7 * al256((size_t)(T / L) * N * 4);
}

int lifb_alif_scan_fwd(const float *I, const float *u0, const float *w0, float *U, float *W, float *S, int64_t T,
                       int64_t N, float beta, float rho, float q, float theta0, float u_r, int64_t L, int64_t Wlead,
                       const float *Wpred, int64_t Cpred, void *workspace, size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_alif_scan_fwd");
    if (T < 0 || N < 0 || L <= 0 || Wlead < 0 || (T > 0 && T % L))
        return fail(LIFB_ERR_INVALID_ARGUMENT,
                    "lifb_alif_scan_fwd: T must be a multiple of the segment length L > 0, W >= 0");
    if (Wpred && (Cpred <= 0 || T % Cpred))
        return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_alif_scan_fwd: Wpred needs T to be a multiple of Cpred > 0");
    if (T / L > 65535) return fail(LIFB_ERR_UNSUPPORTED, "lifb_alif_scan_fwd: more than 65535 segments");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !w0 || !U || !W || !S) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_alif_scan_fwd: null pointer");
    cudaStream_t s = (cudaStream_t)stream;
    const lifb::AlifP p{beta, rho, q, theta0, u_r};
    const int64_t NS = T / L;
    if (NS == 1 || Wlead == 0) {
        lifb::alif_serial(I, u0, w0, U, W, S, T, N, p, s);
        return done("lifb_alif_scan_fwd");
    }
    const size_t one = al256((size_t)NS * N * 4);
    if (!workspace || (uintptr_t)workspace % 256 || workspace_bytes < 7 * one)
        return fail(LIFB_ERR_WORKSPACE, "lifb_alif_scan_fwd: workspace missing, misaligned or too small "
                                        "(lifb_alif_scan_fwd_workspace_bytes)");
    char *b = (char *)workspace;
    float *SU = (float *)b, *SW = (float *)(b + one), *EU = (float *)(b + 2 * one), *EW = (float *)(b + 3 * one);
    float *EUn = (float *)(b + 4 * one), *EWn = (float *)(b + 5 * one);
    int32_t *Changed = (int32_t *)(b + 6 * one);
    if (lifb::alif_fwd_tma(I, u0, w0, nullptr, nullptr, U, W, S, EU, EW, T, N, L, p, Wlead, SU, SW, Wpred, Cpred, s)) {
        const unsigned nb = (unsigned)((N + lifb::kAlifFixBlock - 1) / lifb::kAlifFixBlock);
        lifb::count_launches(2);
        lifb::k_alif_fixup_par<<<dim3(nb, (unsigned)(NS - 1)), lifb::kAlifFixBlock, 0, s>>>(
            I, SU, SW, U, W, S, EU, EW, EUn, EWn, Changed, N, L, p);
        lifb::k_alif_fixup_seq<<<nb, lifb::kAlifFixBlock, 0, s>>>(I, U, W, S, EU, EW, EUn, EWn, Changed, N, NS, L, p);
    } else {
        // the TMA path does not apply: the serial pass (exact, no fix-up needed)
        lifb::alif_serial(I, u0, w0, U, W, S, T, N, p, s);
    }
    return done("lifb_alif_scan_fwd");
}

int lifb_alif_warm_predict(const float *I, const float *u0, const float *w0, float *WP, const float *UI,
                           const float *WI, int64_t T, int64_t N, int64_t C, int64_t Wn, float u_init, float w_init,
                           float beta, float rho, float q, float theta0, float u_r, void *stream)
{
    LIFB_RANGE("lifb_alif_warm_predict");
    if (T < 0 || N < 0 || C <= 0 || Wn < 0 || T % C)
        return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_alif_warm_predict: T must be a multiple of C > 0, Wn >= 0");
    if (T / C > 65535) return fail(LIFB_ERR_UNSUPPORTED, "lifb_alif_warm_predict: more than 65535 chunks");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !w0 || !WP || (UI && !WI) || (WI && !UI))
        return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_alif_warm_predict: null pointer (UI and WI go together)");
    lifb::count_launches(1);
    dim3 g((unsigned)((N + lifb::kAlifBlock - 1) / lifb::kAlifBlock), (unsigned)(T / C));
    lifb::k_alif_warm<<<g, lifb::kAlifBlock, 0, (cudaStream_t)stream>>>(
        I, u0, w0, WP, UI, WI, N, C, Wn, u_init, w_init, lifb::AlifP{beta, rho, q, theta0, u_r});
    return done("lifb_alif_warm_predict");
}

size_t lifb_alif_bwd_scan_workspace_bytes(int64_t T, int64_t N, int64_t C)
{
    if (T <= 0 || N <= 0 || C <= 0 || T % C || T / C < 2) return 0;
    return 7 * al256((size_t)(T / C) * N * 4);
}

int lifb_alif_bwd_scan(const float *I, const float *u0, const float *w0, const float *U, const float *W,
                       const float *S, const float *GS, float *LV, float *LW, float *lw_m1, double *param_sums,
                       int64_t T, int64_t N, float beta, float rho, float q, float theta0, float alpha, int64_t C,
                       void *workspace, size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_alif_bwd_scan");
    if (T < 0 || N < 0 || C <= 0 || (T > 0 && T % C))
        return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_alif_bwd_scan: T must be a multiple of the chunk length C > 0");
    if (T / C > 65535) return fail(LIFB_ERR_UNSUPPORTED, "lifb_alif_bwd_scan: more than 65535 chunks");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !w0 || !U || !W || !GS || !LV)
        return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_alif_bwd_scan: null pointer");
    const int64_t M = T / C;
    float *Map = nullptr, *LVE = nullptr, *LWE = nullptr;
    int64_t mst = 0;
    if (M > 1) {
        const size_t one = al256((size_t)M * N * 4);
        if (!workspace || (uintptr_t)workspace % 256 || workspace_bytes < 7 * one)
            return fail(LIFB_ERR_WORKSPACE, "lifb_alif_bwd_scan: workspace missing, misaligned or too small "
                                            "(lifb_alif_bwd_scan_workspace_bytes)");
        char *b = (char *)workspace;
        Map = (float *)b;  // 5 arrays of [M][N], `one` bytes apart
        mst = (int64_t)(one / 4);
        LVE = (float *)(b + 5 * one);
        LWE = (float *)(b + 6 * one);
    }
    const lifb::AlifP p{beta, rho, q, theta0, 0.0f};
    cudaStream_t s = (cudaStream_t)stream;
    if (lifb::alif_bwd_tma(I, u0, w0, U, W, S, GS, LV, LW, lw_m1, param_sums, T, N, C, Map, mst, LVE, LWE, p, alpha,
                           s))
        return done("lifb_alif_bwd_scan");
    // the plain sweep over the whole sequence: its sums go to chunk 0's slots
    if (param_sums && M > 1 && cudaMemsetAsync(param_sums, 0, (size_t)4 * M * N * sizeof(double), s) != cudaSuccess)
        return fail(LIFB_ERR_CUDA, "lifb_alif_bwd_scan: memset failed");
    lifb::count_launches(1);
    lifb::k_alif_bwd<8><<<(unsigned)((N + lifb::kAlifBlock - 1) / lifb::kAlifBlock), lifb::kAlifBlock, 0, s>>>(
        I, u0, w0, U, W, S, GS, LV, LW, lw_m1, param_sums, M * N, T, N, p, alpha);
    return done("lifb_alif_bwd_scan");
}

int lifb_alif_bwd(const float *I, const float *u0, const float *w0, const float *U, const float *W, const float *S,
                  const float *GS, float *LV, float *LW, float *lw_m1, double *param_sums, int64_t T, int64_t N,
                  float beta, float rho, float q, float theta0, float alpha, void *stream)
{
    LIFB_RANGE("lifb_alif_bwd");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_alif_bwd: negative size");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !w0 || !U || !W || !GS || !LV) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_alif_bwd: null pointer");
    return lifb_alif_bwd_scan(I, u0, w0, U, W, S, GS, LV, LW, lw_m1, param_sums, T, N, beta, rho, q, theta0, alpha,
                              T, nullptr, 0, stream);
}

}  // extern "C"
