// TMA-pipelined chunk kernels: the forward replay (which is also the serial
// forward: one chunk of T rows starting from u0) and the reverse adjoint
// sweep (the serial backward: one chunk ending at lam = 0), both streaming
// HBM once.
//
// CTA = one warp owning NB = 32*NPL consecutive neurons (NPL = 4: a float4 of
// four independent recurrences per lane; NPL = 1: one per lane, for more
// warps on narrow N) and one chunk m of C rows (blockIdx.y).  Time tiles of
// R rows x NB neurons stream into a ring of S shared-memory stages with 2-D
// TMA loads (cp.async.bulk.tensor, no multicast) completing on one mbarrier
// per stage; lane 0 refills a stage once the warp has consumed it.  Results
// are written into a double-buffered shared-memory tile and leave with one
// TMA bulk-tensor store per tile, so a step costs one shared load, the
// recurrence and one shared store per output; no per-step address math or
// predicates on full tiles.  The ragged last tile (C % R rows) and the tile
// holding t = 0 of the adjoint take a checked path with direct stores.
//
//   k_fwd_tma  replay of chunk m from Starts[m] (or u0): U, S rows and Ends[m]
//              = fwd_tiled_kernel (lifscan/triton_lif.py:353-379); with M = 1 it is
//              serial_forward_tiled (:460-466), bit-identical to fast.py:69-81.
//   k_bwd_tma  reverse sweep of lam_t = a_t lam_{t+1} + b_t over chunk m with the
//              surrogate fused (_coef :42-50):
//                kReplay:  from LamEnd[m] (or 0), writes Lam (= bwd_tiled_kernel
//                          :382-418; with M = 1 bwd_tiled_pf_kernel :1087-1127)
//                kCompose: chunk map lam_start = P*lam_end + Q (= bwd_chunk_tiled_kernel :421-457)
//              With S == NULL the spike s_t is recomputed as [v_t >= theta] from the
//              recomputed v_t (bit-identical to the forward's S), saving 4 B/step.
//
// The launchers fall back (return false) unless N % 4 == 0 and every tensor
// is 16-byte aligned (TMA stride rule and vector accesses).
#include <type_traits>

#include "lifb_common.cuh"
#include "lifb_internal.h"
#include "tma.cuh"
#include "vec.cuh"

namespace lifb {

// ===================================================================== forward
// Chunk m starts from Starts[m * start_stride] (rows of N) or u0.  With
// lead > 0 (a multiple of R, with C a multiple of R) chunk m >= 1 instead
// runs the `lead` rows before it first, without stores, from u_r (from u0
// when they reach row 0, where the start is then exact), streamed through the
// same TMA ring, and records that guessed start in LeadStarts[m]; chunk 0
// starts from Starts[0] or u0 as before.  VOUT: the U output receives the
// pre-reset potential v_t instead of u_t (Ends still hold u).  AFF: the affine
// reset u = fl(fl(gamma*v) + delta) instead of u_r (gamma = 1, delta = -theta:
// the soft reset).
template <int NPL, int R, int S, bool VOUT, bool AFF>
__global__ void __launch_bounds__(32) k_fwd_tma(const __grid_constant__ CUtensorMap tI,
                                                const __grid_constant__ CUtensorMap tU,
                                                const __grid_constant__ CUtensorMap tS, const float *__restrict__ u0,
                                                const float *__restrict__ Starts, int64_t start_stride,
                                                float *__restrict__ U, float *__restrict__ Sout,
                                                float *__restrict__ Ends, int64_t N, int64_t C, float beta,
                                                float theta, float u_r, int64_t lead, float *__restrict__ LeadStarts,
                                                float gamma, float delta, int *status, int64_t m0)
{
    constexpr int NB = 32 * NPL;
    constexpr int kTile = R * NB;  // floats per tile
    constexpr uint32_t kStageBytes = kTile * 4;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    float *ring = reinterpret_cast<float *>(smem_raw);  // S input tiles
    float *obuf = ring + S * kTile;                      // 2 x (U tile, S tile)
    __shared__ __align__(8) uint64_t full[S];
    const int lane = threadIdx.x;
    const int64_t n0 = (int64_t)blockIdx.x * NB;
    const int64_t m = blockIdx.y + m0;  // chunks m0..M-1 (m0 > 0: the caller runs the first ones)
    const int64_t row0 = m * C;
    const int64_t nfull = C / R;
    const int rem = (int)(C - nfull * R);
    const int64_t ntiles = nfull + (rem ? 1 : 0);
    // lead-in tiles before the chunk's own: rows [lrow0, row0)
    const bool leading = lead > 0 && m > 0;
    const int64_t lrow0 = leading ? (row0 > lead ? row0 - lead : 0) : row0;
    const int64_t nlead = (row0 - lrow0) / R;
    const int64_t ntot = nlead + ntiles;
    auto tile_row = [&](int64_t k) { return k < nlead ? lrow0 + k * R : row0 + (k - nlead) * R; };

    if (lane == 0) {
        prefetch_tmap(&tI);
        prefetch_tmap(&tU);
        prefetch_tmap(&tS);
        for (int s = 0; s < S; s++) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncwarp();
    // V path: the adjoint reads V next, so V's lines are kept in L2 ahead of I's and S's, which nothing
    // in the layer reads again
    const uint64_t pol_first = VOUT ? l2_evict_first() : 0, pol_last = VOUT ? l2_evict_last() : 0;
    auto load_i = [&](int s, int64_t k) {
        if constexpr (VOUT) tma_load_2d_hint(ring + s * kTile, &tI, (int)n0, (int)tile_row(k), &full[s], pol_first);
        else tma_load_2d(ring + s * kTile, &tI, (int)n0, (int)tile_row(k), &full[s]);
    };
    if (lane == 0) {
        for (int s = 0; s < S && s < ntot; s++) {
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            load_i(s, s);
        }
    }
    const int64_t nl = n0 + NPL * lane;
    const bool act = nl < N;
    Vec<NPL> u;
    if (act) {
        if (leading) {
            if (lrow0 == 0 && u0) {  // without u0, a lead-in from row 0 starts from u_r too
                u = ld_vec<NPL>(u0 + nl);
            } else {
#pragma unroll
                for (int i = 0; i < NPL; i++) u.v[i] = u_r;
            }
        } else {
            u = ld_vec<NPL>((Starts ? Starts + m * start_stride * N : u0) + nl);
        }
    } else {
#pragma unroll
        for (int i = 0; i < NPL; i++) u.v[i] = 0.f;
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
            for (int i = 0; i < NPL; i++)
                u.v[i] = step_r_u<AFF>(u.v[i], x[r].v[i], beta, theta, u_r, gamma, delta);
        // the stage's rows are consumed (every lane used them): refill it
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0 && k + S < ntot) {
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            load_i(s, k + S);
        }
    }
    if (leading && ok && LeadStarts && act) st_vec<NPL>(LeadStarts + m * N + nl, u);

    for (int64_t kk = 0; kk < nfull && ok; kk++) {
        const int64_t k = nlead + kk;  // ring index
        const int s = (int)(k % S);
        if (!mbar_wait(&full[s], (uint32_t)((k / S) & 1))) { ok = false; break; }
        const float *in = ring + s * kTile + NPL * lane;
        Vec<NPL> x[R];
#pragma unroll
        for (int r = 0; r < R; r++) x[r] = ld_vec<NPL>(in + r * NB);
        float *ou = obuf + (int)(kk & 1) * 2 * kTile;
        float *os = ou + kTile;
        if (kk >= 2) {  // the store issued two tiles ago must have read this buffer
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
            Vec<NPL> sp, vv;
#pragma unroll
            for (int i = 0; i < NPL; i++) {
                const float v = __fadd_rn(__fmul_rn(beta, u.v[i]), x[r].v[i]);
                const bool f = v >= theta;
                u.v[i] = f ? (AFF ? __fadd_rn(__fmul_rn(gamma, v), delta) : u_r) : v;
                sp.v[i] = f ? 1.0f : 0.0f;
                vv.v[i] = v;
            }
            st_vec<NPL>(ou + r * NB + NPL * lane, VOUT ? vv : u);
            st_vec<NPL>(os + r * NB + NPL * lane, sp);
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
            if constexpr (VOUT) {
                tma_store_2d_hint(&tU, (int)n0, (int)(row0 + kk * R), ou, pol_last);
                tma_store_2d_hint(&tS, (int)n0, (int)(row0 + kk * R), os, pol_first);
            } else {
                tma_store_2d(&tU, (int)n0, (int)(row0 + kk * R), ou);
                tma_store_2d(&tS, (int)n0, (int)(row0 + kk * R), os);
            }
            bulk_commit();
            if (k + S < ntot) {
                mbar_arrive_expect_tx(&full[s], kStageBytes);
                load_i(s, k + S);
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
                Vec<NPL> sp, vv;
#pragma unroll
                for (int i = 0; i < NPL; i++) {
                    const float v = __fadd_rn(__fmul_rn(beta, u.v[i]), x.v[i]);
                    const bool f = v >= theta;
                    u.v[i] = f ? (AFF ? __fadd_rn(__fmul_rn(gamma, v), delta) : u_r) : v;
                    sp.v[i] = f ? 1.0f : 0.0f;
                    vv.v[i] = v;
                }
                if (act) {
                    const int64_t o = (row0 + nfull * R + r) * N + nl;
                    st_vec<NPL>(U + o, VOUT ? vv : u);
                    st_vec<NPL>(Sout + o, sp);
                }
            }
        }
    }
    if (!ok && status) atomicCAS(status, 0, (int)kStatusTmaWaitTimeout);
    if (ok && Ends && act) st_vec<NPL>(Ends + m * N + nl, u);
    if (lane == 0) bulk_wait_all();
}

// ==================================================================== backward
enum BwdMode { kReplay = 0, kCompose = 1 };

// Input tensors per stage, in ring order: I, U (one row earlier), [S], GS, [GU];
// FROM_V (the forward saved v_t = fl(fl(beta*u_{t-1}) + x_t) in place of U):
// V (slot kI), GS.
template <bool READ_S, bool HAS_GU, bool FROM_V = false>
struct BwdLayout {
    static constexpr int kI = 0, kU = 1, kS = 2;
    static constexpr int kGS = FROM_V ? 1 : (READ_S ? 3 : 2);
    static constexpr int kGU = kGS + 1;
    static constexpr int NT = FROM_V ? 2 : 3 + (READ_S ? 1 : 0) + (HAS_GU ? 1 : 0);
};

// log2(e): e^x = 2^(x log2 e), so the surrogate's exponential is one ex2.
constexpr float kLog2e = 1.4426950408889634f;

// Adjoint coefficients of one neuron-step: lam_t = a*lam_{t+1} + c with the
// forward's v = fl(fl(beta*u_{t-1}) + x_t) (bit for bit), s = S or [v >= theta],
// the sigmoid surrogate sg = alpha*sig*(1 - sig), sig = 1/(1 + e),
// e = exp(-alpha (v - theta)) = 2^(k2 (theta - v)) with k2 = alpha*log2(e), and
// J = 1 - s (+ (u_r - v) sg for the attached reset), a = beta*J, c = gs*sg + J*gu.
// k2 = alpha*log2(e), k2t = k2*theta: the exponent k2*(theta - v) is one FMA.
// sig*(1 - sig) = sig - sig^2 (one FMA).  DET: the detached reset, known at
// compile time (the V path has no other).
template <bool READ_S, bool HAS_GU, bool DET = false, bool AFF = false>
__device__ __forceinline__ void adj_coef_v(float v, float sread, float gs, float gu, float beta, float theta,
                                           float u_r, float alpha, float k2, float k2t, bool detach, float &a,
                                           float &c, float bgamma = 0.0f)
{
    const float e = ex2_approx(fmaf(-k2, v, k2t));
    const float sig = rcp_approx(1.0f + e);
    const float sg = alpha * fmaf(-sig, sig, sig);
    float cc = gs * sg;
    if (AFF) {  // detached affine reset: du_t/dv_t = gamma at a spike, 1 elsewhere (bgamma = beta*gamma)
        a = v >= theta ? bgamma : beta;
    } else if (!READ_S && (DET || detach)) {  // s in {0, 1}: a = beta*(1 - s) and J*gu as selects
        const bool spk = v >= theta;
        a = spk ? 0.0f : beta;
        if constexpr (HAS_GU) cc = spk ? cc : cc + gu;
    } else {
        const float s = READ_S ? sread : (v >= theta ? 1.0f : 0.0f);
        float J = 1.0f - s;
        if (!detach) J = J + (u_r - v) * sg;
        a = beta * J;
        if constexpr (HAS_GU) cc = cc + J * gu;
    }
    c = cc;
}

// The forward's v, bit for bit, from U[t-1] and I[t]; or read (FROM_V).
template <int NPL, bool FROM_V, typename Ly>
__device__ __forceinline__ Vec<NPL> bwd_v(const float *b, int kTile, int off, const Vec<NPL> *up_override, float beta)
{
    Vec<NPL> v = ld_vec<NPL>(b + Ly::kI * kTile + off);
    if constexpr (!FROM_V) {
        const Vec<NPL> up = up_override ? *up_override : ld_vec<NPL>(b + Ly::kU * kTile + off);
#pragma unroll
        for (int i = 0; i < NPL; i++) v.v[i] = __fadd_rn(__fmul_rn(beta, up.v[i]), v.v[i]);
    }
    return v;
}

// Coefficients of NPL neurons at in-tile offset `off` (no dependence on lam,
// so a whole tile is computed ahead of the chain); vout, when given, receives
// the forward's v of the row.
template <int NPL, bool READ_S, bool HAS_GU, bool FROM_V, bool AFF = false>
__device__ __forceinline__ void bwd_coef(const float *b, int kTile, int off, Vec<NPL> &a, Vec<NPL> &c, float beta,
                                         float theta, float u_r, float alpha, float k2, float k2t, bool detach,
                                         float bgamma = 0.0f, Vec<NPL> *vout = nullptr)
{
    using Ly = BwdLayout<READ_S, HAS_GU, FROM_V>;
    const Vec<NPL> v = bwd_v<NPL, FROM_V, Ly>(b, kTile, off, nullptr, beta);
    if (vout) *vout = v;
    const Vec<NPL> gs = ld_vec<NPL>(b + Ly::kGS * kTile + off);
    Vec<NPL> sv, gu;
    if constexpr (READ_S) sv = ld_vec<NPL>(b + Ly::kS * kTile + off);
    if constexpr (HAS_GU) gu = ld_vec<NPL>(b + Ly::kGU * kTile + off);
#pragma unroll
    for (int i = 0; i < NPL; i++)
        adj_coef_v<READ_S, HAS_GU, FROM_V, AFF>(v.v[i], READ_S ? sv.v[i] : 0.0f, gs.v[i], HAS_GU ? gu.v[i] : 0.0f,
                                                beta, theta, u_r, alpha, k2, k2t, detach, a.v[i], c.v[i], bgamma);
}

// One reverse step for NPL neurons at in-tile offset `off`; pp (the running
// product of a) only when the chunk map is tracked.
template <int NPL, bool READ_S, bool HAS_GU, bool TRACK, bool FROM_V, bool AFF = false>
__device__ __forceinline__ void bwd_step(const float *b, int kTile, int off, const Vec<NPL> *up_override,
                                         Vec<NPL> &lam, Vec<NPL> &pp, float beta, float theta, float u_r,
                                         float alpha, float k2, float k2t, bool detach, float bgamma = 0.0f)
{
    using Ly = BwdLayout<READ_S, HAS_GU, FROM_V>;
    const Vec<NPL> v = bwd_v<NPL, FROM_V, Ly>(b, kTile, off, up_override, beta);
    const Vec<NPL> gs = ld_vec<NPL>(b + Ly::kGS * kTile + off);
    Vec<NPL> sv, gu;
    if constexpr (READ_S) sv = ld_vec<NPL>(b + Ly::kS * kTile + off);
    if constexpr (HAS_GU) gu = ld_vec<NPL>(b + Ly::kGU * kTile + off);
#pragma unroll
    for (int i = 0; i < NPL; i++) {
        float a, c;
        adj_coef_v<READ_S, HAS_GU, FROM_V, AFF>(v.v[i], READ_S ? sv.v[i] : 0.0f, gs.v[i], HAS_GU ? gu.v[i] : 0.0f,
                                                beta, theta, u_r, alpha, k2, k2t, detach, a, c, bgamma);
        lam.v[i] = c + a * lam.v[i];
        if constexpr (TRACK) pp.v[i] = a * pp.v[i];
    }
}

template <int NPL, int R, int S, bool READ_S, bool HAS_GU, int MODE, bool TRACK, bool FROM_V, bool AFF = false,
          bool PG = false>
__global__ void __launch_bounds__(32) k_bwd_tma(const __grid_constant__ CUtensorMap tI,
                                                const __grid_constant__ CUtensorMap tU,
                                                const __grid_constant__ CUtensorMap tS,
                                                const __grid_constant__ CUtensorMap tGS,
                                                const __grid_constant__ CUtensorMap tGU,
                                                const __grid_constant__ CUtensorMap tLam,
                                                const float *__restrict__ u0, const float *__restrict__ LamEnd,
                                                float *__restrict__ Lam, float *__restrict__ P, float *__restrict__ Q,
                                                int32_t *__restrict__ D, int64_t N, int64_t C, float beta, float theta,
                                                float u_r, float alpha, bool detach, float gamma, float delta,
                                                double *__restrict__ PGout, int *status)
{
    static_assert(!PG || (FROM_V && AFF && MODE == kReplay && !TRACK), "parameter sums: affine V path only");
    using Ly = BwdLayout<READ_S, HAS_GU, FROM_V>;
    constexpr int NB = 32 * NPL;
    constexpr int NT = Ly::NT;
    constexpr int kTile = R * NB;
    constexpr uint32_t kStageBytes = NT * kTile * 4;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    float *ring = reinterpret_cast<float *>(smem_raw);
    float *obuf = ring + (size_t)S * NT * kTile;  // 2 Lam tiles (kReplay)
    __shared__ __align__(8) uint64_t full[S];
    const int lane = threadIdx.x;
    const int64_t n0 = (int64_t)blockIdx.x * NB;
    const int64_t m = blockIdx.y;
    const int64_t cstart = m * C, cend = (m + 1) * C;
    const int64_t nfull = C / R;
    const int rem = (int)(C - nfull * R);
    const int64_t ntiles = nfull + (rem ? 1 : 0);

    const uint64_t pol_first = FROM_V ? l2_evict_first() : 0;  // V and GS are read once
    auto issue = [&](int s, int64_t k) {
        const int row = (int)(cend - (k + 1) * R);  // may be negative: zero-filled
        float *b = ring + (size_t)s * NT * kTile;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        if constexpr (FROM_V) {
            tma_load_2d_hint(b + Ly::kI * kTile, &tI, (int)n0, row, &full[s], pol_first);
            if (READ_S) tma_load_2d_hint(b + Ly::kS * kTile, &tS, (int)n0, row, &full[s], pol_first);
            tma_load_2d_hint(b + Ly::kGS * kTile, &tGS, (int)n0, row, &full[s], pol_first);
            if (HAS_GU) tma_load_2d_hint(b + Ly::kGU * kTile, &tGU, (int)n0, row, &full[s], pol_first);
            return;
        }
        tma_load_2d(b + Ly::kI * kTile, &tI, (int)n0, row, &full[s]);
        if (!FROM_V) tma_load_2d(b + Ly::kU * kTile, &tU, (int)n0, row - 1, &full[s]);
        if (READ_S) tma_load_2d(b + Ly::kS * kTile, &tS, (int)n0, row, &full[s]);
        tma_load_2d(b + Ly::kGS * kTile, &tGS, (int)n0, row, &full[s]);
        if (HAS_GU) tma_load_2d(b + Ly::kGU * kTile, &tGU, (int)n0, row, &full[s]);
    };

    if (lane == 0) {
        prefetch_tmap(&tI);
        prefetch_tmap(&tU);
        prefetch_tmap(&tGS);
        if (READ_S) prefetch_tmap(&tS);
        if (HAS_GU) prefetch_tmap(&tGU);
        if (MODE == kReplay) prefetch_tmap(&tLam);
        for (int s = 0; s < S; s++) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncwarp();
    if (lane == 0)
        for (int s = 0; s < S && s < ntiles; s++) issue(s, s);

    const int64_t nl = n0 + NPL * lane;
    const bool act = nl < N;
    Vec<NPL> uz, lam, pp;
    // dn: rows, counted from the chunk's last row, whose running product of a
    // is still nonzero (the rows a lam entering from above changes)
    int dn[NPL];
#pragma unroll
    for (int i = 0; i < NPL; i++) { uz.v[i] = 0.f; lam.v[i] = 0.f; pp.v[i] = 1.f; dn[i] = 0; }
    if (act) {
        if (!FROM_V) uz = ld_vec<NPL>(u0 + nl);
        if (MODE == kReplay && LamEnd) lam = ld_vec<NPL>(LamEnd + m * N + nl);
    }
    bool ok = true;
    const float k2 = alpha * kLog2e, k2t = k2 * theta, bgamma = beta * gamma;
    // PG: sums of dL/dbeta = sum_t lam_{t+1} u_t (+ lam_0 u0), dL/dgamma =
    // beta sum_t s_t v_t lam_{t+1}, dL/ddelta = beta sum_t s_t lam_{t+1}, taken
    // at row t before lam is stepped (lam then holds lam_{t+1}); each tile's
    // rows are summed in fp32 (tb, tg, td) and folded into fp64 totals, where
    // the factor beta of the last two is applied
    double pb[NPL], pgm[NPL], pdl[NPL];
    float tb[NPL], tg[NPL], td[NPL];
#pragma unroll
    for (int i = 0; i < NPL; i++) { pb[i] = 0.0; pgm[i] = 0.0; pdl[i] = 0.0; tb[i] = tg[i] = td[i] = 0.0f; }
    auto pg_row = [&](const Vec<NPL> &v) {
#pragma unroll
        for (int i = 0; i < NPL; i++) {
            const bool spk = v.v[i] >= theta;
            const float u = spk ? __fadd_rn(__fmul_rn(gamma, v.v[i]), delta) : v.v[i];
            tb[i] = fmaf(lam.v[i], u, tb[i]);
            const float ls = spk ? lam.v[i] : 0.0f;
            td[i] += ls;
            tg[i] = fmaf(v.v[i], ls, tg[i]);
        }
    };
    auto pg_fold = [&]() {
#pragma unroll
        for (int i = 0; i < NPL; i++) {
            pb[i] += (double)tb[i];
            pgm[i] = fma((double)beta, (double)tg[i], pgm[i]);
            pdl[i] = fma((double)beta, (double)td[i], pdl[i]);
            tb[i] = tg[i] = td[i] = 0.0f;
        }
    };

    for (int64_t k = 0; k < ntiles; k++) {
        const int s = (int)(k % S);
        if (!mbar_wait(&full[s], (uint32_t)((k / S) & 1))) { ok = false; break; }
        const float *b = ring + (size_t)s * NT * kTile;
        const int64_t rbase = cend - (k + 1) * R;  // global row of in-tile row 0
        const bool fast = k < nfull && rbase > 0;  // full tile, no row 0 inside
        if (fast) {
            float *ol = obuf + (int)(k & 1) * kTile;
            Vec<NPL> av[R], cv[R];
            // PG: v of every row kept in registers and the rows that spiked
            // (bit rr), found with the coefficients.  The chain adds one FMA
            // per row, lam_{t+1} v_t; the spiking rows, where u_t differs from
            // v_t, add lam_{t+1} (u_t - v_t) to the dbeta sum afterwards
            Vec<NPL> vk[PG ? R : 1];
            uint32_t smask[NPL];
#pragma unroll
            for (int i = 0; i < NPL; i++) smask[i] = 0u;
            static_assert(!PG || R <= 32, "spike mask holds 32 rows");
#pragma unroll
            for (int rr = 0; rr < R; rr++) {
                if constexpr (PG) {
                    bwd_coef<NPL, READ_S, HAS_GU, FROM_V, AFF>(b, kTile, rr * NB + NPL * lane, av[rr], cv[rr], beta,
                                                               theta, u_r, alpha, k2, k2t, detach, bgamma, &vk[rr]);
#pragma unroll
                    for (int i = 0; i < NPL; i++) smask[i] |= vk[rr].v[i] >= theta ? (1u << rr) : 0u;
                } else {
                    bwd_coef<NPL, READ_S, HAS_GU, FROM_V, AFF>(b, kTile, rr * NB + NPL * lane, av[rr], cv[rr], beta,
                                                               theta, u_r, alpha, k2, k2t, detach, bgamma);
                }
            }
            if (MODE == kReplay && k >= 2) {
                if (lane == 0) bulk_wait_read<1>();
                __syncwarp();
            }
            const Vec<NPL> pp_in = pp;
            [[maybe_unused]] const Vec<NPL> lam_in = lam;
#pragma unroll
            for (int rr = R - 1; rr >= 0; rr--) {
#pragma unroll
                for (int i = 0; i < NPL; i++) {
                    if constexpr (PG) tb[i] = fmaf(lam.v[i], vk[rr].v[i], tb[i]);
                    lam.v[i] = cv[rr].v[i] + av[rr].v[i] * lam.v[i];
                    if constexpr (TRACK) pp.v[i] = av[rr].v[i] * pp.v[i];
                }
                if (MODE == kReplay) st_vec<NPL>(ol + rr * NB + NPL * lane, lam);
            }
            if constexpr (PG) {
                // the spiking rows only (a few per tile): lam_{t+1} is the
                // tile's next row in ol (this lane's own stores), or the lam
                // that entered the tile for its top row
#pragma unroll
                for (int i = 0; i < NPL; i++) {
                    uint32_t msk = smask[i];
                    while (msk) {
                        const int rr = __ffs(msk) - 1;
                        msk &= msk - 1u;
                        const float ln = rr == R - 1 ? lam_in.v[i] : ol[(rr + 1) * NB + NPL * lane + i];
                        const float v = b[Ly::kI * kTile + rr * NB + NPL * lane + i];
                        const float u = __fadd_rn(__fmul_rn(gamma, v), delta);
                        tb[i] = fmaf(ln, __fsub_rn(u, v), tb[i]);
                        td[i] += ln;
                        tg[i] = fmaf(v, ln, tg[i]);
                    }
                }
                pg_fold();
            }
            if (TRACK && D) {
#pragma unroll
                for (int i = 0; i < NPL; i++) {
                    if (pp.v[i] != 0.f) {
                        dn[i] += R;
                    } else if (pp_in.v[i] != 0.f) {  // the product reached 0 in this tile: find the row
                        float q = pp_in.v[i];
                        for (int rr = R - 1; rr >= 0; rr--) {
                            q = av[rr].v[i] * q;
                            if (q == 0.f) break;
                            dn[i]++;
                        }
                    }
                }
            }
            if (MODE == kReplay) {
                fence_proxy_async_shared();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tLam, (int)n0, (int)rbase, ol);
                    bulk_commit();
                }
            }
        } else {  // ragged tile or the tile holding t = 0: checked rows, direct stores
            for (int rr = R - 1; rr >= 0; rr--) {
                const int64_t t = rbase + rr;
                if (t < cstart) break;
                if constexpr (PG) pg_row(ld_vec<NPL>(b + Ly::kI * kTile + rr * NB + NPL * lane));
                bwd_step<NPL, READ_S, HAS_GU, TRACK, FROM_V, AFF>(b, kTile, rr * NB + NPL * lane,
                                                            (!FROM_V && t == 0) ? &uz : nullptr, lam, pp, beta,
                                                            theta, u_r, alpha, k2, k2t, detach, bgamma);
                if constexpr (TRACK) {
#pragma unroll
                    for (int i = 0; i < NPL; i++) dn[i] += pp.v[i] != 0.f ? 1 : 0;
                }
                if (MODE == kReplay && act) st_vec<NPL>(Lam + t * N + nl, lam);
            }
            if constexpr (PG) pg_fold();
        }
        __syncwarp();
        if (lane == 0 && k + S < ntiles) issue(s, k + S);
    }
    if (!ok && status) atomicCAS(status, 0, (int)kStatusTmaWaitTimeout);
    // kCompose always writes the chunk map; kReplay writes it when P is given
    // (then P = prod a over the chunk and Q = lam at its first row).
    if (TRACK && ok && P && act) {
        st_vec<NPL>(P + m * N + nl, pp);
        st_vec<NPL>(Q + m * N + nl, lam);
        if (D) {
#pragma unroll
            for (int i = 0; i < NPL; i++) D[m * N + nl + i] = dn[i];
        }
    }
    if constexpr (PG) {
        // one chunk holding row 0: lam is lam_0 and u_{-1} = u0
        if (ok && act) {
            const Vec<NPL> z = ld_vec<NPL>(u0 + nl);
#pragma unroll
            for (int i = 0; i < NPL; i++) {
                pb[i] = fma((double)lam.v[i], (double)z.v[i], pb[i]);
                PGout[nl + i] = pb[i];
                PGout[N + nl + i] = pgm[i];
                PGout[2 * N + nl + i] = pdl[i];
            }
        }
    }
    if (MODE == kReplay && lane == 0) bulk_wait_all();
}

// ================================================================= host side
// Tile rows R and ring depth S per lane width (build-time tunables, chosen by
// a sweep on B200: longer tiles amortise the per-tile barrier/TMA work for
// one-neuron lanes; float4 lanes move 4x the bytes per tile already).
#ifndef LIFB_FWD1_R
#define LIFB_FWD1_R 32
#endif
#ifndef LIFB_FWD1_S
#define LIFB_FWD1_S 4
#endif
#ifndef LIFB_FWD4_R
#define LIFB_FWD4_R 16
#endif
#ifndef LIFB_FWD4_S
#define LIFB_FWD4_S 6
#endif
#ifndef LIFB_BWD1_R
#define LIFB_BWD1_R 16
#endif
#ifndef LIFB_BWD1_S
#define LIFB_BWD1_S 4
#endif
#ifndef LIFB_BWD4_R
#define LIFB_BWD4_R 8
#endif
#ifndef LIFB_BWD4_S
#define LIFB_BWD4_S 6
#endif
// float4 lanes once there are at least this many 128-neuron CTAs per SM
#ifndef LIFB_FWD_NPL4_MIN_CTAS_PER_SM
#define LIFB_FWD_NPL4_MIN_CTAS_PER_SM 2
#endif
#ifndef LIFB_BWD_NPL4_MIN_CTAS_PER_SM
#define LIFB_BWD_NPL4_MIN_CTAS_PER_SM 1000000
#endif
#ifndef LIFB_FORCE_NPL
#define LIFB_FORCE_NPL 0
#endif
// Single-chunk forward with one neuron per lane (the streaming pass over a
// whole sequence): a deeper ring, measured 32.8 us against 34.8 us for the
// V-saving forward at T = 1024, N = 16384.
#ifndef LIFB_FWD1_DEEP_S
#define LIFB_FWD1_DEEP_S 8
#endif
// Adjoint from V (two input arrays, V and GS) with one neuron per lane:
// taller tiles keep twice the rows in flight; measured 36.9 us against 45.1 us
// at T = 1024, N = 16384 (the three-array layouts are slower with them).
#ifndef LIFB_BWDV1_R
#define LIFB_BWDV1_R 32
#endif
#ifndef LIFB_BWDV1_S
#define LIFB_BWDV1_S 4
#endif
template <int NPL, bool DEEP = false>
struct FwdTile {
    static constexpr int R = NPL == 4 ? LIFB_FWD4_R : LIFB_FWD1_R;
    static constexpr int S = NPL == 4 ? LIFB_FWD4_S : (DEEP ? LIFB_FWD1_DEEP_S : LIFB_FWD1_S);
};
template <int NPL, bool FROM_V = false>
struct BwdTile {
    static constexpr int R = NPL == 4 ? LIFB_BWD4_R : (FROM_V ? LIFB_BWDV1_R : LIFB_BWD1_R);
    static constexpr int S = NPL == 4 ? LIFB_BWD4_S : (FROM_V ? LIFB_BWDV1_S : LIFB_BWD1_S);
};
static int bwd_rows(int npl, bool from_v)
{
    if (npl == 4) return from_v ? BwdTile<4, true>::R : BwdTile<4>::R;
    return from_v ? BwdTile<1, true>::R : BwdTile<1>::R;
}

bool tma_ok(const void *const *ptrs, int n, int64_t N)
{
    if (N % 4) return false;
    for (int i = 0; i < n; i++)
        if (ptrs[i] && ((uintptr_t)ptrs[i] & 15)) return false;
    return true;
}

// float4 lanes when there are enough 128-neuron CTAs per SM; otherwise one
// neuron per lane (4x more warps for narrow problems).
int pick_npl(int64_t N, int64_t M, int min_ctas_per_sm)
{
    if (LIFB_FORCE_NPL == 1 || LIFB_FORCE_NPL == 4) return LIFB_FORCE_NPL;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return ((N + 127) / 128) * M >= (int64_t)min_ctas_per_sm * sms ? 4 : 1;
}

template <int NPL, bool VOUT, bool AFF, bool DEEP>
static void launch_fwd(const CUtensorMap *maps, const float *u0, const float *Starts, int64_t start_stride, float *U,
                       float *S, float *Ends, int64_t N, int64_t M, int64_t C, float beta, float theta, float u_r,
                       int64_t lead, float *LeadStarts, float gamma, float delta, int *status, cudaStream_t s,
                       int64_t m0)
{
    constexpr int NB = 32 * NPL;
    constexpr int R = FwdTile<NPL, DEEP>::R, ST = FwdTile<NPL, DEEP>::S;
    const size_t smem = (size_t)(ST + 4) * R * NB * 4;
    auto kern = k_fwd_tma<NPL, R, ST, VOUT, AFF>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 g((unsigned)((N + NB - 1) / NB), (unsigned)(M - m0));
    count_launches(1);
    kern<<<g, 32, smem, s>>>(maps[0], maps[1], maps[2], u0, Starts, start_stride, U, S, Ends, N, C, beta, theta, u_r,
                             lead, LeadStarts, gamma, delta, status, m0);
}

bool fwd_replay_tma(const float *I, const float *u0, const float *Starts, float *U, float *S, float *Ends,
                    int64_t T, int64_t N, int64_t C, float beta, float theta, float u_r, cudaStream_t s,
                    int64_t start_stride, int64_t lead, float *LeadStarts, bool vout, Reset rs, int64_t first_chunk)
{
    const bool aff = rs.aff;
    const float gamma = rs.gamma, delta = rs.delta;
    const void *p[] = {I, u0, Starts, U, S, Ends, LeadStarts};
    if (!tma_ok(p, 7, N) || C <= 0 || T % C) return false;
    const int64_t M = T / C;
    if (M > 65535 || first_chunk < 0 || first_chunk >= M) return false;
    const int npl = pick_npl(N, M - first_chunk, LIFB_FWD_NPL4_MIN_CTAS_PER_SM);
    const int R = npl == 4 ? FwdTile<4>::R : FwdTile<1>::R;
    if (lead > 0) {  // lead-in tiles: whole tiles inside whole chunks
        if (C % R) return false;
        lead = (lead + R - 1) / R * R;
    }
    CUtensorMap maps[3];
    if (!make_tmap_2d(&maps[0], I, N, T, 32 * npl, R) || !make_tmap_2d(&maps[1], U, N, T, 32 * npl, R) ||
        !make_tmap_2d(&maps[2], S, N, T, 32 * npl, R))
        return false;
    int *status = device_status_ptr();
    // one chunk, one neuron per lane: the deeper ring
    const bool deep = npl == 1 && M == 1 && lead == 0 && first_chunk == 0;
    auto go = [&](auto npl_c, auto vout_c, auto aff_c) {
        constexpr int kNpl = decltype(npl_c)::value;
        constexpr bool kV = decltype(vout_c)::value, kA = decltype(aff_c)::value;
        if (kNpl == 1 && deep)
            launch_fwd<kNpl, kV, kA, true>(maps, u0, Starts, start_stride, U, S, Ends, N, M, C, beta, theta, u_r,
                                           lead, LeadStarts, gamma, delta, status, s, first_chunk);
        else
            launch_fwd<kNpl, kV, kA, false>(maps, u0, Starts, start_stride, U, S, Ends, N, M, C, beta, theta, u_r,
                                            lead, LeadStarts, gamma, delta, status, s, first_chunk);
    };
    using I1 = std::integral_constant<int, 1>;
    using I4 = std::integral_constant<int, 4>;
    using BT = std::true_type;
    using BF = std::false_type;
    auto go2 = [&](auto npl_c, auto vout_c) { aff ? go(npl_c, vout_c, BT{}) : go(npl_c, vout_c, BF{}); };
    if (npl == 4) vout ? go2(I4{}, BT{}) : go2(I4{}, BF{});
    else vout ? go2(I1{}, BT{}) : go2(I1{}, BF{});
    return true;
}

template <int NPL, bool READ_S, bool HAS_GU, int MODE, bool TRACK, bool FROM_V = false, bool AFF = false,
          bool PG = false>
static void launch_bwd(const CUtensorMap *maps, const float *u0, const float *LamEnd, float *Lam, float *P, float *Q,
                       int32_t *D, int64_t N, int64_t M, int64_t C, float beta, float theta, float u_r, float alpha,
                       bool detach, int *status, cudaStream_t s, float gamma = 0.0f, float delta = 0.0f,
                       double *PGout = nullptr)
{
    constexpr int NB = 32 * NPL;
    constexpr int NT = BwdLayout<READ_S, HAS_GU, FROM_V>::NT;
    constexpr int R = BwdTile<NPL, FROM_V>::R, ST = BwdTile<NPL, FROM_V>::S;
    const size_t smem = ((size_t)ST * NT + (MODE == kReplay ? 2 : 0)) * R * NB * 4;
    auto kern = k_bwd_tma<NPL, R, ST, READ_S, HAS_GU, MODE, TRACK, FROM_V, AFF, PG>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 g((unsigned)((N + NB - 1) / NB), (unsigned)M);
    count_launches(1);
    kern<<<g, 32, smem, s>>>(maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], u0, LamEnd, Lam, P, Q, D, N, C,
                             beta, theta, u_r, alpha, detach, gamma, delta, PGout, status);
}

template <int NPL, int MODE, bool TRACK>
static void launch_bwd_v(bool read_s, bool has_gu, const CUtensorMap *maps, const float *u0, const float *LamEnd,
                         float *Lam, float *P, float *Q, int32_t *D, int64_t N, int64_t M, int64_t C, float beta,
                         float theta, float u_r, float alpha, bool detach, int *status, cudaStream_t s)
{
    if (read_s) {
        if (has_gu) launch_bwd<NPL, true, true, MODE, TRACK>(maps, u0, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, u_r, alpha, detach, status, s);
        else launch_bwd<NPL, true, false, MODE, TRACK>(maps, u0, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, u_r, alpha, detach, status, s);
    } else {
        if (has_gu) launch_bwd<NPL, false, true, MODE, TRACK>(maps, u0, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, u_r, alpha, detach, status, s);
        else launch_bwd<NPL, false, false, MODE, TRACK>(maps, u0, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, u_r, alpha, detach, status, s);
    }
}

// Adjoint from V (the forward's pre-reset potentials), GS: detached reset,
// S recomputed as [v >= theta], no GU.  Same outputs as bwd_tma mode 0.
bool bwd_tma_v(const float *V, const float *GS, float *Lam, float *P, float *Q, int32_t *D, int64_t T, int64_t N,
               int64_t C, float beta, float theta, float alpha, cudaStream_t s, const float *LamEnd)
{
    const void *p[] = {V, GS, Lam, P, Q, D, LamEnd};
    if (!tma_ok(p, 7, N) || C <= 0 || T % C) return false;
    const int64_t M = T / C;
    if (M > 65535) return false;
    const int npl = pick_npl(N, M, LIFB_BWD_NPL4_MIN_CTAS_PER_SM);
    const int nb = 32 * npl;
    const int R = bwd_rows(npl, true);
    CUtensorMap maps[6];
    if (!make_tmap_2d(&maps[0], V, N, T, nb, R) || !make_tmap_2d(&maps[3], GS, N, T, nb, R) ||
        !make_tmap_2d(&maps[5], Lam, N, T, nb, R))
        return false;
    maps[1] = maps[2] = maps[4] = maps[0];
    int *status = device_status_ptr();
    if (P) {
        if (npl == 4) launch_bwd<4, false, false, kReplay, true, true>(maps, nullptr, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, 0.f, alpha, true, status, s);
        else launch_bwd<1, false, false, kReplay, true, true>(maps, nullptr, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, 0.f, alpha, true, status, s);
    } else {
        if (npl == 4) launch_bwd<4, false, false, kReplay, false, true>(maps, nullptr, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, 0.f, alpha, true, status, s);
        else launch_bwd<1, false, false, kReplay, false, true>(maps, nullptr, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, 0.f, alpha, true, status, s);
    }
    return true;
}

// Affine-reset adjoint over one chunk of T rows (detached reset): lam_t =
// gs_t sigma'(v_t) + a_t lam_{t+1}, a_t = beta*gamma at a spike, beta elsewhere
// (gamma = 1: the soft reset); v_t from U[t-1] and I[t] (from_v: V given).
bool bwd_tma_aff(const float *IV, const float *u0, const float *U, const float *GS, float *Lam, int64_t T, int64_t N,
                 float beta, float theta, float alpha, float gamma, bool from_v, cudaStream_t s)
{
    const void *p[] = {IV, u0, U, GS, Lam};
    if (!tma_ok(p, 5, N) || T <= 0) return false;
    const int npl = pick_npl(N, 1, LIFB_BWD_NPL4_MIN_CTAS_PER_SM);
    const int nb = 32 * npl;
    const int R = bwd_rows(npl, from_v);
    CUtensorMap maps[6];
    if (!make_tmap_2d(&maps[0], IV, N, T, nb, R) || !make_tmap_2d(&maps[3], GS, N, T, nb, R) ||
        !make_tmap_2d(&maps[5], Lam, N, T, nb, R))
        return false;
    if (from_v) {
        maps[1] = maps[0];
    } else if (!make_tmap_2d(&maps[1], U, N, T, nb, R)) {
        return false;
    }
    maps[2] = maps[4] = maps[0];
    int *status = device_status_ptr();
    if (from_v) {
        if (npl == 4) launch_bwd<4, false, false, kReplay, false, true, true>(maps, nullptr, nullptr, Lam, nullptr, nullptr, nullptr, N, 1, T, beta, theta, 0.f, alpha, true, status, s, gamma);
        else launch_bwd<1, false, false, kReplay, false, true, true>(maps, nullptr, nullptr, Lam, nullptr, nullptr, nullptr, N, 1, T, beta, theta, 0.f, alpha, true, status, s, gamma);
    } else {
        if (npl == 4) launch_bwd<4, false, false, kReplay, false, false, true>(maps, u0, nullptr, Lam, nullptr, nullptr, nullptr, N, 1, T, beta, theta, 0.f, alpha, true, status, s, gamma);
        else launch_bwd<1, false, false, kReplay, false, false, true>(maps, u0, nullptr, Lam, nullptr, nullptr, nullptr, N, 1, T, beta, theta, 0.f, alpha, true, status, s, gamma);
    }
    return true;
}

// Affine-reset adjoint from V over one chunk of T rows with the parameter
// sums fused in: PGout[3][N] (fp64) receives per neuron (dbeta, dgamma,
// ddelta); u0 [N] supplies the u_{-1} of the dbeta sum.
bool bwd_tma_aff_pg(const float *V, const float *u0, const float *GS, float *Lam, double *PGout, int64_t T, int64_t N,
                    float beta, float theta, float alpha, float gamma, float delta, cudaStream_t s)
{
    const void *p[] = {V, u0, GS, Lam};
    if (!tma_ok(p, 4, N) || T <= 0 || (uintptr_t)PGout % 8) return false;
    const int npl = pick_npl(N, 1, LIFB_BWD_NPL4_MIN_CTAS_PER_SM);
    const int nb = 32 * npl;
    const int R = bwd_rows(npl, true);
    CUtensorMap maps[6];
    if (!make_tmap_2d(&maps[0], V, N, T, nb, R) || !make_tmap_2d(&maps[3], GS, N, T, nb, R) ||
        !make_tmap_2d(&maps[5], Lam, N, T, nb, R))
        return false;
    maps[1] = maps[2] = maps[4] = maps[0];
    int *status = device_status_ptr();
    if (npl == 4)
        launch_bwd<4, false, false, kReplay, false, true, true, true>(maps, u0, nullptr, Lam, nullptr, nullptr, nullptr,
                                                                      N, 1, T, beta, theta, 0.f, alpha, true, status, s,
                                                                      gamma, delta, PGout);
    else
        launch_bwd<1, false, false, kReplay, false, true, true, true>(maps, u0, nullptr, Lam, nullptr, nullptr, nullptr,
                                                                      N, 1, T, beta, theta, 0.f, alpha, true, status, s,
                                                                      gamma, delta, PGout);
    return true;
}

bool bwd_tma(int mode, const float *I, const float *u0, const float *U, const float *S, const float *GS,
             const float *GU, const float *LamEnd, float *Lam, float *P, float *Q, int64_t T, int64_t N, int64_t C,
             float beta, float theta, float u_r, float alpha, bool detach, cudaStream_t s, int32_t *D)
{
    const void *p[] = {I, u0, U, S, GS, GU, LamEnd, Lam, P, Q};
    if (!tma_ok(p, 10, N) || C <= 0 || T % C) return false;
    const int64_t M = T / C;
    if (M > 65535) return false;
    const int npl = pick_npl(N, M, LIFB_BWD_NPL4_MIN_CTAS_PER_SM);
    const int nb = 32 * npl;
    const int R = bwd_rows(npl, false);
    // maps: I, U, S, GS, GU, Lam (unused slots repeat a valid map)
    CUtensorMap maps[6];
    if (!make_tmap_2d(&maps[0], I, N, T, nb, R) || !make_tmap_2d(&maps[1], U, N, T, nb, R) ||
        !make_tmap_2d(&maps[3], GS, N, T, nb, R))
        return false;
    maps[2] = maps[0];
    maps[4] = maps[0];
    maps[5] = maps[0];
    if (S && !make_tmap_2d(&maps[2], S, N, T, nb, R)) return false;
    if (GU && !make_tmap_2d(&maps[4], GU, N, T, nb, R)) return false;
    if (mode == kReplay && !make_tmap_2d(&maps[5], Lam, N, T, nb, R)) return false;
    int *status = device_status_ptr();
    const bool rs = S != nullptr, g = GU != nullptr;
    if (mode == kReplay && P) {
        if (npl == 4) launch_bwd_v<4, kReplay, true>(rs, g, maps, u0, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, u_r, alpha, detach, status, s);
        else launch_bwd_v<1, kReplay, true>(rs, g, maps, u0, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, u_r, alpha, detach, status, s);
    } else if (mode == kReplay) {
        if (npl == 4) launch_bwd_v<4, kReplay, false>(rs, g, maps, u0, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, u_r, alpha, detach, status, s);
        else launch_bwd_v<1, kReplay, false>(rs, g, maps, u0, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, u_r, alpha, detach, status, s);
    } else {
        if (npl == 4) launch_bwd_v<4, kCompose, true>(rs, g, maps, u0, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, u_r, alpha, detach, status, s);
        else launch_bwd_v<1, kCompose, true>(rs, g, maps, u0, LamEnd, Lam, P, Q, D, N, M, C, beta, theta, u_r, alpha, detach, status, s);
    }
    return true;
}

}  // namespace lifb
