// Fix-up passes that make segment-parallel replays exact.
//
// Forward (k_fwd_fixup_par + k_fwd_fixup_seq).  The replay kernel runs every segment of L rows from
// the start the map carry gave it; a carried start can be off by a few ulps
// (the affine piece A*u+B is not rounded like L separate steps) or, near a
// breakpoint, select a neighbouring piece.  Hard resets resynchronise
// trajectories: once the replay from the exact start produces the same
// (u_t, s_t) as the stored one, every later row is identical.  So, per
// neuron and in time order, each segment whose stored start differs (bit for
// bit) from the exact end of the previous segment is replayed from that end
// only until it resynchronises; a segment that never does gets a new end,
// which is then checked against the next segment.  This is the reference's
// repair loop (lifscan/triton_lif.py:805-811) done once, in Gauss-Seidel order,
// touching only the rows that change.
//
// Adjoint (k_bwd_fixup, detached reset).  lam_t = c_t + a_t lam_{t+1} with
// a_t = beta*(1 - s_t) = 0 exactly at a spike, so rows at and below the last
// spike of a chunk do not depend on the lam that enters the chunk from above.
// The replay pass ran every chunk from lam_end = 0 and recorded its chunk map
// (P = prod a, Q = lam at its first row).  The true lam_end of chunk m is Q of
// the next chunk that contains a spike, carried back through the spike-free
// chunks in between with their (P, Q); only the rows above chunk m's last
// spike are then recomputed.  (bwd_carry_kernel lifscan/triton_lif.py:197-208
// is the general form of this carry.)
#include "lifb_common.cuh"
#include "lifb_internal.h"
#include "tma.cuh"

namespace lifb {

constexpr int kFixBlock = 128;

__device__ __forceinline__ bool same_bits(float a, float b) { return __float_as_uint(a) == __float_as_uint(b); }

// Replays rows [r0, r0 + L) of one neuron per lane from u (active lanes
// only) with coalesced batched loads, comparing (u, s) with the stored rows:
// a lane stops at the first row that matches (everything after it is already
// right) and otherwise rewrites the row.  Returns true for lanes that
// resynchronised; u then holds the state of the matching row.
template <int kB>
__device__ __forceinline__ bool replay_until_sync(const float *__restrict__ I, float *__restrict__ U,
                                                  float *__restrict__ S, int64_t N, int64_t n, bool act, int64_t r0,
                                                  int64_t L, float &u, bool active, float beta, float theta,
                                                  float u_r, Reset rs = {})
{
    const unsigned full = 0xffffffffu;
    bool synced = !active;
    if (!__any_sync(full, active)) return synced;
    // rows of batch b are loaded while batch b - kB is replayed
    float x[kB], uo[kB], so[kB];
#pragma unroll
    for (int q = 0; q < kB; q++) {
        if (act && q < L) {
            const int64_t o = (r0 + q) * N + n;
            x[q] = __ldg(I + o);
            uo[q] = U[o];
            so[q] = S[o];
        }
    }
    for (int64_t b = 0; b < L; b += kB) {
        if (!__any_sync(full, active)) break;
        float xn[kB], un_[kB], sn[kB];
#pragma unroll
        for (int q = 0; q < kB; q++) {
            if (act && b + kB + q < L) {
                const int64_t o = (r0 + b + kB + q) * N + n;
                xn[q] = __ldg(I + o);
                un_[q] = U[o];
                sn[q] = S[o];
            }
        }
#pragma unroll
        for (int q = 0; q < kB; q++) {
            if (active && b + q < L) {
                bool f;
                const float un = step_any(u, x[q], beta, theta, u_r, rs.aff, rs.gamma, rs.delta, f);
                const float fs = f ? 1.0f : 0.0f;
                u = un;
                if (same_bits(un, uo[q]) && fs == so[q]) {
                    active = false;  // identical from here on
                    synced = true;
                } else {
                    const int64_t o = (r0 + b + q) * N + n;
                    U[o] = un;
                    S[o] = fs;
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kB; q++) {
            x[q] = xn[q];
            uo[q] = un_[q];
            so[q] = sn[q];
        }
    }
    return synced;
}

// Parallel pass over segment boundaries (blockIdx.y = segment sg >= 1):
// assumes the replay's end of segment sg-1 is exact and fixes segment sg from
// it.  Segments whose rows never resynchronise get a new end (EndsNew) and a
// flag; the sequential pass below redoes whatever followed them.
__global__ void __launch_bounds__(kFixBlock) k_fwd_fixup_par(const float *__restrict__ I,
                                                             const float *__restrict__ Starts, int64_t start_stride,
                                                             float *__restrict__ U, float *__restrict__ S,
                                                             const float *__restrict__ Ends, float *__restrict__ EndsNew,
                                                             int32_t *__restrict__ Changed, int64_t N, int64_t L,
                                                             float beta, float theta, float u_r, Reset rs)
{
    const int64_t n = (int64_t)blockIdx.x * kFixBlock + threadIdx.x;
    const int64_t sg = (int64_t)blockIdx.y + 1;
    const bool act = n < N;
    const float prev = act ? Ends[(sg - 1) * N + n] : 0.0f;
    const float st = act ? Starts[sg * start_stride * N + n] : 0.0f;
    const bool need = act && !same_bits(prev, st);
    if (!__any_sync(0xffffffffu, need)) {
        if (act) Changed[sg * N + n] = 0;
        return;
    }
    float u = prev;
    const bool synced = replay_until_sync<16>(I, U, S, N, n, act, sg * L, L, u, need, beta, theta, u_r, rs);
    if (act) {
        Changed[sg * N + n] = synced ? 0 : 1;
        if (!synced) EndsNew[sg * N + n] = u;
    }
}

// Sequential pass per neuron: a segment whose fix did not resynchronise has a
// new end, so the segment after it is redone from that end (and so on).
__global__ void __launch_bounds__(kFixBlock) k_fwd_fixup_seq(const float *__restrict__ I, float *__restrict__ U,
                                                             float *__restrict__ S, float *__restrict__ Ends,
                                                             const float *__restrict__ EndsNew,
                                                             const int32_t *__restrict__ Changed, int64_t N,
                                                             int64_t NS, int64_t L, float beta, float theta, float u_r,
                                                             int *__restrict__ longest_chain, Reset rs)
{
    const int64_t n = (int64_t)blockIdx.x * kFixBlock + threadIdx.x;
    const bool act = n < N;
    // nothing to carry unless some lane has a segment whose fix did not
    // resynchronise: check all flags first (independent loads)
    bool any_ch = false;
    for (int64_t s0 = 1; s0 < NS && !__any_sync(0xffffffffu, any_ch); s0 += 16) {
#pragma unroll
        for (int q = 0; q < 16; q++)
            if (act && s0 + q < NS) any_ch |= Changed[(s0 + q) * N + n] != 0;
    }
    if (!__any_sync(0xffffffffu, any_ch)) return;
    bool carry = false;  // the previous segment's end differs from the replay's
    float end = 0.0f;
    int run = 0, longest = 0;
    for (int64_t sg = 1; sg < NS; sg++) {
        // end of the rows currently stored for segment sg: the parallel pass's
        // new end if its fix never resynchronised, else the replay's end
        bool ch = act && Changed[sg * N + n] != 0;
        float e = ch ? EndsNew[sg * N + n] : (act ? Ends[sg * N + n] : 0.0f);
        if (__any_sync(0xffffffffu, carry)) {
            // redo segment sg from the previous segment's new end
            float u = end;
            const bool synced = replay_until_sync<16>(I, U, S, N, n, act, sg * L, L, u, carry, beta, theta, u_r,
                                                      rs);
            if (carry && !synced) {  // synced lanes rejoined the stored rows: (ch, e) stand
                ch = true;
                e = u;
            }
        }
        if (ch && act) Ends[sg * N + n] = e;
        run = ch ? run + 1 : 0;
        longest = run > longest ? run : longest;
        carry = ch;
        end = e;
    }
    if (longest_chain && act && longest) atomicMax(longest_chain, longest);
}

// Cross-slice repair: rows [0, T) were replayed (and fixed) from an entry
// state that may differ from the exact one; replay from the exact entry until
// (u, s) rejoins the stored rows.  Neurons that never rejoin get a new end.
__global__ void __launch_bounds__(kFixBlock) k_entry_repair(const float *__restrict__ I,
                                                            const float *__restrict__ entry, float *__restrict__ U,
                                                            float *__restrict__ S, float *__restrict__ end,
                                                            int32_t *__restrict__ changed, int64_t T, int64_t N,
                                                            float beta, float theta, float u_r)
{
    const int64_t n = (int64_t)blockIdx.x * kFixBlock + threadIdx.x;
    const bool act = n < N;
    float u = act ? entry[n] : 0.0f;
    // the stored rows started from the state before row 0, which the caller
    // compares: every active lane is assumed to differ
    const bool synced = replay_until_sync<16>(I, U, S, N, n, act, 0, T, u, act, beta, theta, u_r);
    if (act) {
        changed[n] = synced ? 0 : 1;
        if (!synced) end[n] = u;
    }
}

void entry_repair(const float *I, const float *entry, float *U, float *S, float *end, int32_t *changed, int64_t T,
                  int64_t N, float beta, float theta, float u_r, cudaStream_t s)
{
    count_launches(1);
    k_entry_repair<<<(unsigned)((N + kFixBlock - 1) / kFixBlock), kFixBlock, 0, s>>>(I, entry, U, S, end, changed, T,
                                                                                      N, beta, theta, u_r);
}

// Adjoint coefficients with the same arithmetic as k_bwd_tma (bwd_coef).
__device__ __forceinline__ void coef_fix(float up, float s, float x, float gs, float gu, float beta, float theta,
                                         float alpha, float &a, float &c)
{
    const float v = __fadd_rn(__fmul_rn(beta, up), x);
    if (s < 0.0f) s = v >= theta ? 1.0f : 0.0f;
    const float e = ex2_approx(alpha * 1.4426950408889634f * (theta - v));  // exp(-alpha (v - theta))
    const float sig = rcp_approx(1.0f + e);
    const float sg = alpha * sig * (1.0f - sig);
    const float J = 1.0f - s;
    a = beta * J;
    c = gs * sg + J * gu;
}

// lam_top (nullable): lam entering the last chunk from above (0 when NULL).
__global__ void __launch_bounds__(kFixBlock) k_bwd_fixup(const float *__restrict__ I, const float *__restrict__ u0,
                                                         const float *__restrict__ U, const float *__restrict__ S,
                                                         const float *__restrict__ GS, const float *__restrict__ GU,
                                                         const float *__restrict__ P, const float *__restrict__ Q,
                                                         const int32_t *__restrict__ D,
                                                         const float *__restrict__ lam_top, float *__restrict__ Lam,
                                                         int64_t N, int64_t M, int64_t C, float beta, float theta,
                                                         float alpha)
{
    const int64_t n = (int64_t)blockIdx.x * kFixBlock + threadIdx.x;
    const int64_t m = blockIdx.y;
    if (n >= N) return;
    const float top = lam_top ? lam_top[n] : 0.0f;
    float lam;
    if (m + 1 >= M) {
        lam = top;  // the last chunk: lam_end is the lam entering from above
    } else {
        // first chunk e > m whose first-row lam is exact: it holds a spike
        // (P = 0), or it is the last chunk (exact from `top`)
        int64_t e = m + 1;
        while (e + 1 < M && P[e * N + n] != 0.0f) e++;
        lam = Q[e * N + n];
        if (e + 1 == M && top != 0.0f) lam = lam + P[e * N + n] * top;
        for (int64_t i = e - 1; i > m; i--) lam = Q[i * N + n] + P[i * N + n] * lam;
    }
    if (lam == 0.0f) return;  // the replay's lam_end = 0 was already right
    if (D) {
        // rows above the chunk's last spike: a = beta exactly, so the replay's
        // rows differ from the exact ones by lam_end * beta^k (k = 1 at the
        // chunk's last row); rows at and below the spike are already exact
        const int64_t d = D[m * N + n];
        constexpr int kB = 16;
        float f = lam;
        for (int64_t k0 = 0; k0 < d && f != 0.0f; k0 += kB) {
            float l[kB];
#pragma unroll
            for (int q = 0; q < kB; q++)
                if (k0 + q < d) l[q] = Lam[((m + 1) * C - 1 - k0 - q) * N + n];
#pragma unroll
            for (int q = 0; q < kB; q++) {
                if (k0 + q < d) {
                    f = beta * f;
                    Lam[((m + 1) * C - 1 - k0 - q) * N + n] = l[q] + f;
                }
            }
        }
        return;
    }
    const float un0 = u0[n];
    constexpr int kB = 8;  // rows loaded ahead of the dependent chain
    bool running = true;
    for (int64_t t0 = (m + 1) * C - 1; t0 >= m * C && running; t0 -= kB) {
        float up[kB], sv[kB], x[kB], gs[kB], gu[kB];
#pragma unroll
        for (int q = 0; q < kB; q++) {
            const int64_t t = t0 - q;
            if (t >= m * C) {
                const int64_t o = t * N + n;
                up[q] = t > 0 ? U[o - N] : un0;
                sv[q] = S ? S[o] : -1.0f;
                x[q] = I[o];
                gs[q] = GS[o];
                gu[q] = GU ? GU[o] : 0.0f;
            }
        }
#pragma unroll
        for (int q = 0; q < kB; q++) {
            const int64_t t = t0 - q;
            if (running && t >= m * C) {
                float a, c;
                coef_fix(up[q], sv[q], x[q], gs[q], gu[q], beta, theta, alpha, a, c);
                lam = c + a * lam;
                Lam[t * N + n] = lam;
                if (a == 0.0f) running = false;  // spike row: every row below is already exact
            }
        }
    }
}

void fwd_fixup(const float *I, const float *Starts, int64_t start_stride, float *U, float *S, float *Ends,
               float *EndsNew, int32_t *Changed, int64_t N, int64_t NS, int64_t L, float beta, float theta, float u_r,
               int *longest_chain, cudaStream_t s, Reset rs)
{
    if (NS < 2) return;
    const unsigned nb = (unsigned)((N + kFixBlock - 1) / kFixBlock);
    count_launches(2);
    k_fwd_fixup_par<<<dim3(nb, (unsigned)(NS - 1)), kFixBlock, 0, s>>>(I, Starts, start_stride, U, S, Ends, EndsNew,
                                                                       Changed, N, L, beta, theta, u_r, rs);
    k_fwd_fixup_seq<<<nb, kFixBlock, 0, s>>>(I, U, S, Ends, EndsNew, Changed, N, NS, L, beta, theta, u_r,
                                             longest_chain, rs);
}

void bwd_fixup(const float *I, const float *u0, const float *U, const float *S, const float *GS, const float *GU,
               const float *P, const float *Q, const int32_t *D, float *Lam, int64_t N, int64_t M, int64_t C,
               float beta, float theta, float alpha, cudaStream_t s)
{
    if (M < 2) return;
    count_launches(1);
    dim3 g((unsigned)((N + kFixBlock - 1) / kFixBlock), (unsigned)(M - 1));
    k_bwd_fixup<<<g, kFixBlock, 0, s>>>(I, u0, U, S, GS, GU, P, Q, D, nullptr, Lam, N, M, C, beta, theta, alpha);
}

void bwd_fixup_top(const float *I, const float *u0, const float *U, const float *S, const float *GS, const float *GU,
                   const float *P, const float *Q, const int32_t *D, const float *lam_top, float *Lam, int64_t N,
                   int64_t M, int64_t C, float beta, float theta, float alpha, cudaStream_t s)
{
    count_launches(1);
    dim3 g((unsigned)((N + kFixBlock - 1) / kFixBlock), (unsigned)M);
    k_bwd_fixup<<<g, kFixBlock, 0, s>>>(I, u0, U, S, GS, GU, P, Q, D, lam_top, Lam, N, M, C, beta, theta, alpha);
}

}  // namespace lifb
