// Grid-level exact scan forward (any T, any N): the two-level (v3) and
// three-level (v4) schedules as a sequence of kernels over [M, N] map arrays.
//
// Phases and the reference code each one follows (lifscan/triton_lif.py):
//   k_env_chunk    envelope map of every chunk            env_chunk_kernel   :698-719
//   k_env_carry    envelope prefix -> Lo[m]               env_carry_kernel   :722-733
//   k_build<KM>    pruned capacity-K chunk map            build3_kernel      :736-779
//   k_carry        maps evaluated in order -> Starts      carry2_kernel      :578-606
//   k_compose<KM2> G chunk maps -> super map (v4)         compose_group      :828-899
//   k_carry_inner  supers' chunk starts (v4)              carry_inner_kernel :902-932
//   k_replay       replay chunks -> U, S, Ends            fwd_tiled_kernel   :353-379
//   k_repair       Jacobi repair until exact              host loop          :805-811
// Threads run along the neuron index (coalesced rows of [T, N]); the chunk
// index is blockIdx.y.  Map arithmetic rounds exactly like the CPU oracle, so
// maps, starts and stats equal the reference's; U and S equal the serial
// recurrence bit for bit after repair.
#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace lifb {

constexpr int kBlock = 128;

__device__ __forceinline__ void stats_add_maps(lifb_stats *st, int cnt, int ovf, bool act, bool super_level)
{
    if (st == nullptr) return;
    unsigned full = 0xffffffffu;
    unsigned c = act ? (unsigned)cnt : 0u;
    unsigned o = act ? (unsigned)ovf : 0u;
    unsigned a = act ? 1u : 0u;
    unsigned sc = __reduce_add_sync(full, c);
    unsigned so = __reduce_add_sync(full, o);
    unsigned sa = __reduce_add_sync(full, a);
    unsigned mc = __reduce_max_sync(full, c);
    if ((threadIdx.x & 31) == 0 && sa) {
        if (super_level) {
            atomicAdd((unsigned long long *)&st->sum_super_cnt, (unsigned long long)sc);
            atomicAdd((unsigned long long *)&st->n_super_overflow, (unsigned long long)so);
            atomicAdd((unsigned long long *)&st->n_super, (unsigned long long)sa);
            atomicMax(&st->max_super_cnt, (int)mc);
        } else {
            atomicAdd((unsigned long long *)&st->sum_cnt, (unsigned long long)sc);
            atomicAdd((unsigned long long *)&st->n_overflow, (unsigned long long)so);
            atomicAdd((unsigned long long *)&st->n_maps, (unsigned long long)sa);
            atomicMax(&st->max_cnt, (int)mc);
        }
    }
}

// ---------------------------------------------------------------- envelope
__global__ void __launch_bounds__(kBlock) k_env_chunk(const float *__restrict__ I, float *__restrict__ EC,
                                                      float *__restrict__ EA, float *__restrict__ EB,
                                                      int64_t N, int C, float beta, float u_r)
{
    int64_t n = (int64_t)blockIdx.x * kBlock + threadIdx.x;
    if (n >= N) return;
    int64_t m = blockIdx.y;
    const float *p = I + (m * C) * N + n;
    float c = kInf, a = 1.0f, b = 0.0f;
#pragma unroll 8
    for (int j = 0; j < C; j++) {
        float x = __ldg(p + (int64_t)j * N);
        float cc = mul_add_rn(beta, c, x);
        c = u_r < cc ? u_r : cc;
        a = __fmul_rn(beta, a);
        b = mul_add_rn(beta, b, x);
    }
    EC[m * N + n] = c;
    EA[m * N + n] = a;
    EB[m * N + n] = b;
}

__global__ void __launch_bounds__(kBlock) k_env_carry(const float *__restrict__ u0, const float *__restrict__ EC,
                                                      const float *__restrict__ EA, const float *__restrict__ EB,
                                                      float *__restrict__ Lo, int64_t N, int64_t M, float margin)
{
    int64_t n = (int64_t)blockIdx.x * kBlock + threadIdx.x;
    if (n >= N) return;
    float l = u0[n];
#pragma unroll 4
    for (int64_t m = 0; m < M; m++) {
        Lo[m * N + n] = __fsub_rn(l, __fmul_rn(margin, __fadd_rn(fabsf(l), 1.0f)));
        float c = EC[m * N + n], a = EA[m * N + n], b = EB[m * N + n];
        float lin = mul_add_rn(a, l, b);
        l = c < lin ? c : lin;
    }
}

// ---------------------------------------------------------------- chunk maps
// One (chunk, neuron) per thread; capacity K <= KM slots in registers.  Only
// the slots that are live in some lane of the warp are pushed each step.
template <int KM>
__global__ void __launch_bounds__(kBlock) k_build(const float *__restrict__ I, const float *__restrict__ Lo,
                                                  const float *__restrict__ u0, float *__restrict__ MA,
                                                  float *__restrict__ MB, float *__restrict__ MX,
                                                  float *__restrict__ MC, int32_t *__restrict__ MN,
                                                  int32_t *__restrict__ OVF, int64_t N, int C, int K, float beta,
                                                  float theta, float u_r, lifb_stats *st)
{
    int64_t n0 = (int64_t)blockIdx.x * kBlock + threadIdx.x;
    bool act = n0 < N;
    int64_t n = act ? n0 : N - 1;  // idle lanes mirror the last neuron, store nothing
    int64_t m = blockIdx.y;
    float lo = Lo[m * N + n];
    float hi = fmaxf(u0[n], fmaxf(theta, u_r));
    float A = 1.0f, B = 0.0f, xmin = kInf;
    int cnt = 0, ovf = 0;
    float xd[KM], cd[KM];
#pragma unroll
    for (int i = 0; i < KM; i++) { xd[i] = kInf; cd[i] = 0.0f; }
    const float *p = I + (m * C) * N + n;
    for (int j = 0; j < C; j++) {
        float x = __ldg(p + (int64_t)j * N);
        int cmax = (int)__reduce_max_sync(0xffffffffu, (unsigned)cnt);
#pragma unroll
        for (int i = 0; i < KM; i++) {
            if (i >= cmax) break;
            cd[i] = lif_step_u(cd[i], x, beta, theta, u_r);
        }
        if (xmin > lo) {
            float num = __fsub_rn(__fsub_rn(theta, x), __fmul_rn(beta, B));
            float den = __fmul_rn(beta, A);
            float z = den == 0.0f ? (num > 0.0f ? kInf : -kInf) : __fdiv_rn(num, den);
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
    if (act) {
        int64_t o = m * N + n;
        MA[o] = A; MB[o] = B; MN[o] = cnt; OVF[o] = ovf;
#pragma unroll
        for (int i = 0; i < KM; i++) {
            if (i < cnt) {
                MX[(m * K + i) * N + n] = xd[i];
                MC[(m * K + i) * N + n] = cd[i];
            }
        }
    }
    stats_add_maps(st, cnt, ovf, act, false);
}

// Map evaluation (lifscan/fast.py:242-251): breakpoints are strictly
// descending, so k = number of leading breakpoints above u.
__device__ __forceinline__ float eval_map_g(const float *__restrict__ MX, const float *__restrict__ MC, float A,
                                           float B, int cnt, int64_t m, int K, int64_t N, int64_t n, float u)
{
    int k = 0;
    while (k < cnt && MX[(m * K + k) * N + n] > u) k++;
    if (k == cnt) return mul_add_rn(A, u, B);
    return MC[(m * K + k) * N + n];
}

// Sequential carry over M maps (chunk or super level); L = rows per map for
// the serial overflow fallback (lifscan/triton_lif.py:600-605).
__global__ void __launch_bounds__(kBlock) k_carry(const float *__restrict__ I, const float *__restrict__ u0,
                                                  const float *__restrict__ MA, const float *__restrict__ MB,
                                                  const float *__restrict__ MX, const float *__restrict__ MC,
                                                  const int32_t *__restrict__ MN, const int32_t *__restrict__ OVF,
                                                  float *__restrict__ Starts, int64_t N, int64_t M, int64_t L, int K,
                                                  float beta, float theta, float u_r)
{
    int64_t n = (int64_t)blockIdx.x * kBlock + threadIdx.x;
    if (n >= N) return;
    float u = u0[n];
    for (int64_t m = 0; m < M; m++) {
        int64_t o = m * N + n;
        Starts[o] = u;
        if (m + 1 == M) break;  // the last map's value is never used
        float nu;
        if (OVF[o]) {
            float w = u;
            const float *p = I + (m * L) * N + n;
            for (int64_t j = 0; j < L; j++) w = lif_step_u(w, __ldg(p + j * N), beta, theta, u_r);
            nu = w;
        } else {
            nu = eval_map_g(MX, MC, MA[o], MB[o], MN[o], m, K, N, n, u);
        }
        u = nu;
    }
}

// ---------------------------------------------------------------- v4 compose
// H (capacity K2 <= KM2, registers) := chunk map s*G, then H := g o H for the
// next G-1 chunk maps g (read from global memory).
template <int KM2>
__global__ void __launch_bounds__(kBlock) k_compose(const float *__restrict__ MA, const float *__restrict__ MB,
                                                    const float *__restrict__ MX, const float *__restrict__ MC,
                                                    const int32_t *__restrict__ MN, const int32_t *__restrict__ OVF,
                                                    const float *__restrict__ Lo, const float *__restrict__ u0,
                                                    float *__restrict__ SA, float *__restrict__ SB,
                                                    float *__restrict__ SX, float *__restrict__ SC,
                                                    int32_t *__restrict__ SN, int32_t *__restrict__ SOVF,
                                                    int64_t N, int G, int K, int K2, float theta, float u_r,
                                                    lifb_stats *st, int64_t lo_stride)
{
    int64_t n0 = (int64_t)blockIdx.x * kBlock + threadIdx.x;
    bool act = n0 < N;
    int64_t n = act ? n0 : N - 1;
    int64_t s = blockIdx.y;
    int64_t m0 = s * G;
    float lo = Lo[m0 * lo_stride * N + n];
    float hi = fmaxf(u0[n], fmaxf(theta, u_r));
    float A = MA[m0 * N + n], B = MB[m0 * N + n];
    int nH = MN[m0 * N + n];
    int ovf = OVF[m0 * N + n];
    float xd[KM2], cd[KM2];
#pragma unroll
    for (int i = 0; i < KM2; i++) {
        bool live = i < nH;
        xd[i] = live ? MX[(m0 * K + i) * N + n] : kInf;
        cd[i] = live ? MC[(m0 * K + i) * N + n] : 0.0f;
    }
    // breakpoints are descending: the smallest live one is the last
    float xmin = kInf;
#pragma unroll
    for (int i = 0; i < KM2; i++)
        if (i < nH) xmin = xd[i];
    for (int jj = 1; jj < G; jj++) {
        int64_t m = m0 + jj;
        int64_t o = m * N + n;
        float Ag = MA[o], Bg = MB[o];
        int ng = MN[o];
        ovf |= OVF[o];
        const float *yd = MX + (m * K) * N + n;
        const float *dd = MC + (m * K) * N + n;
        // 1) push H's constants through g
#pragma unroll
        for (int i = 0; i < KM2; i++) {
            if (i < nH) {
                float c = cd[i];
                int k = 0;
                while (k < ng && yd[(int64_t)k * N] > c) k++;
                cd[i] = (k == ng) ? mul_add_rn(Ag, c, Bg) : dd[(int64_t)k * N];
            }
        }
        // 2) pull g's breakpoints back through H's affine part
        for (int j = 0; j < ng; j++) {
            float num = __fsub_rn(yd[(int64_t)j * N], B);
            float z = A == 0.0f ? (num > 0.0f ? kInf : -kInf) : __fdiv_rn(num, A);
            if (z < xmin && z <= hi && xmin > lo) {
                if (nH >= K2) {
                    ovf = 1;
                } else {
                    float dj = dd[(int64_t)j * N];
#pragma unroll
                    for (int i = 0; i < KM2; i++)
                        if (i == nH) { xd[i] = z; cd[i] = dj; }
                    nH++;
                    xmin = z;
                }
            }
        }
        // 3) affine part
        B = mul_add_rn(Ag, B, Bg);
        A = __fmul_rn(Ag, A);
    }
    if (act) {
        int64_t o = s * N + n;
        SA[o] = A; SB[o] = B; SN[o] = nH; SOVF[o] = ovf;
#pragma unroll
        for (int i = 0; i < KM2; i++) {
            if (i < nH) {
                SX[(s * K2 + i) * N + n] = xd[i];
                SC[(s * K2 + i) * N + n] = cd[i];
            }
        }
    }
    stats_add_maps(st, nH, ovf, act, true);
}

__global__ void __launch_bounds__(kBlock) k_carry_inner(const float *__restrict__ I, const float *__restrict__ SStarts,
                                                        const float *__restrict__ MA, const float *__restrict__ MB,
                                                        const float *__restrict__ MX, const float *__restrict__ MC,
                                                        const int32_t *__restrict__ MN,
                                                        const int32_t *__restrict__ OVF, float *__restrict__ Starts,
                                                        int64_t N, int64_t Mtot, int G, int C, int K, float beta,
                                                        float theta, float u_r)
{
    int64_t n = (int64_t)blockIdx.x * kBlock + threadIdx.x;
    if (n >= N) return;
    int64_t s = blockIdx.y;
    float u = SStarts[s * N + n];
    for (int jj = 0; jj < G; jj++) {
        int64_t m = s * G + jj;
        int64_t o = m * N + n;
        Starts[o] = u;
        if (m + 1 >= Mtot) break;  // the last chunk's map is never used
        float nu;
        if (OVF[o]) {
            float w = u;
            const float *p = I + (m * C) * N + n;
            for (int j = 0; j < C; j++) w = lif_step_u(w, __ldg(p + (int64_t)j * N), beta, theta, u_r);
            nu = w;
        } else {
            nu = eval_map_g(MX, MC, MA[o], MB[o], MN[o], m, K, N, n, u);
        }
        u = nu;
    }
}

// ---------------------------------------------------------------- replay
__global__ void __launch_bounds__(kBlock) k_replay(const float *__restrict__ I, const float *__restrict__ Starts,
                                                   float *__restrict__ U, float *__restrict__ S,
                                                   float *__restrict__ Ends, int64_t N, int C, float beta,
                                                   float theta, float u_r)
{
    int64_t n = (int64_t)blockIdx.x * kBlock + threadIdx.x;
    if (n >= N) return;
    int64_t m = blockIdx.y;
    float u = Starts[m * N + n];
    int64_t base = (m * C) * N + n;
#pragma unroll 8
    for (int j = 0; j < C; j++) {
        int64_t o = base + (int64_t)j * N;
        bool s;
        u = lif_step(u, __ldg(I + o), beta, theta, u_r, s);
        U[o] = u;
        S[o] = s ? 1.0f : 0.0f;
    }
    Ends[m * N + n] = u;
}

// Jacobi repair per neuron (neurons are independent, so the global round
// count is the maximum over neurons).  Round r: for m = M-1 .. 0 the new
// start is Ends[m-1] of round r-1 (or u0); a chunk whose start changed is
// replayed again.  Converges in at most M rounds for NaN-free input.
__global__ void __launch_bounds__(kBlock) k_repair(const float *__restrict__ I, const float *__restrict__ u0,
                                                   float *__restrict__ Starts, float *__restrict__ Ends,
                                                   float *__restrict__ U, float *__restrict__ S, int64_t N,
                                                   int64_t M, int C, int max_rounds, float beta, float theta,
                                                   float u_r, lifb_stats *st)
{
    int64_t n = (int64_t)blockIdx.x * kBlock + threadIdx.x;
    if (n >= N) return;
    int it = 0;
    for (int r = 1; r <= max_rounds; r++) {
        bool changed = false;
        for (int64_t m = M - 1; m >= 0; m--) {
            float ns = m > 0 ? Ends[(m - 1) * N + n] : u0[n];
            if (ns != Starts[m * N + n]) {
                Starts[m * N + n] = ns;
                float u = ns;
                int64_t base = (m * C) * N + n;
                for (int j = 0; j < C; j++) {
                    int64_t o = base + (int64_t)j * N;
                    bool s;
                    u = lif_step(u, __ldg(I + o), beta, theta, u_r, s);
                    U[o] = u;
                    S[o] = s ? 1.0f : 0.0f;
                }
                Ends[m * N + n] = u;
                changed = true;
            }
        }
        if (!changed) break;
        it = r;
    }
    if (st != nullptr && it > 0) atomicMax(&st->repair_iters, it);
}

// ---------------------------------------------------------------- launchers
template <int KM>
static void launch_build(dim3 g, cudaStream_t s, const float *I, const float *Lo, const float *u0, float *MA,
                         float *MB, float *MX, float *MC, int32_t *MN, int32_t *OVF, int64_t N, int C, int K,
                         float beta, float theta, float u_r, lifb_stats *st)
{
    count_launches(1);
    k_build<KM><<<g, kBlock, 0, s>>>(I, Lo, u0, MA, MB, MX, MC, MN, OVF, N, C, K, beta, theta, u_r, st);
}

template <int KM2>
static void launch_compose(dim3 g, cudaStream_t s, const FwdMaps &mp, const SuperMaps &sp, const float *u0,
                           int64_t N, int G, int K, int K2, float theta, float u_r, lifb_stats *st, int64_t lo_stride)
{
    count_launches(1);
    k_compose<KM2><<<g, kBlock, 0, s>>>(mp.MA, mp.MB, mp.MX, mp.MC, mp.MN, mp.OVF, mp.Lo, u0, sp.SA, sp.SB, sp.SX,
                                        sp.SC, sp.SN, sp.SOVF, N, G, K, K2, theta, u_r, st, lo_stride);
}

static inline unsigned nblk(int64_t N) { return (unsigned)((N + kBlock - 1) / kBlock); }

void grid_envelope(const float *I, const float *u0, FwdMaps &mp, int64_t M, int64_t N, int C, float beta,
                   float u_r, cudaStream_t s)
{
    // EC/EA/EB live in the Starts/Ends/MB slots, which are written later.
    count_launches(1);
    k_env_chunk<<<dim3(nblk(N), (unsigned)M), kBlock, 0, s>>>(I, mp.Starts, mp.Ends, mp.MB, N, C, beta, u_r);
    grid_envelope_carry(u0, mp, M, N, s);
}

void grid_envelope_carry(const float *u0, FwdMaps &mp, int64_t M, int64_t N, cudaStream_t s)
{
    const float *EC = mp.Starts, *EA = mp.Ends, *EB = mp.MB;
    if (!env_carry_staged(u0, EC, EA, EB, mp.Lo, N, M, 1e-5f, s)) {
        count_launches(1);
        k_env_carry<<<nblk(N), kBlock, 0, s>>>(u0, EC, EA, EB, mp.Lo, N, M, 1e-5f);
    }
}

// Composition of the chunk envelope maps of a slice (one thread per neuron):
// g2 o g1 = (min(c2, a2*c1 + b2), a2*a1, a2*b1 + b2).  env = [c | a | b] rows.
__global__ void __launch_bounds__(kBlock) k_env_compose(const float *__restrict__ EC, const float *__restrict__ EA,
                                                        const float *__restrict__ EB, float *__restrict__ env,
                                                        int64_t N, int64_t M)
{
    int64_t n = (int64_t)blockIdx.x * kBlock + threadIdx.x;
    if (n >= N) return;
    float c = kInf, a = 1.0f, b = 0.0f;
#pragma unroll 8
    for (int64_t m = 0; m < M; m++) {
        const float c2 = EC[m * N + n], a2 = EA[m * N + n], b2 = EB[m * N + n];
        const float cc = mul_add_rn(a2, c, b2);
        c = c2 < cc ? c2 : cc;
        b = mul_add_rn(a2, b, b2);
        a = __fmul_rn(a2, a);
    }
    env[n] = c;
    env[N + n] = a;
    env[2 * N + n] = b;
}

void env_compose(const float *EC, const float *EA, const float *EB, float *env, int64_t N, int64_t M, cudaStream_t s)
{
    count_launches(1);
    k_env_compose<<<nblk(N), kBlock, 0, s>>>(EC, EA, EB, env, N, M);
}

void env_chunks(const float *I, float *EC, float *EA, float *EB, int64_t N, int64_t M, int C, float beta, float u_r,
                cudaStream_t s)
{
    count_launches(1);
    k_env_chunk<<<dim3(nblk(N), (unsigned)M), kBlock, 0, s>>>(I, EC, EA, EB, N, C, beta, u_r);
}

void grid_build(const float *I, const float *u0, FwdMaps &mp, int64_t M, int64_t N, int C, int K, float beta,
                float theta, float u_r, lifb_stats *st, cudaStream_t s)
{
    dim3 g(nblk(N), (unsigned)M);
    int km = K <= 2 ? 2 : K <= 4 ? 4 : K <= 8 ? 8 : K <= 16 ? 16 : K <= 32 ? 32 : 64;
    switch (km) {
    case 2: launch_build<2>(g, s, I, mp.Lo, u0, mp.MA, mp.MB, mp.MX, mp.MC, mp.MN, mp.OVF, N, C, K, beta, theta, u_r, st); break;
    case 4: launch_build<4>(g, s, I, mp.Lo, u0, mp.MA, mp.MB, mp.MX, mp.MC, mp.MN, mp.OVF, N, C, K, beta, theta, u_r, st); break;
    case 8: launch_build<8>(g, s, I, mp.Lo, u0, mp.MA, mp.MB, mp.MX, mp.MC, mp.MN, mp.OVF, N, C, K, beta, theta, u_r, st); break;
    case 16: launch_build<16>(g, s, I, mp.Lo, u0, mp.MA, mp.MB, mp.MX, mp.MC, mp.MN, mp.OVF, N, C, K, beta, theta, u_r, st); break;
    case 32: launch_build<32>(g, s, I, mp.Lo, u0, mp.MA, mp.MB, mp.MX, mp.MC, mp.MN, mp.OVF, N, C, K, beta, theta, u_r, st); break;
    default: launch_build<64>(g, s, I, mp.Lo, u0, mp.MA, mp.MB, mp.MX, mp.MC, mp.MN, mp.OVF, N, C, K, beta, theta, u_r, st); break;
    }
}

void grid_carry(const float *I, const float *u0, const float *MA, const float *MB, const float *MX, const float *MC,
                const int32_t *MN, const int32_t *OVF, float *Starts, int64_t N, int64_t M, int64_t L, int K,
                float beta, float theta, float u_r, cudaStream_t s)
{
    count_launches(1);
    k_carry<<<nblk(N), kBlock, 0, s>>>(I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, L, K, beta, theta, u_r);
}

void grid_compose(const FwdMaps &mp, const SuperMaps &sp, const float *u0, int64_t M2, int64_t N, int G,
                  int K, int K2, float theta, float u_r, lifb_stats *st, cudaStream_t s, int64_t lo_stride)
{
    dim3 g(nblk(N), (unsigned)M2);
    int km = K2 <= 2 ? 2 : K2 <= 4 ? 4 : K2 <= 8 ? 8 : K2 <= 16 ? 16 : K2 <= 32 ? 32 : 64;
    switch (km) {
    case 2: launch_compose<2>(g, s, mp, sp, u0, N, G, K, K2, theta, u_r, st, lo_stride); break;
    case 4: launch_compose<4>(g, s, mp, sp, u0, N, G, K, K2, theta, u_r, st, lo_stride); break;
    case 8: launch_compose<8>(g, s, mp, sp, u0, N, G, K, K2, theta, u_r, st, lo_stride); break;
    case 16: launch_compose<16>(g, s, mp, sp, u0, N, G, K, K2, theta, u_r, st, lo_stride); break;
    case 32: launch_compose<32>(g, s, mp, sp, u0, N, G, K, K2, theta, u_r, st, lo_stride); break;
    default: launch_compose<64>(g, s, mp, sp, u0, N, G, K, K2, theta, u_r, st, lo_stride); break;
    }
}

void grid_carry_inner(const float *I, const FwdMaps &mp, const float *SStarts, int64_t T, int64_t N, int C, int G,
                      int K, float beta, float theta, float u_r, cudaStream_t s)
{
    int64_t M2 = T / C / G;
    count_launches(1);
    k_carry_inner<<<dim3(nblk(N), (unsigned)M2), kBlock, 0, s>>>(I, SStarts, mp.MA, mp.MB, mp.MX, mp.MC, mp.MN,
                                                                mp.OVF, mp.Starts, N, T / C, G, C, K, beta, theta,
                                                                u_r);
}

void replay_any(const float *I, const float *u0, const float *Starts, float *U, float *S, float *Ends, int64_t T,
                int64_t N, int64_t L, float beta, float theta, float u_r, cudaStream_t s)
{
    if (fwd_replay_tma(I, u0, Starts, U, S, Ends, T, N, L, beta, theta, u_r, s)) return;
    count_launches(1);
    k_replay<<<dim3(nblk(N), (unsigned)(T / L)), kBlock, 0, s>>>(I, Starts, U, S, Ends, N, (int)L, beta, theta,
                                                                u_r);
}

void grid_replay_repair(const float *I, const float *u0, FwdMaps &mp, float *U, float *S, int64_t T, int64_t N,
                        int C, int max_repair, float beta, float theta, float u_r, lifb_stats *st,
                        cudaStream_t s)
{
    int64_t M = T / C;
    if (!fwd_replay_tma(I, u0, mp.Starts, U, S, mp.Ends, T, N, C, beta, theta, u_r, s)) {
        count_launches(1);
        k_replay<<<dim3(nblk(N), (unsigned)M), kBlock, 0, s>>>(I, mp.Starts, U, S, mp.Ends, N, C, beta, theta, u_r);
    }
    int rounds = max_repair < 0 ? (int)(M + 1) : max_repair;
    if (rounds > 0) {
        count_launches(1);
        k_repair<<<nblk(N), kBlock, 0, s>>>(I, u0, mp.Starts, mp.Ends, U, S, N, M, C, rounds, beta, theta, u_r,
                                            st);
    }
}

}  // namespace lifb
