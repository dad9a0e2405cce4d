// Time-sharded exact scan: each GPU owns one slice of the time axis and runs
// these phases; the host exchanges the small per-slice results with NCCL
// all-gathers (hard_resets_compose_b200/tshard.py).
//
//   envelope   the slice's envelope map min(c, a*u + b), all its chunk maps composed
//   slice_map  chunk maps -> super maps (G) -> one slice map (capacity K3), pruned
//              with the slice's entry envelope bound (from the gathered envelopes)
//   apply      entry state from the gathered slice maps of the earlier slices, then
//              the super carry, the super replay and the local fix-up
//   repair     replay from the exact entry until the rows resynchronise
//   bwd        adjoint of the slice, chunks replayed from lam = 0, and the slice's
//              adjoint map (q, p): lam at its first row = q + p * lam entering it
//   bwd_fix    fix-up of the rows above each chunk's last spike given the lam that
//              enters the slice from the next one (folded from the gathered maps)
// The map algebra is the v4 three-level scan (lifscan/triton_lif.py:828-983)
// applied one level further, across GPUs.
#include <cstdio>

#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace lifb {

constexpr int kTsBlock = 128;

// Slice map layout [4 + 2*K3, N]: A, B, count (int32 bits), overflow (int32
// bits), K3 breakpoint rows, K3 constant rows.
static SuperMaps slice_map_view(float *map, int64_t N, int K3)
{
    SuperMaps v;
    v.SA = map;
    v.SB = map + N;
    v.SN = reinterpret_cast<int32_t *>(map + 2 * N);
    v.SOVF = reinterpret_cast<int32_t *>(map + 3 * N);
    v.SX = map + 4 * N;
    v.SC = map + (4 + (int64_t)K3) * N;
    v.SStarts = nullptr;
    return v;
}

// l = u0 folded through the envelope maps of slices 0..r-1 ([r][3][N]).
__global__ void k_env_prefix(const float *__restrict__ envs, int r, const float *__restrict__ u0,
                             float *__restrict__ l_entry, int64_t N)
{
    const int64_t n = (int64_t)blockIdx.x * kTsBlock + threadIdx.x;
    if (n >= N) return;
    float l = u0[n];
    for (int q = 0; q < r; q++) {
        const float *e = envs + (int64_t)q * 3 * N;
        const float lin = mul_add_rn(e[N + n], l, e[2 * N + n]);
        l = e[n] < lin ? e[n] : lin;
    }
    l_entry[n] = l;
}

// Entry state of slice r: u0 through the slice maps of slices 0..r-1.  A map
// that overflowed is still used below its lowest breakpoint (no rows of other
// slices are here to replay): the result is then a guess the repair corrects.
__global__ void k_map_prefix(const float *__restrict__ maps, int r, int K3, const float *__restrict__ u0,
                             float *__restrict__ entry, int64_t N)
{
    const int64_t n = (int64_t)blockIdx.x * kTsBlock + threadIdx.x;
    if (n >= N) return;
    float u = u0[n];
    const int64_t rows = 4 + 2 * (int64_t)K3;
    for (int q = 0; q < r; q++) {
        const float *m = maps + (int64_t)q * rows * N;
        const int cnt = __float_as_int(m[2 * N + n]);
        int k = 0;
        while (k < cnt && m[(4 + k) * N + n] > u) k++;
        u = (k == cnt) ? mul_add_rn(m[n], u, m[N + n]) : m[(4 + (int64_t)K3 + k) * N + n];
    }
    entry[n] = u;
}

// The slice's adjoint as one affine map lam_0 = q + p * lam_T, from the chunk
// maps (P, Q) of the replay with lam_T = 0, folded from the first chunk:
// q = Q0 + P0*(Q1 + P1*(...)).  The running product is exactly 0 after the
// first chunk that holds a spike, where the fold stops.  lam_pq = [q | p].
__global__ void k_slice_adjoint(const float *__restrict__ P, const float *__restrict__ Q, float *__restrict__ lam_pq,
                                int64_t N, int64_t M)
{
    const int64_t n = (int64_t)blockIdx.x * kTsBlock + threadIdx.x;
    if (n >= N) return;
    float q = 0.0f, p = 1.0f;
    for (int64_t m = 0; m < M && p != 0.0f; m++) {
        q = q + p * Q[m * N + n];
        p = p * P[m * N + n];
    }
    lam_pq[n] = q;
    lam_pq[N + n] = p;
}

}  // namespace lifb

namespace {

constexpr size_t kAl = 256;
size_t al(size_t x) { return (x + kAl - 1) / kAl * kAl; }

struct TsLayout {
    lifb::FwdMaps mp;
    lifb::SuperMaps sp;
    float *tmp;
    size_t bytes;
};

TsLayout ts_layout(void *base, int64_t T, int64_t N, int C, int G, int K, int K2)
{
    TsLayout L{};
    const int64_t M = T / C, M2 = M / G;
    char *b = (char *)base;
    size_t off = 0;
    auto take = [&](size_t n_bytes) {
        void *p = b ? (void *)(b + off) : nullptr;
        off = al(off + n_bytes);
        return p;
    };
    L.mp.Lo = (float *)take((size_t)M * N * 4);
    L.mp.MA = (float *)take((size_t)M * N * 4);
    L.mp.MB = (float *)take((size_t)M * N * 4);
    L.mp.MX = (float *)take((size_t)M * K * N * 4);
    L.mp.MC = (float *)take((size_t)M * K * N * 4);
    L.mp.MN = (int32_t *)take((size_t)M * N * 4);
    L.mp.OVF = (int32_t *)take((size_t)M * N * 4);
    L.mp.Starts = (float *)take((size_t)M * N * 4);
    L.mp.Ends = (float *)take((size_t)M * N * 4);
    L.sp.SA = (float *)take((size_t)M2 * N * 4);
    L.sp.SB = (float *)take((size_t)M2 * N * 4);
    L.sp.SX = (float *)take((size_t)M2 * K2 * N * 4);
    L.sp.SC = (float *)take((size_t)M2 * K2 * N * 4);
    L.sp.SN = (int32_t *)take((size_t)M2 * N * 4);
    L.sp.SOVF = (int32_t *)take((size_t)M2 * N * 4);
    L.sp.SStarts = (float *)take((size_t)M2 * N * 4);
    L.tmp = (float *)take((size_t)N * 4);
    L.bytes = off;
    return L;
}

int ts_fail(int status, const char *msg)
{
    lifb::set_last_error(msg);
    return status;
}

int ts_check(const char *what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        lifb::set_last_error(what);
        return LIFB_ERR_CUDA;
    }
    lifb::set_last_error("");
    return LIFB_OK;
}

int ts_args(int64_t T, int64_t N, int C, int G, int K, int K2, void *ws, size_t bytes)
{
    if (T <= 0 || N <= 0 || C <= 0 || G <= 0 || T % ((int64_t)C * G))
        return ts_fail(LIFB_ERR_INVALID_ARGUMENT, "time-sharded scan: the slice length must be a positive multiple of C*G");
    if (K < 1 || K > 64 || K2 < 1 || K2 > 64)
        return ts_fail(LIFB_ERR_INVALID_ARGUMENT, "time-sharded scan: capacities must be in 1..64");
    if (T / C > 65535) return ts_fail(LIFB_ERR_UNSUPPORTED, "time-sharded scan: more than 65535 chunks per slice");
    if (!ws || (uintptr_t)ws % kAl) return ts_fail(LIFB_ERR_WORKSPACE, "time-sharded scan: workspace missing or misaligned");
    if (bytes < ts_layout(nullptr, T, N, C, G, K, K2).bytes)
        return ts_fail(LIFB_ERR_WORKSPACE, "time-sharded scan: workspace too small");
    return LIFB_OK;
}

}  // namespace

extern "C" {

size_t lifb_tshard_workspace_bytes(int64_t T, int64_t N, int C, int G, int K, int K2)
{
    if (T <= 0 || N <= 0 || C <= 0 || G <= 0 || T % ((int64_t)C * G)) return 0;
    return ts_layout(nullptr, T, N, C, G, K, K2).bytes;
}

int lifb_tshard_envelope(const float *I, int64_t T, int64_t N, int C, int G, int K, int K2, float beta, float u_r,
                         float *env, void *ws, size_t bytes, void *stream)
{
    LIFB_RANGE("lifb_tshard_envelope");
    int st = ts_args(T, N, C, G, K, K2, ws, bytes);
    if (st) return st;
    TsLayout L = ts_layout(ws, T, N, C, G, K, K2);
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t M = T / C;
    lifb::env_chunks(I, L.mp.Starts, L.mp.Ends, L.mp.MB, N, M, C, beta, u_r, s);
    lifb::env_compose(L.mp.Starts, L.mp.Ends, L.mp.MB, env, N, M, s);
    return ts_check("lifb_tshard_envelope");
}

int lifb_tshard_slice_map(const float *I, const float *envs, int rank, const float *u0, int64_t T, int64_t N,
                          float beta, float theta, float u_r, int C, int G, int K, int K2, int K3, float *map, void *ws,
                          size_t bytes, void *stream)
{
    LIFB_RANGE("lifb_tshard_slice_map");
    int st = ts_args(T, N, C, G, K, K2, ws, bytes);
    if (st) return st;
    if (K3 < 1 || K3 > 64) return ts_fail(LIFB_ERR_INVALID_ARGUMENT, "time-sharded scan: K3 must be in 1..64");
    TsLayout L = ts_layout(ws, T, N, C, G, K, K2);
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t M = T / C, M2 = M / G;
    const unsigned nb = (unsigned)((N + lifb::kTsBlock - 1) / lifb::kTsBlock);
    // entry envelope bound of this slice, then the slice's chunk bounds
    lifb::count_launches(1);
    lifb::k_env_prefix<<<nb, lifb::kTsBlock, 0, s>>>(envs, rank, u0, L.tmp, N);
    lifb::grid_envelope_carry(L.tmp, L.mp, M, N, s);  // chunk envelopes from lifb_tshard_envelope
    lifb::grid_build(I, u0, L.mp, M, N, C, K, beta, theta, u_r, nullptr, s);
    lifb::grid_compose(L.mp, L.sp, u0, M2, N, G, K, K2, theta, u_r, nullptr, s);
    // all super maps of the slice composed into one map
    lifb::FwdMaps sup{};
    sup.Lo = L.mp.Lo;  // the slice's entry bound is Lo of its first chunk
    sup.MA = L.sp.SA;
    sup.MB = L.sp.SB;
    sup.MX = L.sp.SX;
    sup.MC = L.sp.SC;
    sup.MN = L.sp.SN;
    sup.OVF = L.sp.SOVF;
    lifb::SuperMaps out = lifb::slice_map_view(map, N, K3);
    lifb::grid_compose(sup, out, u0, 1, N, (int)M2, K2, K3, theta, u_r, nullptr, s);
    return ts_check("lifb_tshard_slice_map");
}

int lifb_tshard_apply(const float *I, const float *maps, int rank, int K3, const float *u0, float *entry, float *U,
                      float *S, float *end, int64_t T, int64_t N, float beta, float theta, float u_r, int C, int G,
                      int K, int K2, void *ws, size_t bytes, void *stream)
{
    LIFB_RANGE("lifb_tshard_apply");
    int st = ts_args(T, N, C, G, K, K2, ws, bytes);
    if (st) return st;
    TsLayout L = ts_layout(ws, T, N, C, G, K, K2);
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t M = T / C, M2 = M / G;
    const unsigned nb = (unsigned)((N + lifb::kTsBlock - 1) / lifb::kTsBlock);
    lifb::count_launches(1);
    lifb::k_map_prefix<<<nb, lifb::kTsBlock, 0, s>>>(maps, rank, K3, u0, entry, N);
    // super carry from the entry state, super replay, local fix-up
    if (!lifb::carry_staged(I, entry, L.sp.SA, L.sp.SB, L.sp.SX, L.sp.SC, L.sp.SN, L.sp.SOVF, L.sp.SStarts, N, M2,
                            (int64_t)C * G, K2, beta, theta, u_r, s))
        lifb::grid_carry(I, entry, L.sp.SA, L.sp.SB, L.sp.SX, L.sp.SC, L.sp.SN, L.sp.SOVF, L.sp.SStarts, N, M2,
                         (int64_t)C * G, K2, beta, theta, u_r, s);
    if (!lifb::fwd_replay_tma(I, entry, L.sp.SStarts, U, S, L.mp.Ends, T, N, (int64_t)C * G, beta, theta, u_r, s,
                              1))
        return ts_fail(LIFB_ERR_UNSUPPORTED, "time-sharded scan: needs N % 4 == 0 and 16-byte aligned tensors");
    lifb::fwd_fixup(I, L.sp.SStarts, 1, U, S, L.mp.Ends, L.mp.Lo, L.mp.MN, N, M2, (int64_t)C * G, beta, theta, u_r,
                    nullptr, s);
    cudaMemcpyAsync(end, U + (T - 1) * N, (size_t)N * 4, cudaMemcpyDeviceToDevice, s);
    return ts_check("lifb_tshard_apply");
}

int lifb_tshard_repair(const float *I, const float *entry, float *U, float *S, float *end, int32_t *changed,
                       int64_t T, int64_t N, float beta, float theta, float u_r, void *stream)
{
    LIFB_RANGE("lifb_tshard_repair");
    if (T <= 0 || N <= 0) return ts_fail(LIFB_ERR_INVALID_ARGUMENT, "time-sharded repair: empty slice");
    lifb::entry_repair(I, entry, U, S, end, changed, T, N, beta, theta, u_r, (cudaStream_t)stream);
    return ts_check("lifb_tshard_repair");
}

size_t lifb_tshard_bwd_workspace_bytes(int64_t T, int64_t N, int C)
{
    if (T <= 0 || N <= 0 || C <= 0 || T % C) return 0;
    return 3 * al((size_t)(T / C) * N * 4);
}

int lifb_tshard_bwd(const float *I, const float *u_prev, const float *U, const float *GS, float *Lam, float *lam_pq,
                    int64_t T, int64_t N, float beta, float theta, float u_r, float alpha, int C, void *ws,
                    size_t bytes, void *stream)
{
    LIFB_RANGE("lifb_tshard_bwd");
    if (T <= 0 || N <= 0 || C <= 0 || T % C)
        return ts_fail(LIFB_ERR_INVALID_ARGUMENT, "time-sharded adjoint: T must be a positive multiple of C");
    if (T / C > 65535) return ts_fail(LIFB_ERR_UNSUPPORTED, "time-sharded adjoint: more than 65535 chunks per slice");
    if (!ws || (uintptr_t)ws % kAl || bytes < lifb_tshard_bwd_workspace_bytes(T, N, C))
        return ts_fail(LIFB_ERR_WORKSPACE, "time-sharded adjoint: workspace missing, misaligned or too small");
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t M = T / C;
    const size_t one = al((size_t)M * N * 4);
    float *P = (float *)ws, *Q = (float *)((char *)ws + one);
    int32_t *D = (int32_t *)((char *)ws + 2 * one);
    if (!lifb::bwd_tma(0, I, u_prev, U, nullptr, GS, nullptr, nullptr, Lam, P, Q, T, N, C, beta, theta, u_r, alpha,
                       true, s, D)) {
        char msg[256];
        snprintf(msg, sizeof msg,
                 "time-sharded adjoint: needs N %% 4 == 0 and 16-byte aligned tensors (N=%lld; address mod 16: "
                 "I %u, u_prev %u, U %u, GS %u, Lam %u)",
                 (long long)N, (unsigned)((uintptr_t)I & 15), (unsigned)((uintptr_t)u_prev & 15),
                 (unsigned)((uintptr_t)U & 15), (unsigned)((uintptr_t)GS & 15), (unsigned)((uintptr_t)Lam & 15));
        return ts_fail(LIFB_ERR_UNSUPPORTED, msg);
    }
    const unsigned nb = (unsigned)((N + lifb::kTsBlock - 1) / lifb::kTsBlock);
    lifb::count_launches(1);
    lifb::k_slice_adjoint<<<nb, lifb::kTsBlock, 0, s>>>(P, Q, lam_pq, N, M);
    return ts_check("lifb_tshard_bwd");
}

int lifb_tshard_bwd_fix(const float *I, const float *u_prev, const float *U, const float *GS, const float *lam_top,
                        float *Lam, int64_t T, int64_t N, float beta, float theta, float alpha, int C, void *ws,
                        size_t bytes, void *stream)
{
    LIFB_RANGE("lifb_tshard_bwd_fix");
    if (T <= 0 || N <= 0 || C <= 0 || T % C)
        return ts_fail(LIFB_ERR_INVALID_ARGUMENT, "time-sharded adjoint: T must be a positive multiple of C");
    if (!ws || (uintptr_t)ws % kAl || bytes < lifb_tshard_bwd_workspace_bytes(T, N, C))
        return ts_fail(LIFB_ERR_WORKSPACE, "time-sharded adjoint: workspace missing, misaligned or too small");
    const int64_t M = T / C;
    const size_t one = al((size_t)M * N * 4);
    const float *P = (const float *)ws, *Q = (const float *)((const char *)ws + one);
    const int32_t *D = (const int32_t *)((const char *)ws + 2 * one);
    lifb::bwd_fixup_top(I, u_prev, U, nullptr, GS, nullptr, P, Q, D, lam_top, Lam, N, M, C, beta, theta, alpha,
                        (cudaStream_t)stream);
    return ts_check("lifb_tshard_bwd_fix");
}

}  // extern "C"
