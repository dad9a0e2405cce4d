// Speculative segment forward for long sequences with few neurons.
//
// The serial recurrence over T rows for N neurons has N independent chains;
// when N is small (config 4: N = 1024 on 148 SMs) one pass cannot fill the GPU
// and runs at the latency of one dependent step per row.  Hard resets make a
// trajectory forget its start: two trajectories of the same neuron driven by
// the same input end up bit-identical once they spike in the same row (or
// their difference rounds away), typically within a few hundred rows.  So:
//
//   lead-in   the start of each segment of L rows, guessed by running the W rows
//             before it from u_r ("just reset"); segment 0 starts from u0, and
//             a lead-in that reaches row 0 starts from u0 too (then it is exact).
//             Normally inside the replay kernel (k_fwd_tma streams the lead-in
//             rows through its TMA ring before the segment's own); k_leadin
//             below does it as a separate pass for a halo (rows before row 0,
//             e.g. the end of the previous time slice) and the two-call form.
//   replay    every segment from its guessed start (k_fwd_tma: TMA-staged rows,
//             TMA-store epilogue), all segments at once
//   fix-up    per neuron, in time order, every segment whose guessed start
//             differs bit for bit from the previous segment's exact end is
//             replayed from that end until its rows rejoin (scan_fixup.cu)
//
// U and S equal the serial recurrence bit for bit whatever the guesses were;
// the guesses decide only how much the fix-up replays.  The map scan of the
// reference (lifscan/triton_lif.py:782-983) computes exact segment starts
// instead; this path trades its map build for a W-row lead-in.
#include <cstdio>

#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace lifb {

constexpr int kLeadBlock = 128;
// Rows per batch; the next batch is loaded while this one is stepped, so 2 x
// kLeadB loads per thread are in flight.  A batch of 64 steps (~1300 cycles
// of dependent arithmetic) covers the load latency; 16 left it exposed
// (a 4096-row lead-in took ~250 us).
constexpr int kLeadB = 64;

// blockIdx.y = s.  s < NS: Starts[s] for segment s.  Segment 0 starts from
// u0 (when given), or, with a halo of W_halo rows before row 0, from u0 (u_r
// when NULL) run through the halo.  Segment s >= 1 starts from a lead-in over
// rows [s*L - W, s*L) from u_r; one that reaches row 0 starts there from u0
// (u_r when NULL).  s == NS (when end_guess is given): the same lead-in over
// the last W rows, a guess of the state after row T-1 for whatever follows.
__global__ void __launch_bounds__(kLeadBlock) k_leadin(const float *__restrict__ I, const float *__restrict__ u0,
                                                       const float *__restrict__ I_halo, int64_t W_halo,
                                                       float *__restrict__ Starts, float *__restrict__ end_guess,
                                                       int64_t N, int64_t NS, int64_t L, int64_t W, float beta,
                                                       float theta, float u_r, Reset rs)
{
    const int64_t n = (int64_t)blockIdx.x * kLeadBlock + threadIdx.x;
    const int64_t s = blockIdx.y;
    if (n >= N) return;
    const float *p;
    int64_t len;
    float u;
    if (s == 0) {
        u = u0 ? u0[n] : u_r;
        if (!I_halo || W_halo <= 0) {
            if (u0) Starts[n] = u;
            return;
        }
        p = I_halo + n;
        len = W_halo;
    } else {
        const int64_t t1 = s * L;  // s == NS: t1 = T
        int64_t t0 = t1 - W;
        u = u_r;
        if (t0 <= 0) {
            t0 = 0;
            u = u0 ? u0[n] : u_r;
        }
        p = I + t0 * N + n;
        len = t1 - t0;
    }
    float cur[kLeadB], nxt[kLeadB];
#pragma unroll
    for (int q = 0; q < kLeadB; q++) cur[q] = q < len ? __ldg(p + q * N) : 0.0f;
    for (int64_t b = 0; b < len; b += kLeadB) {
        const int64_t nb = b + kLeadB;
#pragma unroll
        for (int q = 0; q < kLeadB; q++) nxt[q] = nb + q < len ? __ldg(p + (nb + q) * N) : 0.0f;
#pragma unroll
        for (int q = 0; q < kLeadB; q++)
            if (b + q < len) {
                bool f;
                u = step_any(u, cur[q], beta, theta, u_r, rs.aff, rs.gamma, rs.delta, f);
            }
#pragma unroll
        for (int q = 0; q < kLeadB; q++) cur[q] = nxt[q];
    }
    if (s < NS) Starts[s * N + n] = u;
    else end_guess[n] = u;
}

void leadin_starts(const float *I, const float *u0, const float *I_halo, int64_t W_halo, float *Starts,
                   float *end_guess, int64_t N, int64_t NS, int64_t L, int64_t W, float beta, float theta, float u_r,
                   cudaStream_t s, Reset rs)
{
    count_launches(1);
    const unsigned ny = (unsigned)(NS + (end_guess ? 1 : 0));
    k_leadin<<<dim3((unsigned)((N + kLeadBlock - 1) / kLeadBlock), ny), kLeadBlock, 0, s>>>(
        I, u0, I_halo, W_halo, Starts, end_guess, N, NS, L, W, beta, theta, u_r, rs);
}

__global__ void k_copy_row(const float *__restrict__ src, float *__restrict__ dst, int64_t N)
{
    const int64_t n = (int64_t)blockIdx.x * kLeadBlock + threadIdx.x;
    if (n < N) dst[n] = src[n];
}

}  // namespace lifb

namespace {
constexpr size_t kAl = 256;
size_t al(size_t x) { return (x + kAl - 1) / kAl * kAl; }
}  // namespace

extern "C" {

size_t lifb_scan_fwd_spec_workspace_bytes(int64_t T, int64_t N, int64_t L)
{
    if (T <= 0 || N <= 0 || L <= 0 || T % L) return 0;
    const size_t one = al((size_t)(T / L) * N * 4);
    return 4 * one;
}

static int spec_check(const char *who, int64_t T, int64_t N, int64_t L, int64_t W, int64_t W_halo)
{
    char msg[160];
    if (T < 0 || N < 0 || L <= 0 || W < 0 || W_halo < 0 || (T > 0 && T % L)) {
        snprintf(msg, sizeof msg, "%s: T must be a multiple of the segment length L > 0, W >= 0", who);
        lifb::set_last_error(msg);
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (T / L > 65535) {
        snprintf(msg, sizeof msg, "%s: more than 65535 segments", who);
        lifb::set_last_error(msg);
        return LIFB_ERR_UNSUPPORTED;
    }
    return LIFB_OK;
}

static int spec_ws(const char *who, int64_t T, int64_t N, int64_t L, void *workspace, size_t workspace_bytes)
{
    if (!workspace || (uintptr_t)workspace % kAl || workspace_bytes < lifb_scan_fwd_spec_workspace_bytes(T, N, L)) {
        char msg[160];
        snprintf(msg, sizeof msg, "%s: workspace missing, misaligned or too small", who);
        lifb::set_last_error(msg);
        return LIFB_ERR_WORKSPACE;
    }
    return LIFB_OK;
}

static int spec_done(const char *who)
{
    if (cudaGetLastError() != cudaSuccess) {
        char msg[160];
        snprintf(msg, sizeof msg, "%s: launch failed", who);
        lifb::set_last_error(msg);
        return LIFB_ERR_CUDA;
    }
    lifb::set_last_error("");
    return LIFB_OK;
}

struct SpecScratch {
    float *Starts, *Ends, *EndsNew;
    int32_t *Changed;
};

static SpecScratch spec_carve(void *workspace, int64_t NS, int64_t N)
{
    char *b = (char *)workspace;
    const size_t one = al((size_t)NS * N * 4);
    return {(float *)b, (float *)(b + one), (float *)(b + 2 * one), (int32_t *)(b + 3 * one)};
}

int lifb_scan_fwd_spec(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                       float theta, float u_r, int64_t L, int64_t W, const float *I_halo, int64_t W_halo,
                       void *workspace, size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_scan_fwd_spec");
    int st = spec_check("lifb_scan_fwd_spec", T, N, L, W, W_halo);
    if (st) return st;
    if (T == 0 || N == 0) return LIFB_OK;
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t NS = T / L;
    if (NS == 1 && (!I_halo || W_halo == 0)) {
        lifb::serial_fwd(I, u0, U, S, T, N, beta, theta, u_r, s);
    } else if (!(I_halo && W_halo > 0) && L <= 256 &&
               lifb::scan_block(I, u0, U, S, T, N, (int)L, 0, false, W, beta, theta, u_r, nullptr, s)) {
        // short sequences: lead-ins, replay and fix-up of one 32-neuron slab
        // per CTA on chip (scan_block.cu), no workspace used
    } else {
        if ((st = spec_ws("lifb_scan_fwd_spec", T, N, L, workspace, workspace_bytes))) return st;
        SpecScratch w = spec_carve(workspace, NS, N);
        // one launch when it applies: each segment's CTA streams its lead-in
        // rows through the replay's own TMA ring and records its start
        const bool fused = !(I_halo && W_halo > 0) && W > 0 &&
                           lifb::fwd_replay_tma(I, u0, nullptr, U, S, w.Ends, T, N, L, beta, theta, u_r, s, 1, W,
                                                w.Starts);
        if (!fused) {
            lifb::leadin_starts(I, u0, I_halo, W_halo, w.Starts, nullptr, N, NS, L, W, beta, theta, u_r, s);
            lifb::replay_any(I, u0, w.Starts, U, S, w.Ends, T, N, L, beta, theta, u_r, s);
        }
        lifb::fwd_fixup(I, w.Starts, 1, U, S, w.Ends, w.EndsNew, w.Changed, N, NS, L, beta, theta, u_r, nullptr, s);
    }
    return spec_done("lifb_scan_fwd_spec");
}

int lifb_tshard_fwd_tail(const float *I, float *U, float *S, int64_t T, int64_t N, float beta, float theta, float u_r,
                         int64_t L, int64_t W, float *end_guess, void *workspace, size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_tshard_fwd_tail");
    int st = spec_check("lifb_tshard_fwd_tail", T, N, L, W, 0);
    if (st) return st;
    if (T == 0 || N == 0) return LIFB_OK;
    if (T / L < 2 || W <= 0 || !end_guess) {
        lifb::set_last_error("lifb_tshard_fwd_tail: needs at least two segments, W > 0 and end_guess");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if ((st = spec_ws("lifb_tshard_fwd_tail", T, N, L, workspace, workspace_bytes))) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t NS = T / L;
    SpecScratch w = spec_carve(workspace, NS, N);
    // segments 1..NS-1, each from its W-row lead-in (from u_r: the slice's
    // entry is not known yet), streamed through the replay's TMA ring;
    // segment 0 waits for the entry (_head)
    if (!lifb::fwd_replay_tma(I, nullptr, nullptr, U, S, w.Ends, T, N, L, beta, theta, u_r, s, 1, W, w.Starts, false,
                              {}, 1)) {
        lifb::set_last_error("lifb_tshard_fwd_tail: needs N % 4 == 0, 16-byte aligned tensors and L a multiple of "
                             "the replay's tile");
        return LIFB_ERR_UNSUPPORTED;
    }
    cudaMemcpyAsync(end_guess, w.Ends + (NS - 1) * N, (size_t)N * 4, cudaMemcpyDeviceToDevice, s);
    return spec_done("lifb_tshard_fwd_tail");
}

int lifb_tshard_fwd_head(const float *I, const float *entry, float *U, float *S, float *end, int64_t T, int64_t N,
                         float beta, float theta, float u_r, int64_t L, void *workspace, size_t workspace_bytes,
                         void *stream)
{
    LIFB_RANGE("lifb_tshard_fwd_head");
    int st = spec_check("lifb_tshard_fwd_head", T, N, L, 0, 0);
    if (st) return st;
    if (T == 0 || N == 0) return LIFB_OK;
    if (T / L < 2 || !entry || !end) {
        lifb::set_last_error("lifb_tshard_fwd_head: needs at least two segments, entry and end");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if ((st = spec_ws("lifb_tshard_fwd_head", T, N, L, workspace, workspace_bytes))) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t NS = T / L;
    SpecScratch w = spec_carve(workspace, NS, N);
    // segment 0 from the entry (one chain of L rows: the caller keeps L
    // short), then every segment whose start differs from the exact end
    // before it, replayed until its rows rejoin
    cudaMemcpyAsync(w.Starts, entry, (size_t)N * 4, cudaMemcpyDeviceToDevice, s);
    if (!lifb::fwd_replay_tma(I, entry, nullptr, U, S, w.Ends, L, N, L, beta, theta, u_r, s)) {
        lifb::set_last_error("lifb_tshard_fwd_head: needs N % 4 == 0 and 16-byte aligned tensors");
        return LIFB_ERR_UNSUPPORTED;
    }
    lifb::fwd_fixup(I, w.Starts, 1, U, S, w.Ends, w.EndsNew, w.Changed, N, NS, L, beta, theta, u_r, nullptr, s);
    cudaMemcpyAsync(end, U + (T - 1) * N, (size_t)N * 4, cudaMemcpyDeviceToDevice, s);
    return spec_done("lifb_tshard_fwd_head");
}

int lifb_scan_fwd_spec_begin(const float *I, int64_t T, int64_t N, float beta, float theta, float u_r, int64_t L,
                             int64_t W, float *end_guess, void *workspace, size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_scan_fwd_spec_begin");
    int st = spec_check("lifb_scan_fwd_spec_begin", T, N, L, W, 0);
    if (st) return st;
    if (T == 0 || N == 0) return LIFB_OK;
    if ((st = spec_ws("lifb_scan_fwd_spec_begin", T, N, L, workspace, workspace_bytes))) return st;
    SpecScratch w = spec_carve(workspace, T / L, N);
    lifb::leadin_starts(I, nullptr, nullptr, 0, w.Starts, end_guess, N, T / L, L, W, beta, theta, u_r,
                        (cudaStream_t)stream);
    return spec_done("lifb_scan_fwd_spec_begin");
}

int lifb_scan_fwd_spec_finish(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                              float theta, float u_r, int64_t L, void *workspace, size_t workspace_bytes,
                              void *stream)
{
    LIFB_RANGE("lifb_scan_fwd_spec_finish");
    int st = spec_check("lifb_scan_fwd_spec_finish", T, N, L, 0, 0);
    if (st) return st;
    if (T == 0 || N == 0) return LIFB_OK;
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t NS = T / L;
    if (NS == 1) {
        lifb::serial_fwd(I, u0, U, S, T, N, beta, theta, u_r, s);
        return spec_done("lifb_scan_fwd_spec_finish");
    }
    if ((st = spec_ws("lifb_scan_fwd_spec_finish", T, N, L, workspace, workspace_bytes))) return st;
    SpecScratch w = spec_carve(workspace, NS, N);
    lifb::count_launches(1);
    lifb::k_copy_row<<<(unsigned)((N + lifb::kLeadBlock - 1) / lifb::kLeadBlock), lifb::kLeadBlock, 0, s>>>(
        u0, w.Starts, N);
    lifb::replay_any(I, u0, w.Starts, U, S, w.Ends, T, N, L, beta, theta, u_r, s);
    lifb::fwd_fixup(I, w.Starts, 1, U, S, w.Ends, w.EndsNew, w.Changed, N, NS, L, beta, theta, u_r, nullptr, s);
    return spec_done("lifb_scan_fwd_spec_finish");
}

}  // extern "C"
