// Internal declarations shared by the CUDA translation units of liblifb.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>

#include "../../include/lifscan_b200.h"

namespace lifb {

// An NVTX range over a library call or one of its phases, so that profilers
// which read NVTX attribute each kernel to the call and phase that launched
// it.  NVTX is header-only here; without an attached tool a range costs one
// predictable branch.
struct NvtxRange {
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};
#define LIFB_RANGE_CAT2(a, b) a##b
#define LIFB_RANGE_CAT(a, b) LIFB_RANGE_CAT2(a, b)
// Opens a range named `name` until the end of the enclosing scope.
#define LIFB_RANGE(name) ::lifb::NvtxRange LIFB_RANGE_CAT(lifb_range_, __LINE__)(name)

// Adds n to the library's launch counter (lifb_kernel_launches).
void count_launches(int n);
// Sets the calling thread's lifb_last_error() text.
void set_last_error(const char *msg);

// Chunk-level scratch of the forward scan, carved from the caller's workspace.
// All arrays are [M, N] (MX/MC: [M, K, N]) with the neuron index fastest.
struct FwdMaps {
    float *Lo, *MA, *MB, *MX, *MC, *Starts, *Ends;
    int32_t *MN, *OVF;
};

// Super-map scratch of the three-level forward (v4): [M2, N] / [M2, K2, N].
struct SuperMaps {
    float *SA, *SB, *SX, *SC, *SStarts;
    int32_t *SN, *SOVF;
};

// The reset rule of one scan, uniform across the grid: hard (u' = u_r) unless
// aff, else the affine reset u' = fl(fl(gamma*v) + delta) (gamma = 1, delta =
// -theta: the soft reset u' = v - theta, bit for bit).
struct Reset {
    bool aff = false;
    float gamma = 0.0f, delta = 0.0f;
};
inline Reset affine_reset(float gamma, float delta)
{
    Reset r;
    r.aff = true;
    r.gamma = gamma;
    r.delta = delta;
    return r;
}

// runtime.cu
bool make_tmap_2d(CUtensorMap *m, const float *base, int64_t N, int64_t T, int box_x, int box_y);
// 2-D map of a [T, N] array of 4-byte elements (fp32, or int32 when int32 is true).
bool make_tmap_2d_typed(CUtensorMap *m, const void *base, bool int32, int64_t N, int64_t T, int box_x, int box_y);
// 3-D map of a [d2, d1, d0] array of 32-bit words (d0 innermost), box
// (b0, b1, b2); false unless d0 * 4 is a multiple of 16 and base is 16-byte
// aligned.
// 2-D float map [T rows, N columns] with boxes of one swizzle row (swz_bytes
// = 64 or 128 bytes of columns) x box_y rows, in the swizzled shared-memory
// layout of the tensor cores' K-major operands.
bool make_tmap_2d_swz(CUtensorMap *m, const float *base, int64_t N, int64_t T, int box_y, int swz_bytes);
bool make_tmap_3d_u32(CUtensorMap *m, const void *base, int64_t d0, int64_t d1, int64_t d2, int b0, int b1, int b2);
int *device_status_ptr();                 // status word of the current device
int read_device_status(bool reset);       // synchronous read (current device)
// Non-blocking: the word as of the last completed asynchronous read of the
// current device (0 before any), or -1 on a CUDA error; starts the next read.
int poll_device_status();

// chunk_tma.cu: true when N % 4 == 0 and every non-null pointer is 16-byte
// aligned (the TMA kernels' requirement).
bool tma_ok(const void *const *ptrs, int n, int64_t N);
// 4 neurons per lane when there are at least min_ctas_per_sm 128-neuron CTAs
// (times M chunks) per SM, else 1.
int pick_npl(int64_t N, int64_t M, int min_ctas_per_sm);

// chunk_tma.cu: TMA-pipelined chunk kernels; false when the TMA path does not
// apply (N % 4 != 0, a misaligned tensor, more than 65535 chunks).
// Forward replay of M = T/C chunks from Starts (NULL: one chunk from u0).
// Chunk m starts from Starts[m * start_stride] (in rows of N).
// lead > 0: chunk m >= 1 starts from a lead-in over the `lead` rows before it
// (from u_r, or from u0 when they reach row 0), streamed through the same
// ring, and records that start in LeadStarts[m] (Starts is then ignored for
// m >= 1); requires C % R == 0 (false otherwise), lead is rounded up to R.
// first_chunk > 0: only chunks first_chunk..M-1 run (the caller runs the
// earlier ones); a lead-in that reaches row 0 starts from u_r when u0 is NULL.
bool fwd_replay_tma(const float *I, const float *u0, const float *Starts, float *U, float *S, float *Ends,
                    int64_t T, int64_t N, int64_t C, float beta, float theta, float u_r, cudaStream_t s,
                    int64_t start_stride = 1, int64_t lead = 0, float *LeadStarts = nullptr, bool vout = false,
                    Reset rs = {}, int64_t first_chunk = 0);
// Reverse adjoint sweep per chunk: mode 0 writes Lam from LamEnd (NULL: 0)
// and, when P is given, also the chunk maps; mode 1 writes only P, Q.
// P[m] = prod of a_t over chunk m, Q[m] = lam at the chunk's first row.
// D (optional, with P): per chunk and neuron, the rows counted from the
// chunk's last row whose running product of a is nonzero, i.e. the rows that
// a lam entering the chunk from above changes.
bool bwd_tma(int mode, const float *I, const float *u0, const float *U, const float *S, const float *GS,
             const float *GU, const float *LamEnd, float *Lam, float *P, float *Q, int64_t T, int64_t N, int64_t C,
             float beta, float theta, float u_r, float alpha, bool detach, cudaStream_t s, int32_t *D = nullptr);

// chunk_tma.cu: the adjoint from V (the forward's pre-reset potentials v_t)
// and GS only: detached reset, s recomputed as [v >= theta], no GU.  P, Q, D
// as bwd_tma when P is given; false when the TMA path does not apply.
// LamEnd (optional, [T/C, N]): the lam entering chunk m from the row after
// it (lam_{(m+1)C}); NULL: 0.
bool bwd_tma_v(const float *V, const float *GS, float *Lam, float *P, float *Q, int32_t *D, int64_t T, int64_t N,
               int64_t C, float beta, float theta, float alpha, cudaStream_t s, const float *LamEnd = nullptr);

// chunk_tma.cu: the affine-reset adjoint (detached reset: a = beta*gamma at a
// spike, beta elsewhere) over one chunk of T rows, v from U and I (u0 for row
// 0) or from V (from_v); false when the TMA path does not apply.
bool bwd_tma_aff(const float *IV, const float *u0, const float *U, const float *GS, float *Lam, int64_t T, int64_t N,
                 float beta, float theta, float alpha, float gamma, bool from_v, cudaStream_t s);
// The same from V with the parameter sums fused in: PGout [3][N] fp64 =
// (dbeta, dgamma, ddelta) per neuron, u0 for the u_{-1} term of dbeta.
bool bwd_tma_aff_pg(const float *V, const float *u0, const float *GS, float *Lam, double *PGout, int64_t T, int64_t N,
                    float beta, float theta, float alpha, float gamma, float delta, cudaStream_t s);

// serial.cu
void serial_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                float theta, float u_r, cudaStream_t s);
void serial_bwd(const float *I, const float *u0, const float *U, const float *S, const float *GS,
                const float *GU, float *Lam, int64_t T, int64_t N, float beta, float theta, float u_r,
                float alpha, bool detach, cudaStream_t s);
// The same forward writing V (pre-reset potentials v_t) in place of U, and
// the adjoint from V and GS (detached reset, s = [v >= theta], no GU).
void serial_fwd_v(const float *I, const float *u0, float *V, float *S, int64_t T, int64_t N, float beta,
                  float theta, float u_r, cudaStream_t s);
void serial_bwd_v(const float *V, const float *GS, float *Lam, int64_t T, int64_t N, float beta, float theta,
                  float alpha, cudaStream_t s);
// Affine-reset (u' = gamma*v + delta) serial forward (U, or V when vout) and
// adjoint (from U and I, or from V); PGout (optional, [3][N] fp64, needs u0):
// the per-neuron parameter sums (dbeta, dgamma, ddelta) of the same sweep.
void serial_fwd_aff(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                    float theta, float gamma, float delta, bool vout, cudaStream_t s);
void serial_bwd_aff(const float *IV, const float *u0, const float *U, const float *GS, float *Lam, int64_t T,
                    int64_t N, float beta, float theta, float alpha, float gamma, bool from_v, cudaStream_t s,
                    float delta = 0.0f, double *PGout = nullptr);

// aff.cu: the exact speculative forward of the affine reset over segments of
// L rows with W-row lead-ins (serial pass when T == L, W == 0 or the TMA path
// does not apply); workspace as lifb_scan_fwd_spec.  False: workspace missing,
// misaligned or too small (nothing launched).
bool aff_scan_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta, float theta,
                  float gamma, float delta, int64_t L, int64_t W, void *workspace, size_t workspace_bytes,
                  cudaStream_t s);

// scan_fwd_grid.cu
// grid_envelope / grid_build / grid_compose work on the first M chunks (M2
// supers) only; the last chunk's map is needed only for the stats.
void grid_envelope(const float *I, const float *u0, FwdMaps &mp, int64_t M, int64_t N, int C, float beta,
                   float u_r, cudaStream_t s);
// The prefix half of grid_envelope: Lo from chunk envelope maps already in
// the Starts / Ends / MB slots of `mp` (EC / EA / EB).
void grid_envelope_carry(const float *u0, FwdMaps &mp, int64_t M, int64_t N, cudaStream_t s);
void grid_build(const float *I, const float *u0, FwdMaps &mp, int64_t M, int64_t N, int C, int K, float beta,
                float theta, float u_r, lifb_stats *st, cudaStream_t s);
void grid_carry(const float *I, const float *u0, const float *MA, const float *MB, const float *MX,
                const float *MC, const int32_t *MN, const int32_t *OVF, float *Starts, int64_t N, int64_t M,
                int64_t L, int K, float beta, float theta, float u_r, cudaStream_t s);
// Composes groups of G maps of `mp` (capacity K) into `sp` (capacity K2); the
// pruning bound of group s is Lo[(s*G) * lo_stride].
void grid_compose(const FwdMaps &mp, const SuperMaps &sp, const float *u0, int64_t M2, int64_t N, int G,
                  int K, int K2, float theta, float u_r, lifb_stats *st, cudaStream_t s, int64_t lo_stride = 1);
void grid_carry_inner(const float *I, const FwdMaps &mp, const float *SStarts, int64_t T, int64_t N, int C, int G,
                      int K, float beta, float theta, float u_r, cudaStream_t s);
void grid_replay_repair(const float *I, const float *u0, FwdMaps &mp, float *U, float *S, int64_t T, int64_t N,
                        int C, int max_repair, float beta, float theta, float u_r, lifb_stats *st,
                        cudaStream_t s);

// Replay of T/L segments of L rows from Starts (TMA kernel, or the plain
// kernel when the TMA path does not apply); writes U, S and Ends [T/L, N].
void replay_any(const float *I, const float *u0, const float *Starts, float *U, float *S, float *Ends, int64_t T,
                int64_t N, int64_t L, float beta, float theta, float u_r, cudaStream_t s);

// scan_spec.cu: Starts[s] of NS segments of L rows guessed by a W-row lead-in
// from u_r (Starts[0] = u0; lead-ins that reach row 0 start from u0).
// end_guess (optional): the same lead-in over the last W rows (a guess of the
// state after row T-1).  u0 NULL: lead-ins that reach row 0 start from u_r
// and Starts[0] is left to the caller.
void leadin_starts(const float *I, const float *u0, const float *I_halo, int64_t W_halo, float *Starts,
                   float *end_guess, int64_t N, int64_t NS, int64_t L, int64_t W, float beta, float theta, float u_r,
                   cudaStream_t s, Reset rs = {});

// scan_block.cu: the block-level fused forward, one CTA per 32-neuron slab
// holding all T rows in shared memory (T % C == 0, 2 <= T/C <= 16 with maps
// and K <= 16, <= 32 without, C <= 256, N % 4 == 0, 16-byte aligned tensors,
// the slab and its maps within the opt-in shared memory).  maps: the
// two-level map scan (envelope, build, carry, replay, fix-up) with chunk
// length C and capacity K, stats accumulated into st when given; otherwise
// W-row lead-ins guess each chunk's start.  False when it does not apply
// (nothing launched).
bool scan_block_applies(int64_t T, int64_t N, int C, int K, bool maps);
bool scan_block(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, int C, int K, bool maps,
                int64_t W, float beta, float theta, float u_r, lifb_stats *st, cudaStream_t s);

// host_pipeline.cu
size_t host_pipe_workspace_bytes(int64_t T, int64_t N, int64_t block_n);
int host_pipe_run(const float *I_h, const float *GS_h, const float *u0_h, float *S_h, float *dI_h, float *du0_h,
                  int64_t T, int64_t N, float beta, float theta, float u_r, float alpha, int64_t block_n,
                  void *workspace, cudaStream_t cs, const char **err);
// The same over blocks of block_t time rows (contiguous copies; N % 4 == 0).
int64_t host_pipe_rows_default_block(int64_t T, int64_t N);
size_t host_pipe_rows_workspace_bytes(int64_t T, int64_t N, int64_t block_t);
int host_pipe_run_rows(const float *I_h, const float *GS_h, const float *u0_h, float *S_h, float *dI_h,
                       float *du0_h, int64_t T, int64_t N, float beta, float theta, float u_r, float alpha,
                       int64_t block_t, void *workspace, cudaStream_t cs, const char **err);

// carry_tma.cu: sequential map carry with TMA-staged map windows; false when
// it does not apply (N % 4 != 0, K > 64).  Writes Starts[m] for m < M.
bool carry_staged(const float *I, const float *u0, const float *MA, const float *MB, const float *MX, const float *MC,
                  const int32_t *MN, const int32_t *OVF, float *Starts, int64_t N, int64_t M, int64_t L, int K,
                  float beta, float theta, float u_r, cudaStream_t s);

// carry_tma.cu: envelope of a whole slice: the chunk envelope maps (c, a, b)
// composed in order (min(c2, a2*c1 + b2), a2*a1, a2*b1 + b2).
void env_compose(const float *EC, const float *EA, const float *EB, float *env, int64_t N, int64_t M, cudaStream_t s);
// k_env_chunk over M chunks of C rows (EC/EA/EB [M, N]).
void env_chunks(const float *I, float *EC, float *EA, float *EB, int64_t N, int64_t M, int C, float beta, float u_r,
                cudaStream_t s);
// scan_fixup.cu: replay-until-resynchronised of rows [0, T) from new entry
// states (cross-slice repair); changed[n] = 1 and end[n] updated for neurons
// whose rows never resynchronise.
void entry_repair(const float *I, const float *entry, float *U, float *S, float *end, int32_t *changed, int64_t T,
                  int64_t N, float beta, float theta, float u_r, cudaStream_t s);
// Lam fix-up given the lam entering the slice from above (lam_top, per neuron).
void bwd_fixup_top(const float *I, const float *u0, const float *U, const float *S, const float *GS, const float *GU,
                   const float *P, const float *Q, const int32_t *D, const float *lam_top, float *Lam, int64_t N,
                   int64_t M, int64_t C, float beta, float theta, float alpha, cudaStream_t s);

// carry_tma.cu: envelope prefix with TMA-staged (c, a, b) windows.
bool env_carry_staged(const float *u0, const float *EC, const float *EA, const float *EB, float *Lo, int64_t N,
                      int64_t M, float margin, cudaStream_t s);

// scan_fixup.cu
// EndsNew [NS, N] float and Changed [NS, N] int32 are scratch.
// rs: the reset rule (default: hard reset to u_r).
void fwd_fixup(const float *I, const float *Starts, int64_t start_stride, float *U, float *S, float *Ends,
               float *EndsNew, int32_t *Changed, int64_t N, int64_t NS, int64_t L, float beta, float theta, float u_r,
               int *longest_chain, cudaStream_t s, Reset rs = {});
// With D (from bwd_tma) the rows above each chunk's last spike, where every
// a is exactly beta (detached reset), are corrected in place by
// lam_end * beta^k instead of being recomputed from I, U and GS.
void bwd_fixup(const float *I, const float *u0, const float *U, const float *S, const float *GS, const float *GU,
               const float *P, const float *Q, const int32_t *D, float *Lam, int64_t N, int64_t M, int64_t C,
               float beta, float theta, float alpha, cudaStream_t s);

// scan_bwd.cu
struct BwdScratch {
    float *P, *Q, *LamEnd;
};
void grid_scan_bwd(const float *I, const float *u0, const float *U, const float *S, const float *GS,
                   const float *GU, float *Lam, BwdScratch &w, int64_t T, int64_t N, int C, float beta,
                   float theta, float u_r, float alpha, bool detach, cudaStream_t s);

}  // namespace lifb
