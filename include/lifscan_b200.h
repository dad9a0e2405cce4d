/*
 * lifscan_b200.h -- C ABI of the B200 (sm_100a) exact hard-reset LIF scan.
 *
 * The reference (cheshireyang/hard-resets-compose) exposes this path only as
 * Python functions in lifscan/triton_lif.py; it has no native FFI.  Each entry
 * point below is what a ctypes/cffi binding of that Python API binds: the same
 * tensors as raw device pointers, the same scalars, the same sizes.  The
 * reference function each one replaces is cited beside it.
 *
 * Conventions (identical to the reference, lifscan/triton_lif.py:3):
 *   - I, U, S, GS, GU, Lam are [T, N] fp32, row-major, contiguous, neuron index
 *     fastest (element (t, n) at t*N + n); N = batch x neurons.
 *   - u0 is [N] fp32.  S holds 0.0f / 1.0f.
 *   - All pointers are CUDA device pointers on the current device; the work is
 *     enqueued on `stream` (a cudaStream_t passed as void*, NULL = legacy
 *     default stream) and the call returns without synchronising.
 *   - beta, theta, u_r, alpha are used as fp32 (the reference casts its Python
 *     floats to fp32 once).
 *   - Scratch memory is caller-provided: query *_workspace_bytes, pass a device
 *     buffer of at least that size (256-byte aligned).  The library allocates
 *     nothing on these paths.
 *   - Forward outputs are bit-identical to the serial fp32 recurrence
 *     v = fl(fl(beta*u) + x); s = v >= theta; u = s ? u_r : v
 *     (lifscan/fast.py:69-81) for every input without NaN.
 * Every function returns LIFB_OK (0) or a nonzero status; it never throws and
 * never aborts.  lifb_last_error() returns a message for the calling thread.
 */
#ifndef LIFSCAN_B200_H
#define LIFSCAN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LIFB_OK 0
#define LIFB_ERR_INVALID_ARGUMENT 1 /* shape, capacity or parameter out of range */
#define LIFB_ERR_CUDA 2             /* a CUDA runtime call or launch failed */
#define LIFB_ERR_WORKSPACE 3        /* workspace NULL, too small or misaligned */
#define LIFB_ERR_UNSUPPORTED 4      /* valid request this build cannot serve */
#define LIFB_ERR_DEVICE 5           /* a kernel reported a device-side error (lifb_check_device) */

/* Device-resident counters filled by the scan forward when a stats pointer is
 * given; they give the reference's `stats` dict (triton_lif.py:812-816 for v3,
 * :976-982 for v4):
 *   repair_iters        = repair_iters
 *   overflow_frac       = n_overflow / n_maps
 *   mean_pieces         = sum_cnt / n_maps + 1
 *   max_pieces          = max_cnt + 1
 *   super_overflow_frac = n_super_overflow / n_super           (v4)
 *   super_mean_pieces   = sum_super_cnt / n_super + 1          (v4)
 *   super_max_pieces    = max_super_cnt + 1                    (v4)
 * The struct lives in device memory; copy it to the host after the stream
 * has finished.  The call zeroes it before counting. */
typedef struct lifb_stats {
    int32_t repair_iters;
    int32_t max_cnt;
    int32_t max_super_cnt;
    int32_t status; /* 0, or a nonzero device-side status code */
    int64_t n_maps;
    int64_t n_overflow;
    int64_t sum_cnt;
    int64_t n_super;
    int64_t n_super_overflow;
    int64_t sum_super_cnt;
} lifb_stats;

/* ABI version of this header; bumped on any signature change. */
int lifb_abi_version(void);

/* Number of CUDA kernels this library has launched in this process (all
 * devices, all threads).  Diagnostic: lets a caller count the library's own
 * launches inside a timed region. */
uint64_t lifb_kernel_launches(void);

/* Device-side status of the current CUDA device: 0 when no kernel of this
 * library has reported a problem, else the code of the first one (101 = a
 * bounded wait for an asynchronous copy expired; the kernel stopped early and
 * its outputs are incomplete).  Synchronous (reads device memory); reset != 0
 * clears the word afterwards.  Returns -1 if the read itself failed. */
int lifb_device_status(int reset);

/* The device-side status folded into a return code: LIFB_OK when no kernel
 * of this library on the current device has reported a problem since the
 * word was last cleared, LIFB_ERR_DEVICE when one has (lifb_last_error() then
 * names the code, e.g. 101: a bounded wait for an asynchronous copy expired,
 * so the outputs of the calls before this check may be incomplete), or
 * LIFB_ERR_CUDA when the read failed.  Synchronous, like lifb_device_status;
 * reset != 0 clears the word after reading it.  No reference counterpart (the
 * reference's Triton kernels never wait on a copy). */
int lifb_check_device(int reset);

/* The same check without blocking: returns the status word as of the last
 * read that has completed (LIFB_OK before any) and starts a new asynchronous
 * read on a private stream of the library, so a problem shows up at most one
 * poll late.  The word stays set until lifb_check_device(1) or
 * lifb_device_status(1) clears it.  Not for use while a stream of the calling
 * thread is being captured into a CUDA graph. */
int lifb_poll_device(void);

/* Human-readable text of a status code, and the last error message recorded
 * on the calling host thread (empty string if none). */
const char *lifb_status_string(int status);
const char *lifb_last_error(void);

/* Serial forward: one recurrence per neuron, time-tiled.
 * Replaces serial_forward_auto (lifscan/triton_lif.py:1221-1225), which is
 * serial_forward_tiled (:460-466) over fwd_tiled_kernel (:353-379), and
 * serial_forward (:246-251). */
int lifb_serial_fwd(const float *I, const float *u0, float *U, float *S,
                    int64_t T, int64_t N, float beta, float theta, float u_r,
                    void *stream);

/* Serial adjoint: lam_t = a_t lam_{t+1} + b_t swept backwards, with the
 * sigmoid surrogate (alpha) and the detached (detach != 0) or attached reset.
 * GU may be NULL (all zeros, the lif_tuned path).  S may be NULL when it is
 * the forward's own output: s_t is then recomputed as [v_t >= theta] from
 * v_t = fl(fl(beta*U[t-1]) + I[t]), which equals the stored spike bit for bit,
 * and the kernel reads 16 instead of 20 bytes per neuron-step.
 * Replaces serial_backward_auto (lifscan/triton_lif.py:1199-1203), i.e.
 * bwd_tiled_pf_kernel (:1087-1127), and serial_backward (:254-259). */
int lifb_serial_bwd(const float *I, const float *u0, const float *U, const float *S,
                    const float *GS, const float *GU, float *Lam,
                    int64_t T, int64_t N, float beta, float theta, float u_r,
                    float alpha, int detach, void *stream);

/* Two-level exact scan forward with envelope-pruned chunk maps.
 * C = chunk length (T % C == 0), K = map capacity (1..64).
 * max_repair < 0: repair until converged (always within T/C rounds), the
 * default of the Python layer; max_repair >= 0 caps the rounds like the
 * reference's `repair` argument.
 * Replaces scan_forward_v3 (lifscan/triton_lif.py:782-817). */
size_t lifb_scan_fwd_v3_workspace_bytes(int64_t T, int64_t N, int C, int K);
int lifb_scan_fwd_v3(const float *I, const float *u0, float *U, float *S,
                     int64_t T, int64_t N, float beta, float theta, float u_r,
                     int C, int K, int max_repair,
                     void *workspace, size_t workspace_bytes,
                     lifb_stats *stats_dev, void *stream);

/* Three-level exact scan forward: chunk maps (C, K) composed in groups of G
 * into super maps of capacity K2 (1..64); T % (C*G) == 0.
 * Replaces scan_forward_v4 (lifscan/triton_lif.py:935-983). */
size_t lifb_scan_fwd_v4_workspace_bytes(int64_t T, int64_t N, int C, int G, int K, int K2);
int lifb_scan_fwd_v4(const float *I, const float *u0, float *U, float *S,
                     int64_t T, int64_t N, float beta, float theta, float u_r,
                     int C, int G, int K, int K2, int max_repair,
                     void *workspace, size_t workspace_bytes,
                     lifb_stats *stats_dev, void *stream);

/* Tiled affine-scan backward with the surrogate fused in; C = chunk length
 * (T % C == 0).  GU may be NULL (zeros); S may be NULL as for lifb_serial_bwd.
 * Replaces scan_backward_tiled (lifscan/triton_lif.py:512-526) and, with the
 * reference's choice of C, scan_backward_auto (:1235-1239). */
size_t lifb_scan_bwd_workspace_bytes(int64_t T, int64_t N, int C);
int lifb_scan_bwd(const float *I, const float *u0, const float *U, const float *S,
                  const float *GS, const float *GU, float *Lam,
                  int64_t T, int64_t N, float beta, float theta, float u_r,
                  float alpha, int detach, int C,
                  void *workspace, size_t workspace_bytes, void *stream);

/* lif_tuned's layer with V saved instead of U (lifscan/triton_lif.py:654-683):
 * lifb_serial_fwd_v is lifb_serial_fwd writing V[t] = v_t = fl(fl(beta*u_{t-1})
 * + x_t) (the potential before the reset) in place of U; S is the same.
 * lifb_lif_bwd_v is the detached-reset adjoint from V and GS alone
 * (s_t = [v_t >= theta] recomputed, GU = 0): Lam = dL/dI, du0 = beta*Lam[0],
 * reading 8 bytes per neuron-step instead of 12.  C = T: one sweep (no
 * workspace); C < T: T/C chunks at once plus the fix-up
 * (lifb_lif_bwd_v_workspace_bytes). */
int lifb_serial_fwd_v(const float *I, const float *u0, float *V, float *S, int64_t T, int64_t N,
                      float beta, float theta, float u_r, void *stream);
size_t lifb_lif_bwd_v_workspace_bytes(int64_t T, int64_t N, int C);
int lifb_lif_bwd_v(const float *V, const float *GS, float *Lam, int64_t T, int64_t N, float beta,
                   float theta, float alpha, int C, void *workspace, size_t workspace_bytes,
                   void *stream);

/* lif_tuned forward + backward for HOST-resident tensors (the layer of
 * lifscan/triton_lif.py:654-683 with the detached sigmoid surrogate, called
 * with tensors that live in host memory).  Inputs I_host, GS_host [T, N] and
 * u0_host [N]; outputs S_host [T, N] (spikes), dI_host [T, N] (= Lam = dL/dI)
 * and du0_host [N] (= beta * Lam[0]).  Host buffers should be pinned
 * (cudaHostAlloc / page-locked) for the copies to overlap.  The neurons are
 * processed in column blocks of block_n (a multiple of 4): while block b runs
 * forward and adjoint on `stream` (the forward as soon as its I has arrived,
 * the adjoint once GS has), later blocks are copied in and earlier ones out on
 * two library-owned copy streams (S of a block leaves as soon as its forward
 * is done), so both PCIe directions stay busy at once.  The workspace is
 * device memory of at least lifb_lif_fwd_bwd_host_workspace_bytes(T, N,
 * block_n) bytes (three staging slots).  Work is ordered after what is already
 * queued on `stream`; the outputs are complete once `stream` has reached the
 * end of this call. */
size_t lifb_lif_fwd_bwd_host_workspace_bytes(int64_t T, int64_t N, int64_t block_n);
int lifb_lif_fwd_bwd_host(const float *I_host, const float *GS_host, const float *u0_host,
                          float *S_host, float *dI_host, float *du0_host,
                          int64_t T, int64_t N, float beta, float theta, float u_r, float alpha,
                          int64_t block_n, void *workspace, size_t workspace_bytes, void *stream);

/* Input gradient of a dense layer, dX [R, Din] = dY [R, Dout] . W [Dout, Din]
 * (row-major fp32; W is the Linear layer's weight), on the tensor cores as
 * three TF32 products (the operands split into TF32 high and low parts, the
 * product of the low parts dropped) accumulated in fp32: within about 1e-6
 * relative of an fp32 GEMM, not bit-equal to one.  This is the backward of
 * the Linear feeding a LIF layer in the consumer network (lifscan/shdnet.py:
 * 30-50, where torch computes it as an fp32 GEMM).  Needs Dout % 4 == 0 and
 * Din in {64, 128, 256} (LIFB_ERR_UNSUPPORTED otherwise) and 16-byte aligned
 * pointers; the workspace (lifb_dense_dgrad_workspace_bytes) holds W's
 * transposed high and low parts.  A non-finite element of dY or W makes the
 * outputs it reaches non-finite (NaN where an fp32 GEMM may give +-inf). */
size_t lifb_dense_dgrad_workspace_bytes(int64_t Din, int64_t Dout);
int lifb_dense_dgrad(const float *dY, const float *W, float *dX, int64_t R, int64_t Din, int64_t Dout,
                     void *workspace, size_t workspace_bytes, void *stream);

/* The same call pipelined over blocks of block_t time rows instead of neuron
 * columns (N % 4 == 0; LIFB_ERR_UNSUPPORTED otherwise).  A block of rows is one
 * contiguous range of each host array, so every copy is one linear transfer.
 * The forward runs the blocks in time order, each from the state the previous
 * block ended in; the adjoint runs them in reverse order, each from the lam
 * the block after it left.  Results equal lifb_lif_fwd_bwd_host's bit for bit.
 * V of all rows stays in the workspace between the two sweeps, so the
 * workspace (lifb_lif_fwd_bwd_host_rows_workspace_bytes) is T*N*4 bytes plus
 * four staging slots of 4*block_t*N*4 bytes.  lifb_lif_fwd_bwd_host_rows_block
 * gives the default block_t (blocks of about 16 MiB per array). */
int64_t lifb_lif_fwd_bwd_host_rows_block(int64_t T, int64_t N);
size_t lifb_lif_fwd_bwd_host_rows_workspace_bytes(int64_t T, int64_t N, int64_t block_t);
int lifb_lif_fwd_bwd_host_rows(const float *I_host, const float *GS_host, const float *u0_host,
                               float *S_host, float *dI_host, float *du0_host,
                               int64_t T, int64_t N, float beta, float theta, float u_r, float alpha,
                               int64_t block_t, void *workspace, size_t workspace_bytes, void *stream);

/* No-allocation variant of lifb_scan_fwd_v3 (no counterpart in the
 * reference, which only runs inside PyTorch and always allocates).
 * For callers that cannot allocate device memory when they call in: a plain
 * C or FFI host with no device allocator, an application whose device memory
 * is already committed to another pool or capped, or a latency-critical loop
 * that must never call cudaMalloc (which can block on the device).  The
 * arguments are those of lifb_scan_fwd_v3 without the workspace: its scratch
 * is a fixed array of LIFB_NOALLOC_SCRATCH_BYTES (64 MiB) inside the library,
 * held by every GPU that loads the library until the process exits.  The call
 * allocates nothing.
 *   - Requests whose lifb_scan_fwd_v3_workspace_bytes(T, N, C, K) exceed the
 *     maximum return LIFB_ERR_INVALID_ARGUMENT (the message gives the size)
 *     without touching the GPU.  At C = 64, K = 16 that is T*N up to about
 *     27 million neuron-steps.
 *   - The first call on each device looks up the array's device address
 *     (once per device, with that device current); make that first call
 *     before any stream capture on the device.
 *   - All calls on a device share the one array: calls that can overlap on
 *     the GPU (other streams, or other host threads without ordering) race
 *     on it and corrupt each other's results.  Issue them on one stream.
 *   - Nothing needs clearing between calls: each call writes every scratch
 *     word before reading it. */
#define LIFB_NOALLOC_SCRATCH_BYTES (64ull << 20)
int lifb_scan_fwd_v3_noalloc(const float *I, const float *u0, float *U, float *S,
                             int64_t T, int64_t N, float beta, float theta, float u_r,
                             int C, int K, int max_repair, lifb_stats *stats_dev, void *stream);

/* Speculative segment forward for long sequences (used by the B200 policy of
 * scan_forward_auto, lifscan/triton_lif.py:1228-1232, when N is too small to
 * fill the GPU with one pass): T/L segments of L rows (T % L == 0), each
 * started from a guess made by running the W rows before it from u_r, all
 * replayed at once, then every segment whose guessed start differs from the
 * previous segment's exact end is replayed from that end until its rows
 * rejoin.  U and S are bit-identical to the serial recurrence for every L and
 * W; L = T is the serial pass.  Optional halo: I_halo [W_halo, N], the rows
 * just before row 0 when u0 is only a guess of the state before the halo (a
 * time slice after the first); segment 0 then starts from u0 run through the
 * halo, and the outputs are exact for that start. */
size_t lifb_scan_fwd_spec_workspace_bytes(int64_t T, int64_t N, int64_t L);
int lifb_scan_fwd_spec(const float *I, const float *u0, float *U, float *S,
                       int64_t T, int64_t N, float beta, float theta, float u_r,
                       int64_t L, int64_t W, const float *I_halo, int64_t W_halo,
                       void *workspace, size_t workspace_bytes, void *stream);
/* The same forward in two calls, for a time slice whose start state comes
 * from elsewhere (the previous GPU): _begin runs the lead-ins of segments
 * 1..T/L-1 (those reaching row 0 start from u_r) and, when end_guess [N] is
 * given, the lead-in over the last W rows, a guess of the slice's final state
 * to hand to the next slice; _finish replays every segment, segment 0 from
 * u0, and fixes them up (same workspace, same L).  _finish alone is exact for
 * u0 whatever _begin guessed. */
int lifb_scan_fwd_spec_begin(const float *I, int64_t T, int64_t N, float beta, float theta,
                             float u_r, int64_t L, int64_t W, float *end_guess,
                             void *workspace, size_t workspace_bytes, void *stream);
int lifb_scan_fwd_spec_finish(const float *I, const float *u0, float *U, float *S, int64_t T,
                              int64_t N, float beta, float theta, float u_r, int64_t L,
                              void *workspace, size_t workspace_bytes, void *stream);

/* Parameter gradients of the fitting layer (lifscan/fit.py:15-61, LIFParamFn):
 * from the adjoint Lam of a detached-reset backward, per chunk of rows and
 * neuron, the fp64 partial sums of
 *   dL/dbeta = sum_t Lam_t u_{t-1},  dL/dtheta = -sum_t GS_t sigma'(v_t - theta),
 *   dL/du_r  = sum_t s_t beta Lam_{t+1}
 * into partials [3][M][N] (the caller sums each [M][N] block); s_t and v_t
 * are recomputed from U and I bit for bit.  M = lifb_param_grad_chunks(T, N)
 * (or any 1..65535).  Reads I, U, GS, Lam once (16 B per neuron-step). */
int lifb_param_grad_chunks(int64_t T, int64_t N);
int lifb_param_grad_partials(const float *I, const float *u0, const float *U, const float *GS,
                             const float *Lam, double *partials, int64_t T, int64_t N,
                             float beta, float theta, float alpha, int M, void *stream);

/* ---- Soft-reset LIF (subtractive reset u <- v - theta) ----------------------
 * The reference's second model class (lifscan/triton_lif.py:1035-1082 and
 * 1139-1198, lifscan/triton_soft.py): v = fl(fl(beta*u) + x); s = v >= theta;
 * u' = s ? fl(v - theta) : v.  Forward outputs are bit-identical to the
 * reference's fp32 soft recurrence.
 *   lifb_soft_serial_fwd  soft_serial_forward / soft_serial_forward_tiled
 *   lifb_soft_scan_fwd    soft_scan_forward, exact: T/L segments with W-row
 *                         lead-ins and the fix-up (workspace:
 *                         lifb_scan_fwd_spec_workspace_bytes(T, N, L))
 *   lifb_soft_serial_bwd  soft_serial_backward(_auto): the detached-reset
 *                         adjoint lam_t = GS_t sigma'(v_t) + beta lam_{t+1}
 *                         from U, I and u0 (Lam = dL/dI, du0 = beta*Lam[0])
 *   lifb_soft_adjoint_v   soft_adjoint_fft: the same adjoint from V (the
 *                         pre-reset potentials), fp32 (the reference: float64 FFT) */
int lifb_soft_serial_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N,
                         float beta, float theta, void *stream);
int lifb_soft_scan_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N,
                       float beta, float theta, int64_t L, int64_t W, void *workspace,
                       size_t workspace_bytes, void *stream);
int lifb_soft_serial_bwd(const float *I, const float *u0, const float *U, const float *GS, float *Lam,
                         int64_t T, int64_t N, float beta, float theta, float alpha, void *stream);
int lifb_soft_adjoint_v(const float *V, const float *GS, float *Lam, int64_t T, int64_t N, float beta,
                        float theta, float alpha, void *stream);

/* ---- Affine-reset LIF (u <- gamma*v + delta on a spike, 0 <= gamma <= 1) ----
 * lifscan/triton_affine.py: v = fl(fl(beta*u) + x); s = v >= theta;
 * u' = s ? fl(fl(gamma*v) + delta) : v (gamma = 0, delta = u_r: the hard
 * reset; gamma = 1, delta = -theta: the soft reset, bit for bit).
 *   lifb_aff_serial_fwd   aff_serial_forward (triton_affine.py:158-162)
 *   lifb_aff_scan_fwd     aff_scan_forward (:165-199), exact: T/L segments with
 *                         W-row lead-ins and the fix-up (workspace:
 *                         lifb_scan_fwd_spec_workspace_bytes(T, N, L)); gamma
 *                         outside [0, 1] is LIFB_ERR_INVALID_ARGUMENT
 *   lifb_aff_adjoint      LIFAffineFn.backward's adjoint (:230-238): lam_t =
 *                         GS_t sigma'(v_t) + a_t lam_{t+1}, a_t = beta*gamma at
 *                         a spike, beta elsewhere, lam_T = 0; s, v recomputed
 *                         from U, I and u0 (Lam = dL/dI, du0 = beta*Lam[0])
 *   lifb_aff_param_grad_partials  as lifb_param_grad_partials with a fourth
 *                         block: partials[4][M][N] = (dbeta, dtheta, ddelta,
 *                         dgamma), ddelta = sum s beta lam_{t+1}, dgamma = sum
 *                         s v beta lam_{t+1}
 *   lifb_reverse_linear_scan  reverse_affine_scan (:202-211) for [T][N] a, b:
 *                         out_t = a_t out_{t+1} + b_t, out_T = 0 (fp32 in order) */
int lifb_aff_serial_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N,
                        float beta, float theta, float gamma, float delta, void *stream);
int lifb_aff_scan_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N,
                      float beta, float theta, float gamma, float delta, int64_t L, int64_t W,
                      void *workspace, size_t workspace_bytes, void *stream);
int lifb_aff_adjoint(const float *I, const float *u0, const float *U, const float *GS, float *Lam,
                     int64_t T, int64_t N, float beta, float theta, float alpha, float gamma,
                     void *stream);
int lifb_aff_param_grad_partials(const float *I, const float *u0, const float *U, const float *GS,
                                 const float *Lam, double *partials, int64_t T, int64_t N,
                                 float beta, float theta, float alpha, int M, void *stream);
int lifb_reverse_linear_scan(const float *A, const float *B, float *Out, int64_t T, int64_t N,
                             void *stream);
/* The affine layer's single-pass path (the layer saves V instead of U):
 *   lifb_aff_serial_fwd_v  the serial forward writing V[t] = v_t (the
 *                          potential before the reset) in place of U
 *   lifb_aff_adjoint_v     lifb_aff_adjoint from V (s_t = [v_t >= theta],
 *                          u_t = s_t ? gamma v_t + delta : v_t bit for bit);
 *                          param_sums (optional, [3][N] double, needs u0)
 *                          receives per neuron (dbeta, dgamma, ddelta) of
 *                          the same sweep, dbeta including lam_0 * u0 */
int lifb_aff_serial_fwd_v(const float *I, const float *u0, float *V, float *S, int64_t T, int64_t N,
                          float beta, float theta, float gamma, float delta, void *stream);
int lifb_aff_adjoint_v(const float *V, const float *u0, const float *GS, float *Lam, double *param_sums,
                       int64_t T, int64_t N, float beta, float theta, float alpha, float gamma,
                       float delta, void *stream);

/* ---- Adaptive-threshold LIF (ALIF) ------------------------------------------
 * lifscan/triton_alif.py: state (u, w);
 *   v = fl(fl(beta*u) + x); s = v >= fl(theta0 + w);
 *   u' = s ? u_r : v;       w' = s ? fl(fl(rho*w) + q) : fl(rho*w).
 * U, W, S are [T][N] (the state after each row); u0, w0 are [N].
 *   lifb_alif_serial_fwd   alif_serial_forward (triton_alif.py:263-273), one pass
 *   lifb_alif_scan_fwd     alif_scan_forward (:301-363), exact: T/L segments,
 *                          each started from a Wlead-row lead-in from (u_r, w
 *                          guess) with the guess Wpred[row / Cpred] ([T/Cpred][N],
 *                          optional: 0 without), replayed at once, then a fix-up
 *                          until every segment's (u, w, s) rows match the serial
 *                          recurrence (workspace: lifb_alif_scan_fwd_workspace_bytes)
 *   lifb_alif_warm_predict alif_warm_predict (:74-92, 276-285): WP[m] ([T/C][N])
 *                          = w after the Wn chunks of C rows before chunk m, run
 *                          from (u_init, w_init), or from (UI, WI)[m - Wn] when
 *                          given, or from (u0, w0) when they reach row 0
 *   lifb_alif_bwd          the detached-reset adjoint (:359-364, 443-487) in one
 *                          reverse sweep: LV[t] = dL/dv_t, LW[t] = dL/dw_t
 *                          (optional), with d_t = GS_t + q lw_t, lv_t = (1 - s_t)
 *                          beta lv_{t+1} + sg_t d_t, lw_{t-1} = rho lw_t - sg_t d_t,
 *                          sg_t = alpha sig (1 - sig) at v_t - theta0 - w_{t-1};
 *                          S optional (NULL: recomputed from U, W, I bit for bit);
 *                          lw_m1 [N] (optional) = dL/dw0; param_sums [4][N] double
 *                          (optional) = per-neuron (dbeta, drho, dq, dtheta0) of
 *                          ALIFFn.backward (:542-554) */
int lifb_alif_serial_fwd(const float *I, const float *u0, const float *w0, float *U, float *W, float *S,
                         int64_t T, int64_t N, float beta, float rho, float q, float theta0, float u_r,
                         void *stream);
size_t lifb_alif_scan_fwd_workspace_bytes(int64_t T, int64_t N, int64_t L);
int lifb_alif_scan_fwd(const float *I, const float *u0, const float *w0, float *U, float *W, float *S,
                       int64_t T, int64_t N, float beta, float rho, float q, float theta0, float u_r,
                       int64_t L, int64_t Wlead, const float *Wpred, int64_t Cpred, void *workspace,
                       size_t workspace_bytes, void *stream);
int lifb_alif_warm_predict(const float *I, const float *u0, const float *w0, float *WP, const float *UI,
                           const float *WI, int64_t T, int64_t N, int64_t C, int64_t Wn, float u_init,
                           float w_init, float beta, float rho, float q, float theta0, float u_r,
                           void *stream);
int lifb_alif_bwd(const float *I, const float *u0, const float *w0, const float *U, const float *W,
                  const float *S, const float *GS, float *LV, float *LW, float *lw_m1, double *param_sums,
                  int64_t T, int64_t N, float beta, float rho, float q, float theta0, float alpha,
                  void *stream);
/* The same adjoint over T/C chunks of C rows (alif_backward's "scan", :505-521):
 * each step is affine in (lv, lw) with the upper-triangular matrix
 * [[(1 - s) beta, sg q], [0, rho - sg q]], so every chunk's map (5 numbers per
 * neuron) is composed in parallel, a carry gives every chunk its entering
 * (lv, lw), and every chunk is replayed from it.  param_sums is [4][T/C][N]
 * (per chunk and neuron; the caller sums).  C = T is lifb_alif_bwd.  Workspace:
 * lifb_alif_bwd_scan_workspace_bytes(T, N, C) (0 when T/C < 2). */
size_t lifb_alif_bwd_scan_workspace_bytes(int64_t T, int64_t N, int64_t C);
int lifb_alif_bwd_scan(const float *I, const float *u0, const float *w0, const float *U, const float *W,
                       const float *S, const float *GS, float *LV, float *LW, float *lw_m1,
                       double *param_sums, int64_t T, int64_t N, float beta, float rho, float q,
                       float theta0, float alpha, int64_t C, void *workspace, size_t workspace_bytes,
                       void *stream);

/* Spike mask of a [R, D] fp32 tensor (a spike raster: R = T*B rows (t, b)),
 * D <= 1024: mask [R, lifb_spike_mask_stride(D)] 32-bit words, 16-byte
 * aligned.  Word k of a row has bit q set when element 32k + q is nonzero
 * (NaN counts, -0 does not); word ceil(D/32) has bit 0 set when a nonzero
 * element of the row is not exactly 1.0 (consumers then read that row's values
 * from the dense tensor); the remaining words are padding, so that a row is a
 * whole number of 16-byte TMA units.  The format is this library's own: the
 * reference keeps spike rasters dense (lifscan/shdnet.py:12-27). */
int64_t lifb_spike_mask_stride(int64_t D);
int lifb_spike_mask(const float *X, uint32_t *mask, int64_t R, int64_t D, void *stream);

/* Fused forward of one layer of a spiking network: a Linear layer on a spike
 * input followed by the hard-reset LIF.  X [T, B, Din] and its spike mask
 * Xmask (lifb_spike_mask, or the Smask of the layer before), W [Dout, Din] and
 * bias [Dout] (NULL: none) as torch.nn.Linear holds them, u0 [B*Dout] (NULL:
 * zeros); writes V (pre-reset potentials, for the adjoint from V) and S, both
 * [T, B*Dout] with neuron b*Dout + j, the layout of fc(x).reshape(T, -1)
 * (lifscan/shdnet.py:39), and, when Smask is not NULL, the spike mask of S
 * ([T*B, lifb_spike_mask_stride(Dout)]) for the next layer.  I = X W^T + bias
 * is formed in shared memory and consumed there, never written: each element
 * sums the active inputs' weights in input order from 0 and adds the bias
 * last, the order of cuBLAS's fp32 GEMM on such an input, so S equals the
 * unfused Linear -> lif_tuned (lifscan/shdnet.py:38-45,
 * triton_lif.py:654-687) bit for bit.  Needs Dout % 32 == 0 and Din <= 1024
 * (LIFB_ERR_UNSUPPORTED otherwise; the caller then runs the unfused layer).
 * Replaces the forward of shdnet.LIFLayer (lifscan/shdnet.py:30-50). */
int lifb_spike_linear_lif_fwd(const float *X, const uint32_t *Xmask, const float *W,
                              const float *bias, const float *u0, float *V, float *S,
                              uint32_t *Smask, int64_t T, int64_t B, int64_t Din,
                              int64_t Dout, float beta, float theta, float u_r, void *stream);

/* Weight and bias gradients of a Linear layer on a spike input: gW [Dout, Din]
 * = dI^T X and gb [Dout] = sum over rows of dI (gb NULL: skipped), from dI
 * [R, Dout] (Dout % 4 == 0) and the input X [R, Din] with its spike mask; only the active
 * (row, input) pairs are visited.  The sums run over rows in a fixed order
 * that follows from the shape alone (row chunks sized for about one CTA per
 * SM, then the chunks' sums in a fixed grouping), so the result is deterministic;
 * it differs from a GEMM's by rounding only.  Workspace:
 * lifb_spike_linear_wgrad_workspace_bytes(R, Din, Dout).  Replaces the weight
 * and bias gradients torch's Linear backward computes for shdnet.LIFLayer
 * (lifscan/shdnet.py:33,39). */
size_t lifb_spike_linear_wgrad_workspace_bytes(int64_t R, int64_t Din, int64_t Dout);
int lifb_spike_linear_wgrad(const float *dI, const float *X, const uint32_t *Xmask, float *gW,
                            float *gb, int64_t R, int64_t Din, int64_t Dout, void *workspace,
                            size_t workspace_bytes, void *stream);

/* Leaky (non-spiking) integrator over time, [T, M] row-major fp32: _fwd
 * writes Y with y_t = beta * y_{t-1} + z_t (y_{-1} = 0); _bwd writes
 * GZ = the adjoint lam_t = gy_t + beta * lam_{t+1} (lam_T = 0).  Time is split
 * into 64-row chunks with one carried value between them, so the result equals
 * the sequential recurrence up to fp32 rounding.  Needs T <= 1024
 * (LIFB_ERR_UNSUPPORTED otherwise).  The leaky readout of the network in
 * config 3 (a deviation from lifscan/shdnet.py:66's mean readout that the
 * benchmark configuration names). */
int lifb_leaky_fwd(const float *Z, float *Y, int64_t T, int64_t M, float beta, void *stream);
int lifb_leaky_bwd(const float *GY, float *GZ, int64_t T, int64_t M, float beta, void *stream);

/* Time-sharded forward, the two halves of a slice's replay around the hand-over
 * of its end state (workspace: lifb_scan_fwd_spec_workspace_bytes(T, N, L)).
 * _tail replays segments 1..T/L-1 of the slice at once, each from a W-row
 * lead-in from u_r streamed through the replay (no separate lead-in pass),
 * and writes end_guess = the last segment's end: the slice's final state
 * whenever that segment's guessed start was right, the next slice's entry
 * guess.  _head, once this slice's entry is known, replays segment 0 from it,
 * then every segment whose start differs bit for bit from the exact end
 * before it until its rows rejoin, and writes end = U[T-1].  U, S are then
 * exact for `entry`.  The time-sharded scan has no reference counterpart (the
 * reference scans a whole sequence on one device, lifscan/triton_lif.py:935-983). */
int lifb_tshard_fwd_tail(const float *I, float *U, float *S, int64_t T, int64_t N,
                         float beta, float theta, float u_r, int64_t L, int64_t W,
                         float *end_guess, void *workspace, size_t workspace_bytes,
                         void *stream);
int lifb_tshard_fwd_head(const float *I, const float *entry, float *U, float *S,
                         float *end, int64_t T, int64_t N, float beta, float theta,
                         float u_r, int64_t L, void *workspace, size_t workspace_bytes,
                         void *stream);

/* ---- Time-sharded scan (one slice of the time axis per GPU) ----------------
 * The reference scans one sequence on one device (lifscan/triton_lif.py:
 * 944-983, scan_forward_v4; :512-526, scan_backward_tiled).  These phases
 * split [T_total, N] into P slices of T rows; the caller exchanges the small
 * per-slice results (all-gather over ranks) between phases.  Every pointer is
 * device memory of the calling GPU; `ws` comes from the *_workspace_bytes
 * query with the same sizes.  I/U/S/GS/Lam are the slice's [T, N] rows.
 *
 * Forward: envelope -> all-gather envs [P][3][N] -> slice_map -> all-gather
 * maps [P][4 + 2*K3][N] -> apply -> repeat { all-gather ends; repair from
 * the previous slice's end } until no slice end changes.
 * Backward: bwd -> all-gather lam_pq [P][2][N] -> lam_top = fold of the later
 * slices' (q, p) -> bwd_fix.  Forward U/S are bit-identical to the serial
 * recurrence over T_total rows; Lam equals its adjoint within rounding. */
size_t lifb_tshard_workspace_bytes(int64_t T, int64_t N, int C, int G, int K, int K2);
/* env[3][N] = the slice's envelope map (c, a, b): l -> min(c, a*l + b). */
int lifb_tshard_envelope(const float *I, int64_t T, int64_t N, int C, int G, int K, int K2,
                         float beta, float u_r, float *env, void *ws, size_t bytes, void *stream);
/* map[4 + 2*K3][N] = the slice's composed map (A, B, count, overflow,
 * breakpoints, constants), pruned with the entry bound folded from envs of
 * slices 0..rank-1 (envs: [P][3][N], gathered).  Reuses the chunk envelopes
 * that lifb_tshard_envelope left in ws, and leaves the slice's super maps
 * there for lifb_tshard_apply. */
int lifb_tshard_slice_map(const float *I, const float *envs, int rank, const float *u0, int64_t T,
                          int64_t N, float beta, float theta, float u_r, int C, int G, int K, int K2,
                          int K3, float *map, void *ws, size_t bytes, void *stream);
/* entry[N] = u0 through maps of slices 0..rank-1; U, S, end[N] (U's last row)
 * from that entry, with the super maps of the slice_map call on the same ws. */
int lifb_tshard_apply(const float *I, const float *maps, int rank, int K3, const float *u0,
                      float *entry, float *U, float *S, float *end, int64_t T, int64_t N, float beta,
                      float theta, float u_r, int C, int G, int K, int K2, void *ws, size_t bytes,
                      void *stream);
/* Replays from a new entry[N] until the rows rejoin U/S; changed[n] = 1 and
 * end[n] updated where they never rejoin. */
int lifb_tshard_repair(const float *I, const float *entry, float *U, float *S, float *end,
                       int32_t *changed, int64_t T, int64_t N, float beta, float theta, float u_r,
                       void *stream);
size_t lifb_tshard_bwd_workspace_bytes(int64_t T, int64_t N, int C);
/* Detached-reset adjoint of the slice with lam = 0 entering from above;
 * u_prev[N] = U of the row before the slice (u0 on the first slice).
 * lam_pq[2][N] = (q, p): lam at row 0 = q + p * lam entering from above. */
int lifb_tshard_bwd(const float *I, const float *u_prev, const float *U, const float *GS, float *Lam,
                    float *lam_pq, int64_t T, int64_t N, float beta, float theta, float u_r,
                    float alpha, int C, void *ws, size_t bytes, void *stream);
/* Lam made exact for lam_top[N] entering from the next slice (after bwd, same ws). */
int lifb_tshard_bwd_fix(const float *I, const float *u_prev, const float *U, const float *GS,
                        const float *lam_top, float *Lam, int64_t T, int64_t N, float beta,
                        float theta, float alpha, int C, void *ws, size_t bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LIFSCAN_B200_H */
