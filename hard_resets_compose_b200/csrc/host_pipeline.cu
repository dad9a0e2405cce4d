// lifb_lif_fwd_bwd_host: forward + adjoint of the lif_tuned layer for
// host-resident tensors, pipelined over blocks of neurons.
//
// Neuron columns of [T, N] are independent recurrences, so the problem splits
// into column blocks of `block_n` neurons.  Block b moves through three
// streams: an input stream copies its columns of u0 and I, then of GS,
// host->device (cudaMemcpy2DAsync, pitched); the caller's stream runs the
// forward as soon as I has arrived (saving V, the pre-reset potentials, as
// lif_tuned does) and the adjoint from V and GS once GS has; an output stream
// copies S back as soon as the forward is done, then dI and du0.  Three
// staging slots in the caller's device workspace keep both PCIe directions
// busy at once (B200: ~55 GB/s each way alone, ~95 GB/s both ways together),
// so the call is bound by their joint rate instead of the sum of both.
//
// lifb_lif_fwd_bwd_host_rows: the same over blocks of time rows.  A block of
// rows of a row-major [T, N] array is one contiguous range of host memory, so
// every copy is a single linear transfer, and the first output can leave as
// soon as the first (small) input block has arrived.  The forward runs block
// after block in time order, each from the state the previous one ended in
// (the replay kernel's end states); the adjoint runs the blocks in reverse
// order, each from the lam its successor left in its first row.  V of all
// rows stays on the device between the two sweeps; I, S, GS and Lam pass
// through four staging slots.  The input stream copies I in time order, then
// GS in reverse order; the output stream returns S in time order, then dI in
// reverse order, each one block behind.
#include <mutex>

#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace lifb {

namespace {

constexpr int kMaxDev = 64;
constexpr int kSlots = 3;     // column blocks
constexpr int kRowSlots = 4;  // row blocks
constexpr int kEv = kRowSlots;

// Rows per block of the row form: blocks of about this many bytes per array.
#ifndef LIFB_HOST_BLOCK_BYTES
#define LIFB_HOST_BLOCK_BYTES (16 << 20)
#endif

struct HostPipe {
    cudaStream_t in = nullptr, out = nullptr;
    cudaEvent_t ev_in[kEv] = {}, ev_gs[kEv] = {}, ev_fwd[kEv] = {}, ev_done[kEv] = {}, ev_free[kEv] = {},
                ev_sout[kEv] = {}, ev_start = nullptr, ev_last = nullptr;
    bool ready = false;
};
HostPipe g_pipe[kMaxDev];
std::mutex g_pipe_mu;

// Destroys whatever handles of q were created (a set that failed half-way).
void destroy_pipe(HostPipe &q)
{
    if (q.in) cudaStreamDestroy(q.in);
    if (q.out) cudaStreamDestroy(q.out);
    cudaEvent_t *sets[] = {q.ev_in, q.ev_gs, q.ev_fwd, q.ev_done, q.ev_free, q.ev_sout};
    for (cudaEvent_t *set : sets)
        for (int i = 0; i < kEv; i++)
            if (set[i]) cudaEventDestroy(set[i]);
    if (q.ev_start) cudaEventDestroy(q.ev_start);
    if (q.ev_last) cudaEventDestroy(q.ev_last);
    q = HostPipe{};
}

// Streams and events of the current device, created once (no memory is
// allocated); a set that cannot be created completely is released again and
// the next call tries anew.
HostPipe *pipe_for_current_device()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
    std::lock_guard<std::mutex> g(g_pipe_mu);
    HostPipe &p = g_pipe[dev];
    if (!p.ready) {
        HostPipe q;
        bool ok = cudaStreamCreateWithFlags(&q.in, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&q.out, cudaStreamNonBlocking) == cudaSuccess;
        for (int i = 0; ok && i < kEv; i++)
            ok = cudaEventCreateWithFlags(&q.ev_in[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&q.ev_gs[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&q.ev_fwd[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&q.ev_done[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&q.ev_free[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&q.ev_sout[i], cudaEventDisableTiming) == cudaSuccess;
        ok = ok && cudaEventCreateWithFlags(&q.ev_last, cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&q.ev_start, cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            destroy_pipe(q);
            return nullptr;
        }
        q.ready = true;
        p = q;
    }
    return &p;
}

// du0 = beta * Lam[0] for one block.
__global__ void k_scale_row(const float *__restrict__ row, float beta, float *__restrict__ out, int64_t n)
{
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = beta * row[i];
}

struct Slot {
    float *I, *GS, *V, *S, *Lam, *u0, *du0;
};

}  // namespace

size_t host_pipe_workspace_bytes(int64_t T, int64_t N, int64_t block_n)
{
    if (T <= 0 || N <= 0 || block_n <= 0) return 0;
    const int64_t nb = block_n < N ? block_n : N;
    // each array 256-byte aligned
    const size_t per = ((size_t)T * nb * 4 + 255) / 256 * 256 * 5 + ((size_t)nb * 4 + 255) / 256 * 256 * 2;
    return per * kSlots;
}

int host_pipe_run(const float *I_h, const float *GS_h, const float *u0_h, float *S_h, float *dI_h, float *du0_h,
                  int64_t T, int64_t N, float beta, float theta, float u_r, float alpha, int64_t block_n,
                  void *workspace, cudaStream_t cs, const char **err)
{
    HostPipe *p = pipe_for_current_device();
    if (!p) {
        *err = "could not create the copy streams/events of the current device";
        return LIFB_ERR_CUDA;
    }
    const int64_t nb_max = block_n < N ? block_n : N;
    const size_t big = ((size_t)T * nb_max * 4 + 255) / 256 * 256;
    const size_t small = ((size_t)nb_max * 4 + 255) / 256 * 256;
    Slot slot[kSlots];
    char *w = (char *)workspace;
    for (int i = 0; i < kSlots; i++) {
        slot[i].I = (float *)w; w += big;
        slot[i].GS = (float *)w; w += big;
        slot[i].V = (float *)w; w += big;
        slot[i].S = (float *)w; w += big;
        slot[i].Lam = (float *)w; w += big;
        slot[i].u0 = (float *)w; w += small;
        slot[i].du0 = (float *)w; w += small;
    }
    // nothing of this call starts before the work already queued on the
    // caller's stream (a previous call may still be using the staging slots)
    cudaEventRecord(p->ev_start, cs);
    cudaStreamWaitEvent(p->in, p->ev_start, 0);
    cudaStreamWaitEvent(p->out, p->ev_start, 0);
    const size_t hp = (size_t)N * 4;  // host pitch
    // The first block's input and the last block's output cross PCIe with
    // nothing to overlap: make those two blocks half as wide (4-neuron aligned).
    const int64_t half = nb_max >= 8 ? (nb_max / 2) / 4 * 4 : nb_max;
    const bool split_ends = N > 2 * nb_max;
    int64_t n0 = 0;
    for (int64_t b = 0; n0 < N; b++) {
        const int k = (int)(b % kSlots);
        int64_t nb = nb_max;
        if (split_ends && (b == 0 || N - n0 <= half)) nb = half;
        if (nb > N - n0) nb = N - n0;
        if (split_ends && N - n0 - nb > 0 && N - n0 - nb < half) nb = N - n0 - half;  // leave a half block last
        const size_t dp = (size_t)nb * 4;  // device pitch (block is contiguous [T, nb])
        Slot &s = slot[k];
        // input: wait until the slot's previous outputs have left the device
        if (b >= kSlots) cudaStreamWaitEvent(p->in, p->ev_free[k], 0);
        cudaMemcpyAsync(s.u0, u0_h + n0, dp, cudaMemcpyHostToDevice, p->in);
        cudaMemcpy2DAsync(s.I, dp, I_h + n0, hp, dp, (size_t)T, cudaMemcpyHostToDevice, p->in);
        cudaEventRecord(p->ev_in[k], p->in);
        cudaMemcpy2DAsync(s.GS, dp, GS_h + n0, hp, dp, (size_t)T, cudaMemcpyHostToDevice, p->in);
        cudaEventRecord(p->ev_gs[k], p->in);
        // compute on the caller's stream: the forward needs I only
        cudaStreamWaitEvent(cs, p->ev_in[k], 0);
        serial_fwd_v(s.I, s.u0, s.V, s.S, T, nb, beta, theta, u_r, cs);
        cudaEventRecord(p->ev_fwd[k], cs);
        cudaStreamWaitEvent(cs, p->ev_gs[k], 0);
        serial_bwd_v(s.V, s.GS, s.Lam, T, nb, beta, theta, alpha, cs);
        count_launches(1);
        k_scale_row<<<(unsigned)((nb + 255) / 256), 256, 0, cs>>>(s.Lam, beta, s.du0, nb);
        cudaEventRecord(p->ev_done[k], cs);
        // output: S as soon as the forward is done, then dI and du0
        cudaStreamWaitEvent(p->out, p->ev_fwd[k], 0);
        cudaMemcpy2DAsync(S_h + n0, hp, s.S, dp, dp, (size_t)T, cudaMemcpyDeviceToHost, p->out);
        cudaStreamWaitEvent(p->out, p->ev_done[k], 0);
        cudaMemcpy2DAsync(dI_h + n0, hp, s.Lam, dp, dp, (size_t)T, cudaMemcpyDeviceToHost, p->out);
        cudaMemcpyAsync(du0_h + n0, s.du0, dp, cudaMemcpyDeviceToHost, p->out);
        cudaEventRecord(p->ev_free[k], p->out);
        n0 += nb;
    }
    // the caller's stream completes only after the last output copy
    cudaEventRecord(p->ev_last, p->out);
    cudaStreamWaitEvent(cs, p->ev_last, 0);
    return LIFB_OK;
}

namespace {

size_t al256(size_t b) { return (b + 255) / 256 * 256; }

// Workspace of the row form: V [T, N], then per slot I, S, GS, Lam blocks
// [block_t, N], then u0, two end-state buffers and du0 [N].
struct RowWs {
    float *V, *I[kRowSlots], *S[kRowSlots], *GS[kRowSlots], *Lam[kRowSlots], *u0, *ust[2], *du0;
};

size_t row_ws_layout(int64_t T, int64_t N, int64_t bt, void *base, RowWs *w)
{
    const size_t full = al256((size_t)T * N * 4), blk = al256((size_t)bt * N * 4), vec = al256((size_t)N * 4);
    if (w) {
        char *c = (char *)base;
        w->V = (float *)c; c += full;
        for (int j = 0; j < kRowSlots; j++) {
            w->I[j] = (float *)c; c += blk;
            w->S[j] = (float *)c; c += blk;
            w->GS[j] = (float *)c; c += blk;
            w->Lam[j] = (float *)c; c += blk;
        }
        w->u0 = (float *)c; c += vec;
        w->ust[0] = (float *)c; c += vec;
        w->ust[1] = (float *)c; c += vec;
        w->du0 = (float *)c;
    }
    return full + (size_t)kRowSlots * 4 * blk + 4 * vec;
}

}  // namespace

int64_t host_pipe_rows_default_block(int64_t T, int64_t N)
{
    if (T <= 0 || N <= 0) return 0;
    int64_t bt = (int64_t)LIFB_HOST_BLOCK_BYTES / (N * 4);
    if (bt < 1) bt = 1;
    return bt < T ? bt : T;
}

size_t host_pipe_rows_workspace_bytes(int64_t T, int64_t N, int64_t block_t)
{
    if (T <= 0 || N <= 0 || block_t <= 0) return 0;
    return row_ws_layout(T, N, block_t < T ? block_t : T, nullptr, nullptr);
}

int host_pipe_run_rows(const float *I_h, const float *GS_h, const float *u0_h, float *S_h, float *dI_h,
                       float *du0_h, int64_t T, int64_t N, float beta, float theta, float u_r, float alpha,
                       int64_t block_t, void *workspace, cudaStream_t cs, const char **err)
{
    if (N % 4) {
        *err = "the row-block pipeline needs N % 4 == 0";
        return LIFB_ERR_UNSUPPORTED;
    }
    HostPipe *p = pipe_for_current_device();
    if (!p) {
        *err = "could not create the copy streams/events of the current device";
        return LIFB_ERR_CUDA;
    }
    const int64_t bt = block_t < T ? block_t : T;
    const int64_t nblk = (T + bt - 1) / bt;
    RowWs w;
    row_ws_layout(T, N, bt, workspace, &w);
    const size_t row_bytes = (size_t)N * 4;
    auto rows_of = [&](int64_t k) { return (k + 1) * bt <= T ? bt : T - k * bt; };

    cudaEventRecord(p->ev_start, cs);
    cudaStreamWaitEvent(p->in, p->ev_start, 0);
    cudaStreamWaitEvent(p->out, p->ev_start, 0);
    cudaMemcpyAsync(w.u0, u0_h, row_bytes, cudaMemcpyHostToDevice, p->in);
    // forward, blocks in time order
    for (int64_t k = 0; k < nblk; k++) {
        const int j = (int)(k % kRowSlots);
        const int64_t r = rows_of(k), off = k * bt * N;
        if (k >= kRowSlots) cudaStreamWaitEvent(p->in, p->ev_fwd[j], 0);  // I slot j consumed
        cudaMemcpyAsync(w.I[j], I_h + off, (size_t)r * row_bytes, cudaMemcpyHostToDevice, p->in);
        cudaEventRecord(p->ev_in[j], p->in);
        cudaStreamWaitEvent(cs, p->ev_in[j], 0);
        if (k >= kRowSlots) cudaStreamWaitEvent(cs, p->ev_sout[j], 0);  // S slot j copied out
        const float *uin = k == 0 ? w.u0 : w.ust[(k - 1) & 1];
        if (!fwd_replay_tma(w.I[j], uin, nullptr, w.V + off, w.S[j], w.ust[k & 1], r, N, r, beta, theta, u_r, cs,
                            1, 0, nullptr, true)) {
            *err = "the TMA forward refused a row block";
            return LIFB_ERR_CUDA;
        }
        cudaEventRecord(p->ev_fwd[j], cs);
        cudaStreamWaitEvent(p->out, p->ev_fwd[j], 0);
        cudaMemcpyAsync(S_h + off, w.S[j], (size_t)r * row_bytes, cudaMemcpyDeviceToHost, p->out);
        cudaEventRecord(p->ev_sout[j], p->out);
    }
    // adjoint, blocks in reverse order; q counts the blocks processed
    for (int64_t q = 0; q < nblk; q++) {
        const int64_t k = nblk - 1 - q;
        const int j = (int)(q % kRowSlots);
        const int64_t r = rows_of(k), off = k * bt * N;
        if (q >= kRowSlots) cudaStreamWaitEvent(p->in, p->ev_done[j], 0);  // GS slot j consumed
        cudaMemcpyAsync(w.GS[j], GS_h + off, (size_t)r * row_bytes, cudaMemcpyHostToDevice, p->in);
        cudaEventRecord(p->ev_gs[j], p->in);
        cudaStreamWaitEvent(cs, p->ev_gs[j], 0);
        if (q >= kRowSlots) cudaStreamWaitEvent(cs, p->ev_free[j], 0);  // Lam slot j copied out
        // lam entering from the row after the block: row 0 of the block processed before
        const float *lam_end = q == 0 ? nullptr : w.Lam[(q - 1) % kRowSlots];
        if (!bwd_tma_v(w.V + off, w.GS[j], w.Lam[j], nullptr, nullptr, nullptr, r, N, r, beta, theta, alpha, cs,
                       lam_end)) {
            *err = "the TMA adjoint refused a row block";
            return LIFB_ERR_CUDA;
        }
        if (k == 0) {
            count_launches(1);
            k_scale_row<<<(unsigned)((N + 255) / 256), 256, 0, cs>>>(w.Lam[j], beta, w.du0, N);
        }
        cudaEventRecord(p->ev_done[j], cs);
        cudaStreamWaitEvent(p->out, p->ev_done[j], 0);
        cudaMemcpyAsync(dI_h + off, w.Lam[j], (size_t)r * row_bytes, cudaMemcpyDeviceToHost, p->out);
        if (k == 0) cudaMemcpyAsync(du0_h, w.du0, row_bytes, cudaMemcpyDeviceToHost, p->out);
        cudaEventRecord(p->ev_free[j], p->out);
    }
    cudaEventRecord(p->ev_last, p->out);
    cudaStreamWaitEvent(cs, p->ev_last, 0);
    return LIFB_OK;
}

}  // namespace lifb
