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
#include <mutex>

#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace lifb {

namespace {

constexpr int kMaxDev = 64;
constexpr int kSlots = 3;

struct HostPipe {
    cudaStream_t in = nullptr, out = nullptr;
    cudaEvent_t ev_in[kSlots] = {}, ev_gs[kSlots] = {}, ev_fwd[kSlots] = {}, ev_done[kSlots] = {},
                ev_free[kSlots] = {}, ev_start = nullptr, ev_last = nullptr;
    bool ready = false;
};
HostPipe g_pipe[kMaxDev];
std::mutex g_pipe_mu;

// Destroys whatever handles of q were created (a set that failed half-way).
void destroy_pipe(HostPipe &q)
{
    if (q.in) cudaStreamDestroy(q.in);
    if (q.out) cudaStreamDestroy(q.out);
    cudaEvent_t *sets[] = {q.ev_in, q.ev_gs, q.ev_fwd, q.ev_done, q.ev_free};
    for (cudaEvent_t *set : sets)
        for (int i = 0; i < kSlots; i++)
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
        for (int i = 0; ok && i < kSlots; i++)
            ok = cudaEventCreateWithFlags(&q.ev_in[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&q.ev_gs[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&q.ev_fwd[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&q.ev_done[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&q.ev_free[i], cudaEventDisableTiming) == cudaSuccess;
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

}  // namespace lifb
