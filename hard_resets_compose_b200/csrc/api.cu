// extern "C" entry points of liblifb (declared in include/lifscan_b200.h).
// Argument checks, workspace carving and kernel dispatch; no allocation, no
// synchronisation, no exceptions across the ABI.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <string>

#include "lifb_internal.h"
#include "tma.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

int fail(int status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int status, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int check_launch(const char *what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(LIFB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    g_last_error.clear();
    return LIFB_OK;
}

constexpr size_t kAlign = 256;

// Carves aligned sub-arrays from one workspace; with base == nullptr it only
// measures.
struct Carver {
    char *base;
    size_t off = 0;
    explicit Carver(void *b) : base((char *)b) {}
    template <class T>
    T *take(int64_t count)
    {
        off = (off + kAlign - 1) / kAlign * kAlign;
        T *p = base ? (T *)(base + off) : nullptr;
        off += (size_t)count * sizeof(T);
        return p;
    }
};

void carve_fwd(Carver &c, lifb::FwdMaps &mp, int64_t M, int64_t N, int K)
{
    mp.Lo = c.take<float>(M * N);
    mp.MA = c.take<float>(M * N);
    mp.MB = c.take<float>(M * N);
    mp.MX = c.take<float>(M * K * N);
    mp.MC = c.take<float>(M * K * N);
    mp.MN = c.take<int32_t>(M * N);
    mp.OVF = c.take<int32_t>(M * N);
    mp.Starts = c.take<float>(M * N);
    mp.Ends = c.take<float>(M * N);
}

void carve_super(Carver &c, lifb::SuperMaps &sp, int64_t M2, int64_t N, int K2)
{
    sp.SA = c.take<float>(M2 * N);
    sp.SB = c.take<float>(M2 * N);
    sp.SX = c.take<float>(M2 * K2 * N);
    sp.SC = c.take<float>(M2 * K2 * N);
    sp.SN = c.take<int32_t>(M2 * N);
    sp.SOVF = c.take<int32_t>(M2 * N);
    sp.SStarts = c.take<float>(M2 * N);
}

int check_common(const void *I, const void *u0, const void *U, const void *S, int64_t T, int64_t N,
                 bool s_optional = false)
{
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "negative shape T=%lld N=%lld", (long long)T, (long long)N);
    if (T > 0 && N > 0 && (!I || !u0 || !U || (!S && !s_optional)))
        return fail(LIFB_ERR_INVALID_ARGUMENT, "null tensor pointer");
    return LIFB_OK;
}

int check_ws(void *ws, size_t have, size_t need)
{
    if (need == 0) return LIFB_OK;
    if (!ws) return fail(LIFB_ERR_WORKSPACE, "workspace is NULL (need %zu bytes)", need);
    if ((uintptr_t)ws % kAlign) return fail(LIFB_ERR_WORKSPACE, "workspace not %zu-byte aligned", kAlign);
    if (have < need) return fail(LIFB_ERR_WORKSPACE, "workspace too small: %zu < %zu bytes", have, need);
    return LIFB_OK;
}

constexpr int64_t kMaxGridY = 65535;

// Chunks per replay segment for the fast v3 path: the largest power of two
// dividing M that still leaves enough (segment, 32-neuron) warps to keep every
// SM busy (about 8 per SM), so each warp replays one long segment.
int64_t segment_chunks(int64_t M, int64_t N)
{
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t warps_per_seg = (N + 31) / 32;
    const int64_t want = (8 * (int64_t)sms + warps_per_seg - 1) / warps_per_seg;  // segments wanted
    int64_t g = 1;
    while ((M % (2 * g)) == 0 && M / (2 * g) >= want) g *= 2;
    return g;
}

// Sequential carry: the TMA-staged kernel when it applies, else the plain one.
void carry_any(const float *I, const float *u0, const float *MA, const float *MB, const float *MX, const float *MC,
               const int32_t *MN, const int32_t *OVF, float *Starts, int64_t N, int64_t M, int64_t L, int K,
               float beta, float theta, float u_r, cudaStream_t s)
{
    if (!lifb::carry_staged(I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, L, K, beta, theta, u_r, s))
        lifb::grid_carry(I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, L, K, beta, theta, u_r, s);
}

}  // namespace

namespace lifb {
void count_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }
void set_last_error(const char *msg) { g_last_error = msg ? msg : ""; }
}  // namespace lifb

extern "C" {

int lifb_abi_version(void) { return 1; }

uint64_t lifb_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

const char *lifb_status_string(int status)
{
    switch (status) {
    case LIFB_OK: return "ok";
    case LIFB_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LIFB_ERR_CUDA: return "CUDA error";
    case LIFB_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case LIFB_ERR_UNSUPPORTED: return "unsupported configuration";
    case LIFB_ERR_DEVICE: return "device-side error reported by a kernel";
    default: return "unknown status";
    }
}

const char *lifb_last_error(void) { return g_last_error.c_str(); }

int lifb_device_status(int reset) { return lifb::read_device_status(reset != 0); }

static int device_code_status(int code, const char *who)
{
    if (code < 0) return fail(LIFB_ERR_CUDA, "%s: the device status could not be read", who);
    if (code == 0) {
        g_last_error.clear();
        return LIFB_OK;
    }
    if (code == lifb::kStatusTmaWaitTimeout)
        return fail(LIFB_ERR_DEVICE, "%s: device status %d: a bounded wait for an asynchronous copy expired; the "
                    "outputs of the calls before this check may be incomplete", who, code);
    return fail(LIFB_ERR_DEVICE, "%s: device status %d", who, code);
}

int lifb_check_device(int reset) { return device_code_status(lifb::read_device_status(reset != 0), "lifb_check_device"); }

int lifb_poll_device(void) { return device_code_status(lifb::poll_device_status(), "lifb_poll_device"); }

int lifb_serial_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                    float theta, float u_r, void *stream)
{
    LIFB_RANGE("lifb_serial_fwd");
    int st = check_common(I, u0, U, S, T, N);
    if (st) return st;
    if (T == 0 || N == 0) return LIFB_OK;
    lifb::serial_fwd(I, u0, U, S, T, N, beta, theta, u_r, (cudaStream_t)stream);
    return check_launch("lifb_serial_fwd");
}

int lifb_serial_bwd(const float *I, const float *u0, const float *U, const float *S, const float *GS,
                    const float *GU, float *Lam, int64_t T, int64_t N, float beta, float theta, float u_r,
                    float alpha, int detach, void *stream)
{
    LIFB_RANGE("lifb_serial_bwd");
    int st = check_common(I, u0, U, S, T, N, true);
    if (st) return st;
    if (T == 0 || N == 0) return LIFB_OK;
    if (!GS || !Lam) return fail(LIFB_ERR_INVALID_ARGUMENT, "null GS or Lam");
    lifb::serial_bwd(I, u0, U, S, GS, GU, Lam, T, N, beta, theta, u_r, alpha, detach != 0, (cudaStream_t)stream);
    return check_launch("lifb_serial_bwd");
}

size_t lifb_scan_fwd_v3_workspace_bytes(int64_t T, int64_t N, int C, int K)
{
    if (T <= 0 || N <= 0 || C <= 0 || K <= 0 || T % C) return 0;
    Carver c(nullptr);
    lifb::FwdMaps mp;
    carve_fwd(c, mp, T / C, N, K);
    return c.off;
}

static int check_scan_args(int64_t T, int C, int K, int64_t &M)
{
    if (C <= 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "chunk length C=%d must be positive", C);
    if (T % C) return fail(LIFB_ERR_INVALID_ARGUMENT, "T=%lld is not a multiple of C=%d", (long long)T, C);
    if (K < 1 || K > 64) return fail(LIFB_ERR_INVALID_ARGUMENT, "map capacity K=%d outside 1..64", K);
    M = T / C;
    if (M > kMaxGridY) return fail(LIFB_ERR_UNSUPPORTED, "T/C=%lld chunks exceeds %lld", (long long)M, (long long)kMaxGridY);
    return LIFB_OK;
}

int lifb_scan_fwd_v3(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                     float theta, float u_r, int C, int K, int max_repair, void *workspace,
                     size_t workspace_bytes, lifb_stats *stats_dev, void *stream)
{
    LIFB_RANGE("lifb_scan_fwd_v3");
    int st = check_common(I, u0, U, S, T, N);
    if (st) return st;
    int64_t M = 0;
    if ((st = check_scan_args(T, C, K, M))) return st;
    cudaStream_t s = (cudaStream_t)stream;
    if (stats_dev && cudaMemsetAsync(stats_dev, 0, sizeof(lifb_stats), s) != cudaSuccess)
        return check_launch("lifb_scan_fwd_v3: stats reset");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!stats_dev && max_repair < 0 && M > 1) {
        // When the slab of 32 neurons x T rows and its maps fit on chip, one
        // launch runs every phase (scan_block.cu) and needs no workspace.
        LIFB_RANGE("block scan");
        if (lifb::scan_block(I, u0, U, S, T, N, C, K, true, 0, beta, theta, u_r, nullptr, s))
            return check_launch("lifb_scan_fwd_v3");
    }
    size_t need = lifb_scan_fwd_v3_workspace_bytes(T, N, C, K);
    if ((st = check_ws(workspace, workspace_bytes, need))) return st;
    // Without stats the last chunk's map is never evaluated: build M-1 maps.
    // One chunk and no stats: the start is u0 and the scan is its replay alone.
    const int64_t Mb = stats_dev ? M : M - 1;
    if (Mb == 0) {
        lifb::serial_fwd(I, u0, U, S, T, N, beta, theta, u_r, s);
        return check_launch("lifb_scan_fwd_v3");
    }
    Carver c(workspace);
    lifb::FwdMaps mp;
    carve_fwd(c, mp, M, N, K);
    {
        LIFB_RANGE("envelope");
        lifb::grid_envelope(I, u0, mp, Mb, N, C, beta, u_r, s);
    }
    {
        LIFB_RANGE("chunk maps");
        lifb::grid_build(I, u0, mp, Mb, N, C, K, beta, theta, u_r, stats_dev, s);
    }
    if (!stats_dev && max_repair < 0) {
        // Fast path: carry every chunk start, replay segments of G chunks from
        // every G-th start, then fix the few segments whose start was not exact.
        {
            LIFB_RANGE("carry");
            carry_any(I, u0, mp.MA, mp.MB, mp.MX, mp.MC, mp.MN, mp.OVF, mp.Starts, N, M, C, K, beta, theta, u_r, s);
        }
        LIFB_RANGE("replay and fix-up");
        const int64_t G = segment_chunks(M, N);
        if (lifb::fwd_replay_tma(I, u0, mp.Starts, U, S, mp.Ends, T, N, (int64_t)C * G, beta, theta, u_r, s, G)) {
            // Lo and MN are free once the maps are built and carried
            lifb::fwd_fixup(I, mp.Starts, G, U, S, mp.Ends, mp.Lo, mp.MN, N, M / G, (int64_t)C * G, beta, theta, u_r,
                            nullptr, s);
            return check_launch("lifb_scan_fwd_v3");
        }
    } else {
        LIFB_RANGE("carry");
        lifb::grid_carry(I, u0, mp.MA, mp.MB, mp.MX, mp.MC, mp.MN, mp.OVF, mp.Starts, N, M, C, K, beta, theta, u_r,
                         s);
    }
    // chunk-level replay and the reference's round-by-round repair (stats, caps on rounds)
    LIFB_RANGE("replay and repair");
    lifb::grid_replay_repair(I, u0, mp, U, S, T, N, C, max_repair, beta, theta, u_r, stats_dev, s);
    return check_launch("lifb_scan_fwd_v3");
}

size_t lifb_scan_fwd_v4_workspace_bytes(int64_t T, int64_t N, int C, int G, int K, int K2)
{
    if (T <= 0 || N <= 0 || C <= 0 || G <= 0 || K <= 0 || K2 <= 0 || T % ((int64_t)C * G)) return 0;
    Carver c(nullptr);
    lifb::FwdMaps mp;
    lifb::SuperMaps sp;
    carve_fwd(c, mp, T / C, N, K);
    carve_super(c, sp, T / C / G, N, K2);
    return c.off;
}

int lifb_scan_fwd_v4(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                     float theta, float u_r, int C, int G, int K, int K2, int max_repair, void *workspace,
                     size_t workspace_bytes, lifb_stats *stats_dev, void *stream)
{
    LIFB_RANGE("lifb_scan_fwd_v4");
    int st = check_common(I, u0, U, S, T, N);
    if (st) return st;
    int64_t M = 0;
    if ((st = check_scan_args(T, C, K, M))) return st;
    if (G <= 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "group size G=%d must be positive", G);
    if (M % G) return fail(LIFB_ERR_INVALID_ARGUMENT, "T=%lld must be divisible by C*G=%lld", (long long)T, (long long)C * G);
    if (K2 < 1 || K2 > 64) return fail(LIFB_ERR_INVALID_ARGUMENT, "super capacity K2=%d outside 1..64", K2);
    cudaStream_t s = (cudaStream_t)stream;
    if (stats_dev && cudaMemsetAsync(stats_dev, 0, sizeof(lifb_stats), s) != cudaSuccess)
        return check_launch("lifb_scan_fwd_v4: stats reset");
    if (T == 0 || N == 0) return LIFB_OK;
    int64_t M2 = M / G;
    size_t need = lifb_scan_fwd_v4_workspace_bytes(T, N, C, G, K, K2);
    if ((st = check_ws(workspace, workspace_bytes, need))) return st;
    // Without stats the last chunk map and the last super map are never
    // evaluated, so they are not built.
    const int64_t Mb = stats_dev ? M : M - 1;
    const int64_t M2c = stats_dev ? M2 : M2 - 1;
    if (Mb == 0) {
        lifb::serial_fwd(I, u0, U, S, T, N, beta, theta, u_r, s);
        return check_launch("lifb_scan_fwd_v4");
    }
    Carver c(workspace);
    lifb::FwdMaps mp;
    lifb::SuperMaps sp;
    carve_fwd(c, mp, M, N, K);
    carve_super(c, sp, M2, N, K2);
    {
        LIFB_RANGE("envelope");
        lifb::grid_envelope(I, u0, mp, Mb, N, C, beta, u_r, s);
    }
    {
        LIFB_RANGE("chunk maps");
        lifb::grid_build(I, u0, mp, Mb, N, C, K, beta, theta, u_r, stats_dev, s);
    }
    if (M2c > 0) {
        LIFB_RANGE("super maps");
        lifb::grid_compose(mp, sp, u0, M2c, N, G, K, K2, theta, u_r, stats_dev, s);
    }
    if (!stats_dev && max_repair < 0) {
        // Fast path: carry the super maps, replay each super (C*G rows) from its
        // carried start, then fix the few supers whose start was not exact.
        {
            LIFB_RANGE("carry");
            carry_any(I, u0, sp.SA, sp.SB, sp.SX, sp.SC, sp.SN, sp.SOVF, sp.SStarts, N, M2, (int64_t)C * G, K2,
                      beta, theta, u_r, s);
        }
        LIFB_RANGE("replay and fix-up");
        if (lifb::fwd_replay_tma(I, u0, sp.SStarts, U, S, mp.Ends, T, N, (int64_t)C * G, beta, theta, u_r, s, 1)) {
            lifb::fwd_fixup(I, sp.SStarts, 1, U, S, mp.Ends, mp.Lo, mp.MN, N, M2, (int64_t)C * G, beta, theta, u_r,
                            nullptr, s);
            return check_launch("lifb_scan_fwd_v4");
        }
    }
    {
        LIFB_RANGE("carry");
        lifb::grid_carry(I, u0, sp.SA, sp.SB, sp.SX, sp.SC, sp.SN, sp.SOVF, sp.SStarts, N, M2, (int64_t)C * G, K2,
                         beta, theta, u_r, s);
        lifb::grid_carry_inner(I, mp, sp.SStarts, T, N, C, G, K, beta, theta, u_r, s);
    }
    LIFB_RANGE("replay and repair");
    lifb::grid_replay_repair(I, u0, mp, U, S, T, N, C, max_repair, beta, theta, u_r, stats_dev, s);
    return check_launch("lifb_scan_fwd_v4");
}

size_t lifb_scan_bwd_workspace_bytes(int64_t T, int64_t N, int C)
{
    if (T <= 0 || N <= 0 || C <= 0 || T % C) return 0;
    Carver c(nullptr);
    int64_t M = T / C;
    c.take<float>(M * N);
    c.take<float>(M * N);
    c.take<float>(M * N);
    return c.off;
}

int lifb_scan_bwd(const float *I, const float *u0, const float *U, const float *S, const float *GS,
                  const float *GU, float *Lam, int64_t T, int64_t N, float beta, float theta, float u_r,
                  float alpha, int detach, int C, void *workspace, size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_scan_bwd");
    int st = check_common(I, u0, U, S, T, N, true);
    if (st) return st;
    if (C <= 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "chunk length C=%d must be positive", C);
    if (T % C) return fail(LIFB_ERR_INVALID_ARGUMENT, "T=%lld is not a multiple of C=%d", (long long)T, C);
    if (T == 0 || N == 0) return LIFB_OK;
    if (!GS || !Lam) return fail(LIFB_ERR_INVALID_ARGUMENT, "null GS or Lam");
    int64_t M = T / C;
    if (M > kMaxGridY) return fail(LIFB_ERR_UNSUPPORTED, "T/C=%lld chunks exceeds %lld", (long long)M, (long long)kMaxGridY);
    if (M == 1) {  // one chunk: lam = 0 at its end, the scan is its replay alone
        lifb::serial_bwd(I, u0, U, S, GS, GU, Lam, T, N, beta, theta, u_r, alpha, detach != 0, (cudaStream_t)stream);
        return check_launch("lifb_scan_bwd");
    }
    size_t need = lifb_scan_bwd_workspace_bytes(T, N, C);
    if ((st = check_ws(workspace, workspace_bytes, need))) return st;
    Carver c(workspace);
    lifb::BwdScratch w;
    w.P = c.take<float>(M * N);
    w.Q = c.take<float>(M * N);
    w.LamEnd = c.take<float>(M * N);
    int32_t *D = reinterpret_cast<int32_t *>(w.LamEnd);  // the fast path needs no LamEnd
    bool replayed = false;
    if (detach) {
        LIFB_RANGE("chunks from lam_end = 0");
        replayed = lifb::bwd_tma(0, I, u0, U, S, GS, GU, nullptr, Lam, w.P, w.Q, T, N, C, beta, theta, u_r, alpha,
                                 true, (cudaStream_t)stream, D);
    }
    if (replayed) {
        // Detached reset: every chunk replayed from lam_end = 0 is exact at and
        // below its last spike; the fix-up corrects only the rows above it.
        LIFB_RANGE("fix-up above the last spikes");
        lifb::bwd_fixup(I, u0, U, S, GS, GU, w.P, w.Q, D, Lam, N, M, C, beta, theta, alpha, (cudaStream_t)stream);
        return check_launch("lifb_scan_bwd");
    }
    LIFB_RANGE("compose, carry, replay");
    lifb::grid_scan_bwd(I, u0, U, S, GS, GU, Lam, w, T, N, C, beta, theta, u_r, alpha, detach != 0,
                        (cudaStream_t)stream);
    return check_launch("lifb_scan_bwd");
}

size_t lifb_lif_fwd_bwd_host_workspace_bytes(int64_t T, int64_t N, int64_t block_n)
{
    return lifb::host_pipe_workspace_bytes(T, N, block_n);
}

int lifb_lif_fwd_bwd_host(const float *I_host, const float *GS_host, const float *u0_host, float *S_host,
                          float *dI_host, float *du0_host, int64_t T, int64_t N, float beta, float theta, float u_r,
                          float alpha, int64_t block_n, void *workspace, size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_lif_fwd_bwd_host");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "negative shape T=%lld N=%lld", (long long)T, (long long)N);
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I_host || !GS_host || !u0_host || !S_host || !dI_host || !du0_host)
        return fail(LIFB_ERR_INVALID_ARGUMENT, "null host pointer");
    if (block_n <= 0 || block_n % 4) return fail(LIFB_ERR_INVALID_ARGUMENT, "block_n=%lld must be a positive multiple of 4", (long long)block_n);
    int st;
    size_t need = lifb::host_pipe_workspace_bytes(T, N, block_n);
    if ((st = check_ws(workspace, workspace_bytes, need))) return st;
    const char *err = nullptr;
    st = lifb::host_pipe_run(I_host, GS_host, u0_host, S_host, dI_host, du0_host, T, N, beta, theta, u_r, alpha,
                             block_n, workspace, (cudaStream_t)stream, &err);
    if (st) return fail(st, "lifb_lif_fwd_bwd_host: %s", err ? err : "error");
    return check_launch("lifb_lif_fwd_bwd_host");
}

int64_t lifb_lif_fwd_bwd_host_rows_block(int64_t T, int64_t N)
{
    return lifb::host_pipe_rows_default_block(T, N);
}

size_t lifb_lif_fwd_bwd_host_rows_workspace_bytes(int64_t T, int64_t N, int64_t block_t)
{
    return lifb::host_pipe_rows_workspace_bytes(T, N, block_t);
}

int lifb_lif_fwd_bwd_host_rows(const float *I_host, const float *GS_host, const float *u0_host, float *S_host,
                               float *dI_host, float *du0_host, int64_t T, int64_t N, float beta, float theta,
                               float u_r, float alpha, int64_t block_t, void *workspace, size_t workspace_bytes,
                               void *stream)
{
    LIFB_RANGE("lifb_lif_fwd_bwd_host_rows");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "negative shape T=%lld N=%lld", (long long)T, (long long)N);
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I_host || !GS_host || !u0_host || !S_host || !dI_host || !du0_host)
        return fail(LIFB_ERR_INVALID_ARGUMENT, "null host pointer");
    if (block_t <= 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "block_t=%lld must be positive", (long long)block_t);
    if (N % 4) return fail(LIFB_ERR_UNSUPPORTED, "lifb_lif_fwd_bwd_host_rows needs N %% 4 == 0 (N=%lld)", (long long)N);
    int st;
    size_t need = lifb::host_pipe_rows_workspace_bytes(T, N, block_t);
    if ((st = check_ws(workspace, workspace_bytes, need))) return st;
    const char *err = nullptr;
    st = lifb::host_pipe_run_rows(I_host, GS_host, u0_host, S_host, dI_host, du0_host, T, N, beta, theta, u_r,
                                  alpha, block_t, workspace, (cudaStream_t)stream, &err);
    if (st) return fail(st, "lifb_lif_fwd_bwd_host_rows: %s", err ? err : "error");
    return check_launch("lifb_lif_fwd_bwd_host_rows");
}

}  // extern "C"
