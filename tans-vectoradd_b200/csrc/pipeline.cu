// pipeline.cu — host-memory front end of the fused decode + add
// (tans_b200_fp8_vecadd_fused_host): chunked host->device copies, the
// fused kernel on each chunk's stream range, and device->host copies of the
// output, pipelined over three CUDA streams so that the two copy directions
// and the kernels overlap.  Host code only; the kernel is reached through
// tans_b200_fp8_vecadd_fused_range.
//
// Chunks are whole 128-stream encoder blocks, so each chunk's compressed
// bytes are one contiguous range [offsets[b0], offsets[b1]); its
// sign/mantissa tiles and output tiles are column ranges of [N/16][K][8] /
// [N/16][K][16], copied with one 2D copy each.  The small metadata (offsets,
// states, partial counts, table) is copied whole before the first chunk.
// The device copies live at the same offsets in a caller-owned workspace,
// so the kernel sees the full-size layout.

#include "../../include/tans_b200.h"
#include "internal.h"

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

using tans_b200::fail;

namespace {

constexpr int64_t kBlk = TANS_B200_BLOCK_STREAMS;
constexpr int kPipeStreams = 3;
constexpr int kMaxDevices = 64;

struct Layout {  // workspace byte offsets
    int64_t a_comp, b_comp, a_off, b_off, a_st, b_st, a_part, b_part, a_sm, b_sm, table, out,
        total;
};

int64_t up256(int64_t x) { return (x + 255) & ~(int64_t)255; }

Layout layout(int64_t K, int64_t N, int64_t a_bytes, int64_t b_bytes) {
    const int64_t B = (K + kBlk - 1) / kBlk;
    Layout l;
    int64_t o = 0;
    auto take = [&](int64_t n) {
        const int64_t at = o;
        o = up256(o + n);
        return at;
    };
    l.a_comp = take(a_bytes);
    l.b_comp = take(b_bytes);
    l.a_off = take(4 * (B + 1));
    l.b_off = take(4 * (B + 1));
    l.a_st = take(2 * K);
    l.b_st = take(2 * K);
    l.a_part = take(K);
    l.b_part = take(K);
    l.a_sm = take(K * (N / 2));
    l.b_sm = take(K * (N / 2));
    l.table = take(4 * TANS_B200_TABLE_SIZE);
    l.out = take(K * N);
    l.total = o;
    return l;
}

// Per-device streams and events, created on first use and kept for the
// life of the process.
struct DevicePipe {
    bool ready = false;
    cudaStream_t s[kPipeStreams];
    cudaEvent_t fork, meta, join[kPipeStreams];
};
std::mutex g_pipe_mu;
DevicePipe g_pipe[kMaxDevices];

int cuda_fail(const char *what, cudaError_t e) {
    return fail(TANS_B200_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int pipe_for_device(DevicePipe **out) {
    int dev;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
    if (dev < 0 || dev >= kMaxDevices) return fail(TANS_B200_ERR_CUDA, "device id out of range");
    DevicePipe &p = g_pipe[dev];
    if (!p.ready) {
        for (int i = 0; i < kPipeStreams; i++) {
            if ((e = cudaStreamCreateWithFlags(&p.s[i], cudaStreamNonBlocking)) != cudaSuccess)
                return cuda_fail("cudaStreamCreateWithFlags", e);
            if ((e = cudaEventCreateWithFlags(&p.join[i], cudaEventDisableTiming)) != cudaSuccess)
                return cuda_fail("cudaEventCreateWithFlags", e);
        }
        if ((e = cudaEventCreateWithFlags(&p.fork, cudaEventDisableTiming)) != cudaSuccess ||
            (e = cudaEventCreateWithFlags(&p.meta, cudaEventDisableTiming)) != cudaSuccess)
            return cuda_fail("cudaEventCreateWithFlags", e);
        p.ready = true;
    }
    *out = &p;
    return TANS_B200_OK;
}

#define PIPE_CHECK(call)                                   \
    do {                                                   \
        cudaError_t e_ = (call);                           \
        if (e_ != cudaSuccess) return cuda_fail(#call, e_); \
    } while (0)

// Host-side checks of one input's offsets: monotone, 512-byte multiples,
// inside the compressed buffer (the kernel re-checks per block).
bool offsets_ok(const int32_t *off, int64_t B, int64_t bytes) {
    if (off[0] < 0) return false;
    for (int64_t b = 0; b < B; b++)
        if (off[b + 1] < off[b] || (off[b + 1] - off[b]) % 512 != 0) return false;
    return off[B] <= bytes;
}

}  // namespace

extern "C" int tans_b200_fp8_vecadd_fused_host_workspace_bytes(int64_t n_streams,
                                                               int64_t n_fp8_per_stream,
                                                               int64_t a_compressed_bytes,
                                                               int64_t b_compressed_bytes,
                                                               int64_t *bytes) {
    tans_b200::clear_error();
    if (!bytes || n_streams < 0 || n_fp8_per_stream < 0 || a_compressed_bytes < 0 ||
        b_compressed_bytes < 0)
        return fail(TANS_B200_ERR_INVALID, "fused_host_workspace_bytes: bad arguments");
    *bytes = layout(n_streams, n_fp8_per_stream, a_compressed_bytes, b_compressed_bytes).total;
    return TANS_B200_OK;
}

extern "C" int tans_b200_fp8_vecadd_fused_host(
    const uint8_t *a_comp, int64_t a_bytes, const int32_t *a_off, const uint16_t *a_st,
    const uint8_t *a_part, const uint8_t *a_sm, const uint8_t *b_comp, int64_t b_bytes,
    const int32_t *b_off, const uint16_t *b_st, const uint8_t *b_part, const uint8_t *b_sm,
    const int32_t *table, uint8_t *out, int64_t K, int64_t N, int64_t chunk_streams,
    void *workspace, int64_t workspace_bytes, int32_t *status, void *stream) {
    tans_b200::clear_error();
    if (N < 0 || N % 16 != 0)
        return fail(TANS_B200_ERR_INVALID, "n_fp8_per_stream must be divisible by 16");
    if (a_bytes < 0 || b_bytes < 0 || a_bytes % 4 != 0 || b_bytes % 4 != 0)
        return fail(TANS_B200_ERR_INVALID,
                    "compressed tensors must have byte lengths divisible by 4");
    if (K < 0) return fail(TANS_B200_ERR_INVALID, "n_streams must be >= 0");
    if (K == 0 || N == 0) return TANS_B200_OK;
    if (!a_comp || !a_off || !a_st || !a_part || !a_sm || !b_comp || !b_off || !b_st ||
        !b_part || !b_sm || !table || !out || !workspace)
        return fail(TANS_B200_ERR_INVALID, "fp8_vecadd_fused_host: null pointer");
    const Layout l = layout(K, N, a_bytes, b_bytes);
    if (workspace_bytes < l.total || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(TANS_B200_ERR_INVALID,
                    "fp8_vecadd_fused_host: workspace needs %lld bytes, 256-byte aligned",
                    (long long)l.total);
    const int64_t B = (K + kBlk - 1) / kBlk;
    if (!offsets_ok(a_off, B, a_bytes) || !offsets_ok(b_off, B, b_bytes))
        return fail(TANS_B200_ERR_INVALID, "fp8_vecadd_fused_host: malformed block offsets");
    int64_t chunk = chunk_streams > 0 ? chunk_streams : (K + 7) / 8;
    chunk = ((chunk + kBlk - 1) / kBlk) * kBlk;

    std::lock_guard<std::mutex> lk(g_pipe_mu);
    DevicePipe *p;
    int rc = pipe_for_device(&p);
    if (rc) return rc;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    uint8_t *d_a_comp = ws + l.a_comp, *d_b_comp = ws + l.b_comp;
    int32_t *d_a_off = reinterpret_cast<int32_t *>(ws + l.a_off);
    int32_t *d_b_off = reinterpret_cast<int32_t *>(ws + l.b_off);
    uint16_t *d_a_st = reinterpret_cast<uint16_t *>(ws + l.a_st);
    uint16_t *d_b_st = reinterpret_cast<uint16_t *>(ws + l.b_st);
    uint8_t *d_a_part = ws + l.a_part, *d_b_part = ws + l.b_part;
    uint8_t *d_a_sm = ws + l.a_sm, *d_b_sm = ws + l.b_sm;
    int32_t *d_table = reinterpret_cast<int32_t *>(ws + l.table);
    uint8_t *d_out = ws + l.out;
    const cudaStream_t user = (cudaStream_t)stream;
    const int64_t tiles = N / 16;

    // fork: every pipeline stream starts after the caller's prior work;
    // stream 0 brings the offsets and the table, the others wait for them
    PIPE_CHECK(cudaEventRecord(p->fork, user));
    for (int i = 0; i < kPipeStreams; i++) PIPE_CHECK(cudaStreamWaitEvent(p->s[i], p->fork, 0));
    // the small per-stream and per-block metadata goes over in one piece
    // each up front (a few hundred KB); the chunks carry only the bulk data
    PIPE_CHECK(cudaMemcpyAsync(d_a_off, a_off, 4 * (B + 1), cudaMemcpyHostToDevice, p->s[0]));
    PIPE_CHECK(cudaMemcpyAsync(d_b_off, b_off, 4 * (B + 1), cudaMemcpyHostToDevice, p->s[0]));
    PIPE_CHECK(cudaMemcpyAsync(d_table, table, 4 * TANS_B200_TABLE_SIZE, cudaMemcpyHostToDevice,
                               p->s[0]));
    PIPE_CHECK(cudaMemcpyAsync(d_a_st, a_st, 2 * K, cudaMemcpyHostToDevice, p->s[0]));
    PIPE_CHECK(cudaMemcpyAsync(d_b_st, b_st, 2 * K, cudaMemcpyHostToDevice, p->s[0]));
    PIPE_CHECK(cudaMemcpyAsync(d_a_part, a_part, K, cudaMemcpyHostToDevice, p->s[0]));
    PIPE_CHECK(cudaMemcpyAsync(d_b_part, b_part, K, cudaMemcpyHostToDevice, p->s[0]));
    PIPE_CHECK(cudaEventRecord(p->meta, p->s[0]));
    for (int i = 1; i < kPipeStreams; i++) PIPE_CHECK(cudaStreamWaitEvent(p->s[i], p->meta, 0));

    int c = 0;
    for (int64_t s0 = 0; s0 < K; s0 += chunk, c++) {
        const int64_t s1 = s0 + chunk < K ? s0 + chunk : K;
        const int64_t b0 = s0 / kBlk, b1 = (s1 + kBlk - 1) / kBlk;
        const cudaStream_t st = p->s[c % kPipeStreams];
        const int64_t ns = s1 - s0;
        PIPE_CHECK(cudaMemcpyAsync(d_a_comp + a_off[b0], a_comp + a_off[b0], a_off[b1] - a_off[b0],
                                   cudaMemcpyHostToDevice, st));
        PIPE_CHECK(cudaMemcpyAsync(d_b_comp + b_off[b0], b_comp + b_off[b0], b_off[b1] - b_off[b0],
                                   cudaMemcpyHostToDevice, st));
        PIPE_CHECK(cudaMemcpy2DAsync(d_a_sm + 8 * s0, 8 * K, a_sm + 8 * s0, 8 * K, 8 * ns, tiles,
                                     cudaMemcpyHostToDevice, st));
        PIPE_CHECK(cudaMemcpy2DAsync(d_b_sm + 8 * s0, 8 * K, b_sm + 8 * s0, 8 * K, 8 * ns, tiles,
                                     cudaMemcpyHostToDevice, st));
        rc = tans_b200_fp8_vecadd_fused_range(d_a_comp, a_bytes, d_a_off, d_a_st, d_a_part, d_a_sm,
                                              d_b_comp, b_bytes, d_b_off, d_b_st, d_b_part, d_b_sm,
                                              d_table, d_out, K, N, s0, s1, status, st);
        if (rc) return rc;
        PIPE_CHECK(cudaMemcpy2DAsync(out + 16 * s0, 16 * K, d_out + 16 * s0, 16 * K, 16 * ns, tiles,
                                     cudaMemcpyDeviceToHost, st));
    }
    // join: the caller's stream waits for every pipeline stream
    for (int i = 0; i < kPipeStreams; i++) {
        PIPE_CHECK(cudaEventRecord(p->join[i], p->s[i]));
        PIPE_CHECK(cudaStreamWaitEvent(user, p->join[i], 0));
    }
    return TANS_B200_OK;
}
