/*
 * tans_b200.h — C ABI of the B200 (sm_100a) tANS FP8 decode library.
 *
 * Every entry point takes plain pointers and sizes, returns an int status
 * (TANS_B200_OK == 0) and never allocates device memory: callers own every
 * buffer.  Device entry points enqueue work on the given CUDA stream
 * (cudaStream_t passed as void*; NULL = legacy default stream) on the device
 * that is current on the calling thread, and return without synchronising.
 * On failure, tans_b200_last_error() returns a message for the calling thread.
 *
 * Data formats are those of the reference (doublewordai/tans-vectoradd):
 *   - pair symbols: sym = exp(elem 2i) << 4 | exp(elem 2i+1), alphabet 256,
 *     rans_vectoradd/tans_codec.py:109-124
 *   - sign/mantissa pairs: sm = sm(elem 2i) | sm(elem 2i+1) << 4,
 *     rans_vectoradd/tans_codec.py:110-113
 *   - slab layout: 128-stream encoder blocks, G_b uint32 slabs per stream,
 *     slab g of stream t at byte offsets[b] + g*512 + 4*t, streams top-aligned,
 *     csrc/tans_codec.cpp:139-181
 *   - decode table: int32[4096], sym | nb << 8 | base << 16,
 *     rans_vectoradd/tans_codec.py:63-87, csrc/tans_decode.cu:23-59
 */
#ifndef TANS_B200_H
#define TANS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define TANS_B200_OK 0
#define TANS_B200_ERR_INVALID 1 /* bad argument (size, alignment, null)   */
#define TANS_B200_ERR_CUDA 2    /* a CUDA runtime call failed            */
#define TANS_B200_ERR_HOST 3    /* host-side failure (allocation, ...)   */

/* Device-side data-error bits, OR-ed into the optional `status` word that
 * the decode entry points take (a device int32, may be NULL).  Malformed
 * metadata never makes a kernel read out of bounds; it is reported here. */
#define TANS_B200_DATA_BAD_OFFSETS 1 /* block offsets not monotone/in range */
#define TANS_B200_DATA_BAD_STATE 2   /* initial state outside [L, 2L)       */
#define TANS_B200_DATA_BAD_TABLE 4   /* spread/freqs/table entry malformed  */
#define TANS_B200_DATA_TIMEOUT 8     /* a bounded in-kernel wait ran out    */

/* Table size L = M (tans_codec.py:24-25).  4096 is the reference's and the
 * parity build; the library is also built with -DTANS_B200_TABLE_SIZE=2048
 * (table_log 11, libtans_b200_l11.so) as a labelled extra. */
#ifndef TANS_B200_TABLE_SIZE
#define TANS_B200_TABLE_SIZE 4096
#endif
#define TANS_B200_BLOCK_STREAMS 128 /* tans_codec.py:27          */

/* Message for the last failed call on this thread ("" if none). */
const char *tans_b200_last_error(void);
/* L of this build (4096, or 2048 for the table_log 11 build).  The
 * reference fixes L = 4096 (tans_codec.py:24-25); no counterpart. */
int tans_b200_table_size(void);
/* Library version string. */
const char *tans_b200_version(void);

/* ---------------------------------------------------------------- host */

/* Build the reference decode table (tans_codec.py:63-87; its C++ twin is
 * csrc/tans_decode.cu:23-59).  spread[4096] slot->symbol, freqs[n_syms]
 * summing to 4096.  Writes table[4096]. */
int tans_b200_build_decode_table_host(const int32_t *spread,
                                      const int32_t *freqs, int64_t n_syms,
                                      int32_t *table);

/* CPU slab encoder: replaces `tans_encode_interleaved`
 * (csrc/tans_codec.cpp:69-196).  Two-phase so that the caller allocates the
 * outputs:
 *   1. tans_b200_encode(...) encodes symbols[K][N] (host, row-major) with
 *      OpenMP over streams and returns an opaque handle;
 *   2. tans_b200_encoded_sizes() reports the compressed byte count and the
 *      number of encoder blocks B = ceil(K/128);
 *   3. tans_b200_encoded_export() copies compressed[bytes] (uint8),
 *      states[K] (uint16), offsets[B+1] (int32), partial[K] (uint8) into
 *      caller buffers; output bytes are identical to the reference's;
 *   4. tans_b200_encoded_free() releases the handle.
 * `symbols` is borrowed: it must stay valid and unchanged until export.
 * n_threads <= 0 uses the OpenMP default.  A symbol with zero frequency, a
 * spread inconsistent with freqs, or freqs not summing to 4096 is an error
 * (TANS_B200_ERR_INVALID). */
typedef struct tans_b200_encoded tans_b200_encoded;
int tans_b200_encode(const uint8_t *symbols, int64_t K, int64_t N,
                     const int32_t *freqs, int64_t n_syms,
                     const int32_t *spread, int n_threads,
                     tans_b200_encoded **out);
int tans_b200_encoded_sizes(const tans_b200_encoded *enc,
                            int64_t *compressed_bytes, int64_t *n_blocks);
int tans_b200_encoded_export(const tans_b200_encoded *enc, uint8_t *compressed,
                             uint16_t *states, int32_t *offsets,
                             uint8_t *partial);
void tans_b200_encoded_free(tans_b200_encoded *enc);

/* Split e4m3 bytes fp8[K][N] (N even) into the encoder's inputs, as
 * rans_vectoradd/tans_codec.py:105-124 does with torch ops:
 *   pair_syms[K][N/2] = exp(2i) << 4 | exp(2i+1),  exp = (b >> 3) & 15
 *   sm = sm(2i) | sm(2i+1) << 4,  sm = ((b >> 4) & 8) | (b & 7), laid out
 *   [N/2/tile][K][tile] when tile > 0, else [N/2][K]
 * exp_hist[16] (optional) is incremented by the exponent histogram.
 * Either output may be NULL. */
int tans_b200_split_fp8(const uint8_t *fp8, int64_t K, int64_t N,
                        int64_t tile, uint8_t *pair_syms, uint8_t *sm,
                        int64_t *exp_hist, int n_threads);

/* -------------------------------------------------------------- device */

/* Number of SMs of the current device (cached per device). */
int tans_b200_sm_count(int *sm_count);

/* C = A: replaces `fp8_memcpy` (csrc/fp8_memcpy.cu:45-64).
 * n bytes, n % 16 == 0, 16-byte aligned pointers. */
int tans_b200_fp8_memcpy(const uint8_t *a, uint8_t *c, int64_t n,
                         void *stream);

/* C[i] = e4m3_satfinite(A[i] + B[i]): replaces `fp8_vecadd_raw`
 * (csrc/vecadd.cu:268-288).  n % 16 == 0, 16-byte aligned pointers. */
int tans_b200_fp8_vecadd_raw(const uint8_t *a, const uint8_t *b, uint8_t *c,
                             int64_t n, void *stream);

/* Build the reference-format decode table on the device from device copies
 * of spread[4096] and freqs[n_syms] (n_syms <= 256).  This is the step that
 * `gpu_tans_decode` performs on the host for every call
 * (csrc/tans_decode.cu:23-59, :389).  table: device int32[4096].
 * status: optional device int32; TANS_B200_DATA_BAD_TABLE is OR-ed in when
 * spread/freqs are inconsistent (the entries concerned are written as 0). */
int tans_b200_build_decode_table(const int32_t *spread, const int32_t *freqs,
                                 int64_t n_syms, int32_t *table,
                                 int32_t *status, void *stream);

/* Standalone decode: replaces `gpu_tans_decode` (csrc/tans_decode.cu:159-210)
 * given a device decode table.
 *   compressed[compressed_bytes], offsets[B+1], states[K], partial[K],
 *   sign_mantissa[N/2][K] -> out[N][K] (element j of stream k at j*K + k).
 * N = n_fp8_per_stream (even).  status: optional device int32 (OR-ed data
 * error bits), may be NULL. */
int tans_b200_decode(const uint8_t *compressed, int64_t compressed_bytes,
                     const int32_t *offsets, const uint16_t *states,
                     const uint8_t *partial, const uint8_t *sign_mantissa,
                     const int32_t *decode_table, uint8_t *out,
                     int64_t n_streams, int64_t n_fp8_per_stream,
                     int32_t *status, void *stream);

/* Standalone decode of split streams (format of
 * tans_b200_fp8_vecadd_fused_split: K*P/S sub-streams of S pair symbols,
 * segment-major; sign_mantissa [N/2][K] and out [N][K] unchanged).
 * segment_pairs divides N/2; more than one segment needs K % 32 == 0. */
int tans_b200_decode_split(const uint8_t *compressed, int64_t compressed_bytes,
                           const int32_t *offsets, const uint16_t *states,
                           const uint8_t *partial, const uint8_t *sign_mantissa,
                           const int32_t *decode_table, uint8_t *out,
                           int64_t n_streams, int64_t n_fp8_per_stream,
                           int64_t segment_pairs, int32_t *status,
                           void *stream);

/* Fused decode + FP8 add: replaces `fp8_vecadd_fused_tans`
 * (csrc/vecadd.cu:290-393).  Both inputs share decode_table and the stream
 * count K; sm tensors are tiled [N/16][K][8]; out is tiled [N/16][K][16]
 * (element 16j+t of stream k at (j*K + k)*16 + t).  N % 16 == 0.
 * status: optional device int32, may be NULL. */
int tans_b200_fp8_vecadd_fused(
    const uint8_t *a_compressed, int64_t a_compressed_bytes,
    const int32_t *a_offsets, const uint16_t *a_states,
    const uint8_t *a_partial, const uint8_t *a_sm,
    const uint8_t *b_compressed, int64_t b_compressed_bytes,
    const int32_t *b_offsets, const uint16_t *b_states,
    const uint8_t *b_partial, const uint8_t *b_sm,
    const int32_t *decode_table, uint8_t *out, int64_t n_streams,
    int64_t n_fp8_per_stream, int32_t *status, void *stream);

/* The same on the streams [stream_begin, stream_end) of the K-stream layout
 * only (stream_begin a multiple of 128: whole encoder blocks).  All pointers
 * and K are those of the full tensors; only the range is read and written.
 * No reference counterpart: it lets callers split one call across CUDA
 * streams or pipeline it with host transfers. */
int tans_b200_fp8_vecadd_fused_range(
    const uint8_t *a_compressed, int64_t a_compressed_bytes,
    const int32_t *a_offsets, const uint16_t *a_states,
    const uint8_t *a_partial, const uint8_t *a_sm,
    const uint8_t *b_compressed, int64_t b_compressed_bytes,
    const int32_t *b_offsets, const uint16_t *b_states,
    const uint8_t *b_partial, const uint8_t *b_sm,
    const int32_t *decode_table, uint8_t *out, int64_t n_streams,
    int64_t n_fp8_per_stream, int64_t stream_begin, int64_t stream_end,
    int32_t *status, void *stream);

/* Fused decode + FP8 add on split streams (a format extension; no
 * reference counterpart).  Each stream of P = N/2 pair symbols is encoded as
 * P/S independent sub-streams of S = segment_pairs pair symbols, sub-stream
 * (segment j, stream k) at index j*K + k of the compressed/offsets/states/
 * partial arrays (K*P/S entries, ceil(K*P/S / 128) + 1 offsets) — exactly
 * what tans_b200_encode produces from the pair-symbol matrix rearranged to
 * [P/S * K][S].  The sign/mantissa tensors and the output keep the
 * unsplit layouts ([N/16][K][8], [N/16][K][16]).  Long streams then decode
 * as P/S times as many chains.  segment_pairs: a multiple of 8 dividing
 * N/2 (segment_pairs == N/2 is the unsplit format); with more than one
 * segment K must be a multiple of 32. */
int tans_b200_fp8_vecadd_fused_split(
    const uint8_t *a_compressed, int64_t a_compressed_bytes,
    const int32_t *a_offsets, const uint16_t *a_states,
    const uint8_t *a_partial, const uint8_t *a_sm,
    const uint8_t *b_compressed, int64_t b_compressed_bytes,
    const int32_t *b_offsets, const uint16_t *b_states,
    const uint8_t *b_partial, const uint8_t *b_sm,
    const int32_t *decode_table, uint8_t *out, int64_t n_streams,
    int64_t n_fp8_per_stream, int64_t segment_pairs, int32_t *status,
    void *stream);

/* Fused decode + FP8 add from and to HOST memory (no reference counterpart;
 * the reference's op takes device tensors).  All a_* / b_* inputs,
 * decode_table and out are host pointers, in the layouts of
 * tans_b200_fp8_vecadd_fused; page-locked memory lets the copies overlap.
 * The streams are split into chunks of whole encoder blocks
 * (chunk_streams, rounded up to 128; <= 0 picks K/8) and pipelined over
 * three internal CUDA streams: chunk c's host->device copies, its kernel and
 * its device->host copy of the output run while neighbouring chunks copy in
 * the other direction.  The work is ordered after `stream`'s prior work and
 * `stream` waits for all of it, so the call is asynchronous like a
 * cudaMemcpyAsync: host buffers must stay valid until `stream` reaches that
 * point.  `workspace` is a caller-owned device buffer of
 * tans_b200_fp8_vecadd_fused_host_workspace_bytes() bytes (256-byte
 * aligned) that holds the device copies.  Calls on one device enqueue under
 * a library lock; calls whose work overlaps must not share a workspace. */
int tans_b200_fp8_vecadd_fused_host_workspace_bytes(
    int64_t n_streams, int64_t n_fp8_per_stream, int64_t a_compressed_bytes,
    int64_t b_compressed_bytes, int64_t *bytes);

int tans_b200_fp8_vecadd_fused_host(
    const uint8_t *a_compressed, int64_t a_compressed_bytes,
    const int32_t *a_offsets, const uint16_t *a_states,
    const uint8_t *a_partial, const uint8_t *a_sm,
    const uint8_t *b_compressed, int64_t b_compressed_bytes,
    const int32_t *b_offsets, const uint16_t *b_states,
    const uint8_t *b_partial, const uint8_t *b_sm,
    const int32_t *decode_table, uint8_t *out, int64_t n_streams,
    int64_t n_fp8_per_stream, int64_t chunk_streams, void *workspace,
    int64_t workspace_bytes, int32_t *status, void *stream);

/* Fused tANS-decode GEMV (no counterpart in the reference; the workload is
 * an e4m3 weight matrix such as a 17408 x 5120 MLP projection):
 *   y[b][r] = bf16(scale[r] * sum_c e4m3(W[r][c]) * x[b][c]), fp32 accumulate,
 * W rows x cols e4m3 stored as tANS streams in the GEMV stream order
 * (rans_vectoradd.tans_gemv.encode_weight): K = rows*4*col_splits streams of
 * cols/col_splits/4 fp8, sign/mantissa tiled [N/16][K][8].  x: bf16
 * [batch][cols], batch 1..8; y: bf16 [batch][rows].  rows % 16 == 0,
 * cols % (64*col_splits) == 0.  With col_splits > 1 the column slices are
 * reduced through `partials` (caller-owned f32 [col_splits][batch][rows]),
 * deterministically.  Launched with programmatic dependent launch: the
 * weight-side set-up may overlap the previous kernel on the stream, x and
 * the outputs are touched only after it completes. */
int tans_b200_gemv(const uint8_t *compressed, int64_t compressed_bytes,
                   const int32_t *offsets, const uint16_t *states,
                   const uint8_t *partial, const uint8_t *sign_mantissa,
                   const int32_t *decode_table, const float *scale,
                   const uint16_t *x, uint16_t *y, float *partials, int64_t rows,
                   int64_t cols, int64_t batch, int64_t col_splits,
                   int32_t *status, void *stream);

/* Uncompressed e4m3 GEMV (no counterpart in the reference; the denominator
 * of the decode-GEMV's amplification, as fp8_vecadd_raw is the fused add's):
 *   y[b][r] = bf16(scale[r] * sum_c e4m3(w[r][c]) * x[b][c]), fp32 accumulate,
 * w e4m3 [rows][cols] row-major (16-byte aligned), x bf16 [batch][cols],
 * batch 1..8, y bf16 [batch][rows]; the same mma.sync f16 path and the same
 * deterministic column-slice reduction as tans_b200_gemv (partials:
 * caller-owned f32 [col_splits][batch][rows]).  rows % 16 == 0,
 * cols % (64*col_splits) == 0. */
int tans_b200_gemv_raw(const uint8_t *w, const float *scale, const uint16_t *x, uint16_t *y,
                       float *partials, int64_t rows, int64_t cols, int64_t batch,
                       int64_t col_splits, void *stream);

/* Decode a GEMV-layout weight (tans_b200_gemv's stream format) to a dense
 * row-major bf16 [rows][cols] matrix of its e4m3 values (unscaled; exact).
 * For batches above 8, where the contraction belongs to a library bf16 GEMM
 * (y = (x @ w^T) * scale); no reference counterpart. */
int tans_b200_gemv_weight_dense(const uint8_t *compressed,
                                int64_t compressed_bytes,
                                const int32_t *offsets, const uint16_t *states,
                                const uint8_t *partial, const uint8_t *sm,
                                const int32_t *decode_table, uint16_t *w_bf16,
                                int64_t rows, int64_t cols, int64_t col_splits,
                                int32_t *status, void *stream);

/* Peer all-gather of a row-sharded GEMV, fused into its epilogue (no
 * NCCL): `world` ranks, one per GPU, each own `rows` rows of W starting at
 * row col0 of the full output; every rank holds the gathered output
 * [batch][y_ld] in memory that the others can store to (peer or symmetric
 * memory, one pointer per rank in the device array y_peers).  flag_peers:
 * device array of each rank's uint32 flag array [world]; flags: this rank's
 * (= flag_peers[rank]); seq, done: this rank's device uint32 counters, both
 * zero before the first gather, flags zero on every rank before any rank
 * starts.  No reference counterpart. */
typedef struct tans_b200_gather {
    int32_t rank, world;
    uint16_t *const *y_peers; /* device array [world] of bf16 [batch][y_ld] buffers */
    int64_t y_ld;             /* row length of the gathered output */
    int64_t col0;             /* this rank's first row (column of the gathered output); even */
    uint32_t *const *flag_peers;
    uint32_t *flags;
    uint32_t *seq, *done;
} tans_b200_gather;

/* y = scale * W @ x^T as tans_b200_gemv (this rank's rows), stored into
 * every rank's gathered buffer at columns [col0, col0 + rows), then this
 * rank's flag raised on every rank.  The kernel first waits until all of
 * this rank's flags have reached the number of gathers it has published, so
 * x may be (and the call may overwrite) the gathered buffer of an earlier
 * step: call it in the same order on every rank.  partials: f32
 * [col_splits][batch][rows], required.  A wait that runs out (a rank that
 * stopped) ORs TANS_B200_DATA_TIMEOUT into the status word. */
int tans_b200_gemv_gather(const uint8_t *compressed, int64_t compressed_bytes,
                          const int32_t *offsets, const uint16_t *states,
                          const uint8_t *partial, const uint8_t *sign_mantissa,
                          const int32_t *decode_table, const float *scale,
                          const uint16_t *x, float *partials, int64_t rows,
                          int64_t cols, int64_t batch, int64_t col_splits,
                          const tans_b200_gather *g, int32_t *status, void *stream);

/* Prefill GEMM with the weight decoded on the fly: y [m][rows] bf16 =
 * scale * W @ x^T for x bf16 [m][cols] (16-byte aligned), W in the GEMV
 * stream format (tans_b200_gemv).  Tensor cores (tcgen05.mma, bf16 in, fp32
 * accumulate in tensor memory); W never goes through HBM decoded.
 * rows % 128 == 0; up to 256 tokens one CTA per 128-row block decodes the
 * weight once; above that, when rows / 128 is even, CTA pairs on 2-SM MMAs
 * decode it once per 512 tokens (else once per 256).  A bounded wait that runs out ORs
 * TANS_B200_DATA_TIMEOUT into the optional status word (no result for that
 * CTA's rows).  No reference
 * counterpart. */
int tans_b200_gemm_tc(const uint8_t *compressed, int64_t compressed_bytes,
                      const int32_t *offsets, const uint16_t *states,
                      const uint8_t *partial, const uint8_t *sign_mantissa,
                      const int32_t *decode_table, const float *scale,
                      const uint16_t *x, uint16_t *y, int64_t rows,
                      int64_t cols, int64_t col_splits, int64_t m,
                      int32_t *status, void *stream);

/* Prefill epilogue: y[m][r] = bf16(acc[m][r] * scale[r]) for an fp32 GEMM
 * output acc [m][rows] (rows % 4 == 0; acc and scale 16-byte aligned, y
 * 8-byte aligned); one rounding. */
int tans_b200_scale_rows_bf16(const float *acc, const float *scale,
                              uint16_t *y, int64_t m, int64_t rows,
                              void *stream);

/* Allocation-free standalone decode.  No counterpart in the reference: it
 * exists for callers that cannot allocate device memory (a runtime that
 * hands the library only buffers carved from a pre-sized pool, or a
 * host-language binding with no device allocator).  Same inputs, output and
 * data-status bits as building the table with tans_b200_build_decode_table
 * and calling tans_b200_decode, but the decode table lives in a fixed
 * file-scope device array of the library: 16 KiB (4096 int32) per GPU that
 * loads the library, held until the process exits.  The caller passes only
 * inputs and outputs (spread[4096] and freqs[n_syms] are device arrays).
 *   - n_syms must be 1..256 (the table's alphabet); anything larger is
 *     rejected with TANS_B200_ERR_INVALID.
 *   - Calls no cudaMalloc/cudaFree and no allocating library routine.
 *   - The first call on a device resolves the array's device address; make
 *     that first call outside any stream capture.
 *   - Every call rewrites the whole table, so nothing is carried over, but
 *     all calls share the one array: calls whose GPU work overlaps (e.g. on
 *     two streams) race on it and must be ordered by the caller. */
int tans_b200_decode_noalloc(const uint8_t *compressed, int64_t compressed_bytes,
                             const int32_t *offsets, const uint16_t *states,
                             const uint8_t *partial, const uint8_t *sign_mantissa,
                             const int32_t *spread, const int32_t *freqs,
                             int64_t n_syms, uint8_t *out, int64_t n_streams,
                             int64_t n_fp8_per_stream, int32_t *status,
                             void *stream);

/* ------------------------------------------------------- device encoder */

/* GPU slab encoder (sm_100a).  The reference encodes on the CPU only
 * (tans_encode_interleaved, csrc/tans_codec.cpp:69-196, reached through
 * rans_vectoradd/tans_codec.py:90-143 `encode`); these entry points produce
 * the same bytes from device-resident input, and with FP8 input also do the
 * nibble split of tans_codec.py:106-124 in the same pass.
 *
 * Input kinds:
 *   TANS_B200_ENC_INPUT_FP8      in = e4m3 bytes [K][n], n even; pair i of
 *                                stream k is (in[k][2i], in[k][2i+1]); the
 *                                sign/mantissa pairs go to sm_out, layout
 *                                [n/2][K] (tile 0) or [n/2/tile][K][tile];
 *   TANS_B200_ENC_INPUT_SYMBOLS  in = pair symbols [K][n] (sm_out unused).
 *
 * Sequence (the caller allocates between the calls):
 *   1. tans_b200_encode_device_workspace_bytes(K, n, kind, &bytes); allocate
 *      a device workspace of that size (256-byte aligned): tables, per-stream
 *      slab counts and a staging area of ceil(13 P / 32) slab rows per
 *      encoder block (P = symbols per stream), about 0.8 bytes per FP8 byte;
 *   2. tans_b200_encode_device_plan(...): validates freqs/spread on the host
 *      (same checks and messages as tans_b200_encode), then enqueues the
 *      encode: sm_out, states_out[K], partial_out[K] and offsets_out[B+1]
 *      are written, the slabs are staged in the workspace, and the workspace
 *      header (tans_b200_enc_header at workspace offset 0) gets total_bytes
 *      and error bits;
 *   3. the caller reads the header (16 bytes, device -> host); error_bits
 *      TANS_B200_ENC_BAD_SYMBOL: a symbol with zero frequency occurs (the
 *      smallest one is bad_symbol); TANS_B200_ENC_TOO_LARGE: the compressed
 *      size exceeds the format's int32 offsets;
 *   4. with no error bits, allocate compressed[total_bytes] and call
 *      tans_b200_encode_device_emit(...), which places the staged slabs
 *      (every byte of compressed is written).  With error bits set it writes
 *      nothing.
 * freqs[n_syms] and spread[4096] are HOST pointers.  Streams are limited to
 * 357,913,941 symbols (32-bit per-stream bit counts).
 * segment_pairs > 0 (dividing the symbols per stream) writes the split-stream
 * format of tans_b200_fp8_vecadd_fused_split: K * segments sub-streams,
 * segment-major (states_out, partial_out and offsets sized for them), with
 * sm_out in the unsplit layout; 0 writes the plain format. */
#define TANS_B200_ENC_INPUT_FP8 0
#define TANS_B200_ENC_INPUT_SYMBOLS 1
#define TANS_B200_ENC_TOO_LARGE 1
#define TANS_B200_ENC_BAD_SYMBOL 2

typedef struct tans_b200_enc_header {
    int32_t error_bits;
    int32_t bad_symbol;  /* smallest zero-frequency symbol seen, else INT32_MAX */
    int64_t total_bytes; /* compressed bytes = offsets[B] */
} tans_b200_enc_header;

int tans_b200_encode_device_workspace_bytes(int64_t n_streams,
                                            int64_t n_per_stream,
                                            int input_kind,
                                            int64_t segment_pairs,
                                            int64_t *bytes);

int tans_b200_encode_device_plan(const uint8_t *in, int input_kind,
                                 int64_t n_streams, int64_t n_per_stream,
                                 int64_t tile, int64_t segment_pairs,
                                 const int32_t *freqs, int64_t n_syms,
                                 const int32_t *spread, uint8_t *sm_out,
                                 uint16_t *states_out, uint8_t *partial_out,
                                 int32_t *offsets_out, void *workspace,
                                 void *stream);

int tans_b200_encode_device_emit(int input_kind, int64_t n_streams,
                                 int64_t n_per_stream, int64_t segment_pairs,
                                 const int32_t *offsets, const void *workspace,
                                 uint8_t *compressed, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TANS_B200_H */
