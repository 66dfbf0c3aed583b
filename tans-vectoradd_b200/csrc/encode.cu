// encode.cu — sm_100a slab encoder: the device twin of the CPU encoder
// (host.cpp) and of the reference's tans_encode_interleaved
// (csrc/tans_codec.cpp:69-196), with the FP8 nibble split of
// rans_vectoradd/tans_codec.py:106-124 fused in.  Output bytes are identical
// to both.  The reference has no device encoder; this is the GPU side of the
// same wire format.
//
// Work split.  The format is serial inside a stream (each step's state
// depends on the previous one) and independent across streams, so one
// thread encodes one stream and a CTA of 128 threads is one encoder block.
// Slabs are top-aligned in their block, so a stream's first slab index
// depends on its block's longest stream, which is only known once every
// stream of the block is encoded.  The encoder therefore runs the state
// machine once, into a staging area, and places the slabs afterwards:
//   enc_setup_kernel  copies the alphabet tables into the workspace;
//   enc_stage_kernel  reads the input back to front, writes the
//                     sign/mantissa bytes (FP8 input), the final state, the
//                     partial-slab bit count, and every completed slab into
//                     the stream's staging column bottom-up; records each
//                     stream's slab count and its block's G_b;
//   enc_scan_kernel   exclusive scan of G_b * 512 into the int32 offsets;
//   enc_place_kernel  copies each block's staging rows to their top-aligned
//                     rows of the output, destination row by destination row
//                     (coalesced 512-byte stores), zeroing the rows below
//                     short streams and the unused columns of a partial last
//                     block, so the output needs no memset.
// The host reads the 16-byte workspace header between the scan and the
// placement to size the compressed buffer.  Staging holds ceil(13 P / 32)
// rows per block (13 bits bound every step, the error marker included).
//
// Step (pair symbol s, state x in [4096, 8192), tables in shared memory):
//     k  = (x + delta[s]) >> 13          bits to emit
//     emit x & (2^k - 1), LSB-first
//     x  = next[base[s] + (x >> k)]
// delta and base of a symbol share one 32-bit word (delta << 14 | base as a
// 14-bit two's-complement field), kept in 4 copies interleaved by word so
// that lane l reads copy l % 4: one 4-byte random lookup per step instead
// of an 8-byte one, with fewer bank conflicts.  The word depends only on s,
// so its lookup is off the x dependency chain; the chain is add, shift,
// shift, address, one 16-bit shared load.

#include "../../include/tans_b200.h"
#include "internal.h"

#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>

using tans_b200::EncoderTables;
using tans_b200::fail;

namespace {

constexpr int kL = TANS_B200_TABLE_SIZE;
constexpr int kBlk = TANS_B200_BLOCK_STREAMS;
constexpr int kScanThreads = 1024;

// Workspace layout (bytes).  The header is the public tans_b200_enc_header.
constexpr int kInfoCopies = 4;
constexpr size_t kWsInfo = 16;                                 // uint32[256][4] packed delta/base
constexpr size_t kWsNext = kWsInfo + 256 * 4 * kInfoCopies;    // uint16[L]
constexpr size_t kWsSlabs = 12544;                             // uint32[K]: slabs per stream
static_assert(kWsNext + kL * 2 <= kWsSlabs, "workspace tables overlap");

__host__ __device__ __forceinline__ size_t ws_blocks_offset(int64_t K) {
    return (kWsSlabs + 4 * (size_t)K + 255) & ~(size_t)255;
}
__host__ __device__ __forceinline__ size_t ws_stage_offset(int64_t K) {
    const int64_t B = (K + kBlk - 1) / kBlk;
    return (ws_blocks_offset(K) + 4 * (size_t)B + 4 + 255) & ~(size_t)255;
}
// Staging rows per block: every step emits at most 13 bits.
__host__ __device__ __forceinline__ int64_t stage_rows(int64_t P) {
    const int64_t g = (13 * P + 31) / 32;
    return g > 0 ? g : 1;
}

struct EncArgs {
    const uint8_t *in;    // FP8 bytes [stride][2 row_pairs] or pair symbols [stride][row_pairs]
    int64_t K, P;         // chains (encoded streams), pair symbols per chain
    int64_t stride;       // streams of the input rows and of the sm layout
    int64_t row_pairs;    // pair symbols per input row (P * segments for split streams)
    int64_t tile;         // sm layout: 0 -> [P][K], t -> [P/t][K][t]
    int32_t vec;          // 16-byte (FP8) / 8-byte (symbols) chunk loads allowed
    int32_t sm_vec;       // tile 8 and sm 8-byte aligned: one 8-byte store per chunk
    uint8_t *sm;          // FP8 input only
    uint16_t *states;
    const int32_t *offsets;
    int32_t *offsets_out;
    uint8_t *compressed;
    uint8_t *partial;
    uint8_t *ws;
    int64_t gmax;         // staging rows per block
};

__device__ __forceinline__ tans_b200_enc_header *header(uint8_t *ws) {
    return reinterpret_cast<tans_b200_enc_header *>(ws);
}
__device__ __forceinline__ uint32_t *slabs_of(uint8_t *ws) {
    return reinterpret_cast<uint32_t *>(ws + kWsSlabs);
}

__device__ __forceinline__ uint4 ld_nc_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_nc_v2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// Exponent pair symbols of one word of 4 e4m3 bytes: byte 0 = pair (b0, b1),
// byte 2 = pair (b2, b3), each exp(first) << 4 | exp(second).
__device__ __forceinline__ uint32_t pair_syms_of(uint32_t w) {
    const uint32_t e = (w >> 3) & 0x0F0F0F0Fu;
    return ((e << 4) | (e >> 8)) & 0x00FF00FFu;
}
// Sign/mantissa pairs of the same word in bytes 0 and 2:
// sm(first) | sm(second) << 4 with sm(b) = (b >> 4 & 8) | (b & 7).
__device__ __forceinline__ uint32_t sm_pairs_of(uint32_t w) {
    const uint32_t m = ((w >> 4) & 0x08080808u) | (w & 0x07070707u);
    return m | (m >> 4);
}

// Byte j (0..3) of w, zero-extended.
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int j) { return (w >> (8 * j)) & 0xFFu; }

struct EncTables {
    const uint32_t *info;  // this lane's copy: entry s at info[4 * s]
    const uint16_t *next;
};

__device__ __forceinline__ int32_t info_delta(uint32_t w) { return (int32_t)w >> 14; }
__device__ __forceinline__ int32_t info_base(uint32_t w) {
    int32_t b;
    asm("bfe.s32 %0, %1, 0, 14;" : "=r"(b) : "r"(w));
    return b;
}

// Encoder state: state x, the pending slab lo (fill bits), the largest k
// seen (13 marks a symbol that cannot be coded) and a running pointer to the
// next slab slot of this stream's staging column (stride 512 bytes).
struct Emitter {
    uint32_t x, lo, fill, kmax;
    uint32_t *out;
    __device__ __forceinline__ void step(const EncTables &t, uint32_t s) {
        const uint32_t w = t.info[kInfoCopies * s];
        const uint32_t k = (uint32_t)((int32_t)x + info_delta(w)) >> (tans_b200::kTableLog + 1);
        const uint32_t v = x & ((1u << k) - 1u);
        const uint32_t hi = __funnelshift_l(v, 0u, fill);  // bits that spill past 32
        lo |= v << fill;
        fill += k;
        kmax = max(kmax, k);
        if (fill >= 32) {
            *out = lo;
            out += kBlk;
            lo = hi;
            fill -= 32;
        }
        x = t.next[info_base(w) + (int32_t)(x >> k)];
    }
};

// Sign/mantissa byte of pair i (index within the whole input row) of column col.
__device__ __forceinline__ void store_sm_byte(const EncArgs &a, int64_t col, int64_t i, uint32_t v) {
    if (a.tile == 0)
        a.sm[i * a.stride + col] = (uint8_t)v;
    else
        a.sm[((i / a.tile) * a.stride + col) * a.tile + (i % a.tile)] = (uint8_t)v;
}

// Symbol i of a chain read without chunking (ragged tail, unaligned rows);
// writes the sign/mantissa byte (row pair pbase + i of column col) in pass 1.
template <bool kFp8, bool kPass1>
__device__ __forceinline__ uint32_t scalar_symbol(const EncArgs &a, const uint8_t *row, int64_t col,
                                                  int64_t pbase, int64_t i) {
    if (!kFp8) return row[i];
    const uint32_t b0 = row[2 * i], b1 = row[2 * i + 1];
    if (kPass1) {
        const uint32_t m0 = ((b0 >> 4) & 8u) | (b0 & 7u), m1 = ((b1 >> 4) & 8u) | (b1 & 7u);
        store_sm_byte(a, col, pbase + i, m0 | (m1 << 4));
    }
    return (((b0 >> 3) & 15u) << 4) | ((b1 >> 3) & 15u);
}

// First input byte of chain k: split streams are segment-major (chain
// k = seg * stride + col covers pairs [seg P, (seg + 1) P) of row col).
template <bool kFp8>
__device__ __forceinline__ const uint8_t *chain_row(const EncArgs &a, int64_t k, int64_t *col,
                                                   int64_t *pbase) {
    const int64_t seg = k / a.stride;
    *col = k - seg * a.stride;
    *pbase = seg * a.P;
    return a.in + (*col * a.row_pairs + *pbase) * (kFp8 ? 2 : 1);
}

// Run `m` over chain k from its last pair symbol to its first.
template <bool kFp8, bool kPass1, typename Machine>
__device__ __forceinline__ void run_stream(const EncArgs &a, const EncTables &t, int64_t k,
                                           Machine &m) {
    const int64_t P = a.P;
    int64_t col, pbase;
    const uint8_t *row = chain_row<kFp8>(a, k, &col, &pbase);
    const int64_t chunks = a.vec ? P / 8 : 0;
    for (int64_t i = P - 1; i >= chunks * 8; i--)
        m.step(t, scalar_symbol<kFp8, kPass1>(a, row, col, pbase, i));
    if (chunks == 0) return;
    if (kFp8) {
        const uint8_t *cp = row + (chunks - 1) * 16;
        uint4 w = ld_nc_v4(cp);
        for (int64_t c = chunks - 1; c >= 0; c--) {
            const uint4 cur = w;
            if (c > 0) w = ld_nc_v4(cp - 16);
            cp -= 16;
            const uint32_t s0 = pair_syms_of(cur.x), s1 = pair_syms_of(cur.y);
            const uint32_t s2 = pair_syms_of(cur.z), s3 = pair_syms_of(cur.w);
            if (kPass1) {
                const uint32_t lo = __byte_perm(sm_pairs_of(cur.x), sm_pairs_of(cur.y), 0x6420);
                const uint32_t hi = __byte_perm(sm_pairs_of(cur.z), sm_pairs_of(cur.w), 0x6420);
                if (a.sm_vec) {
                    *reinterpret_cast<uint2 *>(a.sm + ((pbase / 8 + c) * a.stride + col) * 8) =
                        make_uint2(lo, hi);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        store_sm_byte(a, col, pbase + c * 8 + j, byte_of(j < 4 ? lo : hi, j & 3));
                }
            }
            m.step(t, s3 >> 16);
            m.step(t, s3 & 0xFFu);
            m.step(t, s2 >> 16);
            m.step(t, s2 & 0xFFu);
            m.step(t, s1 >> 16);
            m.step(t, s1 & 0xFFu);
            m.step(t, s0 >> 16);
            m.step(t, s0 & 0xFFu);
        }
    } else {
        const uint8_t *cp = row + (chunks - 1) * 8;
        uint2 w = ld_nc_v2(cp);
        for (int64_t c = chunks - 1; c >= 0; c--) {
            const uint2 cur = w;
            if (c > 0) w = ld_nc_v2(cp - 8);
            cp -= 8;
#pragma unroll
            for (int j = 7; j >= 0; j--) m.step(t, byte_of(j < 4 ? cur.x : cur.y, j & 3));
        }
    }
}

__device__ __forceinline__ EncTables load_tables(uint8_t *smem, const uint8_t *ws) {
    // 4 KB of packed delta/base words and 8 KB of next states, 16-byte copies
    const uint4 *src = reinterpret_cast<const uint4 *>(ws + kWsInfo);
    uint4 *dst = reinterpret_cast<uint4 *>(smem);
    for (int i = threadIdx.x; i < (int)((kWsNext - kWsInfo + kL * 2) / 16); i += blockDim.x)
        dst[i] = src[i];
    __syncthreads();
    return EncTables{reinterpret_cast<const uint32_t *>(smem) + (threadIdx.x % kInfoCopies),
                     reinterpret_cast<const uint16_t *>(smem + (kWsNext - kWsInfo))};
}

constexpr int kTableSmem = (int)(kWsNext - kWsInfo) + kL * 2;

__global__ void enc_setup_kernel(const __grid_constant__ EncoderTables t, uint8_t *ws) {
    const int i = threadIdx.x;
    if (i == 0) {
        tans_b200_enc_header *h = header(ws);
        h->error_bits = 0;
        h->bad_symbol = INT_MAX;
        h->total_bytes = 0;
    }
    uint32_t *info = reinterpret_cast<uint32_t *>(ws + kWsInfo);
    for (int s = i; s < 256; s += blockDim.x) {
        const uint32_t w = ((uint32_t)t.delta[s] << 14) | ((uint32_t)t.base[s] & 0x3FFFu);
        for (int c = 0; c < kInfoCopies; c++) info[kInfoCopies * s + c] = w;
    }
    uint16_t *next = reinterpret_cast<uint16_t *>(ws + kWsNext);
    for (int j = i; j < kL; j += blockDim.x) next[j] = t.next[j];
}

template <bool kFp8>
__global__ void __launch_bounds__(kBlk, 8) enc_stage_kernel(const EncArgs a) {
    __shared__ __align__(16) uint8_t smem[kTableSmem];
    __shared__ uint32_t warp_max[kBlk / 32];
    const EncTables t = load_tables(smem, a.ws);
    const int64_t k = (int64_t)blockIdx.x * kBlk + threadIdx.x;
    uint32_t slabs = 0;
    if (k < a.K) {
        uint32_t *col = reinterpret_cast<uint32_t *>(a.ws + ws_stage_offset(a.K)) +
                        (int64_t)blockIdx.x * a.gmax * kBlk + threadIdx.x;
        Emitter e{(uint32_t)kL, 0u, 0u, 0u, col};
        run_stream<kFp8, true>(a, t, k, e);
        if (e.fill > 0) {
            *e.out = e.lo;
            e.out += kBlk;
        }
        a.states[k] = (uint16_t)e.x;
        a.partial[k] = (uint8_t)e.fill;
        slabs = (uint32_t)((e.out - col) / kBlk);
        slabs_of(a.ws)[k] = slabs;
        if (e.kmax >= (uint32_t)tans_b200::kEncoderBadBits) {
            // error path: find the symbols that have no slot and report the smallest
            tans_b200_enc_header *h = header(a.ws);
            atomicOr(&h->error_bits, TANS_B200_ENC_BAD_SYMBOL);
            int64_t col, pbase;
            const uint8_t *row = chain_row<kFp8>(a, k, &col, &pbase);
            for (int64_t i = 0; i < a.P; i++) {
                uint32_t s;
                if (kFp8)
                    s = (((row[2 * i] >> 3) & 15u) << 4) | ((row[2 * i + 1] >> 3) & 15u);
                else
                    s = row[i];
                if (info_delta(t.info[kInfoCopies * s]) ==
                    (tans_b200::kEncoderBadBits << (tans_b200::kTableLog + 1)))
                    atomicMin(&h->bad_symbol, (int)s);
            }
        }
    }
    const uint32_t m = __reduce_max_sync(0xffffffffu, slabs);
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t g = 1;  // an all-empty block still has one slab per stream
        for (int w = 0; w < kBlk / 32; w++) g = max(g, warp_max[w]);
        reinterpret_cast<uint32_t *>(a.ws + ws_blocks_offset(a.K))[blockIdx.x] = g;
    }
}

// offsets[b] = 512 * sum_{c<b} G_c (int64 running sum; a total above
// INT32_MAX is flagged and the offsets are not used).
__global__ void __launch_bounds__(kScanThreads) enc_scan_kernel(const EncArgs a, int64_t B) {
    __shared__ int64_t warp_sum[kScanThreads / 32];
    __shared__ int64_t carry_s;
    const uint32_t *g = reinterpret_cast<const uint32_t *>(a.ws + ws_blocks_offset(a.K));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry_s = 0;
    __syncthreads();
    for (int64_t base = 0; base < B; base += kScanThreads) {
        const int64_t b = base + threadIdx.x;
        const int64_t v = b < B ? (int64_t)g[b] * (kBlk * 4) : 0;
        int64_t incl = v;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int64_t o = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += o;
        }
        if (lane == 31) warp_sum[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int64_t w = warp_sum[lane];
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int64_t o = __shfl_up_sync(0xffffffffu, w, d);
                if (lane >= d) w += o;
            }
            warp_sum[lane] = w;  // inclusive over warps
        }
        __syncthreads();
        const int64_t carry = carry_s;
        const int64_t excl = carry + (warp ? warp_sum[warp - 1] : 0) + incl - v;
        if (b < B) a.offsets_out[b] = (int32_t)excl;
        __syncthreads();
        if (threadIdx.x == 0) carry_s = carry + warp_sum[kScanThreads / 32 - 1];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const int64_t total = carry_s;
        a.offsets_out[B] = (int32_t)total;
        tans_b200_enc_header *h = header(a.ws);
        h->total_bytes = total;
        if (total > INT32_MAX) atomicOr(&h->error_bits, TANS_B200_ENC_TOO_LARGE);
    }
}

// Destination row r of stream t's column holds staging row r - (G_b - G_s)
// (zero below it): stores walk the output row by row, 512 contiguous bytes
// per row and block; the staging reads of a warp fall in a few rows.
__global__ void __launch_bounds__(kBlk) enc_place_kernel(const EncArgs a) {
    if (header(a.ws)->error_bits != 0) return;  // layout not valid: write nothing
    const int64_t k = (int64_t)blockIdx.x * kBlk + threadIdx.x;
    const int64_t off = a.offsets[blockIdx.x];
    const int32_t g_b = (int32_t)((a.offsets[blockIdx.x + 1] - off) / (kBlk * 4));
    const int32_t g_s = k < a.K ? (int32_t)slabs_of(a.ws)[k] : 0;
    const int32_t shift = g_b - g_s;
    const uint32_t *src = reinterpret_cast<const uint32_t *>(a.ws + ws_stage_offset(a.K)) +
                          (int64_t)blockIdx.x * a.gmax * kBlk + threadIdx.x;
    uint32_t *dst = reinterpret_cast<uint32_t *>(a.compressed + off) + threadIdx.x;
    for (int32_t r = 0; r < g_b; r++) {
        const int32_t g = r - shift;
        dst[(int64_t)r * kBlk] = g >= 0 ? src[(int64_t)g * kBlk] : 0u;
    }
}

int launch_status(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(TANS_B200_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
    return TANS_B200_OK;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// 12 bits per pair symbol at most: the per-stream bit count stays in 32 bits.
constexpr int64_t kMaxPairsPerStream = (int64_t)(UINT32_MAX / 12);

int check_shape(int input_kind, int64_t K, int64_t n, int64_t segment_pairs, int64_t *P,
                int64_t *segs) {
    if (input_kind != TANS_B200_ENC_INPUT_FP8 && input_kind != TANS_B200_ENC_INPUT_SYMBOLS)
        return fail(TANS_B200_ERR_INVALID, "encode_device: unknown input kind %d", input_kind);
    if (K < 0 || n < 0) return fail(TANS_B200_ERR_INVALID, "encode: bad arguments");
    if (input_kind == TANS_B200_ENC_INPUT_FP8 && n % 2 != 0)
        return fail(TANS_B200_ERR_INVALID, "encode_device: FP8 bytes per stream must be even");
    const int64_t row = input_kind == TANS_B200_ENC_INPUT_FP8 ? n / 2 : n;
    if (segment_pairs < 0 || (segment_pairs > 0 && row % segment_pairs != 0))
        return fail(TANS_B200_ERR_INVALID,
                    "encode_device: segment_pairs must divide the %lld symbols per stream",
                    (long long)row);
    *P = segment_pairs > 0 ? segment_pairs : row;
    *segs = segment_pairs > 0 ? row / segment_pairs : 1;
    if (*P > kMaxPairsPerStream)
        return fail(TANS_B200_ERR_INVALID, "encode_device: more than %lld symbols per stream",
                    (long long)kMaxPairsPerStream);
    return TANS_B200_OK;
}

}  // namespace

extern "C" int tans_b200_encode_device_workspace_bytes(int64_t K, int64_t n, int input_kind,
                                                       int64_t segment_pairs, int64_t *bytes) {
    tans_b200::clear_error();
    if (!bytes) return fail(TANS_B200_ERR_INVALID, "encode_device_workspace_bytes: bytes is null");
    int64_t P = 0, segs = 0;
    int rc = check_shape(input_kind, K, n, segment_pairs, &P, &segs);
    if (rc) return rc;
    const int64_t chains = K * segs, B = (chains + kBlk - 1) / kBlk;
    *bytes = (int64_t)ws_stage_offset(chains) + B * stage_rows(P) * kBlk * 4;
    return TANS_B200_OK;
}

extern "C" int tans_b200_encode_device_plan(const uint8_t *in, int input_kind, int64_t K,
                                            int64_t n, int64_t tile, int64_t segment_pairs,
                                            const int32_t *freqs, int64_t n_syms,
                                            const int32_t *spread, uint8_t *sm_out,
                                            uint16_t *states_out, uint8_t *partial_out,
                                            int32_t *offsets_out, void *workspace, void *stream) {
    tans_b200::clear_error();
    int64_t P = 0, segs = 0;
    int rc = check_shape(input_kind, K, n, segment_pairs, &P, &segs);
    if (rc) return rc;
    const bool fp8 = input_kind == TANS_B200_ENC_INPUT_FP8;
    const int64_t row_pairs = P * segs, chains = K * segs;
    if (fp8 && tile < 0) return fail(TANS_B200_ERR_INVALID, "encode_device: tile must be >= 0");
    if (fp8 && tile > 0 && P % tile != 0)
        return fail(TANS_B200_ERR_INVALID, "n_pairs=%lld not divisible by tile=%lld", (long long)P,
                    (long long)tile);
    if (!workspace || !offsets_out || (K > 0 && (!states_out || !partial_out)) ||
        (K > 0 && P > 0 && (!in || (fp8 && !sm_out))))
        return fail(TANS_B200_ERR_INVALID, "encode_device: null pointer");
    if (!aligned(workspace, 256) || !aligned(offsets_out, 4) || !aligned(states_out, 2))
        return fail(TANS_B200_ERR_INVALID, "encode_device: misaligned output or workspace");
    EncoderTables tables;
    rc = tans_b200::encoder_tables(freqs, n_syms, spread, &tables);
    if (rc) return rc;
    const int64_t B = (chains + kBlk - 1) / kBlk;
    if (B > INT_MAX) return fail(TANS_B200_ERR_INVALID, "encode_device: too many streams");
    cudaStream_t st = (cudaStream_t)stream;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    enc_setup_kernel<<<1, 256, 0, st>>>(tables, ws);
    if ((rc = launch_status("enc_setup_kernel"))) return rc;
    EncArgs a{};
    a.in = in;
    a.K = chains;
    a.P = P;
    a.stride = K;
    a.row_pairs = row_pairs;
    a.tile = fp8 ? tile : 0;
    a.vec = fp8 ? (aligned(in, 16) && (2 * row_pairs) % 16 == 0 && (2 * P) % 16 == 0)
                : (aligned(in, 8) && row_pairs % 8 == 0 && P % 8 == 0);
    a.sm = sm_out;
    a.sm_vec = fp8 && tile == 8 && aligned(sm_out, 8);
    a.states = states_out;
    a.partial = partial_out;
    a.offsets_out = offsets_out;
    a.ws = ws;
    a.gmax = stage_rows(P);
    if (B > 0) {
        if (fp8)
            enc_stage_kernel<true><<<(unsigned)B, kBlk, 0, st>>>(a);
        else
            enc_stage_kernel<false><<<(unsigned)B, kBlk, 0, st>>>(a);
        if ((rc = launch_status("enc_stage_kernel"))) return rc;
    }
    enc_scan_kernel<<<1, kScanThreads, 0, st>>>(a, B);
    return launch_status("enc_scan_kernel");
}

extern "C" int tans_b200_encode_device_emit(int input_kind, int64_t K, int64_t n,
                                            int64_t segment_pairs, const int32_t *offsets,
                                            const void *workspace, uint8_t *compressed,
                                            void *stream) {
    tans_b200::clear_error();
    int64_t P = 0, segs = 0;
    int rc = check_shape(input_kind, K, n, segment_pairs, &P, &segs);
    if (rc) return rc;
    if (K == 0) return TANS_B200_OK;
    if (!workspace || !offsets || !compressed)
        return fail(TANS_B200_ERR_INVALID, "encode_device: null pointer");
    if (!aligned(workspace, 256) || !aligned(offsets, 4) || !aligned(compressed, 4))
        return fail(TANS_B200_ERR_INVALID, "encode_device: misaligned compressed or workspace");
    const int64_t chains = K * segs, B = (chains + kBlk - 1) / kBlk;
    if (B > INT_MAX) return fail(TANS_B200_ERR_INVALID, "encode_device: too many streams");
    EncArgs a{};
    a.K = chains;
    a.P = P;
    a.stride = K;
    a.row_pairs = P * segs;
    a.offsets = offsets;
    a.compressed = compressed;
    a.ws = static_cast<uint8_t *>(const_cast<void *>(workspace));
    a.gmax = stage_rows(P);
    enc_place_kernel<<<(unsigned)B, kBlk, 0, (cudaStream_t)stream>>>(a);
    return launch_status("enc_place_kernel");
}
