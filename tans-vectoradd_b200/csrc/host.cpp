// host.cpp — host half of libtans_b200: the CPU slab encoder, the host
// decode-table builder, the FP8 nibble splitter and the error plumbing of the
// C ABI declared in include/tans_b200.h.
//
// Encoder design.  The wire format is fixed by the reference
// (csrc/tans_codec.cpp:22-196): every stream is tANS-encoded last symbol
// first with state x in [4096, 8192); renormalisation emits x's low bits
// LSB-first into uint32 slabs; the final partial slab stays LSB-aligned and
// its bit count is reported; 128-stream blocks are padded to the block's
// longest stream and streams are top-aligned inside the block.  This encoder
// produces those bytes with a different structure:
//   * renormalisation emits all k bits of a step at once, with k taken from a
//     per-symbol threshold (k = k1 - 1 + (x >= f << k1), k1 = 12 - log2 f)
//     instead of a bit-by-bit loop;
//   * the next state comes from one flat table indexed by cum[s] + (x' - f);
//   * pass 1 runs the state machine only to size every stream, so the block
//     layout and the output buffer are known up front; pass 2 re-runs it and
//     writes each completed slab straight into its final interleaved slot.
//     No per-stream staging buffers, so memory stays at the output size.
// Both passes are OpenMP-parallel over streams.

#include "../../include/tans_b200.h"
#include "internal.h"

#include <omp.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

namespace {

constexpr uint32_t kL = TANS_B200_TABLE_SIZE;
constexpr int64_t kBlk = TANS_B200_BLOCK_STREAMS;

thread_local std::string g_last_error;

}  // namespace

namespace tans_b200 {

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

void clear_error() { g_last_error.clear(); }

}  // namespace tans_b200

using tans_b200::fail;

extern "C" const char *tans_b200_last_error(void) { return g_last_error.c_str(); }

extern "C" const char *tans_b200_version(void) { return "tans_b200 0.1 (sm_100a)"; }

extern "C" int tans_b200_table_size(void) { return (int)kL; }

// ------------------------------------------------------------ decode table

extern "C" int tans_b200_build_decode_table_host(const int32_t *spread, const int32_t *freqs,
                                                 int64_t n_syms, int32_t *table) {
    if (!spread || !freqs || !table || n_syms <= 0)
        return fail(TANS_B200_ERR_INVALID, "build_decode_table: null pointer or empty alphabet");
    std::vector<int64_t> seen(static_cast<size_t>(n_syms), 0);
    for (uint32_t slot = 0; slot < kL; slot++) {
        int32_t s = spread[slot];
        if (s < 0 || s >= n_syms)
            return fail(TANS_B200_ERR_INVALID, "build_decode_table: spread[%u]=%d outside [0,%lld)",
                        slot, s, (long long)n_syms);
        int64_t xp = static_cast<int64_t>(freqs[s]) + seen[s]++;
        if (xp <= 0 || xp >= 2 * (int64_t)kL)
            return fail(TANS_B200_ERR_INVALID, "build_decode_table: inconsistent freqs for symbol %d",
                        s);
        // nb = shifts that lift xp into [L, 2L): log2 L - floor(log2 xp)
        int nb = tans_b200::kTableLog - (31 - __builtin_clz(static_cast<uint32_t>(xp)));
        if (nb < 0)
            return fail(TANS_B200_ERR_INVALID, "build_decode_table: symbol %d over-subscribed", s);
        uint32_t base = static_cast<uint32_t>(xp) << nb;
        table[slot] = static_cast<int32_t>((static_cast<uint32_t>(s) & 0xFFu) |
                                           (static_cast<uint32_t>(nb) << 8) | (base << 16));
    }
    return TANS_B200_OK;
}

// ----------------------------------------------------------------- encoder

struct tans_b200_encoded {
    const uint8_t *symbols = nullptr;  // borrowed until export
    int64_t K = 0, N = 0;
    int n_threads = 0;
    std::vector<uint32_t> next_state;  // flat: cum[s] + r -> L + slot
    std::vector<uint32_t> cum;         // per-symbol start in next_state
    std::vector<uint32_t> freq;
    std::vector<uint32_t> k1;          // log2 L - floor(log2 f)
    std::vector<uint32_t> thresh;      // f << k1
    std::vector<uint64_t> bits;        // total bits per stream
    std::vector<uint16_t> final_state;
    std::vector<int32_t> offsets;      // [B+1]
    int64_t total_bytes = 0;
};

namespace {

struct SlabSink {  // pass 2: writes completed slabs to their final slots
    uint8_t *block_base;  // compressed + offsets[b]
    int64_t tid;
    int64_t slab;         // next slab index to write (G_b - G_s + g)
    void put(uint32_t w) {
        std::memcpy(block_base + slab * kBlk * 4 + tid * 4, &w, 4);
        slab++;
    }
};

struct NullSink {
    void put(uint32_t) {}
};

// Encode one stream of n pair symbols.  Returns the bit count; writes the
// final state; hands completed slabs (and the final partial one) to `sink`.
template <typename Sink>
inline uint64_t encode_stream(const tans_b200_encoded &e, const uint8_t *sym, int64_t n,
                              Sink &sink, uint16_t *state_out, uint8_t *partial_out) {
    uint32_t x = kL;
    uint64_t acc = 0;  // pending bits, LSB-first
    uint32_t fill = 0;
    uint64_t total = 0;
    const uint32_t *freq = e.freq.data();
    const uint32_t *k1 = e.k1.data();
    const uint32_t *th = e.thresh.data();
    const uint32_t *cum = e.cum.data();
    const uint32_t *nxt = e.next_state.data();
    for (int64_t i = n - 1; i >= 0; i--) {
        uint32_t s = sym[i];
        uint32_t k = k1[s] - 1u + (x >= th[s] ? 1u : 0u);
        acc |= static_cast<uint64_t>(x & ((1u << k) - 1u)) << fill;
        fill += k;
        total += k;
        if (fill >= 32) {
            sink.put(static_cast<uint32_t>(acc));
            acc >>= 32;
            fill -= 32;
        }
        x = nxt[cum[s] + ((x >> k) - freq[s])];
    }
    if (fill > 0) sink.put(static_cast<uint32_t>(acc));
    if (state_out) *state_out = static_cast<uint16_t>(x);
    if (partial_out) *partial_out = static_cast<uint8_t>(fill);
    return total;
}

}  // namespace

extern "C" int tans_b200_encode(const uint8_t *symbols, int64_t K, int64_t N,
                                const int32_t *freqs, int64_t n_syms, const int32_t *spread,
                                int n_threads, tans_b200_encoded **out) {
    tans_b200::clear_error();
    if (!out) return fail(TANS_B200_ERR_INVALID, "encode: out is null");
    *out = nullptr;
    if (K < 0 || N < 0 || (K > 0 && N > 0 && !symbols) || !freqs || !spread || n_syms <= 0)
        return fail(TANS_B200_ERR_INVALID, "encode: bad arguments");
    tans_b200_encoded *e = new (std::nothrow) tans_b200_encoded();
    if (!e) return fail(TANS_B200_ERR_HOST, "encode: out of host memory");
    e->symbols = symbols;
    e->K = K;
    e->N = N;
    e->n_threads = n_threads;

    // frequency checks (csrc/tans_codec.cpp:91-98)
    uint64_t sum = 0;
    e->freq.resize(n_syms);
    e->k1.resize(n_syms);
    e->thresh.resize(n_syms);
    e->cum.resize(n_syms + 1);
    for (int64_t s = 0; s < n_syms; s++) {
        if (freqs[s] < 0) {
            delete e;
            return fail(TANS_B200_ERR_INVALID, "encode: freqs[%lld] is negative", (long long)s);
        }
        e->cum[s] = static_cast<uint32_t>(sum);
        sum += static_cast<uint32_t>(freqs[s]);
        uint32_t f = static_cast<uint32_t>(freqs[s]);
        e->freq[s] = f;
        uint32_t hf = f ? 31u - __builtin_clz(f) : 0u;
        e->k1[s] = f ? (uint32_t)tans_b200::kTableLog - std::min(hf, (uint32_t)tans_b200::kTableLog) : 0u;
        e->thresh[s] = f ? (f << e->k1[s]) : 0u;
    }
    if (sum != kL) {
        delete e;
        return fail(TANS_B200_ERR_INVALID, "freqs must sum to L=%u; got %llu", kL,
                    (unsigned long long)sum);
    }
    e->cum[n_syms] = kL;

    // next-state table from the spread, ranks in slot order
    // (csrc/tans_codec.cpp:100-118)
    e->next_state.assign(kL, 0u);
    std::vector<uint32_t> seen(n_syms, 0u);
    for (uint32_t slot = 0; slot < kL; slot++) {
        int32_t s = spread[slot];
        if (s < 0 || s >= n_syms || seen[s] >= e->freq[s]) {
            delete e;
            return fail(TANS_B200_ERR_INVALID,
                        "encode: spread[%u]=%d inconsistent with freqs (alphabet %lld)", slot, s,
                        (long long)n_syms);
        }
        e->next_state[e->cum[s] + seen[s]++] = kL + slot;
    }

    // symbols must be codable (a zero-frequency symbol has no state)
    std::vector<uint8_t> present(256, 0);
    int bad_sym = -1;
    if (K > 0 && N > 0) {
        const int64_t total = K * N;
#pragma omp parallel num_threads(n_threads > 0 ? n_threads : omp_get_max_threads())
        {
            std::vector<uint8_t> loc(256, 0);
#pragma omp for schedule(static)
            for (int64_t i = 0; i < total; i++) loc[symbols[i]] = 1;
#pragma omp critical
            for (int s = 0; s < 256; s++) present[s] |= loc[s];
        }
        for (int s = 0; s < 256; s++)
            if (present[s] && (s >= n_syms || e->freq[s] == 0)) {
                bad_sym = s;
                break;
            }
    }
    if (bad_sym >= 0) {
        delete e;
        return fail(TANS_B200_ERR_INVALID, "encode: symbol %d occurs but has zero frequency",
                    bad_sym);
    }

    // pass 1: bit counts and final states
    e->bits.assign(K, 0);
    e->final_state.assign(K, 0);
#pragma omp parallel for schedule(static) num_threads(n_threads > 0 ? n_threads : omp_get_max_threads())
    for (int64_t k = 0; k < K; k++) {
        NullSink sink;
        e->bits[k] = encode_stream(*e, symbols + k * N, N, sink, &e->final_state[k], nullptr);
    }

    // block layout (csrc/tans_codec.cpp:139-155)
    const int64_t B = (K + kBlk - 1) / kBlk;
    e->offsets.assign(B + 1, 0);
    int64_t cum_bytes = 0;
    for (int64_t b = 0; b < B; b++) {
        uint64_t g = 0;
        for (int64_t k = b * kBlk; k < std::min(K, (b + 1) * kBlk); k++)
            g = std::max<uint64_t>(g, (e->bits[k] + 31) / 32);
        if (g == 0) g = 1;
        e->offsets[b] = static_cast<int32_t>(cum_bytes);
        cum_bytes += static_cast<int64_t>(g) * kBlk * 4;
        if (cum_bytes > INT32_MAX) {
            delete e;
            return fail(TANS_B200_ERR_INVALID,
                        "encode: compressed size exceeds the int32 offsets of the format");
        }
    }
    e->offsets[B] = static_cast<int32_t>(cum_bytes);
    e->total_bytes = cum_bytes;
    *out = e;
    return TANS_B200_OK;
}

extern "C" int tans_b200_encoded_sizes(const tans_b200_encoded *e, int64_t *compressed_bytes,
                                       int64_t *n_blocks) {
    if (!e) return fail(TANS_B200_ERR_INVALID, "encoded_sizes: null handle");
    if (compressed_bytes) *compressed_bytes = e->total_bytes;
    if (n_blocks) *n_blocks = static_cast<int64_t>(e->offsets.size()) - 1;
    return TANS_B200_OK;
}

extern "C" int tans_b200_encoded_export(const tans_b200_encoded *e, uint8_t *compressed,
                                        uint16_t *states, int32_t *offsets, uint8_t *partial) {
    if (!e) return fail(TANS_B200_ERR_INVALID, "encoded_export: null handle");
    const int64_t K = e->K, N = e->N;
    if (offsets) std::memcpy(offsets, e->offsets.data(), e->offsets.size() * sizeof(int32_t));
    if (states) std::memcpy(states, e->final_state.data(), K * sizeof(uint16_t));
    if (!compressed && !partial) return TANS_B200_OK;
    if (compressed && e->total_bytes) std::memset(compressed, 0, e->total_bytes);
    const int nt = e->n_threads > 0 ? e->n_threads : omp_get_max_threads();
    std::vector<uint8_t> part(K > 0 ? K : 1);
#pragma omp parallel for schedule(static) num_threads(nt)
    for (int64_t k = 0; k < K; k++) {
        const int64_t b = k / kBlk;
        const int64_t g_b = (static_cast<int64_t>(e->offsets[b + 1]) - e->offsets[b]) / (kBlk * 4);
        const int64_t g_s = static_cast<int64_t>((e->bits[k] + 31) / 32);
        if (compressed) {
            SlabSink sink{compressed + e->offsets[b], k % kBlk, g_b - g_s};
            encode_stream(*e, e->symbols + k * N, N, sink, nullptr, &part[k]);
        } else {
            part[k] = static_cast<uint8_t>(e->bits[k] % 32);
        }
    }
    if (partial) std::memcpy(partial, part.data(), K);
    return TANS_B200_OK;
}

extern "C" void tans_b200_encoded_free(tans_b200_encoded *e) { delete e; }

// Tables of the device encoder (layout and meaning in internal.h).
int tans_b200::encoder_tables(const int32_t *freqs, int64_t n_syms, const int32_t *spread,
                              EncoderTables *t) {
    if (!freqs || !spread || !t || n_syms <= 0)
        return fail(TANS_B200_ERR_INVALID, "encode: bad arguments");
    std::vector<uint32_t> cum(n_syms + 1, 0u);
    uint64_t sum = 0;
    for (int64_t s = 0; s < n_syms; s++) {
        if (freqs[s] < 0)
            return fail(TANS_B200_ERR_INVALID, "encode: freqs[%lld] is negative", (long long)s);
        cum[s] = static_cast<uint32_t>(std::min<uint64_t>(sum, kL));
        sum += static_cast<uint32_t>(freqs[s]);
    }
    if (sum != kL)
        return fail(TANS_B200_ERR_INVALID, "freqs must sum to L=%u; got %llu", kL,
                    (unsigned long long)sum);
    std::vector<uint32_t> seen(n_syms, 0u);
    for (uint32_t slot = 0; slot < kL; slot++) {
        int32_t s = spread[slot];
        if (s < 0 || s >= n_syms || seen[s] >= static_cast<uint32_t>(freqs[s]))
            return fail(TANS_B200_ERR_INVALID,
                        "encode: spread[%u]=%d inconsistent with freqs (alphabet %lld)", slot, s,
                        (long long)n_syms);
        t->next[cum[s] + seen[s]++] = static_cast<uint16_t>(kL + slot);
    }
    for (int s = 0; s < 256; s++) {
        const uint32_t f = s < n_syms ? static_cast<uint32_t>(freqs[s]) : 0u;
        if (f == 0) {
            t->delta[s] = kEncoderBadBits << (kTableLog + 1);
            t->base[s] = 0;
            continue;
        }
        const uint32_t lg = (uint32_t)kTableLog;
        const uint32_t k1 = lg - std::min(31u - static_cast<uint32_t>(__builtin_clz(f)), lg);
        t->delta[s] = static_cast<int32_t>(k1 << (kTableLog + 1)) - static_cast<int32_t>(f << k1);
        t->base[s] = static_cast<int32_t>(cum[s]) - static_cast<int32_t>(f);
    }
    return TANS_B200_OK;
}

// ------------------------------------------------------------ FP8 splitter

// Split e4m3 bytes fp8[K][N] (N even) into pair symbols [K][N/2]
// (exp(2i) << 4 | exp(2i+1), tans_codec.py:109,123-124) and packed
// sign/mantissa pairs (sm(2i) | sm(2i+1) << 4, tans_codec.py:110-113) laid
// out tiled [N/2/tile][K][tile] when tile > 0, else [N/2][K]
// (tans_codec.py:115-121).  exp_hist (optional) accumulates the 16-bin
// exponent histogram.
extern "C" int tans_b200_split_fp8(const uint8_t *fp8, int64_t K, int64_t N, int64_t tile,
                                   uint8_t *pair_syms, uint8_t *sm, int64_t *exp_hist,
                                   int n_threads) {
    if (N % 2 != 0) return fail(TANS_B200_ERR_INVALID, "split_fp8: N must be even");
    const int64_t P = N / 2;
    if (tile > 0 && P % tile != 0)
        return fail(TANS_B200_ERR_INVALID, "n_pairs=%lld not divisible by tile=%lld",
                    (long long)P, (long long)tile);
    const int nt = n_threads > 0 ? n_threads : omp_get_max_threads();
    std::vector<int64_t> hist(16, 0);
#pragma omp parallel num_threads(nt)
    {
        int64_t h[16] = {0};
#pragma omp for schedule(static)
        for (int64_t k = 0; k < K; k++) {
            const uint8_t *row = fp8 + k * N;
            for (int64_t i = 0; i < P; i++) {
                const uint8_t b0 = row[2 * i], b1 = row[2 * i + 1];
                const uint8_t e0 = (b0 >> 3) & 15, e1 = (b1 >> 3) & 15;
                const uint8_t m0 = ((b0 >> 4) & 8) | (b0 & 7), m1 = ((b1 >> 4) & 8) | (b1 & 7);
                h[e0]++;
                h[e1]++;
                if (pair_syms) pair_syms[k * P + i] = static_cast<uint8_t>(e0 << 4 | e1);
                if (sm) {
                    const uint8_t v = static_cast<uint8_t>(m0 | m1 << 4);
                    if (tile > 0)
                        sm[((i / tile) * K + k) * tile + (i % tile)] = v;
                    else
                        sm[i * K + k] = v;
                }
            }
        }
#pragma omp critical
        for (int j = 0; j < 16; j++) hist[j] += h[j];
    }
    if (exp_hist)
        for (int j = 0; j < 16; j++) exp_hist[j] += hist[j];
    return TANS_B200_OK;
}
