/*
 * tans_oracle.c — CPU restatement of the reference's tANS FP8 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: tests/, the smoke()
 * entry of __graft_entry__.py and the cpu_baseline leg of bench.py may load
 * it; the product (the rans_vectoradd package and libtans_b200.so) never
 * does.
 *
 * Everything here restates doublewordai/tans-vectoradd in plain C with
 * straightforward loops, deliberately unlike the product kernels:
 *   oracle_fp8_add            csrc/vecadd.cu:27-35   (satfinite RNE e4m3 add)
 *   oracle_compose            csrc/vecadd.cu:37-39, csrc/tans_decode.cu:61-63
 *   oracle_build_decode_table rans_vectoradd/tans_codec.py:63-87
 *   oracle_encode             csrc/tans_codec.cpp:22-60, 69-196
 *   oracle_decode             csrc/tans_decode.cu:65-155
 *   oracle_vecadd_fused       csrc/vecadd.cu:84-154, 156-243
 *   oracle_vecadd_raw         csrc/vecadd.cu:41-73
 *
 * The e4m3 conversion follows the OCP FP8 E4M3 definition (bias 7, no
 * infinities, NaN = S.1111.111) with round-to-nearest-even and the PTX
 * `.satfinite` rule the reference's __nv_fp8_e4m3(float) constructor uses:
 * finite overflow and infinities clamp to +-448, NaN becomes 0x7F.  The sum
 * of two e4m3 values is exact in double, so the single rounding is the
 * conversion back to e4m3.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_L 4096
#define ORACLE_BLOCK 128

/* ------------------------------------------------------------------ e4m3 */

double oracle_e4m3_to_double(uint8_t b) {
    int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
    double v;
    if (e == 15 && m == 7) return NAN;
    if (e == 0)
        v = ldexp((double)m, -9); /* subnormal: m * 2^-9 */
    else
        v = ldexp((double)(8 + m), e - 10); /* (1 + m/8) * 2^(e-7) */
    return s ? -v : v;
}

/* round-half-to-even of a non-negative double that has an exact binary form */
static double rne(double q) {
    double f = floor(q);
    double d = q - f;
    if (d > 0.5) return f + 1.0;
    if (d < 0.5) return f;
    return fmod(f, 2.0) == 0.0 ? f : f + 1.0;
}

uint8_t oracle_e4m3_from_double(double v) {
    uint8_t sign;
    double a, q, r;
    int e2, E;
    if (isnan(v)) return 0x7F;
    sign = signbit(v) ? 0x80 : 0x00;
    a = fabs(v);
    if (a >= 448.0) return (uint8_t)(sign | 0x7E); /* satfinite clamp */
    if (a < 0.015625) {                             /* below 2^-6: subnormal grid 2^-9 */
        r = rne(a * 512.0);                         /* 8 rounds up into the first normal */
        return (uint8_t)(sign | (uint8_t)r);
    }
    frexp(a, &e2);
    E = e2 - 1;             /* a in [2^E, 2^(E+1)) */
    q = ldexp(a, 3 - E);    /* in [8, 16) */
    r = rne(q);
    if (r == 16.0) {
        r = 8.0;
        E += 1;
    }
    return (uint8_t)(sign | ((E + 7) << 3) | ((int)r - 8));
}

uint8_t oracle_fp8_add(uint8_t a, uint8_t b) {
    return oracle_e4m3_from_double(oracle_e4m3_to_double(a) + oracle_e4m3_to_double(b));
}

/* Whole 256x256 add table: out[a*256 + b]. */
void oracle_fp8_add_table(uint8_t *out) {
    for (int a = 0; a < 256; a++)
        for (int b = 0; b < 256; b++) out[a * 256 + b] = oracle_fp8_add((uint8_t)a, (uint8_t)b);
}

uint8_t oracle_compose(uint8_t exp, uint8_t sm) {
    return (uint8_t)(((sm & 8u) << 4) | ((exp & 15u) << 3) | (sm & 7u));
}

void oracle_vecadd_raw(const uint8_t *a, const uint8_t *b, uint8_t *c, int64_t n) {
    uint8_t *tab = (uint8_t *)malloc(65536);
    oracle_fp8_add_table(tab);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) c[i] = tab[(int)a[i] * 256 + b[i]];
    free(tab);
}

/* ---------------------------------------------------------- decode table */

/* tans_codec.py:63-87.  Returns 0, or -1 on inconsistent input. */
int oracle_build_decode_table(const int32_t *spread, const int32_t *freqs, int n_syms,
                              int32_t *table) {
    int64_t *counts = (int64_t *)calloc((size_t)n_syms, sizeof(int64_t));
    for (int slot = 0; slot < ORACLE_L; slot++) {
        int s = spread[slot];
        int64_t rank, x_prev, v, base;
        int nb = 0;
        if (s < 0 || s >= n_syms) {
            free(counts);
            return -1;
        }
        rank = counts[s];
        x_prev = freqs[s] + rank;
        v = x_prev;
        while (v < ORACLE_L) {
            v <<= 1;
            nb++;
        }
        base = x_prev << nb;
        if (base < ORACLE_L || base >= 2 * ORACLE_L) {
            free(counts);
            return -1;
        }
        table[slot] = (int32_t)((uint32_t)(s & 0xFF) | ((uint32_t)(nb & 0xF) << 8) |
                                ((uint32_t)(base & 0xFFFF) << 16));
        counts[s]++;
    }
    free(counts);
    return 0;
}

/* --------------------------------------------------------------- encoder */

/* One stream, bit by bit, exactly as csrc/tans_codec.cpp:22-60 describes:
 * symbols consumed last to first; while x >= 2f emit x's LSB into the current
 * uint32 slab (LSB-first), then x = L + slot(rank x - f).  Slabs are written
 * to `slabs` (capacity cap); returns the slab count, or -1 on overflow. */
static int64_t encode_stream(const uint8_t *sym, int64_t n, const int32_t *freqs,
                             const int32_t *const *enc, uint32_t *slabs, int64_t cap,
                             uint32_t *x_out, uint8_t *partial_out) {
    uint32_t x = ORACLE_L, cur = 0, cnt = 0;
    int64_t ns = 0;
    for (int64_t i = n - 1; i >= 0; i--) {
        int s = sym[i];
        uint32_t f = (uint32_t)freqs[s];
        while (x >= 2u * f) {
            cur |= (x & 1u) << cnt;
            cnt++;
            if (cnt == 32u) {
                if (ns >= cap) return -1;
                slabs[ns++] = cur;
                cur = 0;
                cnt = 0;
            }
            x >>= 1;
        }
        x = (uint32_t)enc[s][x - f];
    }
    *partial_out = (uint8_t)cnt;
    if (cnt > 0) {
        if (ns >= cap) return -1;
        slabs[ns++] = cur;
    }
    *x_out = x;
    return ns;
}

/* csrc/tans_codec.cpp:69-196.  symbols[K][N].  If compressed == NULL only
 * the byte count is computed.  Returns the compressed byte count, or -1. */
int64_t oracle_encode(const uint8_t *symbols, int64_t K, int64_t N, const int32_t *freqs,
                      int n_syms, const int32_t *spread, uint8_t *compressed,
                      uint16_t *states, int32_t *offsets, uint8_t *partial) {
    int64_t n_blocks = (K + ORACLE_BLOCK - 1) / ORACLE_BLOCK;
    int64_t cap = N / 2 + 8; /* >= 12 bits per symbol / 32 + 1 */
    int32_t **enc = (int32_t **)calloc((size_t)n_syms, sizeof(int32_t *));
    int32_t *counts = (int32_t *)calloc((size_t)n_syms, sizeof(int32_t));
    int64_t *nslabs = (int64_t *)calloc((size_t)(K > 0 ? K : 1), sizeof(int64_t));
    uint32_t *all = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(K > 0 ? K : 1) * (size_t)cap);
    uint32_t *xs = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(K > 0 ? K : 1));
    uint8_t *parts = (uint8_t *)malloc((size_t)(K > 0 ? K : 1));
    int64_t total = 0, result = -1, sum = 0;
    int bad = 0;

    for (int s = 0; s < n_syms; s++) {
        if (freqs[s] < 0) goto done;
        sum += freqs[s];
        enc[s] = (int32_t *)calloc((size_t)(freqs[s] > 0 ? freqs[s] : 1), sizeof(int32_t));
    }
    if (sum != ORACLE_L) goto done;
    for (int slot = 0; slot < ORACLE_L; slot++) {
        int s = spread[slot];
        if (s < 0 || s >= n_syms) goto done;
        if (counts[s] >= freqs[s]) goto done;
        enc[s][counts[s]++] = ORACLE_L + slot;
    }

#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t k = 0; k < K; k++) {
        int64_t ns = encode_stream(symbols + k * N, N, freqs, (const int32_t *const *)enc,
                                   all + k * cap, cap, &xs[k], &parts[k]);
        if (ns < 0) bad = 1;
        nslabs[k] = ns;
    }
    if (bad) goto done;

    for (int64_t b = 0; b < n_blocks; b++) {
        int64_t g = 0;
        for (int64_t k = b * ORACLE_BLOCK; k < K && k < (b + 1) * ORACLE_BLOCK; k++)
            if (nslabs[k] > g) g = nslabs[k];
        if (g == 0) g = 1;
        if (offsets) offsets[b] = (int32_t)total;
        total += g * ORACLE_BLOCK * 4;
    }
    if (offsets) offsets[n_blocks] = (int32_t)total;

    if (compressed) {
        memset(compressed, 0, (size_t)total);
        for (int64_t k = 0; k < K; k++) {
            int64_t b = k / ORACLE_BLOCK, t = k % ORACLE_BLOCK;
            int64_t g_b = ((int64_t)offsets[b + 1] - offsets[b]) / (ORACLE_BLOCK * 4);
            for (int64_t g = 0; g < nslabs[k]; g++) {
                int64_t slab = g_b - nslabs[k] + g;
                memcpy(compressed + offsets[b] + slab * ORACLE_BLOCK * 4 + t * 4, &all[k * cap + g],
                       4);
            }
        }
    }
    for (int64_t k = 0; k < K; k++) {
        if (states) states[k] = (uint16_t)xs[k];
        if (partial) partial[k] = parts[k];
    }
    result = total;
done:
    for (int s = 0; s < n_syms; s++) free(enc[s]);
    free(enc);
    free(counts);
    free(nslabs);
    free(all);
    free(xs);
    free(parts);
    return result;
}

/* --------------------------------------------------------------- decoder */

typedef struct {
    uint32_t x, hi, lo, cnt;
    uint32_t L;   /* table size: 4096 (the reference's), 2048 for table_log 11 */
    int64_t slab; /* next slab index to load, or < 0 */
    const uint8_t *blk;
} chain_t;

static uint32_t load_slab(const chain_t *c, int64_t slab, int64_t t) {
    uint32_t w;
    memcpy(&w, c->blk + slab * ORACLE_BLOCK * 4 + t * 4, 4);
    return w;
}

/* tans_decode.cu:65-92 (init_tans_ctx).  Returns -1 on malformed metadata. */
static int chain_init(chain_t *c, const uint8_t *comp, int64_t comp_bytes, const int32_t *offsets,
                      const uint16_t *states, const uint8_t *partial, int64_t sid, uint32_t L) {
    int64_t b = sid / ORACLE_BLOCK, t = sid % ORACLE_BLOCK;
    int64_t base = offsets[b], next = offsets[b + 1], g;
    if (base < 0 || next < base || next > comp_bytes || (next - base) % (ORACLE_BLOCK * 4) != 0)
        return -1;
    g = (next - base) / (ORACLE_BLOCK * 4);
    if (g < 1) return -1;
    if (states[sid] < L || states[sid] >= 2 * L) return -1;
    c->L = L;
    c->blk = comp + base;
    c->x = states[sid];
    c->hi = load_slab(c, g - 1, t);
    c->lo = g >= 2 ? load_slab(c, g - 2, t) : 0u;
    c->slab = g - 3;
    c->cnt = partial[sid] == 0 ? 0u : 32u - partial[sid];
    return 0;
}

/* tans_decode.cu:94-123 (tans_step).  Returns the pair symbol. */
static uint8_t chain_step(chain_t *c, const int32_t *table, int64_t t) {
    uint32_t e = (uint32_t)table[c->x - c->L];
    uint32_t nb = (e >> 8) & 15u, base = (e >> 16) & 0xFFFFu;
    uint32_t window = c->cnt == 0 ? c->hi : (c->hi << c->cnt) | (c->lo >> (32u - c->cnt));
    uint32_t bits = nb == 0 ? 0u : window >> (32u - nb);
    c->x = base | bits;
    c->cnt += nb;
    if (c->cnt >= 32u) {
        c->cnt -= 32u;
        c->hi = c->lo;
        c->lo = c->slab >= 0 ? load_slab(c, c->slab, t) : 0u;
        c->slab -= 1;
    }
    return (uint8_t)(e & 0xFFu);
}

/* tans_decode.cu:125-155: out[N][K], sm[N/2][K].  Returns 0, or -1 if any
 * stream's metadata is malformed (that stream's output is zeroed). */
int oracle_decode_l(const uint8_t *comp, int64_t comp_bytes, const int32_t *offsets,
                    const uint16_t *states, const uint8_t *partial, const uint8_t *sm,
                    const int32_t *table, int64_t K, int64_t N, uint8_t *out, int64_t L) {
    int bad = 0;
    if (L != ORACLE_L && L != ORACLE_L / 2) return -1;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t k = 0; k < K; k++) {
        chain_t c;
        int64_t t = k % ORACLE_BLOCK;
        if (chain_init(&c, comp, comp_bytes, offsets, states, partial, k, (uint32_t)L) != 0) {
            for (int64_t j = 0; j < N; j++) out[j * K + k] = 0;
            bad = 1;
            continue;
        }
        for (int64_t i = 0; i < N / 2; i++) {
            uint8_t s = chain_step(&c, table, t);
            uint8_t m = sm[i * K + k];
            out[(2 * i) * K + k] = oracle_compose(s >> 4, m & 15);
            out[(2 * i + 1) * K + k] = oracle_compose(s & 15, m >> 4);
        }
    }
    return bad ? -1 : 0;
}

/* The reference's table size (tans_codec.py:24-25). */
int oracle_decode(const uint8_t *comp, int64_t comp_bytes, const int32_t *offsets,
                  const uint16_t *states, const uint8_t *partial, const uint8_t *sm,
                  const int32_t *table, int64_t K, int64_t N, uint8_t *out) {
    return oracle_decode_l(comp, comp_bytes, offsets, states, partial, sm, table, K, N, out,
                           ORACLE_L);
}

/* vecadd.cu:156-243: both inputs decoded with one table, composed, added;
 * sm tiled [N/16][K][8], out tiled [N/16][K][16].  Returns 0 or -1.  L is
 * the table size (4096, or 2048 for the table_log 11 extra). */
int oracle_vecadd_fused_l(const uint8_t *a_comp, int64_t a_bytes, const int32_t *a_off,
                          const uint16_t *a_st, const uint8_t *a_part, const uint8_t *a_sm,
                          const uint8_t *b_comp, int64_t b_bytes, const int32_t *b_off,
                          const uint16_t *b_st, const uint8_t *b_part, const uint8_t *b_sm,
                          const int32_t *table, int64_t K, int64_t N, uint8_t *out, int64_t L) {
    uint8_t *tab;
    int bad = 0;
    if (L != ORACLE_L && L != ORACLE_L / 2) return -1;
    tab = (uint8_t *)malloc(65536);
    int64_t n_tiles = N / 16;
    oracle_fp8_add_table(tab);
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t k = 0; k < K; k++) {
        chain_t ca, cb;
        int64_t t = k % ORACLE_BLOCK;
        if (chain_init(&ca, a_comp, a_bytes, a_off, a_st, a_part, k, (uint32_t)L) != 0 ||
            chain_init(&cb, b_comp, b_bytes, b_off, b_st, b_part, k, (uint32_t)L) != 0) {
            for (int64_t j = 0; j < n_tiles; j++) memset(out + (j * K + k) * 16, 0, 16);
            bad = 1;
            continue;
        }
        for (int64_t j = 0; j < n_tiles; j++) {
            for (int p = 0; p < 8; p++) {
                uint8_t sa = chain_step(&ca, table, t), sb = chain_step(&cb, table, t);
                uint8_t ma = a_sm[(j * K + k) * 8 + p], mb = b_sm[(j * K + k) * 8 + p];
                uint8_t a0 = oracle_compose(sa >> 4, ma & 15), a1 = oracle_compose(sa & 15, ma >> 4);
                uint8_t b0 = oracle_compose(sb >> 4, mb & 15), b1 = oracle_compose(sb & 15, mb >> 4);
                out[(j * K + k) * 16 + 2 * p] = tab[a0 * 256 + b0];
                out[(j * K + k) * 16 + 2 * p + 1] = tab[a1 * 256 + b1];
            }
        }
    }
    free(tab);
    return bad ? -1 : 0;
}

int oracle_vecadd_fused(const uint8_t *a_comp, int64_t a_bytes, const int32_t *a_off,
                        const uint16_t *a_st, const uint8_t *a_part, const uint8_t *a_sm,
                        const uint8_t *b_comp, int64_t b_bytes, const int32_t *b_off,
                        const uint16_t *b_st, const uint8_t *b_part, const uint8_t *b_sm,
                        const int32_t *table, int64_t K, int64_t N, uint8_t *out) {
    return oracle_vecadd_fused_l(a_comp, a_bytes, a_off, a_st, a_part, a_sm, b_comp, b_bytes, b_off,
                                 b_st, b_part, b_sm, table, K, N, out, ORACLE_L);
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    extern int omp_get_max_threads(void);
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Thread count of the OpenMP loops above (launchers such as torchrun set
 * OMP_NUM_THREADS=1 in every rank; the timed CPU baseline wants all cores). */
void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    extern void omp_set_num_threads(int);
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
