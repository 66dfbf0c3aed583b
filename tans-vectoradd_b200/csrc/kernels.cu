// kernels.cu — sm_100a device half of libtans_b200 (C ABI in include/tans_b200.h).
//
// Kernels and the reference code each one replaces:
//   memcpy_kernel        csrc/fp8_memcpy.cu:30-41     (practical HBM ceiling)
//   vecadd_raw_kernel    csrc/vecadd.cu:41-73         (uncompressed FP8 add)
//   build_table_kernel   csrc/tans_decode.cu:23-59    (host table build, per call)
//   decode_kernel        csrc/tans_decode.cu:125-155  (standalone decode, [N,K] out)
//   fused_pair_kernel    csrc/vecadd.cu:156-243       (decode A and B + add, tiled out)
//
// Design (B200-first, not a translation of the reference):
//  * FP8 add: e4m3x2 -> f16x2 (exact), add.rn.f16x2, cvt.rn.satfinite.e4m3x2.
//    The f16 sum of two e4m3 values rounded once more to e4m3 equals the
//    reference's f32-sum-then-satfinite-convert for all 65,536 byte pairs (an
//    exhaustive check lives in the tests), at half the instruction count of
//    an f32 path.
//  * tANS decode: the 4096-entry table lives in shared memory as C
//    word-interleaved copies; lane l reads copy l % C, so its lookups land in
//    the 32/C banks of that copy and random lookups from a warp collide less
//    (expected wavefronts per warp lookup 3.51 -> 3.29 for C = 4).  Each
//    entry is re-packed so one lookup yields everything the next step needs:
//        bits  0-4  nb             (also the funnel-shift amount, see below)
//        bits  8-15 pair symbol
//        bits 16-31 byte offset of the successor base entry in this lane's copy
//    The next lookup address is (e >> 16) + (bits << log2(4C)).  bits itself
//    is __funnelshift_l(window, 0, e): the wrap-mode shift uses e & 31 = nb and
//    yields 0 for nb = 0, so no field extraction is needed.
//  * The consumed-bit counter is bumped by the whole entry (bits 5-7 are 0),
//    so its low 5 bits track the position inside the current slab and bit 5
//    flips exactly when a slab is exhausted: one add and one xor-test per step.
//  * Slab refills come from a per-warp shared-memory ring of slab rows that
//    the warp fills ahead of use with cp.async (see Ring); the bit window is
//    the two registers hi:lo.
//  * One thread owns one stream.  In the fused kernel a pair of warps owns a
//    32-stream group, one warp per input, exchanging decoded pair symbols per
//    tile through shared memory.  Grids are persistent and balanced over the
//    SMs: every warp runs the same number of 32-stream groups.
//  * Malformed metadata never causes an out-of-bounds access: offsets, states
//    and table entries are validated or masked in-kernel and reported through
//    an optional device status word.

#include "../../include/tans_b200.h"
#include "internal.h"

#include <cuda.h>  // CUtensorMap and its enums (the encoder is resolved at run time)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>
#include <mutex>
#include <utility>

using tans_b200::fail;

namespace {

constexpr int kL = TANS_B200_TABLE_SIZE;
constexpr int kBlk = TANS_B200_BLOCK_STREAMS;
constexpr int kCopies = 4;  // table copies in shared memory
constexpr int kLog4C = 4;   // log2(4 * kCopies)
constexpr int kTablePairs = 8;  // pairs per fused tile (16 output bytes)
static_assert(4 * kCopies == (1 << kLog4C), "copy count and shift disagree");

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_stream_v4(void *p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint2 ld_stream_v2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Programmatic dependent launch (the GEMV chain: GEMV -> reduce or publish ->
// next GEMV).  A kernel lets the next one in its stream start as soon as all
// of its own CTAs are running, so the next kernel's prologue (the GEMV's
// table load and first row group's set-up, which read only its weight)
// overlaps its tail; the next kernel waits for this one to complete, with
// its memory visible, before it reads anything this one writes.  Every
// global write of these kernels, other than an error bit ORed into the
// status word, comes after their wait.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t ld_stream_u32(const void *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ void st_stream_v2(void *p, uint32_t x, uint32_t y) {
    asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(x), "r"(y) : "memory");
}

__device__ __forceinline__ void st_stream_u32(void *p, uint32_t x) {
    asm volatile("st.global.cs.u32 [%0], %1;" ::"l"(p), "r"(x) : "memory");
}

// Four e4m3 additions: byte i of the result = satfinite_e4m3(a_i + b_i).
__device__ __forceinline__ uint32_t add_e4m3x4(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("{\n\t"
        ".reg .b16 al, ah, bl, bh, rl, rh;\n\t"
        ".reg .b32 fa0, fa1, fb0, fb1, s0, s1;\n\t"
        "mov.b32 {al, ah}, %1;\n\t"
        "mov.b32 {bl, bh}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 fa0, al;\n\t"
        "cvt.rn.f16x2.e4m3x2 fa1, ah;\n\t"
        "cvt.rn.f16x2.e4m3x2 fb0, bl;\n\t"
        "cvt.rn.f16x2.e4m3x2 fb1, bh;\n\t"
        "add.rn.f16x2 s0, fa0, fb0;\n\t"
        "add.rn.f16x2 s1, fa1, fb1;\n\t"
        "cvt.rn.satfinite.e4m3x2.f16x2 rl, s0;\n\t"
        "cvt.rn.satfinite.e4m3x2.f16x2 rh, s1;\n\t"
        "mov.b32 %0, {rl, rh};\n\t"
        "}"
        : "=r"(r)
        : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint4 add_e4m3x16(uint4 a, uint4 b) {
    return make_uint4(add_e4m3x4(a.x, b.x), add_e4m3x4(a.y, b.y), add_e4m3x4(a.z, b.z),
                      add_e4m3x4(a.w, b.w));
}

// -------------------------------------------------------- memcpy / raw add

constexpr int kStreamThreads = 256;
constexpr int kStreamUnroll = 4;

__global__ void __launch_bounds__(kStreamThreads) memcpy_kernel(const uint4 *__restrict__ a,
                                                                uint4 *__restrict__ c,
                                                                int64_t n_vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < n_vec;
         base += stride * kStreamUnroll) {
        uint4 v[kStreamUnroll];
#pragma unroll
        for (int u = 0; u < kStreamUnroll; u++)
            if (base + u * stride < n_vec) v[u] = ld_stream_v4(a + base + u * stride);
#pragma unroll
        for (int u = 0; u < kStreamUnroll; u++)
            if (base + u * stride < n_vec) st_stream_v4(c + base + u * stride, v[u]);
    }
}

__global__ void __launch_bounds__(kStreamThreads) vecadd_raw_kernel(const uint4 *__restrict__ a,
                                                                    const uint4 *__restrict__ b,
                                                                    uint4 *__restrict__ c,
                                                                    int64_t n_vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < n_vec;
         base += stride * kStreamUnroll) {
        uint4 va[kStreamUnroll], vb[kStreamUnroll];
#pragma unroll
        for (int u = 0; u < kStreamUnroll; u++)
            if (base + u * stride < n_vec) {
                va[u] = ld_stream_v4(a + base + u * stride);
                vb[u] = ld_stream_v4(b + base + u * stride);
            }
#pragma unroll
        for (int u = 0; u < kStreamUnroll; u++)
            if (base + u * stride < n_vec)
                st_stream_v4(c + base + u * stride, add_e4m3x16(va[u], vb[u]));
    }
}

// ------------------------------------------------------ decode-table build

// One CTA of kBuildWarps warps (L / 4 threads: 1024 for L = 4096).  Warp w
// owns slots [128w, 128w+128).  A symbol's rank at a slot is the number of
// earlier slots holding it: per-warp histograms, an exclusive scan across
// warps, then in-warp ranks from __match_any_sync, processed in slot order.
constexpr int kBuildWarps = kL / 128;
static_assert(kBuildWarps * 128 == kL && kBuildWarps <= 32, "table builder geometry");
__global__ void __launch_bounds__(kBuildWarps * 32) build_table_kernel(const int32_t *__restrict__ spread,
                                                           const int32_t *__restrict__ freqs,
                                                           int n_syms, int32_t *__restrict__ table,
                                                           int32_t *__restrict__ status) {
    __shared__ uint32_t cnt[kBuildWarps][256];
    __shared__ int32_t fr[256];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < kBuildWarps * 256; i += blockDim.x) (&cnt[0][0])[i] = 0;
    if (tid < 256) fr[tid] = tid < n_syms ? freqs[tid] : 0;
    __syncthreads();
    int sym[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
        int s = spread[warp * 128 + r * 32 + lane];
        if (s < 0 || s >= n_syms) {
            if (status) atomicOr(status, TANS_B200_DATA_BAD_TABLE);
            s = 0;
        }
        sym[r] = s;
        atomicAdd(&cnt[warp][s], 1u);
    }
    __syncthreads();
    if (tid < 256) {  // exclusive scan over warps for symbol tid
        uint32_t run = 0;
        for (int w = 0; w < kBuildWarps; w++) {
            uint32_t v = cnt[w][tid];
            cnt[w][tid] = run;
            run += v;
        }
    }
    __syncthreads();
    const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int s = sym[r];
        const uint32_t peers = __match_any_sync(0xffffffffu, s);
        const uint32_t rank = cnt[warp][s] + __popc(peers & lt);
        __syncwarp();
        if ((peers & lt) == 0) cnt[warp][s] += __popc(peers);
        __syncwarp();
        const int64_t xp = (int64_t)fr[s] + rank;
        uint32_t entry = 0;
        if (xp > 0 && xp < 2 * kL) {
            const int nb = tans_b200::kTableLog - (31 - __clz((uint32_t)xp));
            if (nb >= 0) entry = (uint32_t)s | ((uint32_t)nb << 8) | (((uint32_t)xp << nb) << 16);
        }
        if (entry == 0 && status) atomicOr(status, TANS_B200_DATA_BAD_TABLE);
        table[warp * 128 + r * 32 + lane] = (int32_t)entry;
    }
}

// ------------------------------------------------------------- tANS chain

// Re-pack the reference table (sym | nb << 8 | base << 16) into kCopies
// interleaved copies of the internal entry layout described at the top.
__device__ __forceinline__ void load_table(uint32_t *tbl, const int32_t *__restrict__ ref,
                                           int32_t *status) {
    bool bad = false;
    for (int i = threadIdx.x; i < kL; i += blockDim.x) {
        const uint32_t r = (uint32_t)__ldg(ref + i);
        const uint32_t sym = r & 0xFFu, base = r >> 16;
        uint32_t nb = (r >> 8) & 0xFu;
        const uint32_t bidx = (base - kL) & (kL - 1);
        // a valid entry has base in [L, 2L) with nb low zero bits, so that
        // base | bits stays in [L, 2L); anything else is clamped to nb = 0
        if (base < (uint32_t)kL || base >= 2u * kL || (bidx & ((1u << nb) - 1u)) != 0 ||
            bidx + (1u << nb) > (uint32_t)kL) {
            nb = 0;
            bad = true;
        }
        const uint32_t v = (sym << 8) | nb;
#pragma unroll
        for (int c = 0; c < kCopies; c++)
            tbl[i * kCopies + c] = ((bidx * 4u * kCopies + 4u * c) << 16) | v;
    }
    if (bad && status) atomicOr(status, TANS_B200_DATA_BAD_TABLE);
}

// Integer constants the kernels receive as parameters.  Their values are
// fixed (set by the host), but because ptxas cannot see them it must emit
// IMAD / IMAD.HI for the shifts, adds and moves written with them below.
// Those run on the FMA pipe, which otherwise idles in this kernel, instead of
// the ALU pipe that bounds it.
struct Opq {
    uint32_t one;    // 1
    uint32_t p16;    // 2^16: mul.hi(x, p16) = x >> 16
    uint32_t p31;    // 2^31: mul.hi(x, p31) = x >> 1
    uint32_t p28;    // 2^28: mul.hi(x, p28) = x >> 4
    uint32_t x16;    // 16:   x * 16 = x << 4
    uint32_t x8;     // 8:    x * 8 = x << 3
    uint32_t step;   // 4 * kCopies (bytes between successive entries of a copy)
    int32_t back;    // -128: one slab row down, in words
    int32_t back64;  // -64: one slab row down in the fused kernel's 64-unit rows
    uint32_t p26;    // 2^26: mul.hi.s32(v, p26) = v >> 6 (row of a 64-unit v)
    uint32_t p25;    // 2^25: mul.hi.s32(v, p25) = v >> 7 (row of a 128-unit v)
    uint32_t rmask;  // (R - 1) * 64: ring row offset of a 64-unit v (set per launch)
};

__device__ __forceinline__ uint32_t mul_lo(uint32_t x, uint32_t y) {
    uint32_t r;
    asm("mul.lo.u32 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(y));
    return r;
}
__device__ __forceinline__ uint32_t mul_hi(uint32_t x, uint32_t y) {
    uint32_t r;
    asm("mul.hi.u32 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(y));
    return r;
}

// One stream's decoder state: the bit window hi:lo (next bits at the top of
// hi after skipping cnt bits) and `v`, the word offset (row * 128) of the
// slab that the next advance loads into lo.  Rows count down from the top of
// the encoder block; row r of this lane lives at src[r * 128].
struct Chain {
    uint32_t addr;  // byte offset of the current entry in this lane's table copy
    uint32_t cnt;   // bits 0-4: bits used in hi; bit 5 flips per exhausted slab
    uint32_t hi, lo;
    int32_t v;
    const uint32_t *src;
};

// A chain for a lane with no stream: steps harmlessly, never loads.
__device__ __forceinline__ void chain_idle(Chain &ch, const uint32_t *comp) {
    ch.addr = 0;
    ch.cnt = 0;
    ch.hi = ch.lo = 0;
    ch.v = -kBlk;
    ch.src = comp;
}

// init_tans_ctx (csrc/tans_decode.cu:65-92) with in-kernel validation.
// Returns the block's slab count G (0 if the metadata is malformed).
__device__ __forceinline__ int32_t chain_init(Chain &ch, const uint32_t *__restrict__ comp,
                                              int64_t comp_bytes,
                                              const int32_t *__restrict__ offsets,
                                              const uint16_t *__restrict__ states,
                                              const uint8_t *__restrict__ partial, int64_t sid,
                                              uint32_t lane_off, int32_t *status) {
    const int64_t b = sid / kBlk;
    const int tid = (int)(sid % kBlk);
    const int64_t base = __ldg(offsets + b), next = __ldg(offsets + b + 1);
    const bool ok = base >= 0 && next > base && next <= comp_bytes && ((next - base) % 512) == 0 &&
                    (base % 4) == 0;
    uint32_t x = __ldg(states + sid);
    if (x < (uint32_t)kL || x >= 2u * kL) {
        if (status) atomicOr(status, TANS_B200_DATA_BAD_STATE);
    }
    const uint32_t p = __ldg(partial + sid);
    if (!ok) {
        if (status) atomicOr(status, TANS_B200_DATA_BAD_OFFSETS);
        chain_idle(ch, comp);
        return 0;
    }
    const int32_t G = (int32_t)((next - base) / 512);
    ch.addr = ((x - kL) & (kL - 1)) * (4u * kCopies) + lane_off;
    ch.cnt = p == 0 ? 0u : ((32u - p) & 31u);
    ch.src = comp + base / 4 + tid;
    ch.hi = __ldg(ch.src + (G - 1) * kBlk);
    ch.lo = G >= 2 ? __ldg(ch.src + (G - 2) * kBlk) : 0u;
    ch.v = (G - 3) * kBlk;
    return G;
}

// Table lookup and window update shared by both step flavours.  On a slab
// advance hi <- lo and lo is reloaded by a predicated load; once a chain has
// run past its block's first row nothing is loaded and lo keeps a stale word,
// whose bits lie beyond the end of the stream and are never consumed.
#define TANS_STEP_HEAD                                                            \
    "mul.hi.u32 f, %5, %8;\n\t"          /* f = e >> 16 */                        \
    "shf.l.wrap.b32 w, %3, %2, %1;\n\t"  /* w = top 32 bits of (hi:lo) << cnt */ \
    "shf.l.wrap.b32 bits, w, 0, %5;\n\t" /* bits = w >> (32 - nb), 0 if nb=0 */  \
    "mad.lo.u32 %0, bits, %9, f;\n\t"    /* next entry address */                \
    "mad.lo.u32 c2, %5, %7, %1;\n\t"     /* cnt + e: bit 5 flips per slab */     \
    "xor.b32 t, c2, %1;\n\t"                                                    \
    "and.b32 t, t, 32;\n\t"                                                     \
    "setp.ne.u32 pa, t, 0;\n\t"                                                 \
    "mov.u32 %1, c2;\n\t"

// Refill from global memory (any row, any time).
__device__ __forceinline__ uint32_t chain_step_global(Chain &ch, const uint8_t *tbl_bytes,
                                                      const Opq &q) {
    const uint32_t e = *reinterpret_cast<const uint32_t *>(tbl_bytes + ch.addr);
    asm volatile(
        "{\n\t"
        ".reg .u32 w, bits, f, c2, t;\n\t"
        ".reg .pred pa, pl;\n\t"
        ".reg .u64 ga;\n\t" TANS_STEP_HEAD
        "setp.ge.and.s32 pl, %4, 0, pa;\n\t"
        "mul.wide.s32 ga, %4, 4;\n\t"
        "add.u64 ga, ga, %6;\n\t"
        "@pa mad.lo.u32 %2, %3, %7, 0;\n\t"    /* hi <- lo */
        "@pl ld.global.nc.u32 %3, [ga];\n\t"   /* lo <- next slab of this stream */
        "@pa mad.lo.s32 %4, %7, %10, %4;\n\t"  /* one row down */
        "}"
        : "+r"(ch.addr), "+r"(ch.cnt), "+r"(ch.hi), "+r"(ch.lo), "+r"(ch.v)
        : "r"(e), "l"(ch.src), "r"(q.one), "r"(q.p16), "r"(q.step), "r"(q.back));
    return e;
}

// Refill from this warp's shared-memory row ring: the slot of row r for this
// lane is at ring_lane + (r mod R) * 128, i.e. (v & mask) | ring_lane.
__device__ __forceinline__ uint32_t chain_step_ring(Chain &ch, const uint8_t *tbl_bytes,
                                                    uint32_t ring_lane, uint32_t mask,
                                                    const Opq &q) {
    const uint32_t e = *reinterpret_cast<const uint32_t *>(tbl_bytes + ch.addr);
    asm volatile(
        "{\n\t"
        ".reg .u32 w, bits, f, c2, t, sa;\n\t"
        ".reg .pred pa;\n\t" TANS_STEP_HEAD
        "and.b32 sa, %4, %11;\n\t"
        "or.b32 sa, sa, %12;\n\t"
        "@pa mad.lo.u32 %2, %3, %7, 0;\n\t"    /* hi <- lo */
        "@pa ld.shared.u32 %3, [sa];\n\t"      /* lo <- next slab of this stream */
        "@pa mad.lo.s32 %4, %7, %10, %4;\n\t"  /* one row down */
        "}"
        : "+r"(ch.addr), "+r"(ch.cnt), "+r"(ch.hi), "+r"(ch.lo), "+r"(ch.v)
        : "r"(e), "l"(ch.src), "r"(q.one), "r"(q.p16), "r"(q.step), "r"(q.back), "r"(mask),
          "r"(ring_lane));
    return e;
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src, bool pred) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t"
        "@p cp.async.ca.shared.global [%0], [%1], 4;\n\t}" ::"r"(dst),
        "l"(src), "r"((uint32_t)pred)
        : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Row ring of one chain of one warp.  The warp fills whole rows (each lane
// copies its own column with cp.async, so every row is one coalesced 128-byte
// read and a lane only ever reads data it copied itself), from the top down,
// never over a slot whose row the slowest lane still needs.  A tile may
// refill from the ring only when every row its lanes can reach in that tile
// (at most 3 rows per tile) belongs to a fill group that has completed
// (cp.async.wait_group kRingLag: groups kRingLag tiles old); otherwise the
// tile refills from global memory, which is always exact.
constexpr int kRingLag = 2;
constexpr int32_t kNoRow = -(1 << 30);  // row reported by lanes without a stream
constexpr int kDecodeLag = 1;   // fill-group age read by the decode kernel
constexpr int kRingBurst = 12;  // rows filled when a group starts
constexpr int kRingPerTile = 2; // rows filled per tile after that

template <int kDepth>
struct RingT {
    uint32_t lane_base;        // shared address of this lane's column, row slot 0
    int32_t fill;              // next row to fill (warp-uniform)
    int32_t done[kDepth + 1];  // lowest filled row after the last kDepth + 1 fills
};
using Ring = RingT<kRingLag>;

template <int R, int D>
__device__ __forceinline__ void ring_start(RingT<D> &rg, const Chain &ch, int32_t G, bool live) {
    rg.fill = G - 3;
#pragma unroll
    for (int k = 0; k < kRingBurst; k++) {
        cp_async4(rg.lane_base + ((uint32_t)(rg.fill & (R - 1)) << 7),
                  ch.src + (int64_t)rg.fill * kBlk, live && rg.fill >= 0);
        rg.fill -= rg.fill >= 0 ? 1 : 0;
    }
    // the caller commits and waits for this burst (cp.async.wait_group 0)
    // before the first tile, so every tile can refill from the ring
#pragma unroll
    for (int i = 0; i <= D; i++) rg.done[i] = rg.fill + 1;
}

// This tile's fills; returns the lowest row a lane may refill from during
// the tile (the fast path needs it at or above done[kRingLag]).
template <int R, int D>
__device__ __forceinline__ int32_t ring_fill(RingT<D> &rg, const Chain &ch, bool live) {
    const int32_t row = ch.v >> 7;
    const int32_t r_fast = __reduce_min_sync(0xffffffffu, live ? row : INT_MAX);
    // lanes without a stream report a far-negative row (no overflow in r_slow - R)
    const int32_t r_slow = __reduce_max_sync(0xffffffffu, live ? row : kNoRow);
    const int32_t lim = r_slow - R;
#pragma unroll
    for (int k = 0; k < kRingPerTile; k++) {
        const bool go = rg.fill >= 0 && rg.fill > lim;
        cp_async4(rg.lane_base + ((uint32_t)(rg.fill & (R - 1)) << 7),
                  ch.src + (int64_t)rg.fill * kBlk, live && go);
        rg.fill -= go ? 1 : 0;
    }
#pragma unroll
    for (int i = D; i > 0; i--) rg.done[i] = rg.done[i - 1];
    rg.done[0] = rg.fill + 1;
    return r_fast == INT_MAX ? INT_MAX : max(r_fast - 2, 0);
}

// Pack the pair symbols of four entries into one word (byte k = entry k).
__device__ __forceinline__ uint32_t gather_syms(uint32_t e0, uint32_t e1, uint32_t e2,
                                                uint32_t e3) {
    return __byte_perm(__byte_perm(e0, e1, 0x0051), __byte_perm(e2, e3, 0x0051), 0x5410);
}

// Compose e4m3 bytes from four pair symbols S (byte k = exp(2k) << 4 | exp(2k+1))
// and four sign/mantissa pairs M (byte k = sm(2k) | sm(2k+1) << 4):
// even: byte k = element 2k; odd: byte k = element 2k+1.
// Byte = (sm & 8) << 4 | exp << 3 | (sm & 7)  (csrc/vecadd.cu:37-39).
// Shifts go through the FMA pipe (see Opq).
// Each is two bitwise selects (lop3 (a & m) | (b & ~m), LUT 0xE4) of the
// shifted operands: the sign bit from one, the mantissa bits from another,
// the exponent bits from the third.
__device__ __forceinline__ uint32_t compose_even(uint32_t S, uint32_t M, const Opq &q) {
    uint32_t t, r;
    asm("lop3.b32 %0, %1, %2, 0x80808080, 0xE4;" : "=r"(t) : "r"(mul_lo(M, q.x16)), "r"(mul_hi(S, q.p31)));
    asm("lop3.b32 %0, %1, %2, 0x07070707, 0xE4;" : "=r"(r) : "r"(M), "r"(t));
    return r;
}
__device__ __forceinline__ uint32_t compose_odd(uint32_t S, uint32_t M, const Opq &q) {
    uint32_t t, r;
    asm("lop3.b32 %0, %1, %2, 0x80808080, 0xE4;" : "=r"(t) : "r"(M), "r"(mul_lo(S, q.x8)));
    asm("lop3.b32 %0, %1, %2, 0x07070707, 0xE4;" : "=r"(r) : "r"(mul_hi(M, q.p28)), "r"(t));
    return r;
}

// Persistent-grid geometry: every warp runs `rounds` 32-stream groups.
struct Geometry {
    int grid, warps_per_cta;
};

Geometry balance(int64_t n_groups, int sms, int max_warps_per_cta) {
    if (n_groups <= 0) return {1, 1};
    const int64_t per_round = (int64_t)sms * max_warps_per_cta;
    const int64_t rounds = (n_groups + per_round - 1) / per_round;
    int64_t wpc = (n_groups + (int64_t)sms * rounds - 1) / ((int64_t)sms * rounds);
    if (wpc < 1) wpc = 1;
    const int64_t grid = (n_groups + wpc * rounds - 1) / (wpc * rounds);
    return {(int)grid, (int)wpc};
}

constexpr int kTableBytes = kL * kCopies * 4;
constexpr int kMaxWarps = 16;  // 512 threads per CTA, one CTA per SM
// The decode kernel: up to 7 teams of 4 warps (its registers fit 896
// threads, 72 each, without spills)
constexpr int kDecodeMaxWarps = 28;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// Shared address of warp w's ring area (aligned to its size so that a slot
// address is (v & mask) | lane_base).
template <int R>
__device__ __forceinline__ uint32_t ring_area(const uint8_t *smem, int warp, int chains) {
    const uint32_t bytes = R * 128u;
    const uint32_t first = (smem_addr(smem) + kTableBytes + bytes - 1) & ~(bytes - 1);
    return first + (uint32_t)(warp * chains) * bytes;
}

// ------------------------------------------- two-step chains and slab rings

// Slab ring of the fused kernel.  Each half-warp (16 streams of one input)
// keeps a ring of R slab rows of its 16 stream columns (64 bytes per row) in
// shared memory; row r sits in ring row r mod R.  The warp fills it with
// 16-byte cp.async copies: lane li of half h copies bytes 16 (li % 4) ..
// of row fill - li / 4 of its half's block, so one instruction moves four
// rows of both halves' rings.  A fill never overwrites a row that any lane of
// the half may still read (rows above the slowest lane's next row minus R,
// with one row of margin for a refill load still in flight).  After the copy
// groups one fill old have landed (cp.async.wait_group 1, then __syncwarp so
// that every lane sees the copies of the others), a tile may refill from the
// ring if every row its lanes can reach is at or above that older fill
// frontier; otherwise it waits for the newest group too, and if even that
// does not cover it, it refills from global memory, which is always exact.
constexpr int kPairFillRows = 4;  // rows per half filled by one copy instruction

struct PairRing {
    int32_t fill;    // next row to fill (< 0: every row is filled)
    int32_t done0;   // lowest filled row including the newest group (INT_MIN: all rows)
    int32_t done1;   // ... excluding it (complete once wait_group 1 returns)
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool pred) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t"
        "@p cp.async.cg.shared.global [%0], [%1], 16;\n\t}" ::"r"(dst),
        "l"(src), "r"((uint32_t)pred)
        : "memory");
}

// Copy the rows fill .. fill - 3 of a ring that lie above `lim` and at or
// above row 0; returns the new fill row.  A ring row holds kUnit bytes (64:
// 16 streams, 128: 32 streams) and is copied by kUnit / 16 lanes, 16 bytes
// each, so the li-th lane of the ring's lanes copies piece li % (kUnit/16)
// of row fill - li / (kUnit/16).  `src` is this lane's 16-byte piece of row 0
// of the block (rows 512 bytes apart), `dst` its piece of ring row 0; the
// ring row of row r is at (kUnit r) & mask (the ring is aligned to its size).
template <int kUnit>
__device__ __forceinline__ int32_t ring_fill16(int32_t fill, int32_t lim, bool on, int li,
                                               const uint8_t *src, uint32_t dst, uint32_t mask) {
    const int32_t r = fill - li / (kUnit / 16);
    const bool go = on && r > lim && r >= 0;
    cp_async16(dst | ((uint32_t)(r * kUnit) & mask), src + (int64_t)r * 512, go);
    return on ? min(fill, max(fill - kPairFillRows, max(lim, -1))) : fill;
}

// Two tANS steps with one slab-exhaustion test.  Two steps consume at most 24
// bits and the window w (bits cnt .. cnt + 31 of hi:lo) holds them all, so the
// second step reads w << nb1; cnt < 32 before and < 56 after, so at most one
// slab is exhausted and one refill (hi <- lo, lo <- next row) follows.  Here v
// counts rows in units of 64 (row r: v = 64 r), matching 64-byte ring rows.
// Shifts, adds and moves are multiplies by the opaque constants of Opq so
// that they run on the FMA pipe; the funnel shifts and the slab test stay on
// the ALU.
#define TANS_STEP2_FIRST                                                                  \
    asm("{\n\t.reg .u32 b, f;\n\t"                                                        \
        "shf.l.wrap.b32 %0, %3, %4, %5;\n\t" /* w = top 32 bits of (hi:lo) << cnt */      \
        "shf.l.wrap.b32 b, %0, 0, %2;\n\t"   /* bits1 = w >> (32 - nb1), 0 if nb1 = 0 */ \
        "mul.hi.u32 f, %2, %6;\n\t"          /* e1 >> 16 */                               \
        "mad.lo.u32 %1, b, %7, f;\n\t}"      /* entry of step 2 */                        \
        : "=r"(w), "=r"(a1)                                                               \
        : "r"(e1), "r"(ch.lo), "r"(ch.hi), "r"(ch.cnt), "r"(q.p16), "r"(q.step))

#define TANS_STEP2_HEAD                                                            \
    "shf.l.wrap.b32 w2, 0, %6, %5;\n\t" /* w << nb1 */                             \
    "shf.l.wrap.b32 b, w2, 0, %7;\n\t"  /* bits2 */                                \
    "mul.hi.u32 f, %7, %9;\n\t"                                                    \
    "mad.lo.u32 %0, b, %10, f;\n\t"     /* next entry */                           \
    "mad.lo.u32 c, %5, %8, %1;\n\t"     /* cnt + e1 + e2: bit 5 flips per slab */ \
    "mad.lo.u32 c, %7, %8, c;\n\t"                                                 \
    "xor.b32 t, c, %1;\n\t"                                                        \
    "and.b32 t, t, 32;\n\t"                                                        \
    "setp.ne.u32 pa, t, 0;\n\t"                                                    \
    "mov.u32 %1, c;\n\t"

// Refill from a ring of kUnit-byte rows (64: the fused kernel's half-warp
// rings, v = 64 r; 128: a warp's 32 streams, v = 128 r): the ring row of row
// r = v / kUnit is at (v & mask) | ring_lane, mask = (R - 1) * kUnit (the
// ring is aligned to its size).
template <int kUnit>
__device__ __forceinline__ void chain_step2_ring(Chain &ch, const uint8_t *tb, uint32_t ring_lane,
                                                 uint32_t mask, const Opq &q, uint32_t &e1,
                                                 uint32_t &e2) {
    e1 = *reinterpret_cast<const uint32_t *>(tb + ch.addr);
    uint32_t w, a1;
    TANS_STEP2_FIRST;
    e2 = *reinterpret_cast<const uint32_t *>(tb + a1);
    asm volatile(
        "{\n\t.reg .u32 w2, b, f, c, t, u, sa;\n\t.reg .pred pa;\n\t" TANS_STEP2_HEAD
        "and.b32 u, %4, %12;\n\t"
        "or.b32 sa, u, %13;\n\t"
        "@pa mad.lo.u32 %2, %3, %8, 0;\n\t"    /* hi <- lo */
        "@pa ld.shared.u32 %3, [sa];\n\t"      /* lo <- next row of this stream */
        "@pa mad.lo.s32 %4, %8, %11, %4;\n\t"  /* one row down */
        "}"
        : "+r"(ch.addr), "+r"(ch.cnt), "+r"(ch.hi), "+r"(ch.lo), "+r"(ch.v)
        : "r"(e1), "r"(w), "r"(e2), "r"(q.one), "r"(q.p16), "r"(q.step),
          "r"(kUnit == 64 ? q.back64 : q.back), "r"(mask), "r"(ring_lane));
}

// Refill from a register window (a tile that cannot use the ring): win[0]
// is the next row of this stream, win[1] the one below it, ...; a refill
// takes win[0] and shifts the window down by one row.  kUnit as for
// chain_step2_ring (v counts rows in units of kUnit); NW = 6 covers 16
// steps, NW = 3 covers 8.
template <int kUnit, int NW>
__device__ __forceinline__ void chain_step2_window(Chain &ch, const uint8_t *tb, const Opq &q,
                                                   uint32_t (&win)[NW], uint32_t &e1, uint32_t &e2) {
    static_assert(NW == 3 || NW == 6, "window of 3 or 6 rows");
    e1 = *reinterpret_cast<const uint32_t *>(tb + ch.addr);
    uint32_t w, a1;
    TANS_STEP2_FIRST;
    e2 = *reinterpret_cast<const uint32_t *>(tb + a1);
    uint32_t pa;
    asm volatile(
        "{\n\t.reg .u32 w2, b, f, c, t;\n\t.reg .pred pa;\n\t"
        "shf.l.wrap.b32 w2, 0, %7, %6;\n\t"  /* w << nb1 */
        "shf.l.wrap.b32 b, w2, 0, %8;\n\t"   /* bits2 */
        "mul.hi.u32 f, %8, %10;\n\t"
        "mad.lo.u32 %0, b, %11, f;\n\t"      /* next entry */
        "mad.lo.u32 c, %6, %9, %1;\n\t"      /* cnt + e1 + e2: bit 5 flips per slab */
        "mad.lo.u32 c, %8, %9, c;\n\t"
        "xor.b32 t, c, %1;\n\t"
        "and.b32 t, t, 32;\n\t"
        "setp.ne.u32 pa, t, 0;\n\t"
        "mov.u32 %1, c;\n\t"
        "@pa mad.lo.u32 %2, %3, %9, 0;\n\t"  /* hi <- lo */
        "@pa mad.lo.s32 %4, %9, %12, %4;\n\t" /* one row down */
        "selp.b32 %5, 1, 0, pa;\n\t"
        "}"
        : "+r"(ch.addr), "+r"(ch.cnt), "+r"(ch.hi), "+r"(ch.lo), "+r"(ch.v), "=r"(pa)
        : "r"(e1), "r"(w), "r"(e2), "r"(q.one), "r"(q.p16), "r"(q.step),
          "r"(kUnit == 64 ? q.back64 : q.back));
    if (pa) {  // lo <- win[0], the window moves down one row
        ch.lo = win[0];
#pragma unroll
        for (int k = 0; k + 1 < NW; k++) win[k] = win[k + 1];
    }
}

// This lane's rows row .. row - NW + 1 of its stream (row = the next row it
// refills from; rows below the block's first read as 0 and are never
// consumed), loaded together.
template <int kUnit, int NW>
__device__ __forceinline__ void chain_window_load(const Chain &ch, const Opq &q, uint32_t (&win)[NW]) {
    int32_t r;
    asm("mul.hi.s32 %0, %1, %2;" : "=r"(r) : "r"(ch.v), "r"(kUnit == 64 ? q.p26 : q.p25));
    const uint8_t *col = reinterpret_cast<const uint8_t *>(ch.src);  // row 0 of its column
#pragma unroll
    for (int k = 0; k < NW; k++)
        win[k] = r - k >= 0 ? __ldg(reinterpret_cast<const uint32_t *>(col + (int64_t)(r - k) * 512)) : 0u;
}

// Row of a 64-unit v, on the FMA pipe (arithmetic: rows below 0 stay negative).
__device__ __forceinline__ int32_t row_of(int32_t v, const Opq &q) {
    int32_t r;
    asm("mul.hi.s32 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(q.p26));
    return r;
}
// Row of a 128-unit v.
__device__ __forceinline__ int32_t row_of128(int32_t v, const Opq &q) {
    int32_t r;
    asm("mul.hi.s32 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(q.p25));
    return r;
}

// NP pair steps (NP % 4 == 0), pair symbols packed four to a word.  Without
// the ring, the tile first loads every row its refills can reach (NP steps
// refill at most 3 NP / 8 times; rows below the block's first read as 0 and
// are never consumed) with independent loads, so it pays one memory round
// trip instead of one per refill.
template <bool kRing, int NP>
__device__ __forceinline__ void chain_tile(Chain &ch, const uint8_t *tb, uint32_t ring_lane,
                                           const Opq &q, uint32_t (&S)[NP / 4]) {
    uint32_t win[6];
    if (!kRing) chain_window_load<64, 6>(ch, q, win);
#pragma unroll
    for (int j = 0; j < NP / 4; j++) {
        uint32_t e0, e1, e2, e3;
        if (kRing) {
            chain_step2_ring<64>(ch, tb, ring_lane, q.rmask, q, e0, e1);
            chain_step2_ring<64>(ch, tb, ring_lane, q.rmask, q, e2, e3);
        } else {
            chain_step2_window<64, 6>(ch, tb, q, win, e0, e1);
            chain_step2_window<64, 6>(ch, tb, q, win, e2, e3);
        }
        S[j] = gather_syms(e0, e1, e2, e3);
    }
}

// init_tans_ctx (csrc/tans_decode.cu:65-92) for 64-unit rows, with in-kernel
// validation.  Returns the block's slab count G (0 if the metadata is
// malformed) and in row0 the tensor row of the block's row 0 (-1 when the
// block does not start on a 512-byte row of the buffer).
__device__ __forceinline__ int32_t chain_init64(Chain &ch, const uint32_t *__restrict__ comp,
                                                int64_t comp_bytes,
                                                const int32_t *__restrict__ offsets,
                                                const uint16_t *__restrict__ states,
                                                const uint8_t *__restrict__ partial, int64_t sid,
                                                uint32_t lane_off, int32_t *status, int32_t &row0) {
    const int32_t G = chain_init(ch, comp, comp_bytes, offsets, states, partial, sid, lane_off, status);
    const int64_t base = __ldg(offsets + sid / kBlk);
    row0 = (G > 0 && base % 512 == 0) ? (int32_t)(base / 512) : -1;
    ch.v = (G - 3) * 64;
    return G;
}

// Per-tile upkeep of one warp's ring of 128-byte rows (one chain per lane):
// fill four more rows (never over a row the slowest live lane may still
// read), then vote on whether every live lane's rows for the next 8 steps
// (row .. row - 2) have landed; if not, wait for the newest fill and vote
// again.  false: the tile refills from global memory.
template <int R>
__device__ __forceinline__ bool ring_tile128(PairRing &rg, int32_t row, bool live, bool on,
                                             int lane, const uint8_t *src, uint32_t dst) {
    const uint32_t full = 0xffffffffu;
    const int32_t slow = __reduce_max_sync(full, live ? row : kNoRow);
    const int32_t f = ring_fill16<128>(rg.fill, slow - R + 1, on, lane, src, dst,
                                       (uint32_t)(R - 1) << 7);
    cp_async_commit();
    rg.done1 = rg.done0;
    rg.done0 = f < 0 ? INT_MIN : (f < rg.fill ? f + 1 : rg.done0);
    rg.fill = f;
    cp_async_wait<1>();
    __syncwarp();
    if (__all_sync(full, !live || row - 2 >= rg.done1)) return true;
    cp_async_wait<0>();
    __syncwarp();
    return __all_sync(full, !live || row - 2 >= rg.done0);
}

// Start a warp's ring for one group: row 0 of the warp's 32 stream columns is
// taken from a live lane (all live lanes share the block); the ring serves
// the group when that row is 16-byte aligned and the block has rows below
// its top two, and then gets its first twelve rows at once.
template <int R>
__device__ __forceinline__ bool ring_start128(PairRing &rg, const Chain &ch, int32_t G, bool live,
                                              int lane, uint32_t dst, const uint8_t *&src) {
    const uint32_t full = 0xffffffffu;
    const uint64_t row0 = reinterpret_cast<uint64_t>(ch.src) - 4u * (uint64_t)lane;
    const uint32_t lv = __ballot_sync(full, live);
    const int32_t Gw = __reduce_max_sync(full, live ? G : 0);
    const uint64_t r = __shfl_sync(full, row0, lv ? __ffs(lv) - 1 : 0);
    const bool on = lv != 0 && Gw >= 3 && (r & 15u) == 0;
    src = reinterpret_cast<const uint8_t *>(r) + 16 * (lane & 7);  // unused when !on
    rg.fill = Gw - 3;
    rg.done0 = rg.done1 = Gw >= 3 ? Gw - 2 : INT_MIN;
    if (on) {
#pragma unroll
        for (int i = 0; i < 3; i++)
            rg.fill = ring_fill16<128>(rg.fill, -1, true, lane, src, dst, (uint32_t)(R - 1) << 7);
        cp_async_commit();
        cp_async_wait<0>();
        rg.done0 = rg.done1 = rg.fill < 0 ? INT_MIN : rg.fill + 1;
    }
    __syncwarp();
    return on;
}

// ---------------------------------------------------------------- decode

struct DecodeArgs {
    const uint32_t *comp;
    int64_t comp_bytes;
    const int32_t *offsets;
    const uint16_t *states;
    const uint8_t *partial;
    const uint8_t *sm;  // [N/2][K]
    const int32_t *table;
    uint8_t *out;       // [N][K]
    int64_t K, N;       // K: chains decoded
    int64_t stride;     // streams of the layout: row stride of sm and out
    int64_t seg_pairs;  // pair symbols per chain: N/2, or S for split streams
    int32_t *status;
    Opq q;
    int32_t word_rows;  // stride % 4 == 0 and sm/out 4-byte aligned: word path allowed
};

// 4x4 byte transpose across the four lanes of a quad (lane = 4a + b):
// lane b ends with byte b of each quad lane's word, in lane order.  Two
// exchange rounds (halves with lane b^2, bytes with lane b^1), each one
// shuffle and one byte permute whose selector depends on the lane.
__device__ __forceinline__ uint32_t quad_transpose(uint32_t v, uint32_t sel1, uint32_t sel2) {
    const uint32_t h = __shfl_xor_sync(0xffffffffu, v, 2);
    const uint32_t t = __byte_perm(v, h, sel1);
    const uint32_t u = __shfl_xor_sync(0xffffffffu, t, 1);
    return __byte_perm(t, u, sel2);
}

// Output staging of the team form (kTeams): 4 warps = one 128-stream block
// hand their decoded 16 x 32-byte tile pieces to shared memory, and each
// warp then stores 4 whole 128-byte output rows, instead of each warp
// storing 32-byte row segments (the [N][K] output puts every row K bytes
// apart, and scattered 32-byte pieces cost ~20 % of the kernel on cfg2).
constexpr int kTeamWarps = 4;
constexpr int kStageRowWords = 36;  // 32 + 4 padding: conflict-free staging writes
constexpr int kStageBytes = 2 * 16 * kStageRowWords * 4;  // double-buffered tile

template <int R, bool kTeams>
__global__ void __launch_bounds__(kDecodeMaxWarps * 32, 1) decode_kernel(const DecodeArgs p) {
    extern __shared__ __align__(16) uint8_t smem[];
    load_table(reinterpret_cast<uint32_t *>(smem), p.table, p.status);
    __syncthreads();
    const uint8_t *tb = smem;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int qa = lane >> 2, qb = lane & 3;
    const uint32_t sel1 = (qb & 2) ? 0x3276u : 0x5410u;
    const uint32_t sel2 = (qb & 1) ? 0x3715u : 0x6240u;
    const uint32_t lane_off = 4u * (lane % kCopies);
    const uint32_t mask = (uint32_t)(R - 1) << 7;
    const uint32_t ring = ring_area<R>(smem, warp, 1);
    const uint32_t ring_lane = ring + 4u * lane, ring_dst = ring + 16u * (lane & 7);
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t n_groups = (p.K + 31) / 32;
    const int64_t P = p.seg_pairs, K = p.stride;
    for (int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp; g < n_groups; g += warps) {
        const int64_t sid = g * 32 + lane;
        const bool active = sid < p.K;
        // chain sid is segment seg of output stream col (split streams: chains
        // are segment-major, 32 | stride; otherwise seg = 0 and col = sid)
        const int64_t seg = (g * 32) / K, col0 = g * 32 - seg * K, col = col0 + lane;
        const uint8_t *sm_seg = p.sm + seg * P * K;
        uint8_t *out_seg = p.out + 2 * seg * P * K;
        Chain ch;
        chain_idle(ch, p.comp);
        int32_t G = 0;
        if (active)
            G = chain_init(ch, p.comp, p.comp_bytes, p.offsets, p.states, p.partial, sid, lane_off,
                           p.status);
        const bool live = active && G > 0;
        PairRing rg;
        const uint8_t *ring_src;
        const bool on = ring_start128<R>(rg, ch, G, live, lane, ring_dst, ring_src);
        // Word path, for full warps when rows are 4-byte aligned: the
        // sign/mantissa bytes of 4 streams x 1 pair arrive as one word and are
        // transposed across the lane quad; the composed even/odd output words
        // are transposed back and stored 4 bytes (4 streams) at a time, each
        // warp store covering four full 32-byte row segments.
        const bool words = p.word_rows && g * 32 + 32 <= p.K;
        const int32_t full_tiles = words ? (int32_t)(P / kTablePairs) : 0;
        const uint8_t *smw = sm_seg + qb * K + col0 + 4 * qa;
        uint8_t *ow = out_seg + 2 * qb * K + col0 + 4 * qa;
        // team form: this warp stores rows 4 wi .. 4 wi + 3 of every tile,
        // 128 bytes each (the team's 128 columns)
        const int wi = warp & (kTeamWarps - 1);
        uint32_t *stage = reinterpret_cast<uint32_t *>(
            smem + (ring_area<R>(smem, blockDim.x >> 5, 1) - smem_addr(smem)) +
            (warp / kTeamWarps) * kStageBytes);
        // lane l stores 16 bytes of row 4 wi + l / 8 of the tile (its 128-byte
        // piece is bytes 16 (l % 8) .. of the team's 128 columns)
        uint8_t *otp = out_seg + (int64_t)(4 * wi + (lane >> 3)) * K + (col0 - 32 * wi) + 16 * (lane & 7);
        const int64_t srow = kTablePairs * K, orow = 2 * kTablePairs * K;
        const int64_t k4 = 4 * K, pf_ahead = 3 * srow + (qa & 1) * 4 * K;
        uint32_t w0n = 0, w1n = 0;
        if (full_tiles > 0) {
            w0n = ld_stream_u32(smw);
            w1n = ld_stream_u32(smw + 4 * K);
        }
        for (int32_t t = 0; t < full_tiles; t++) {
            const uint32_t w0 = w0n, w1 = w1n;
            smw += srow;
            if (t + 1 < full_tiles) {
                w0n = ld_stream_u32(smw);
                w1n = ld_stream_u32(smw + k4);
            }
            if (t + 4 < full_tiles) prefetch_l2(smw + pf_ahead);
            uint32_t e[kTablePairs];
            if (ring_tile128<R>(rg, row_of128(ch.v, p.q), live, on, lane, ring_src, ring_dst)) {
#pragma unroll
                for (int j = 0; j < kTablePairs; j += 2)
                    chain_step2_ring<128>(ch, tb, ring_lane, mask, p.q, e[j], e[j + 1]);
            } else {  // rows from a register window loaded at once (8 steps: 3 rows at most)
                uint32_t win[3];
                chain_window_load<128, 3>(ch, p.q, win);
#pragma unroll
                for (int j = 0; j < kTablePairs; j += 2)
                    chain_step2_window<128, 3>(ch, tb, p.q, win, e[j], e[j + 1]);
            }
            const uint32_t M0 = quad_transpose(w0, sel1, sel2);
            const uint32_t M1 = quad_transpose(w1, sel1, sel2);
            const uint32_t S0 = gather_syms(e[0], e[1], e[2], e[3]);
            const uint32_t S1 = gather_syms(e[4], e[5], e[6], e[7]);
            uint32_t E0 = compose_even(S0, M0, p.q), O0 = compose_odd(S0, M0, p.q);
            uint32_t E1 = compose_even(S1, M1, p.q), O1 = compose_odd(S1, M1, p.q);
            if (!live) E0 = O0 = E1 = O1 = 0;
            E0 = quad_transpose(E0, sel1, sel2);
            O0 = quad_transpose(O0, sel1, sel2);
            E1 = quad_transpose(E1, sel1, sel2);
            O1 = quad_transpose(O1, sel1, sel2);
            if (kTeams) {
                uint32_t *sb = stage + (t & 1) * (16 * kStageRowWords) + wi * 8 + qa;
                sb[(2 * qb) * kStageRowWords] = E0;      // element 2b
                sb[(2 * qb + 1) * kStageRowWords] = O0;  // element 2b + 1
                sb[(8 + 2 * qb) * kStageRowWords] = E1;  // element 8 + 2b
                sb[(9 + 2 * qb) * kStageRowWords] = O1;  // element 9 + 2b
                asm volatile("bar.sync %0, %1;" ::"r"(1 + warp / kTeamWarps), "n"(kTeamWarps * 32)
                             : "memory");
                const uint32_t *rb = stage + (t & 1) * (16 * kStageRowWords) +
                                     (4 * wi + (lane >> 3)) * kStageRowWords + 4 * (lane & 7);
                st_stream_v4(otp, *reinterpret_cast<const uint4 *>(rb));
                otp += orow;
            } else {
                st_stream_u32(ow, E0);          // element 2b
                st_stream_u32(ow + K, O0);      // element 2b + 1
                st_stream_u32(ow + 8 * K, E1);  // element 8 + 2b
                st_stream_u32(ow + 9 * K, O1);  // element 9 + 2b
                ow += orow;
            }
        }
        // Byte path: the rest of the stream (all of it for a partial warp or
        // unaligned rows), one pair at a time.
        for (int64_t i = (int64_t)full_tiles * kTablePairs; i < P; i += kTablePairs) {
            uint32_t s8[kTablePairs];
            if (ring_tile128<R>(rg, row_of128(ch.v, p.q), live, on, lane, ring_src, ring_dst)) {
#pragma unroll
                for (int j = 0; j < kTablePairs; j += 2)
                    chain_step2_ring<128>(ch, tb, ring_lane, mask, p.q, s8[j], s8[j + 1]);
            } else {
                uint32_t win[3];
                chain_window_load<128, 3>(ch, p.q, win);
#pragma unroll
                for (int j = 0; j < kTablePairs; j += 2)
                    chain_step2_window<128, 3>(ch, tb, p.q, win, s8[j], s8[j + 1]);
            }
            if (active) {
#pragma unroll
                for (int j = 0; j < kTablePairs; j++) {
                    if (i + j >= P) break;
                    const uint32_t m = live ? __ldg(sm_seg + (i + j) * K + col) : 0u;
                    const uint32_t sy = (s8[j] >> 8) & 0xFFu;
                    const uint32_t v0 = ((m & 8u) << 4) | ((sy >> 4) << 3) | (m & 7u);
                    const uint32_t v1 = (((m >> 4) & 8u) << 4) | ((sy & 15u) << 3) | ((m >> 4) & 7u);
                    out_seg[(2 * (i + j)) * K + col] = live ? (uint8_t)v0 : 0;
                    out_seg[(2 * (i + j) + 1) * K + col] = live ? (uint8_t)v1 : 0;
                }
            }
        }
        cp_async_wait<0>();
    }
}

// ----------------------------------------------------------------- fused

struct FusedArgs {
    const uint32_t *a_comp, *b_comp;
    int64_t a_bytes, b_bytes;
    const int32_t *a_off, *b_off;
    const uint16_t *a_st, *b_st;
    const uint8_t *a_part, *b_part;
    const uint8_t *a_sm, *b_sm;  // [N/16][K][8]
    const int32_t *table;
    uint8_t *out;                // [N/16][K][16]
    int64_t K, N;                // K: chains decoded (pointers start at the first one)
    int64_t stride;              // streams of the layout: row stride of the sm/out tiles
    int64_t seg_tiles;           // 8-pair tiles per chain: N/16, or S/8 for split streams
    int32_t *status;
    Opq q;
};

// Fused kernel, paired-lane form.  A warp owns 16 streams: lane l < 16
// decodes stream l of input A, lane l + 16 the same stream of input B (one
// tANS chain per lane), so 28 warps per SM keep all four schedulers equally
// loaded.  Per 16-pair tile the two halves swap the packed pair symbols they
// do not keep with two shuffles; lane half h then composes, adds and stores
// the 8-pair output tile 2T + h of its stream with one 16-byte store (a warp
// writes two contiguous 256-byte runs), loading the sign/mantissa bytes of
// both inputs for that tile itself.  Slab rows come from a ring per
// half-warp (see PairRing).
constexpr int kPairMaxWarps = 28;

// Per-tile ring upkeep: fill up to four rows of each half's ring, then vote
// on whether every lane's rows for this tile (down to row - 5: 16 steps read
// at most 6 slabs) are in landed fills.
template <int R, bool kAll>
__device__ __forceinline__ bool ring_tile(PairRing &rg, int32_t row, bool live, bool on, int h,
                                          int li, const uint8_t *src, uint32_t dst, const Opq &q) {
    const uint32_t full = 0xffffffffu;
    const int32_t sa = __reduce_max_sync(full, (h == 0 && (kAll || live)) ? row : kNoRow);
    const int32_t sb = __reduce_max_sync(full, (h == 1 && (kAll || live)) ? row : kNoRow);
    const int32_t f = ring_fill16<64>(rg.fill, (h ? sb : sa) - R + 1, on, li, src, dst, q.rmask);
    cp_async_commit();
    rg.done1 = rg.done0;
    rg.done0 = f < 0 ? INT_MIN : (f < rg.fill ? f + 1 : rg.done0);
    rg.fill = f;
    cp_async_wait<1>();
    __syncwarp();
    if (__all_sync(full, (!kAll && !live) || row - 5 >= rg.done1)) return true;
    cp_async_wait<0>();
    __syncwarp();
    return __all_sync(full, (!kAll && !live) || row - 5 >= rg.done0);
}

// The 16-pair tiles (and a last 8-pair tile) of one group.  kAll: every lane
// has a live stream (no masking of loads, outputs or votes).
template <int R, bool kAll>
__device__ __forceinline__ void pair_group(const FusedArgs &p, Chain &ch, PairRing &rg,
                                           const uint8_t *tb, uint32_t ring_lane, bool on, int li,
                                           const uint8_t *fsrc, uint32_t fdst, bool live,
                                           bool active, int h, const uint8_t *so,
                                           const uint8_t *sx, uint8_t *op, int64_t tail) {
    const uint32_t full = 0xffffffffu;
    const int32_t n8 = (int32_t)p.seg_tiles, n16 = n8 / 2;
    const int64_t t8 = p.stride * 8, o8 = p.stride * 16;
    uint2 mo_n = make_uint2(0, 0), mx_n = make_uint2(0, 0);
    if ((kAll || live) && n16 > 0) {
        mo_n = ld_stream_v2(so);
        mx_n = ld_stream_v2(sx);
    }
    for (int32_t t = 0; t < n16; t++) {
        const uint2 mo = mo_n, mx = mx_n;
        so += 2 * t8;
        sx += 2 * t8;
        if ((kAll || live) && t + 1 < n16) {
            mo_n = ld_stream_v2(so);
            mx_n = ld_stream_v2(sx);
        }
        // (no L2 prefetch further ahead: it cost 6 % on cfg1)
        uint32_t S[4];
        if (ring_tile<R, kAll>(rg, row_of(ch.v, p.q), live, on, h, li, fsrc, fdst, p.q))
            chain_tile<true, 16>(ch, tb, ring_lane, p.q, S);
        else
            chain_tile<false, 16>(ch, tb, ring_lane, p.q, S);
        // half h keeps pairs 8h .. 8h + 7 and sends the other eight
        const uint32_t k0 = h ? S[2] : S[0], k1 = h ? S[3] : S[1];
        const uint32_t x0 = __shfl_xor_sync(full, h ? S[0] : S[2], 16);
        const uint32_t x1 = __shfl_xor_sync(full, h ? S[1] : S[3], 16);
        const uint32_t re0 = add_e4m3x4(compose_even(k0, mo.x, p.q), compose_even(x0, mx.x, p.q));
        const uint32_t ro0 = add_e4m3x4(compose_odd(k0, mo.x, p.q), compose_odd(x0, mx.x, p.q));
        const uint32_t re1 = add_e4m3x4(compose_even(k1, mo.y, p.q), compose_even(x1, mx.y, p.q));
        const uint32_t ro1 = add_e4m3x4(compose_odd(k1, mo.y, p.q), compose_odd(x1, mx.y, p.q));
        uint4 o = make_uint4(__byte_perm(re0, ro0, 0x5140), __byte_perm(re0, ro0, 0x7362),
                             __byte_perm(re1, ro1, 0x5140), __byte_perm(re1, ro1, 0x7362));
        if (!kAll && !live) o = make_uint4(0, 0, 0, 0);
        if (kAll || active) st_stream_v4(op, o);
        op += 2 * o8;
    }
    if (n8 & 1) {
        // a last 8-pair tile (element tile `tail` of this stream): half h
        // composes pairs 4h .. 4h + 3 (8 output bytes)
        uint32_t S[2];
        if (ring_tile<R, kAll>(rg, row_of(ch.v, p.q), live, on, h, li, fsrc, fdst, p.q))
            chain_tile<true, 8>(ch, tb, ring_lane, p.q, S);
        else
            chain_tile<false, 8>(ch, tb, ring_lane, p.q, S);
        const uint32_t k0 = h ? S[1] : S[0];
        const uint32_t x0 = __shfl_xor_sync(full, h ? S[0] : S[1], 16);
        const uint8_t *own = h ? p.b_sm : p.a_sm, *oth = h ? p.a_sm : p.b_sm;
        uint32_t mo = 0, mx = 0;
        if (kAll || live) {
            mo = ld_stream_u32(own + tail * 8 + 4 * h);
            mx = ld_stream_u32(oth + tail * 8 + 4 * h);
        }
        const uint32_t re = add_e4m3x4(compose_even(k0, mo, p.q), compose_even(x0, mx, p.q));
        const uint32_t ro = add_e4m3x4(compose_odd(k0, mo, p.q), compose_odd(x0, mx, p.q));
        uint32_t ox = __byte_perm(re, ro, 0x5140), oy = __byte_perm(re, ro, 0x7362);
        if (!kAll && !live) ox = oy = 0;
        if (kAll || active) st_stream_v2(p.out + tail * 16 + 8 * h, ox, oy);
    }
}

template <int R>
__global__ void __launch_bounds__(kPairMaxWarps * 32, 1)
    fused_pair_kernel(const __grid_constant__ FusedArgs p) {
    static_assert(R >= 16 && (R & (R - 1)) == 0, "ring rows: a power of two");
    extern __shared__ __align__(16) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    const int h = lane >> 4, li = lane & 15;
    const uint32_t rbytes = R * 64u;
    const uint32_t rings = (smem_addr(smem) + kTableBytes + rbytes - 1) & ~(rbytes - 1);
    const uint32_t ring_h = rings + (uint32_t)(2 * warp + h) * rbytes;  // this half's ring
    load_table(reinterpret_cast<uint32_t *>(smem), p.table, p.status);
    __syncthreads();
    const uint8_t *tb = smem;
    const uint32_t lane_off = 4u * (lane % kCopies);
    const uint32_t ring_lane = ring_h + 4u * li;                // this lane's column: reads
    const uint32_t fdst = ring_h + 16u * (li & 3);              // this lane's fill piece
    const uint32_t *comp = h ? p.b_comp : p.a_comp;
    const int64_t comp_bytes = h ? p.b_bytes : p.a_bytes;
    const int32_t *off = h ? p.b_off : p.a_off;
    const uint16_t *st = h ? p.b_st : p.a_st;
    const uint8_t *part = h ? p.b_part : p.a_part;
    // sign/mantissa bytes of this lane's own input and of the other input
    const uint8_t *sm_own = h ? p.b_sm : p.a_sm, *sm_oth = h ? p.a_sm : p.b_sm;
    const int32_t *off_oth = h ? p.a_off : p.b_off;
    const int64_t bytes_oth = h ? p.a_bytes : p.b_bytes;
    const int64_t n_groups = (p.K + 15) / 16;
    const int64_t K = p.K, t8 = p.stride * 8, o8 = p.stride * 16;
    const uint32_t full = 0xffffffffu;
    for (int64_t g = (int64_t)blockIdx.x * warps + warp; g < n_groups; g += (int64_t)gridDim.x * warps) {
        const int64_t sid = g * 16 + li;
        const bool active = sid < K;
        Chain ch;
        chain_idle(ch, comp);
        int32_t G = 0, row0 = -1;
        bool ok = false;
        if (active) {
            G = chain_init64(ch, comp, comp_bytes, off, st, part, sid, lane_off, p.status, row0);
            // the other input's block must be valid too (its lane reports its
            // own metadata; this keeps both lanes of a stream in step)
            const int64_t bb = sid / kBlk;
            const int64_t ob = __ldg(off_oth + bb), on = __ldg(off_oth + bb + 1);
            ok = ob >= 0 && on > ob && on <= bytes_oth && ((on - ob) % 512) == 0 && (ob % 4) == 0;
        }
        const bool live = active && ok && G > 0;
        // this half's ring: its block's slab count, and row 0 of the half's
        // 16 stream columns (the same for every live lane of the half), which
        // the ring copies 16 bytes at a time when it is 16-byte aligned
        const uint64_t row0_cols = reinterpret_cast<uint64_t>(ch.src) - 4u * (uint64_t)li;
        const int32_t ga = __reduce_max_sync(full, (live && !h) ? G : 0);
        const int32_t gb = __reduce_max_sync(full, (live && h) ? G : 0);
        const uint32_t hm = (__ballot_sync(full, live && (row0_cols & 15u) == 0) >> (16 * h)) & 0xFFFFu;
        const int32_t Gh = h ? gb : ga;
        const bool on = Gh >= 3 && hm != 0;
        const uint64_t rc = __shfl_sync(full, row0_cols, 16 * h + (hm ? __ffs(hm) - 1 : 0));
        const uint8_t *fsrc = reinterpret_cast<const uint8_t *>(rc) + 16 * (li & 3);  // unused when !on
        if (!live) {
            chain_idle(ch, comp);
            ch.v = -64;
        }
        PairRing rg;
        rg.fill = Gh - 3;
        rg.done0 = rg.done1 = Gh >= 3 ? Gh - 2 : INT_MIN;
        if (on) {
            // the first rows: three fills of four, then wait for all of them
#pragma unroll
            for (int k = 0; k < 3; k++) rg.fill = ring_fill16<64>(rg.fill, -1, true, li, fsrc, fdst, p.q.rmask);
            cp_async_commit();
            cp_async_wait<0>();
            rg.done0 = rg.done1 = rg.fill < 0 ? INT_MIN : rg.fill + 1;
        }
        __syncwarp();
        // chain sid is segment j of output stream col (split streams: chains
        // are segment-major, 16 | stride; otherwise j = 0 and col = sid)
        const int64_t j = (g * 16) / p.stride;
        const int64_t col = sid - j * p.stride, tile0 = j * p.seg_tiles * p.stride;
        const uint8_t *so = sm_own + (tile0 + col) * 8 + h * t8;
        const uint8_t *sx = sm_oth + (tile0 + col) * 8 + h * t8;
        uint8_t *op = p.out + (tile0 + col) * 16 + h * o8;
        const int64_t tail = tile0 + (p.seg_tiles - 1) * p.stride + col;
        if (__all_sync(full, live))
            pair_group<R, true>(p, ch, rg, tb, ring_lane, on, li, fsrc, fdst, live, active, h, so,
                                sx, op, tail);
        else
            pair_group<R, false>(p, ch, rg, tb, ring_lane, on, li, fsrc, fdst, live, active, h, so,
                                 sx, op, tail);
        // every copy lands before the ring is reused
        cp_async_wait<0>();
        __syncwarp();
    }
}

// ------------------------------------------------------------------ GEMV
//
// y[b][r] = bf16(scale[r] * sum_c e4m3(W[r][c]) * x[b][c]), fp32 accumulate,
// with W stored as tANS streams (no counterpart in the reference).
//
// Stream format (built by rans_vectoradd.tans_gemv.encode_weight): rows are
// taken 16 at a time (row group w) and columns in KS slices of CS = C/KS;
// within a slice, 16-column chunk j.  Lane l of a warp (g = l/4, t = l%4)
// owns two streams, chain 0 for row 16w+g and chain 1 for row 16w+g+8, each
// holding columns 16j+2t, 16j+2t+1, 16j+8+2t, 16j+9+2t of every chunk, in
// that order: exactly the A fragment of mma.m16n8k16 (rows g, g+8; k = 2t..,
// 2t+8..).  Stream id = ((w*KS + k)*2 + chain)*32 + l, so each chain of a
// warp is 32 consecutive streams of one encoder block.  A pair symbol of a
// stream is therefore one f16x2 fragment register after a single
// cvt.rn.f16x2.e4m3x2, and one mma.sync per chunk does 16 rows x 8 batch x
// 16 columns.  x (batch <= 8) sits in shared memory as f16 with a row pitch
// of CS + 8 halves, which puts the B-fragment words of the 32 lanes in 32
// different banks.  The work is the tANS decode (as in the vecadd kernel);
// the tensor pipe only replaces 8 x 16 scalar FMAs per chunk.

constexpr int kGemvMaxBatch = 8;

struct GemvArgs {
    const uint32_t *comp;
    int64_t comp_bytes;
    const int32_t *offsets;
    const uint16_t *states;
    const uint8_t *partial;
    const uint8_t *sm;        // [N/16][K][8]
    const int32_t *table;
    const float *scale;       // [R]
    const uint16_t *x;        // bf16 [B][C]
    uint16_t *y;              // bf16 [B][R]   (written directly when !to_partials)
    float *part;              // f32 [KS][B][R] (when to_partials: KS > 1, or a gathering GEMV)
    int64_t R, C, B, KS;
    int32_t *status;
    Opq q;
    // fused all-gather (tans_b200_gemv_gather): wait until every
    // wait_flags[q] has reached *wait_seq before reading x; results go to
    // `part` even for KS == 1
    const uint32_t *wait_flags;
    const uint32_t *wait_seq;
    int32_t wait_n;
    int32_t to_partials;
};

constexpr uint32_t kPeerWaitLimit = 1u << 24;  // polls of ~64 ns or more: >1 s

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait (one thread) until flags[0..n) have all reached `target`
// (wrap-safe); false if the limit ran out.
__device__ __forceinline__ bool peer_wait(const uint32_t *flags, uint32_t target, int n) {
    for (int q = 0; q < n; q++) {
        uint32_t i = 0;
        while ((int32_t)(ld_acquire_sys(flags + q) - target) < 0) {
            if (++i > kPeerWaitLimit) return false;
            __nanosleep(64);
        }
    }
    return true;
}

__device__ __forceinline__ uint32_t cvt_f16x2_e4m3x2(uint32_t v16) {
    uint32_t r;
    asm("{\n\t.reg .b16 h;\n\tcvt.u16.u32 h, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, h;\n\t}"
        : "=r"(r)
        : "r"(v16));
    return r;
}

__device__ __forceinline__ void mma_16x8x16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                            uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Uncompressed e4m3 GEMV (the decode-GEMV's denominator): the same sum with
// the same mma.sync f16 path and the same column-slice reduction, W read as
// plain e4m3 bytes [R][C].  A warp owns 16 rows of one column slice at a
// time; per 64-column chunk lane (g, t) loads 16 contiguous bytes of rows g
// and g + 8 (columns 16t .. 16t + 15).  Inside a chunk the MMA k index is
// permuted: in step s, lane t's k = 2t, 2t+1 / 2t+8, 2t+9 are columns
// 16t + 4s + 0, 1 / 2, 3, and the x (B) fragment follows the same
// permutation, so every product w[r][c] * x[b][c] is summed exactly once.
// Each warp walks its row groups chunk by chunk with four chunks (4 KiB of
// W) in flight, the first four issued before x is staged.  Every warp
// instruction reads 64-byte pieces of 8 rows; that access pattern, not the
// grid shape, bounds it near 3 TB/s (a sweep of column splits and grid caps
// on [17408 x 5120] and [5120 x 17408] all landed at 31-33 us).
constexpr int kRawGemvWarps = 8;  // warps per CTA
constexpr int kRawGemvDepth = 4;  // chunks in flight per warp

struct RawGemvArgs {
    const uint8_t *w;       // e4m3 [R][C]
    const uint16_t *x;      // bf16 [B][C] (16-byte aligned)
    float *part;            // f32 [KS][B][R]
    int64_t R, C, B, KS;
};

__device__ __forceinline__ void raw_chunk(float (&acc)[4], uint4 wa, uint4 wb, const uint16_t *xp) {
    const uint4 x0 = *reinterpret_cast<const uint4 *>(xp);      // halves 4s .. 4s + 3, s = 0, 1
    const uint4 x1 = *reinterpret_cast<const uint4 *>(xp + 8);  // s = 2, 3
    const uint32_t a[4] = {wa.x, wa.y, wa.z, wa.w}, b[4] = {wb.x, wb.y, wb.z, wb.w};
    const uint32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int s = 0; s < 4; s++)
        mma_16x8x16(acc, cvt_f16x2_e4m3x2(a[s] & 0xFFFFu), cvt_f16x2_e4m3x2(b[s] & 0xFFFFu),
                    cvt_f16x2_e4m3x2(a[s] >> 16), cvt_f16x2_e4m3x2(b[s] >> 16), xv[2 * s],
                    xv[2 * s + 1]);
}

__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t v) {
    const __half2 h = __floats2half2_rn(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
    return *reinterpret_cast<const uint32_t *>(&h);
}

__global__ void __launch_bounds__(kRawGemvWarps * 32, 3) gemv_raw_kernel(const RawGemvArgs p) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int64_t CS = p.C / p.KS;
    const int k = blockIdx.y;
    const int64_t pitch = CS + 8;  // halves (rows stay 16-byte aligned)
    uint16_t *xs = reinterpret_cast<uint16_t *>(smem);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int64_t groups = p.R / 16, gstride = (int64_t)gridDim.x * kRawGemvWarps;
    const int64_t rg0 = (int64_t)blockIdx.x * kRawGemvWarps + warp;
    const int32_t nch = (int32_t)(CS / 64);
    const int32_t items = rg0 < groups ? (int32_t)((groups - rg0 + gstride - 1) / gstride) * nch : 0;
    // W of row g (and g + 8), this lane's 16 bytes, column slice k, row group 0
    const uint8_t *wk = p.w + (int64_t)g * p.C + k * CS + 16 * t;
    const int64_t wrow8 = 8 * p.C, wgrp = 16 * p.C;
    int64_t l_rg = rg0;
    int32_t l_c = 0;
    uint4 A[kRawGemvDepth], B[kRawGemvDepth];
#pragma unroll
    for (int u = 0; u < kRawGemvDepth; u++) {
        A[u] = B[u] = make_uint4(0, 0, 0, 0);
        if (u < items) {
            const uint8_t *q = wk + l_rg * wgrp + 64 * l_c;
            A[u] = ld_stream_v4(q);
            B[u] = ld_stream_v4(q + wrow8);
        }
        if (++l_c == nch) {
            l_c = 0;
            l_rg += gstride;
        }
    }
    // x slice -> f16 in shared memory, eight columns per 16-byte load (rows
    // >= B are zero), while the first chunks of W are in flight
    const int64_t c8 = CS / 8;
    for (int64_t i = threadIdx.x; i < kGemvMaxBatch * c8; i += blockDim.x) {
        const int64_t b = i / c8, c = (i - b * c8) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (b < p.B) {
            const uint4 r = *reinterpret_cast<const uint4 *>(p.x + b * p.C + k * CS + c);
            v = make_uint4(bf16x2_to_f16x2(r.x), bf16x2_to_f16x2(r.y), bf16x2_to_f16x2(r.z),
                           bf16x2_to_f16x2(r.w));
        }
        *reinterpret_cast<uint4 *>(xs + b * pitch + c) = v;
    }
    __syncthreads();
    const uint16_t *xp = xs + g * pitch + 16 * t;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int64_t c_rg = rg0;
    int32_t c_c = 0;
    float *pk = p.part + (int64_t)k * p.B * p.R;
    for (int32_t i = 0; i < items; i += kRawGemvDepth) {
#pragma unroll
        for (int u = 0; u < kRawGemvDepth; u++) {
            if (i + u < items) {
                const uint4 a = A[u], b = B[u];
                if (i + u + kRawGemvDepth < items) {
                    const uint8_t *q = wk + l_rg * wgrp + 64 * l_c;
                    A[u] = ld_stream_v4(q);
                    B[u] = ld_stream_v4(q + wrow8);
                }
                if (++l_c == nch) {
                    l_c = 0;
                    l_rg += gstride;
                }
                raw_chunk(acc, a, b, xp + 64 * c_c);
                if (++c_c == nch) {
                    // D fragment: rows g, g + 8; batch columns 2t, 2t + 1
                    const int64_t r0 = c_rg * 16;
                    if (2 * t < p.B) {
                        pk[(2 * t) * p.R + r0 + g] = acc[0];
                        pk[(2 * t) * p.R + r0 + g + 8] = acc[2];
                    }
                    if (2 * t + 1 < p.B) {
                        pk[(2 * t + 1) * p.R + r0 + g] = acc[1];
                        pk[(2 * t + 1) * p.R + r0 + g + 8] = acc[3];
                    }
                    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
                    c_c = 0;
                    c_rg += gstride;
                }
            }
        }
    }
}

// Natural-order e4m3 words of four pairs: lo = pairs 0,1 (bytes e0 e1 e0 e1),
// hi = pairs 2,3.
__device__ __forceinline__ void compose_pairs(uint32_t S, uint32_t M, const Opq &q, uint32_t &lo,
                                              uint32_t &hi) {
    const uint32_t ev = compose_even(S, M, q), od = compose_odd(S, M, q);
    lo = __byte_perm(ev, od, 0x5140);
    hi = __byte_perm(ev, od, 0x7362);
}

constexpr int kGemvMaxWarps = 20;
// Short column slices (at most 512 columns, 8 tiles per stream: the row
// shards of a 4- or 8-way stack) run a build for up to 22 warps, whose
// 80-register allocation suits them better (a 4-way rank's 80 GEMVs: 1.68
// -> 1.51 ms); longer slices keep 20 warps at up to 96 registers.
constexpr int kGemvShortWarps = 22;
constexpr int64_t kGemvShortCols = 512;

// One warp's row group of the GEMV: its two chains (a: rows g, b: rows
// g + 8), their slab rings and the first sign/mantissa words.  Set up from
// the weight alone (nothing an earlier kernel writes).
struct GemvGroup {
    Chain ca, cb;
    PairRing ra, rb;
    const uint8_t *src_a, *src_b;
    const uint8_t *spa, *spb;  // this tile's sign/mantissa words
    uint2 sa_n, sb_n;          // ... loaded one tile ahead
    bool live, on;
};

template <int R>
__device__ __forceinline__ void gemv_group_start(const GemvArgs &p, int64_t w, int k, int lane,
                                                 uint32_t lane_off, uint32_t dst_a, uint32_t dst_b,
                                                 int32_t n_tiles, GemvGroup &gs) {
    const uint32_t full = 0xffffffffu;
    const uint32_t mask = (uint32_t)(R - 1) << 7;
    const int64_t sa_id = ((w * p.KS + k) * 2 + 0) * 32 + lane;
    const int64_t sb_id = sa_id + 32;
    const int32_t ga = chain_init(gs.ca, p.comp, p.comp_bytes, p.offsets, p.states, p.partial,
                                  sa_id, lane_off, p.status);
    const int32_t gb = chain_init(gs.cb, p.comp, p.comp_bytes, p.offsets, p.states, p.partial,
                                  sb_id, lane_off, p.status);
    gs.live = ga > 0 && gb > 0;
    // row 0 of each chain's 32 stream columns, copied 16 bytes at a time
    // when every lane is live and it is 16-byte aligned
    const uintptr_t r0a = reinterpret_cast<uintptr_t>(gs.ca.src) - 4u * lane;
    const uintptr_t r0b = reinterpret_cast<uintptr_t>(gs.cb.src) - 4u * lane;
    const int32_t Ga = __reduce_max_sync(full, gs.live ? ga : 0);
    const int32_t Gb = __reduce_max_sync(full, gs.live ? gb : 0);
    gs.on = __all_sync(full, gs.live && ((r0a | r0b) & 15u) == 0);
    if (!gs.live) {
        chain_idle(gs.ca, p.comp);
        chain_idle(gs.cb, p.comp);
    }
    gs.src_a = reinterpret_cast<const uint8_t *>(r0a) + 16 * (lane & 7);
    gs.src_b = reinterpret_cast<const uint8_t *>(r0b) + 16 * (lane & 7);
    gs.ra.fill = Ga - 3;
    gs.rb.fill = Gb - 3;
    gs.ra.done0 = gs.ra.done1 = Ga >= 3 ? Ga - 2 : INT_MIN;
    gs.rb.done0 = gs.rb.done1 = Gb >= 3 ? Gb - 2 : INT_MIN;
    if (gs.on) {
        // the first rows: three fills of four per chain in one copy group;
        // the first tile's cp.async.wait_group 1 (after it commits its own
        // fills) covers this group before any lane reads the ring
#pragma unroll
        for (int i = 0; i < 3; i++) {
            gs.ra.fill = ring_fill16<128>(gs.ra.fill, -1, true, lane, gs.src_a, dst_a, mask);
            gs.rb.fill = ring_fill16<128>(gs.rb.fill, -1, true, lane, gs.src_b, dst_b, mask);
        }
        cp_async_commit();
        gs.ra.done0 = gs.ra.done1 = gs.ra.fill < 0 ? INT_MIN : gs.ra.fill + 1;
        gs.rb.done0 = gs.rb.done1 = gs.rb.fill < 0 ? INT_MIN : gs.rb.fill + 1;
    }
    __syncwarp();
    gs.spa = p.sm + sa_id * 8;
    gs.spb = p.sm + sb_id * 8;
    gs.sa_n = gs.sb_n = make_uint2(0, 0);
    if (gs.live && n_tiles > 0) {
        gs.sa_n = ld_stream_v2(gs.spa);
        gs.sb_n = ld_stream_v2(gs.spb);
    }
}

template <int R, int kW = kGemvMaxWarps>
__global__ void __launch_bounds__(kW * 32, 1) gemv_kernel(const GemvArgs p) {
    extern __shared__ __align__(16) uint8_t smem[];
    pdl_trigger();
    const int64_t CS = p.C / p.KS;
    const int k = blockIdx.y;
    const int64_t pitch = CS + 8;  // halves
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t lane_off = 4u * (lane % kCopies);
    const uint32_t mask = (uint32_t)(R - 1) << 7;
    const uint32_t xbytes = ((uint32_t)(kGemvMaxBatch * pitch * 2) + 127u) & ~127u;
    // two rings per warp (chain a: rows g, chain b: rows g + 8), R rows of the
    // warp's 32 stream columns (128 bytes per row) each
    uint32_t ring_a, ring_b;
    {
        const uint32_t bytes = R * 128u;
        const uint32_t first =
            (smem_addr(smem) + kTableBytes + xbytes + bytes - 1) & ~(bytes - 1);
        ring_a = first + (uint32_t)(warp * 2) * bytes;
        ring_b = ring_a + bytes;
    }
    const uint32_t lane_a = ring_a + 4u * lane, lane_b = ring_b + 4u * lane;
    const uint32_t dst_a = ring_a + 16u * (lane & 7), dst_b = ring_b + 16u * (lane & 7);
    const int64_t K = p.R * 4 * p.KS;  // streams
    const int64_t N = CS / 4;          // fp8 per stream
    const int32_t n_tiles = (int32_t)(N / 16);  // CS / 64
    const int64_t groups = p.R / 16;
    const int64_t w0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    const int64_t wstep = (int64_t)gridDim.x * (blockDim.x >> 5);
    // The prologue reads only this weight (not written by the kernel before
    // this one): the table, and the first row group's chains, slab-ring
    // fills and sign/mantissa words, all while that kernel may still run.
    load_table(reinterpret_cast<uint32_t *>(smem), p.table, p.status);
    GemvGroup gs;
    if (w0 < groups) gemv_group_start<R>(p, w0, k, lane, lane_off, dst_a, dst_b, n_tiles, gs);
    pdl_wait();
    if (p.wait_n > 0) {  // x is gathered by the peers' epilogues: wait for all of them
        if (threadIdx.x == 0 && !peer_wait(p.wait_flags, *p.wait_seq, p.wait_n) && p.status)
            atomicOr(p.status, TANS_B200_DATA_TIMEOUT);
        __syncthreads();
    }
    uint16_t *xs = reinterpret_cast<uint16_t *>(smem + kTableBytes);
    // x slice -> f16 in shared memory (rows >= B are zero)
    for (int b = 0; b < kGemvMaxBatch; b++) {
        const uint16_t *xr = p.x + b * p.C + k * CS;
        for (int32_t c = threadIdx.x; c < (int32_t)CS; c += blockDim.x) {
            const float v = b < p.B ? __uint_as_float((uint32_t)xr[c] << 16) : 0.f;
            xs[b * pitch + c] = __half_as_ushort(__float2half_rn(v));
        }
    }
    __syncthreads();
    const uint8_t *tb = smem;
    const uint32_t *xw = reinterpret_cast<const uint32_t *>(xs) + g * (pitch / 2) + t;
    const int64_t tstep = K * 8;  // sign/mantissa bytes per tile row
    const uint32_t full = 0xffffffffu;
    for (int64_t w = w0; w < groups; w += wstep) {
        if (w != w0) gemv_group_start<R>(p, w, k, lane, lane_off, dst_a, dst_b, n_tiles, gs);
        Chain &ca = gs.ca, &cb = gs.cb;
        PairRing &ra = gs.ra, &rb = gs.rb;
        const bool live = gs.live, on = gs.on;
        const uint8_t *src_a = gs.src_a, *src_b = gs.src_b;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        uint2 sa_n = gs.sa_n, sb_n = gs.sb_n;
        // running pointers: this tile's sign/mantissa words and x fragments
        const uint8_t *spa = gs.spa, *spb = gs.spb;
        const uint32_t *xp = xw;
        for (int32_t tt = 0; tt < n_tiles; tt++) {
            const uint2 sa = sa_n, sb = sb_n;
            spa += tstep;
            spb += tstep;
            if (live && tt + 1 < n_tiles) {
                sa_n = ld_stream_v2(spa);
                sb_n = ld_stream_v2(spb);
            }
            // ring upkeep: four more rows per chain (never over a row the
            // slowest lane may still read), then vote on this tile's rows
            // (8 steps read at most 3 slabs: row .. row - 2)
            const int32_t rowa = row_of128(ca.v, p.q), rowb = row_of128(cb.v, p.q);
            const int32_t slow_a = __reduce_max_sync(full, live ? rowa : kNoRow);
            const int32_t slow_b = __reduce_max_sync(full, live ? rowb : kNoRow);
            const int32_t fa = ring_fill16<128>(ra.fill, slow_a - R + 1, on, lane, src_a, dst_a, mask);
            const int32_t fb = ring_fill16<128>(rb.fill, slow_b - R + 1, on, lane, src_b, dst_b, mask);
            cp_async_commit();
            ra.done1 = ra.done0;
            rb.done1 = rb.done0;
            ra.done0 = fa < 0 ? INT_MIN : (fa < ra.fill ? fa + 1 : ra.done0);
            rb.done0 = fb < 0 ? INT_MIN : (fb < rb.fill ? fb + 1 : rb.done0);
            ra.fill = fa;
            rb.fill = fb;
            cp_async_wait<1>();
            __syncwarp();
            bool fast = __all_sync(full, !live || (rowa - 2 >= ra.done1 && rowb - 2 >= rb.done1));
            if (!fast) {
                cp_async_wait<0>();
                __syncwarp();
                fast = __all_sync(full, !live || (rowa - 2 >= ra.done0 && rowb - 2 >= rb.done0));
            }
            uint32_t ea[kTablePairs], eb[kTablePairs];
            if (fast) {
#pragma unroll
                for (int j = 0; j < kTablePairs; j += 2) {
                    chain_step2_ring<128>(ca, tb, lane_a, mask, p.q, ea[j], ea[j + 1]);
                    chain_step2_ring<128>(cb, tb, lane_b, mask, p.q, eb[j], eb[j + 1]);
                }
            } else {  // rows from register windows loaded at once (8 steps: 3 rows at most)
                uint32_t wa[3], wb[3];
                chain_window_load<128, 3>(ca, p.q, wa);
                chain_window_load<128, 3>(cb, p.q, wb);
#pragma unroll
                for (int j = 0; j < kTablePairs; j += 2) {
                    chain_step2_window<128, 3>(ca, tb, p.q, wa, ea[j], ea[j + 1]);
                    chain_step2_window<128, 3>(cb, tb, p.q, wb, eb[j], eb[j + 1]);
                }
            }
            uint32_t wa[4], wb[4];
            compose_pairs(gather_syms(ea[0], ea[1], ea[2], ea[3]), sa.x, p.q, wa[0], wa[1]);
            compose_pairs(gather_syms(ea[4], ea[5], ea[6], ea[7]), sa.y, p.q, wa[2], wa[3]);
            compose_pairs(gather_syms(eb[0], eb[1], eb[2], eb[3]), sb.x, p.q, wb[0], wb[1]);
            compose_pairs(gather_syms(eb[4], eb[5], eb[6], eb[7]), sb.y, p.q, wb[2], wb[3]);
#pragma unroll
            for (int j = 0; j < 4; j++) {  // chunk = 16 columns: words 8j (k 0-7) and 8j + 4 (k 8-15)
                const uint32_t b0 = xp[8 * j], b1 = xp[8 * j + 4];
                const uint32_t a0 = cvt_f16x2_e4m3x2(wa[j] & 0xFFFFu);
                const uint32_t a2 = cvt_f16x2_e4m3x2(wa[j] >> 16);
                const uint32_t a1 = cvt_f16x2_e4m3x2(wb[j] & 0xFFFFu);
                const uint32_t a3 = cvt_f16x2_e4m3x2(wb[j] >> 16);
                mma_16x8x16(d, a0, a1, a2, a3, b0, b1);
            }
            xp += 32;  // 64 columns
        }
        cp_async_wait<0>();
        const int64_t r0 = w * 16 + g, r1 = r0 + 8;
        const int64_t b0 = 2 * t, b1 = 2 * t + 1;
        if (!live) d[0] = d[1] = d[2] = d[3] = 0.f;
        if (!p.to_partials) {
            const float s0 = p.scale[r0], s1 = p.scale[r1];
            if (b0 < p.B) {
                p.y[b0 * p.R + r0] = __bfloat16_as_ushort(__float2bfloat16_rn(d[0] * s0));
                p.y[b0 * p.R + r1] = __bfloat16_as_ushort(__float2bfloat16_rn(d[2] * s1));
            }
            if (b1 < p.B) {
                p.y[b1 * p.R + r0] = __bfloat16_as_ushort(__float2bfloat16_rn(d[1] * s0));
                p.y[b1 * p.R + r1] = __bfloat16_as_ushort(__float2bfloat16_rn(d[3] * s1));
            }
        } else {
            float *pk = p.part + (int64_t)k * p.B * p.R;
            if (b0 < p.B) {
                pk[b0 * p.R + r0] = d[0];
                pk[b0 * p.R + r1] = d[2];
            }
            if (b1 < p.B) {
                pk[b1 * p.R + r0] = d[1];
                pk[b1 * p.R + r1] = d[3];
            }
        }
    }
}

// y[b][r] = bf16(scale[r] * sum_k part[k][b][r]) for column-sliced GEMVs.
__global__ void gemv_reduce_kernel(const float *__restrict__ part, const float *__restrict__ scale,
                                   uint16_t *__restrict__ y, int64_t R, int64_t B, int64_t KS) {
    pdl_trigger();
    pdl_wait();
    const int64_t n = R * B;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float acc = 0.f;
        for (int64_t k = 0; k < KS; k++) acc += part[k * n + i];
        y[i] = __bfloat16_as_ushort(__float2bfloat16_rn(acc * scale[i % R]));
    }
}

// Fused all-gather epilogue of a row-sharded GEMV: y[b][r] as in
// gemv_reduce_kernel (same summation order, so the same bits), stored
// straight into every rank's gathered buffer y_peers[q][b][col0 + r] over
// NVLink (plain peer stores, two rows per 4-byte store).  The last CTA to
// finish then publishes: after a system-scope fence it raises this rank's
// flag in every rank's flag array to seq + 1 (release, system scope) and
// advances seq.  A reader that has seen all flags reach its own seq (see
// peer_wait) sees every rank's shard of the step.
struct PublishArgs {
    const float *part;  // f32 [KS][B][R]
    const float *scale; // [R]
    int64_t R, B, KS;
    uint16_t *const *y_peers;
    int64_t y_ld, col0;
    uint32_t *const *flag_peers;
    uint32_t *seq, *done;
    int32_t world, rank;
};

__global__ void gemv_publish_kernel(const PublishArgs p) {
    pdl_trigger();
    pdl_wait();
    const int64_t half = p.R / 2, n = half * p.B, plane = p.R * p.B;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / half, r = 2 * (i - b * half), e = b * p.R + r;
        float a0 = 0.f, a1 = 0.f;
        for (int64_t k = 0; k < p.KS; k++) {
            a0 += p.part[k * plane + e];
            a1 += p.part[k * plane + e + 1];
        }
        const uint32_t v = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a0 * p.scale[r])) |
                           ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a1 * p.scale[r + 1])) << 16);
        const int64_t off = b * p.y_ld + p.col0 + r;
        for (int q = 0; q < p.world; q++)
            *reinterpret_cast<uint32_t *>(p.y_peers[q] + off) = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(p.done, 1u) == gridDim.x - 1) {  // every CTA's stores are fenced
            *p.done = 0;
            __threadfence_system();
            const uint32_t v = *p.seq + 1u;
            for (int q = 0; q < p.world; q++)
                asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.flag_peers[q] + p.rank), "r"(v)
                             : "memory");
            *p.seq = v;
        }
    }
}

// --------------------------------------------------- GEMV weight -> dense
//
// Decode a GEMV-layout weight (streams as in gemv_kernel) to a dense
// row-major bf16 matrix of the e4m3 values (exact: e4m3 -> f16 -> f32 ->
// bf16 loses nothing), for batches beyond the GEMV kernel's 8, where the
// contraction is done by a library bf16 GEMM.  One chain per lane; lane
// (g, t) of a warp holds row 16w + g (+8 for the second chain set) and, per
// 16-column chunk, columns 2t, 2t+1, 8+2t, 9+2t: each composed pair becomes
// one bf16x2 store, and a warp's stores cover 8 rows x 16 contiguous bytes.

struct DenseArgs {
    const uint32_t *comp;
    int64_t comp_bytes;
    const int32_t *offsets;
    const uint16_t *states;
    const uint8_t *partial;
    const uint8_t *sm;  // [N/16][K][8]
    const int32_t *table;
    uint16_t *w;        // bf16 [R][C]
    int64_t R, C, KS;
    int32_t *status;
    Opq q;
};

__device__ __forceinline__ uint32_t cvt_bf16x2_e4m3x2(uint32_t v16) {
    uint32_t r;
    asm("{\n\t.reg .b16 h, l, u;\n\t.reg .b32 f;\n\t.reg .f32 fl, fu;\n\t"
        "cvt.u16.u32 h, %1;\n\t"
        "cvt.rn.f16x2.e4m3x2 f, h;\n\t"
        "mov.b32 {l, u}, f;\n\t"
        "cvt.f32.f16 fl, l;\n\t"
        "cvt.f32.f16 fu, u;\n\t"
        "cvt.rn.bf16x2.f32 %0, fu, fl;\n\t}"
        : "=r"(r)
        : "r"(v16));
    return r;
}

template <int R>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) gemv_dense_kernel(const DenseArgs p) {
    extern __shared__ __align__(16) uint8_t smem[];
    load_table(reinterpret_cast<uint32_t *>(smem), p.table, p.status);
    __syncthreads();
    const uint8_t *tb = smem;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t lane_off = 4u * (lane % kCopies);
    const uint32_t mask = (uint32_t)(R - 1) << 7;
    Ring rg;
    rg.lane_base = ring_area<R>(smem, warp, 1) + 4u * lane;
    const int64_t CS = p.C / p.KS, K = p.R * 4 * p.KS;
    const int32_t n_tiles = (int32_t)(CS / 64);
    const int64_t n_groups = K / 32;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp; g < n_groups; g += warps) {
        const int64_t sid = g * 32 + lane;
        Chain ch;
        const int32_t G = chain_init(ch, p.comp, p.comp_bytes, p.offsets, p.states, p.partial,
                                     sid, lane_off, p.status);
        const bool live = G > 0;
        if (!live) chain_idle(ch, p.comp);
        ring_start<R>(rg, ch, __reduce_max_sync(0xffffffffu, live ? G : 0), live);
        cp_async_commit();
        cp_async_wait<0>();
        // stream group g = (w * KS + k) * 2 + chain
        const int64_t chain = g & 1, wk = g >> 1, k = wk % p.KS, w = wk / p.KS;
        const int64_t row = 16 * w + (lane >> 2) + 8 * chain;
        // warp-private staging of one tile: 8 rows x 64 bf16 (row stride 36
        // words, conflict-free), written back as 16-byte stores that cover
        // whole 128-byte row pieces
        uint32_t *stage = reinterpret_cast<uint32_t *>(
            smem + (ring_area<R>(smem, blockDim.x >> 5, 1) - smem_addr(smem)) + warp * 1152);
        const int64_t row0 = 16 * w + 8 * chain;
        uint8_t *dst = reinterpret_cast<uint8_t *>(p.w + (row0 + (lane >> 3)) * p.C + k * CS) +
                       (lane & 7) * 16;
        (void)row;
        const uint8_t *sp = p.sm + sid * 8;
        const int64_t tstep = K * 8, pf_ahead = 3 * tstep, hstep = 4 * p.C * 2;
        uint2 m_n = live ? ld_stream_v2(sp) : make_uint2(0, 0);
        for (int32_t t = 0; t < n_tiles; t++) {
            const uint2 m = m_n;
            sp += tstep;
            if (live && t + 1 < n_tiles) m_n = ld_stream_v2(sp);
            if (live && t + 4 < n_tiles) prefetch_l2(sp + pf_ahead);
            const int32_t need = ring_fill<R>(rg, ch, live);
            cp_async_commit();
            cp_async_wait<kDecodeLag>();
            uint32_t e[kTablePairs];
            if (need >= rg.done[kDecodeLag]) {
#pragma unroll
                for (int j = 0; j < kTablePairs; j++)
                    e[j] = chain_step_ring(ch, tb, rg.lane_base, mask, p.q);
            } else {
#pragma unroll
                for (int j = 0; j < kTablePairs; j++) e[j] = chain_step_global(ch, tb, p.q);
            }
            uint32_t wd[4];
            compose_pairs(gather_syms(e[0], e[1], e[2], e[3]), m.x, p.q, wd[0], wd[1]);
            compose_pairs(gather_syms(e[4], e[5], e[6], e[7]), m.y, p.q, wd[2], wd[3]);
            uint32_t *sw = stage + (lane >> 2) * kStageRowWords + (lane & 3);
#pragma unroll
            for (int c = 0; c < 4; c++) {  // 16-column chunk 4t + c
                sw[c * 8] = live ? cvt_bf16x2_e4m3x2(wd[c] & 0xFFFFu) : 0u;  // columns 2t, 2t+1
                sw[c * 8 + 4] = live ? cvt_bf16x2_e4m3x2(wd[c] >> 16) : 0u;  // columns 8+2t, 9+2t
            }
            __syncwarp();
            const uint32_t *sr = stage + (lane >> 3) * kStageRowWords + (lane & 7) * 4;
#pragma unroll
            for (int h = 0; h < 2; h++) {  // rows (lane >> 3) + 4h
                const uint4 v = *reinterpret_cast<const uint4 *>(sr + h * 4 * kStageRowWords);
                asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(dst + h * hstep),
                             "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                             : "memory");
            }
            dst += 128;  // 64 bf16 columns
            __syncwarp();
        }
        cp_async_wait<0>();
    }
}

// ------------------------------------------- prefill: decode + tcgen05 MMA
//
// y[m][r] = bf16(scale[r] * sum_c e4m3(W[r][c]) * x[m][c]) for a tile of up
// to kTcMaxTokens tokens, with W read in the GEMV stream layout and never
// written out.  A CTA owns 128 rows of W and walks the columns in 64-column
// chunks through a ring of `stages` shared-memory stages, with the work split
// by warp role:
//   - 16 decode warps (8 row groups x 2 chains, one tANS chain per lane, two
//     steps per slab test, slab rows through a per-warp ring of 128-byte rows
//     filled by 16-byte copies, sign/mantissa words loaded two chunks ahead
//     into registers): per chunk each decodes one 8-pair tile of its streams
//     straight into the stage's bf16 A tile (K-major, 128-byte swizzle), then arrives on the
//     stage's a_full barrier.  A warp waits only for the stage to be empty
//     (the MMAs that last read it have completed), so warps drift up to
//     `stages` chunks apart instead of meeting at a block barrier per chunk;
//   - one MMA warp, whose lane 0 loads the x chunk with a tensor-map copy
//     (cp.async.bulk.tensor, 128-byte swizzle, rows past M zero-filled) into
//     the stage's B tile, waits for a_full and x_full, issues four
//     tcgen05.mma (M = 128, N = tokens, K = 16, bf16 in, fp32 accumulate in
//     tensor memory) and commits them to the stage's `empty` barrier.
// After the last chunk the 16 decode warps read the accumulator back
// (tcgen05.ld; warp w reads lanes 32 (w % 4).. and every fourth 8-column
// group), scale, round once to bf16 and store.  Every mbarrier wait is
// bounded and gives up early once another warp has given up; a wait that
// runs out ORs TANS_B200_DATA_TIMEOUT into the status word, the CTA
// waits (bounded) for its own tensor copies still in flight, skips its
// epilogue and frees its tensor memory.
//
// CTA pairs (CL = 2, batches above one tile): the decode, not the MMA,
// bounds this kernel, so every decoded row must serve as many tokens as the
// tensor memory holds.  Two CTAs of a cluster decode row blocks 2b and 2b + 1
// exactly as above, each into its own stage, and the pair is one 2-SM MMA
// (tcgen05 cta_group::2, M = 256): the first CTA's MMA thread issues it, the
// hardware reads A rows 0-127 from the first CTA's stage and rows 128-255
// from the second's, and x rows (the N dimension) half from each.  Per K
// step two MMAs of mma_n tokens (<= 256 each) fill 2 * mma_n accumulator
// columns in both CTAs' tensor memory, so one decode of W serves up to 512
// tokens and no decoded tile is copied between the CTAs.  The second CTA's
// MMA-warp lane loads its x rows and, once its decode warps and copies have
// finished a chunk, arrives on the first CTA's `pair_full` barrier; the
// first CTA's MMA thread, once the pair's MMAs of a stage are done, arrives
// on the second CTA's `free` barrier, which its decode warps and x loads
// wait on.  A CTA that gives up raises its partner's failure flag; cluster
// barriers after the set-up, after the main loops and before the tensor
// memory is freed keep either CTA from leaving while the other may still
// read or write its shared or tensor memory.

constexpr int kTcWarps = 16;                     // decode warps
constexpr int kTcThreads = (kTcWarps + 1) * 32;  // + the MMA warp
constexpr int kTcMaxTokens = 256;
constexpr int kTcMaxStages = 4;
constexpr int kTcATile = 128 * 128;   // 128 rows x 64 bf16
constexpr uint32_t kTcWaitLimit = 1u << 16;  // polls per wait
constexpr uint32_t kTcPollNs = 10000;        // suspend-time hint per poll (ns): bound ~0.66 s

struct TcArgs {
    CUtensorMap xmap;         // x [M][C] bf16: box 64 columns x brows / halves rows, 128-byte swizzle
    const uint32_t *comp;
    int64_t comp_bytes;
    const int32_t *offsets;
    const uint16_t *states;
    const uint8_t *partial;
    const uint8_t *sm;        // [N/16][K][8]
    const int32_t *table;
    const float *scale;       // [R]
    uint16_t *y;              // bf16 [M][R]
    int64_t R, C, KS, M;
    int32_t brows;            // x rows (tokens) per B stage of this CTA
    int32_t mma_n;            // tokens per MMA (multiple of 16, <= 256)
    int32_t halves;           // MMAs per K step (accumulators of mma_n columns)
    int32_t stages;           // shared-memory stages (2..kTcMaxStages)
    int32_t *status;
    Opq q;
};

// K-major, 128-byte-swizzle shared-memory matrix descriptor: 8-row groups
// 1024 bytes apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Byte offset of bf16 element (row, k) in a 128-row x 64 K-major tile with
// the 128-byte swizzle (16-byte chunk index XOR row % 8).
__device__ __forceinline__ uint32_t tc_swz(uint32_t row, uint32_t k) {
    return (row >> 3) * 1024u + (row & 7u) * 128u + ((((k >> 3) ^ row) & 7u) << 4) + (k & 7u) * 2u;
}

// Wait for the phase of `mbar` with the given parity to complete; false when
// the wait runs out or (checked every 16 polls) *failed became non-zero.
// Each poll lets the hardware suspend the thread for up to kTcPollNs until
// the phase completes, so waiting warps take no issue slots from the
// decoding ones; the whole wait is bounded by kTcWaitLimit polls.
// With kCluster the wait acquires at cluster scope (arrivals released by
// other CTAs of the cluster).
template <bool kCluster = false>
__device__ __forceinline__ bool tc_wait(uint32_t mbar, uint32_t parity, const volatile int32_t *failed) {
    for (uint32_t i = 0; i < kTcWaitLimit; i++) {
        uint32_t done;
        if constexpr (kCluster)
            asm volatile(
                "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 P1, [%1], "
                "%2;\n\tselp.b32 %0, 1, 0, P1;\n\t}"
                : "=r"(done)
                : "r"(mbar), "r"(parity)
                : "memory");
        else
            asm volatile(
                "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2, %3;\n\t"
                "selp.b32 %0, 1, 0, P1;\n\t}"
                : "=r"(done)
                : "r"(mbar), "r"(parity), "n"(kTcPollNs)
                : "memory");
        if (done) return true;
        if ((i & 15u) == 15u && failed && *failed) return false;
    }
    return false;
}

__device__ __forceinline__ void tc_arrive(uint32_t mbar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(mbar)
                 : "memory");
}

// Thread-block cluster helpers: this CTA's rank, the shared::cluster address
// of a shared-memory address in CTA `rank`, a releasing arrive on a cluster
// mbarrier, and a full cluster barrier (every thread of every CTA).
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
    return d;
}
__device__ __forceinline__ void tc_arrive_cluster(uint32_t mbar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(mbar) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}

// One box of x (columns 64c..64c+63, tokens row..) -> shared memory at
// `dst`, completing its bytes on mbarrier `bar` (armed by the caller).
__device__ __forceinline__ void tc_copy_x(const CUtensorMap *map, uint32_t dst, uint32_t bar, int32_t c,
                                          int32_t m0) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
        "{%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c * 64), "r"(m0), "r"(bar)
        : "memory");
}

// Block-wide (CL = 1) or cluster-wide barrier between the main loops and the
// epilogue, ordered after the tensor-core work of every thread.
template <int CL>
__device__ __forceinline__ void tc_fence_sync() {
    if constexpr (CL > 1)
        cluster_sync();
    else
        __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
}

template <int R, int CL>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const __grid_constant__ TcArgs p) {
    static_assert(CL == 1 || CL == 2, "one CTA or a CTA pair per MMA");
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ __align__(8) uint64_t a_full[kTcMaxStages], x_full[kTcMaxStages], empty[kTcMaxStages],
        pair_full[kTcMaxStages], free_[kTcMaxStages];
    __shared__ uint32_t tmem_base_s;
    __shared__ int32_t failed_s;
    volatile int32_t *failed = &failed_s;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int S = p.stages;
    // layout: A stages (1024-byte aligned for the swizzle), B stages, the
    // decode warps' slab rings (each aligned to its size), the decode table
    const uint32_t base_sa = smem_addr(smem);
    const uint32_t a_sa = (base_sa + 1023u) & ~1023u;
    const uint32_t b_bytes = (uint32_t)p.brows * 128u;
    const uint32_t b_sa = a_sa + (uint32_t)S * kTcATile;
    constexpr uint32_t ring_bytes = R * 128u;
    const uint32_t ring0 = (b_sa + (uint32_t)S * b_bytes + ring_bytes - 1u) & ~(ring_bytes - 1u);
    const uint32_t tbl_sa = ring0 + kTcWarps * ring_bytes;
    load_table(reinterpret_cast<uint32_t *>(smem + (tbl_sa - base_sa)), p.table, p.status);
    const uint32_t af0 = smem_addr(&a_full[0]), xf0 = smem_addr(&x_full[0]), em0 = smem_addr(&empty[0]);
    const uint32_t pr0 = smem_addr(&pair_full[0]), fr0 = smem_addr(&free_[0]);
    const uint32_t acc_cols = (uint32_t)(p.halves * p.mma_n);
    const uint32_t ncols = acc_cols <= 32 ? 32u
                                          : (acc_cols <= 64 ? 64u
                                                            : (acc_cols <= 128 ? 128u
                                                                               : (acc_cols <= 256 ? 256u : 512u)));
    const uint32_t rank = CL > 1 ? cluster_rank() : 0u;
    const uint32_t peer = rank ^ 1u;
    if (threadIdx.x == 32 * kTcWarps) {
        for (int s = 0; s < S; s++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(af0 + 8u * s), "r"(kTcWarps));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(xf0 + 8u * s));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(em0 + 8u * s));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(pr0 + 8u * s));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(fr0 + 8u * s));
        }
        asm volatile("fence.mbarrier_init.release.cluster;");
        failed_s = 0;
    }
    if constexpr (CL > 1) cluster_sync();  // the partner's barriers exist before anything arrives on them
    if (warp == 0) {
        if constexpr (CL > 1) {
            // one allocation for the pair: the same columns in both CTAs' tensor memory
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_addr(&tmem_base_s)), "r"(ncols));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_addr(&tmem_base_s)), "r"(ncols));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = tmem_base_s;
    const int64_t CS = p.C / p.KS, K = p.R * 4 * p.KS;
    const int32_t tps = (int32_t)(CS / 64), nchunks = (int32_t)(p.C / 64);
    const int32_t m0 = (int32_t)blockIdx.y * p.halves * p.mma_n;  // first token of this tile
    // a give-up is seen by both CTAs of a pair
    auto give_up = [&]() {
        *failed = 1;
        if constexpr (CL > 1)
            asm volatile("st.relaxed.cluster.shared::cluster.b32 [%0], 1;" ::"r"(
                             cluster_addr(smem_addr(&failed_s), peer))
                         : "memory");
    };
    // x rows of chunk c -> B stage s: one box of all tokens (CL = 1), or per
    // MMA half h this CTA's mma_n / 2 tokens (m0 + h mma_n + rank mma_n / 2 ..)
    auto load_x = [&](int32_t c, int s) {
        const uint32_t dst = b_sa + (uint32_t)s * b_bytes, bar = xf0 + 8u * (uint32_t)s;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(b_bytes)
                     : "memory");
        if constexpr (CL > 1) {
            const int32_t hb = p.mma_n / 2;
            for (int h = 0; h < p.halves; h++)
                tc_copy_x(&p.xmap, dst + (uint32_t)(h * hb) * 128u, bar, c, m0 + h * p.mma_n + (int32_t)rank * hb);
        } else {
            tc_copy_x(&p.xmap, dst, bar, c, m0);
        }
    };

    if (warp == kTcWarps && (CL == 1 || rank == 0)) {
        // ------------------------------------- MMA warp (lane 0): one CTA, or the pair's leader
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.mma_n >> 3) << 17) |
                                   ((uint32_t)((128 * CL) >> 4) << 24);
            bool ok = true;
            int32_t loaded = 0, consumed = 0, issued = 0;  // x chunks issued / waited for; MMA chunks
            for (; loaded < (nchunks < S ? nchunks : S); loaded++) load_x(loaded, loaded);
            int s = 0, ps = 0;          // stage of chunk c and of chunk c - 1
            uint32_t ph = 0, pph = 0;   // their phase parities
            for (int32_t c = 0; c < nchunks && ok; c++) {
                // first release the stage of chunk c - 1 once its MMAs are done
                // (the partner's decode warps and x copies wait for this), and
                // refill its x
                if (c >= 1 && loaded < nchunks) {
                    if (!tc_wait(em0 + 8u * ps, pph, failed)) {
                        ok = false;
                        break;
                    }
                    if constexpr (CL > 1) tc_arrive_cluster(cluster_addr(fr0 + 8u * ps, peer));
                    load_x(loaded, ps);
                    loaded++;
                }
                if (!tc_wait(af0 + 8u * s, ph, failed) || !tc_wait(xf0 + 8u * s, ph, failed)) {
                    ok = false;
                    break;
                }
                if constexpr (CL > 1) {  // the partner's A rows and x rows of chunk c
                    if (!tc_wait<true>(pr0 + 8u * s, ph, failed)) {
                        ok = false;
                        break;
                    }
                }
                consumed = c + 1;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t as = a_sa + (uint32_t)s * kTcATile, bs = b_sa + (uint32_t)s * b_bytes;
                for (int h = 0; h < p.halves; h++) {  // MMA half h -> accumulator columns h * mma_n
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const uint64_t ad = tc_smem_desc(as + 32u * j),
                                       bd = tc_smem_desc(bs + (uint32_t)(h * p.mma_n / CL) * 128u + 32u * j);
                        const uint32_t acc = (uint32_t)(c > 0 || j > 0), d = tmem + (uint32_t)(h * p.mma_n);
                        if constexpr (CL > 1)
                            asm volatile(
                                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, "
                                "%5}, p;\n\t}" ::"r"(d),
                                "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(0u));
                        else
                            asm volatile(
                                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(
                                    d),
                                "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(0u));
                    }
                }
                if constexpr (CL > 1)
                    asm volatile(
                        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                            em0 + 8u * s)
                        : "memory");
                else
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                            em0 + 8u * s)
                        : "memory");
                issued = c + 1;
                ps = s;
                pph = ph;
                if (++s == S) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            // the MMAs complete in order: the last commit covers them all
            if (ok && nchunks > 0) {
                const int32_t cl = nchunks - 1;
                if (!tc_wait(em0 + 8u * (cl % S), (uint32_t)((cl / S) & 1), failed)) ok = false;
            }
            if (!ok) {
                give_up();
                // copies and MMAs still in flight finish before the CTA frees
                // its tensor memory and exits
                for (int32_t c = consumed; c < loaded; c++)
                    tc_wait(xf0 + 8u * (c % S), (uint32_t)((c / S) & 1), nullptr);
                if (issued > 0)
                    tc_wait(em0 + 8u * ((issued - 1) % S), (uint32_t)(((issued - 1) / S) & 1), nullptr);
            }
        }
        __syncwarp();
    } else if (warp == kTcWarps) {
        // ------------------------------------- the pair's second CTA: x rows + readiness (lane 0)
        if constexpr (CL > 1) {
            if (lane == 0) {
                bool ok = true;
                int32_t loaded = 0, consumed = 0;
                const uint32_t lead_pr0 = cluster_addr(pr0, 0u);
                int s = 0;
                uint32_t ph = 0;
                for (int32_t c = 0; c < nchunks && ok; c++) {
                    // the stage is free once the leader's MMAs of chunk c - S are done
                    if (c >= S && !tc_wait<true>(fr0 + 8u * s, ph ^ 1u, failed)) {
                        ok = false;
                        break;
                    }
                    load_x(c, s);
                    loaded = c + 1;
                    if (!tc_wait(af0 + 8u * s, ph, failed) || !tc_wait(xf0 + 8u * s, ph, failed)) {
                        ok = false;
                        break;
                    }
                    consumed = c + 1;
                    tc_arrive_cluster(lead_pr0 + 8u * s);
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) {
                    give_up();
                    for (int32_t c = consumed; c < loaded; c++)
                        tc_wait(xf0 + 8u * (c % S), (uint32_t)((c / S) & 1), nullptr);
                }
            }
            __syncwarp();
        }
    } else {
        // ----------------------------------------------------- decode warps
        // one chain per lane (two tANS steps per slab test), a ring of R
        // 128-byte slab rows per warp filled 16 bytes a copy, the
        // sign/mantissa words of the next two chunks in registers
        const uint8_t *tb = smem + (tbl_sa - base_sa);
        const uint32_t lane_off = 4u * (lane % kCopies);
        const uint32_t mask = (uint32_t)(R - 1) << 7;
        const uint32_t ring = ring0 + (uint32_t)warp * ring_bytes;
        const uint32_t ring_lane = ring + 4u * lane, ring_dst = ring + 16u * (lane & 7);
        uint8_t *a_ptr = smem + (a_sa - base_sa);
        const int g = lane >> 2, t4 = lane & 3;
        const int rgrp = warp >> 1, chain = warp & 1;
        const int64_t wg = (int64_t)blockIdx.x * 8 + rgrp;          // global 16-row group
        const uint32_t row = (uint32_t)(16 * rgrp + g + 8 * chain);  // row within the tile
        const int64_t tstep = K * 8;  // sign/mantissa bytes per chunk row
        Chain ch;
        chain_idle(ch, p.comp);
        PairRing rg{};
        bool live = false, on = false, ok = true;
        const uint8_t *ring_src = nullptr;
        const uint8_t *sp = p.sm;
        uint2 m_n0 = make_uint2(0u, 0u), m_n1 = make_uint2(0u, 0u);
        int32_t kslice = 0, tt = 0;  // slice of chunk c and chunk within it
        int s = 0;                   // stage of chunk c
        uint32_t ph = 0;             // (c / S) & 1
        for (int32_t c = 0; c < nchunks; c++) {
            if (tt == 0) {  // this slice's streams, their first rows and sign/mantissa words
                const int64_t sid = ((wg * p.KS + kslice) * 2 + chain) * 32 + lane;
                const int32_t G = chain_init(ch, p.comp, p.comp_bytes, p.offsets, p.states, p.partial,
                                             sid, lane_off, p.status);
                live = G > 0;
                if (!live) chain_idle(ch, p.comp);
                on = ring_start128<R>(rg, ch, G, live, lane, ring_dst, ring_src);
                sp = p.sm + sid * 8;
                if (live) {
                    m_n0 = ld_stream_v2(sp);
                    if (tps > 1) m_n1 = ld_stream_v2(sp + tstep);
                }
            }
            const uint2 m = m_n0;
            m_n0 = m_n1;
            if (live && tt + 2 < tps) m_n1 = ld_stream_v2(sp + (int64_t)(tt + 2) * tstep);
            uint32_t e[kTablePairs];
            if (ring_tile128<R>(rg, row_of128(ch.v, p.q), live, on, lane, ring_src, ring_dst)) {
#pragma unroll
                for (int j = 0; j < kTablePairs; j += 2)
                    chain_step2_ring<128>(ch, tb, ring_lane, mask, p.q, e[j], e[j + 1]);
            } else {
                uint32_t win[3];
                chain_window_load<128, 3>(ch, p.q, win);
#pragma unroll
                for (int j = 0; j < kTablePairs; j += 2) chain_step2_window<128, 3>(ch, tb, p.q, win, e[j], e[j + 1]);
            }
            uint32_t wd[4];
            compose_pairs(gather_syms(e[0], e[1], e[2], e[3]), m.x, p.q, wd[0], wd[1]);
            compose_pairs(gather_syms(e[4], e[5], e[6], e[7]), m.y, p.q, wd[2], wd[3]);
            // the stage is free once the MMAs of chunk c - S have completed
            // (the leader's, relayed to the pair's second CTA); a wait that
            // gives up is published before this warp arrives
            if (c >= S && ok) {
                const bool got = (CL > 1 && rank == 1) ? tc_wait<true>(fr0 + 8u * s, ph ^ 1u, failed)
                                                       : tc_wait(em0 + 8u * s, ph ^ 1u, failed);
                if (!got) {
                    ok = false;
                    give_up();
                }
            }
            uint8_t *at = a_ptr + s * kTcATile;
#pragma unroll
            for (int j = 0; j < 4; j++) {  // 16-column sub-chunk j: columns 2t, 2t+1 | 8+2t, 9+2t
                const uint32_t lo = live ? cvt_bf16x2_e4m3x2(wd[j] & 0xFFFFu) : 0u;
                const uint32_t hi = live ? cvt_bf16x2_e4m3x2(wd[j] >> 16) : 0u;
                *reinterpret_cast<uint32_t *>(at + tc_swz(row, 16 * j + 2 * t4)) = lo;
                *reinterpret_cast<uint32_t *>(at + tc_swz(row, 16 * j + 8 + 2 * t4)) = hi;
            }
            // the MMAs read the tile through the async proxy
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) tc_arrive(af0 + 8u * s);
            if (++tt == tps) {
                tt = 0;
                kslice++;
            }
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }
        cp_async_wait<0>();
    }
    tc_fence_sync<CL>();  // the leader's MMAs are done before either CTA reads its accumulator
    const bool good = *failed == 0;
    if (warp < kTcWarps && good) {
        // warp w: tensor-memory lanes 32 (w % 4).. (rows of this CTA's
        // block), 8-column groups w / 4, w / 4 + 4, ... (token m0 + column)
        const int quarter = warp & 3;
        const int64_t r = (int64_t)blockIdx.x * 128 + 32 * quarter + lane;
        const float sc = p.scale[r];
        for (int col = 8 * (warp >> 2); col < (int)acc_cols; col += 32) {
            uint32_t v[8];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                  "=r"(v[6]), "=r"(v[7])
                : "r"(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)col));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int64_t mm = (int64_t)m0 + col + k;
                if (mm < p.M)
                    p.y[mm * p.R + r] = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[k]) * sc));
            }
        }
    }
    if (!good && threadIdx.x == 0 && p.status) atomicOr(p.status, TANS_B200_DATA_TIMEOUT);
    asm volatile("tcgen05.fence::before_thread_sync;");
    if constexpr (CL > 1)
        cluster_sync();  // both CTAs have read their accumulators before the pair frees them
    else
        __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        if constexpr (CL > 1)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
    }
}

// ------------------------------------------------------------- host glue

constexpr int kMaxDevices = 64;
int g_sms[kMaxDevices];
bool g_attr_set[kMaxDevices];
std::mutex g_mu;

int current_device(int *dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return fail(TANS_B200_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (*dev < 0 || *dev >= kMaxDevices) return fail(TANS_B200_ERR_CUDA, "device id out of range");
    return TANS_B200_OK;
}

int device_setup(int *sms) {
    int dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_attr_set[dev]) {
        cudaError_t e = cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess)
            return fail(TANS_B200_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
        g_attr_set[dev] = true;
    }
    *sms = g_sms[dev];
    return TANS_B200_OK;
}

int launch_status(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(TANS_B200_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
    return TANS_B200_OK;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Launch with programmatic stream serialisation (see pdl_trigger): the kernel
// may start once the previous kernel in the stream has all its CTAs running
// (at once, if that kernel does not trigger early).
template <typename... P, typename... A>
int launch_pdl(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               const char *name, A &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
    if (e != cudaSuccess) return fail(TANS_B200_ERR_CUDA, "%s launch: %s", name, cudaGetErrorString(e));
    return TANS_B200_OK;
}

constexpr int kSmemMax = 227 * 1024;

// Ring depth by stream length: lanes of a warp drift apart by roughly
// 0.3 * sqrt(pairs) rows over a stream; the ring must cover that spread plus
// the look-ahead (rows outside it fall back to global refills, still exact).
int ring_rows(int64_t pairs) {
    return pairs <= 1024 ? 16 : pairs <= 4096 ? 32 : (pairs <= 16384 ? 64 : 128);
}

template <typename Kernel>
int set_smem(Kernel k, int bytes) {
    // The attribute is a per-device, per-kernel upper bound; raise it only
    // when a launch needs more than this device has already allowed, so the
    // steady state of repeated calls makes no driver call here.
    struct Seen {
        const void *kernel;
        int dev, bytes;
    };
    static std::mutex mu;
    static Seen seen[256];
    static int n_seen = 0;
    int dev = 0;
    const int rc = current_device(&dev);
    if (rc) return rc;
    const void *key = reinterpret_cast<const void *>(k);
    std::lock_guard<std::mutex> lock(mu);
    int slot = -1;
    for (int i = 0; i < n_seen; i++)
        if (seen[i].kernel == key && seen[i].dev == dev) slot = i;
    if (slot >= 0 && seen[slot].bytes >= bytes) return TANS_B200_OK;
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess)
        return fail(TANS_B200_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    if (slot >= 0)
        seen[slot].bytes = bytes;
    else if (n_seen < 256)
        seen[n_seen++] = Seen{key, dev, bytes};
    return TANS_B200_OK;
}

template <int R, typename Args, typename Kernel>
int launch_ring_kernel(Kernel kernel, const Args &args, int chains, int64_t n_streams, int sms,
                       cudaStream_t stream, const char *name) {
    const int per_warp = chains * R * 128;
    int max_w = (kSmemMax - kTableBytes - R * 128) / per_warp;
    if (max_w > kMaxWarps) max_w = kMaxWarps;
    const Geometry geo = balance((n_streams + 31) / 32, sms, max_w);
    const int smem = kTableBytes + R * 128 + geo.warps_per_cta * per_warp;
    int rc = set_smem(kernel, smem);
    if (rc) return rc;
    kernel<<<geo.grid, geo.warps_per_cta * 32, smem, stream>>>(args);
    return launch_status(name);
}

Opq make_opq() {
    Opq q;
    q.one = 1;
    q.p16 = 1u << 16;
    q.p31 = 1u << 31;
    q.p28 = 1u << 28;
    q.x16 = 16;
    q.x8 = 8;
    q.step = 4 * kCopies;
    q.back = -kBlk;
    q.back64 = -64;
    q.p26 = 1u << 26;
    q.p25 = 1u << 25;
    q.rmask = 0;
    return q;
}

int stream_grid(int64_t n_vec, int sms) {
    const int64_t want = (n_vec + (int64_t)kStreamThreads * kStreamUnroll - 1) /
                         ((int64_t)kStreamThreads * kStreamUnroll);
    const int64_t cap = (int64_t)sms * 4;
    return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace

// cuTensorMapEncodeTiled, resolved through the runtime so that the library
// needs no link against the driver library.
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tiled_fn(EncodeTiledFn *fn) {
    static EncodeTiledFn cached = nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!cached) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000,
                                                         cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !f)
            return fail(TANS_B200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable: %s",
                        cudaGetErrorString(e));
        cached = reinterpret_cast<EncodeTiledFn>(f);
    }
    *fn = cached;
    return TANS_B200_OK;
}

template <int R>
int launch_fused_pair(FusedArgs &args, int64_t chains, int sms, cudaStream_t stream) {
    const int per_warp = 2 * R * 64;  // two rings
    int max_w = (kSmemMax - kTableBytes - R * 64) / per_warp;
    if (max_w > kPairMaxWarps) max_w = kPairMaxWarps;
    const Geometry geo = balance((chains + 15) / 16, sms, max_w);
    const int smem = kTableBytes + R * 64 + geo.warps_per_cta * per_warp;
    args.q.rmask = (uint32_t)(R - 1) << 6;
    int rc = set_smem(fused_pair_kernel<R>, smem);
    if (rc) return rc;
    fused_pair_kernel<R><<<geo.grid, geo.warps_per_cta * 32, smem, stream>>>(args);
    return launch_status("fused_pair_kernel");
}

static int launch_fused(FusedArgs &args, int64_t chains, int64_t pairs_per_chain, int sms,
                        cudaStream_t st) {
    switch (ring_rows(pairs_per_chain)) {
        case 16: return launch_fused_pair<16>(args, chains, sms, st);
        case 32: return launch_fused_pair<32>(args, chains, sms, st);
        case 64: return launch_fused_pair<64>(args, chains, sms, st);
        default: return launch_fused_pair<128>(args, chains, sms, st);
    }
}

extern "C" int tans_b200_sm_count(int *sm_count) {
    if (!sm_count) return fail(TANS_B200_ERR_INVALID, "sm_count: null");
    return device_setup(sm_count);
}

extern "C" int tans_b200_fp8_memcpy(const uint8_t *a, uint8_t *c, int64_t n, void *stream) {
    tans_b200::clear_error();
    if (n < 0 || n % 16 != 0) return fail(TANS_B200_ERR_INVALID, "A length must be a multiple of 16");
    if (n == 0) return TANS_B200_OK;
    if (!a || !c || !aligned(a, 16) || !aligned(c, 16))
        return fail(TANS_B200_ERR_INVALID, "fp8_memcpy: pointers must be 16-byte aligned");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    const int64_t n_vec = n / 16;
    memcpy_kernel<<<stream_grid(n_vec, sms), kStreamThreads, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint4 *>(a), reinterpret_cast<uint4 *>(c), n_vec);
    return launch_status("memcpy_kernel");
}

extern "C" int tans_b200_fp8_vecadd_raw(const uint8_t *a, const uint8_t *b, uint8_t *c, int64_t n,
                                        void *stream) {
    tans_b200::clear_error();
    if (n < 0 || n % 16 != 0)
        return fail(TANS_B200_ERR_INVALID, "A/B length must be a multiple of 16");
    if (n == 0) return TANS_B200_OK;
    if (!a || !b || !c || !aligned(a, 16) || !aligned(b, 16) || !aligned(c, 16))
        return fail(TANS_B200_ERR_INVALID, "fp8_vecadd_raw: pointers must be 16-byte aligned");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    const int64_t n_vec = n / 16;
    vecadd_raw_kernel<<<stream_grid(n_vec, sms), kStreamThreads, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint4 *>(a), reinterpret_cast<const uint4 *>(b),
        reinterpret_cast<uint4 *>(c), n_vec);
    return launch_status("vecadd_raw_kernel");
}

extern "C" int tans_b200_build_decode_table(const int32_t *spread, const int32_t *freqs,
                                            int64_t n_syms, int32_t *table, int32_t *status,
                                            void *stream) {
    tans_b200::clear_error();
    if (!spread || !freqs || !table)
        return fail(TANS_B200_ERR_INVALID, "build_decode_table: null pointer");
    if (n_syms <= 0 || n_syms > 256)
        return fail(TANS_B200_ERR_INVALID, "build_decode_table: alphabet must be 1..256 symbols");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    build_table_kernel<<<1, kBuildWarps * 32, 0, (cudaStream_t)stream>>>(spread, freqs, (int)n_syms,
                                                                         table, status);
    return launch_status("build_table_kernel");
}

// Decode launch: the team form (output staged per 128-stream block, 16-byte
// row stores) when rows are word-aligned, the output is 16-byte aligned and
// the layout's stream count is a multiple of 128, else the per-warp form.
template <int R>
int launch_decode(const DecodeArgs &args, int64_t chains, int sms, cudaStream_t st) {
    if (!(args.word_rows && args.stride % (kTeamWarps * 32) == 0 &&
          reinterpret_cast<uintptr_t>(args.out) % 16 == 0))
        return launch_ring_kernel<R>(decode_kernel<R, false>, args, 1, chains, sms, st,
                                     "decode_kernel");
    const int per_team = kTeamWarps * R * 128 + kStageBytes;
    int max_t = (kSmemMax - kTableBytes - R * 128) / per_team;
    if (max_t > kDecodeMaxWarps / kTeamWarps) max_t = kDecodeMaxWarps / kTeamWarps;
    const Geometry geo = balance(chains / (kTeamWarps * 32), sms, max_t);
    const int smem = kTableBytes + R * 128 + geo.warps_per_cta * per_team;
    int rc = set_smem(decode_kernel<R, true>, smem);
    if (rc) return rc;
    decode_kernel<R, true><<<geo.grid, geo.warps_per_cta * kTeamWarps * 32, smem, st>>>(args);
    return launch_status("decode_kernel");
}

static int decode_launch(const uint8_t *compressed, int64_t compressed_bytes,
                         const int32_t *offsets, const uint16_t *states, const uint8_t *partial,
                         const uint8_t *sign_mantissa, const int32_t *decode_table, uint8_t *out,
                         int64_t n_streams, int64_t n_fp8_per_stream, int64_t segment_pairs,
                         int32_t *status, void *stream) {
    if (n_fp8_per_stream < 0 || n_fp8_per_stream % 2 != 0)
        return fail(TANS_B200_ERR_INVALID, "n_fp8_per_stream must be even");
    if (compressed_bytes < 0 || compressed_bytes % 4 != 0)
        return fail(TANS_B200_ERR_INVALID, "compressed length must be divisible by 4 bytes");
    if (n_streams < 0) return fail(TANS_B200_ERR_INVALID, "n_streams must be >= 0");
    if (n_streams == 0 || n_fp8_per_stream == 0) return TANS_B200_OK;
    const int64_t segs = (n_fp8_per_stream / 2) / segment_pairs;
    if (segs > 1 && n_streams % 32 != 0)
        return fail(TANS_B200_ERR_INVALID, "split streams need n_streams divisible by 32");
    if (!compressed || !offsets || !states || !partial || !sign_mantissa || !decode_table || !out)
        return fail(TANS_B200_ERR_INVALID, "decode: null pointer");
    if (!aligned(compressed, 4) || !aligned(offsets, 4) || !aligned(states, 2) ||
        !aligned(decode_table, 4))
        return fail(TANS_B200_ERR_INVALID, "decode: misaligned input");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    const int64_t chains = n_streams * segs;
    DecodeArgs args{reinterpret_cast<const uint32_t *>(compressed), compressed_bytes, offsets,
                    states, partial, sign_mantissa, decode_table, out, chains,
                    n_fp8_per_stream, n_streams, segment_pairs, status, make_opq(),
                    (int32_t)(n_streams % 4 == 0 && aligned(sign_mantissa, 4) && aligned(out, 4))};
    cudaStream_t st = (cudaStream_t)stream;
    switch (ring_rows(segment_pairs)) {
        case 16: return launch_decode<16>(args, chains, sms, st);
        case 32: return launch_decode<32>(args, chains, sms, st);
        case 64: return launch_decode<64>(args, chains, sms, st);
        default: return launch_decode<128>(args, chains, sms, st);
    }
}

extern "C" int tans_b200_decode(const uint8_t *compressed, int64_t compressed_bytes,
                                const int32_t *offsets, const uint16_t *states,
                                const uint8_t *partial, const uint8_t *sign_mantissa,
                                const int32_t *decode_table, uint8_t *out, int64_t n_streams,
                                int64_t n_fp8_per_stream, int32_t *status, void *stream) {
    tans_b200::clear_error();
    return decode_launch(compressed, compressed_bytes, offsets, states, partial, sign_mantissa,
                         decode_table, out, n_streams, n_fp8_per_stream,
                         n_fp8_per_stream > 0 ? n_fp8_per_stream / 2 : 1, status, stream);
}

extern "C" int tans_b200_decode_split(const uint8_t *compressed, int64_t compressed_bytes,
                                      const int32_t *offsets, const uint16_t *states,
                                      const uint8_t *partial, const uint8_t *sign_mantissa,
                                      const int32_t *decode_table, uint8_t *out,
                                      int64_t n_streams, int64_t n_fp8_per_stream,
                                      int64_t segment_pairs, int32_t *status, void *stream) {
    tans_b200::clear_error();
    if (segment_pairs <= 0 || n_fp8_per_stream < 0 || (n_fp8_per_stream / 2) % segment_pairs != 0)
        return fail(TANS_B200_ERR_INVALID,
                    "segment_pairs must be a positive divisor of n_fp8_per_stream/2");
    return decode_launch(compressed, compressed_bytes, offsets, states, partial, sign_mantissa,
                         decode_table, out, n_streams, n_fp8_per_stream, segment_pairs, status,
                         stream);
}

extern "C" int tans_b200_fp8_vecadd_fused(
    const uint8_t *a_compressed, int64_t a_compressed_bytes, const int32_t *a_offsets,
    const uint16_t *a_states, const uint8_t *a_partial, const uint8_t *a_sm,
    const uint8_t *b_compressed, int64_t b_compressed_bytes, const int32_t *b_offsets,
    const uint16_t *b_states, const uint8_t *b_partial, const uint8_t *b_sm,
    const int32_t *decode_table, uint8_t *out, int64_t n_streams, int64_t n_fp8_per_stream,
    int32_t *status, void *stream) {
    return tans_b200_fp8_vecadd_fused_range(
        a_compressed, a_compressed_bytes, a_offsets, a_states, a_partial, a_sm, b_compressed,
        b_compressed_bytes, b_offsets, b_states, b_partial, b_sm, decode_table, out, n_streams,
        n_fp8_per_stream, 0, n_streams, status, stream);
}

extern "C" int tans_b200_fp8_vecadd_fused_range(
    const uint8_t *a_compressed, int64_t a_compressed_bytes, const int32_t *a_offsets,
    const uint16_t *a_states, const uint8_t *a_partial, const uint8_t *a_sm,
    const uint8_t *b_compressed, int64_t b_compressed_bytes, const int32_t *b_offsets,
    const uint16_t *b_states, const uint8_t *b_partial, const uint8_t *b_sm,
    const int32_t *decode_table, uint8_t *out, int64_t n_streams, int64_t n_fp8_per_stream,
    int64_t stream_begin, int64_t stream_end, int32_t *status, void *stream) {
    tans_b200::clear_error();
    if (n_fp8_per_stream < 0 || n_fp8_per_stream % 16 != 0)
        return fail(TANS_B200_ERR_INVALID, "n_fp8_per_stream must be divisible by 16");
    if (a_compressed_bytes < 0 || b_compressed_bytes < 0 || a_compressed_bytes % 4 != 0 ||
        b_compressed_bytes % 4 != 0)
        return fail(TANS_B200_ERR_INVALID,
                    "compressed tensors must have byte lengths divisible by 4");
    if (n_streams < 0) return fail(TANS_B200_ERR_INVALID, "n_streams must be >= 0");
    if (stream_begin < 0 || stream_begin % kBlk != 0 || stream_end < stream_begin ||
        stream_end > n_streams)
        return fail(TANS_B200_ERR_INVALID,
                    "fp8_vecadd_fused: stream range [%lld, %lld) must start on a 128-stream "
                    "block and lie in [0, %lld]",
                    (long long)stream_begin, (long long)stream_end, (long long)n_streams);
    if (n_streams == 0 || n_fp8_per_stream == 0 || stream_end == stream_begin) return TANS_B200_OK;
    if (!a_compressed || !a_offsets || !a_states || !a_partial || !a_sm || !b_compressed ||
        !b_offsets || !b_states || !b_partial || !b_sm || !decode_table || !out)
        return fail(TANS_B200_ERR_INVALID, "fp8_vecadd_fused: null pointer");
    if (!aligned(a_compressed, 4) || !aligned(b_compressed, 4) || !aligned(a_offsets, 4) ||
        !aligned(b_offsets, 4) || !aligned(a_states, 2) || !aligned(b_states, 2) ||
        !aligned(a_sm, 8) || !aligned(b_sm, 8) || !aligned(decode_table, 4) || !aligned(out, 16))
        return fail(TANS_B200_ERR_INVALID,
                    "fp8_vecadd_fused: sm tensors need 8-byte and the output 16-byte alignment");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    // a range is the full layout seen from its first stream: per-stream and
    // per-block arrays start there, tiles keep the full row stride
    const int64_t s0 = stream_begin, b0 = stream_begin / kBlk;
    FusedArgs args{};
    args.a_comp = reinterpret_cast<const uint32_t *>(a_compressed);
    args.b_comp = reinterpret_cast<const uint32_t *>(b_compressed);
    args.a_bytes = a_compressed_bytes;
    args.b_bytes = b_compressed_bytes;
    args.a_off = a_offsets + b0;
    args.b_off = b_offsets + b0;
    args.a_st = a_states + s0;
    args.b_st = b_states + s0;
    args.a_part = a_partial + s0;
    args.b_part = b_partial + s0;
    args.a_sm = a_sm + 8 * s0;
    args.b_sm = b_sm + 8 * s0;
    args.table = decode_table;
    args.out = out + 16 * s0;
    args.K = stream_end - stream_begin;
    args.N = n_fp8_per_stream;
    args.stride = n_streams;
    args.seg_tiles = n_fp8_per_stream / 16;
    args.status = status;
    args.q = make_opq();
    return launch_fused(args, stream_end - stream_begin, n_fp8_per_stream / 2, sms,
                        (cudaStream_t)stream);
}

extern "C" int tans_b200_fp8_vecadd_fused_split(
    const uint8_t *a_compressed, int64_t a_compressed_bytes, const int32_t *a_offsets,
    const uint16_t *a_states, const uint8_t *a_partial, const uint8_t *a_sm,
    const uint8_t *b_compressed, int64_t b_compressed_bytes, const int32_t *b_offsets,
    const uint16_t *b_states, const uint8_t *b_partial, const uint8_t *b_sm,
    const int32_t *decode_table, uint8_t *out, int64_t n_streams, int64_t n_fp8_per_stream,
    int64_t segment_pairs, int32_t *status, void *stream) {
    tans_b200::clear_error();
    if (n_fp8_per_stream < 0 || n_fp8_per_stream % 16 != 0)
        return fail(TANS_B200_ERR_INVALID, "n_fp8_per_stream must be divisible by 16");
    if (segment_pairs <= 0 || segment_pairs % kTablePairs != 0 ||
        (n_fp8_per_stream / 2) % segment_pairs != 0)
        return fail(TANS_B200_ERR_INVALID,
                    "segment_pairs must be a positive multiple of 8 dividing n_fp8_per_stream/2");
    if (a_compressed_bytes < 0 || b_compressed_bytes < 0 || a_compressed_bytes % 4 != 0 ||
        b_compressed_bytes % 4 != 0)
        return fail(TANS_B200_ERR_INVALID,
                    "compressed tensors must have byte lengths divisible by 4");
    if (n_streams < 0) return fail(TANS_B200_ERR_INVALID, "n_streams must be >= 0");
    const int64_t segs = (n_fp8_per_stream / 2) / segment_pairs;
    if (segs > 1 && n_streams % 32 != 0)
        return fail(TANS_B200_ERR_INVALID, "split streams need n_streams divisible by 32");
    if (n_streams == 0 || n_fp8_per_stream == 0) return TANS_B200_OK;
    if (!a_compressed || !a_offsets || !a_states || !a_partial || !a_sm || !b_compressed ||
        !b_offsets || !b_states || !b_partial || !b_sm || !decode_table || !out)
        return fail(TANS_B200_ERR_INVALID, "fp8_vecadd_fused: null pointer");
    if (!aligned(a_compressed, 4) || !aligned(b_compressed, 4) || !aligned(a_offsets, 4) ||
        !aligned(b_offsets, 4) || !aligned(a_states, 2) || !aligned(b_states, 2) ||
        !aligned(a_sm, 8) || !aligned(b_sm, 8) || !aligned(decode_table, 4) || !aligned(out, 16))
        return fail(TANS_B200_ERR_INVALID,
                    "fp8_vecadd_fused: sm tensors need 8-byte and the output 16-byte alignment");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    FusedArgs args{};
    args.a_comp = reinterpret_cast<const uint32_t *>(a_compressed);
    args.b_comp = reinterpret_cast<const uint32_t *>(b_compressed);
    args.a_bytes = a_compressed_bytes;
    args.b_bytes = b_compressed_bytes;
    args.a_off = a_offsets;
    args.b_off = b_offsets;
    args.a_st = a_states;
    args.b_st = b_states;
    args.a_part = a_partial;
    args.b_part = b_partial;
    args.a_sm = a_sm;
    args.b_sm = b_sm;
    args.table = decode_table;
    args.out = out;
    args.K = n_streams * segs;
    args.N = n_fp8_per_stream;
    args.stride = n_streams;
    args.seg_tiles = segment_pairs / kTablePairs;
    args.status = status;
    args.q = make_opq();
    return launch_fused(args, n_streams * segs, segment_pairs, sms, (cudaStream_t)stream);
}

// Geometry and launch of gemv_kernel (the plain GEMV and the gathering one).
static int launch_gemv_kernel(const GemvArgs &args, int sms, cudaStream_t st) {
    const int64_t rows = args.R, cols = args.C, col_splits = args.KS;
    int rc = TANS_B200_OK;
    const int64_t cs = cols / col_splits;
    const int rr = ring_rows(cs / 8);
    const int64_t xbytes = ((kGemvMaxBatch * (cs + 8) * 2) + 127) / 128 * 128;
    const int64_t fixed = kTableBytes + xbytes + rr * 128;
    const int64_t per_warp = 2 * rr * 128;
    const bool short_slices = rr == 16 && cs <= kGemvShortCols;
    const int64_t cap = short_slices ? kGemvShortWarps : kGemvMaxWarps;
    int64_t max_w = (kSmemMax - fixed) / per_warp;
    if (max_w > cap) max_w = cap;
    if (max_w < 1)
        return fail(TANS_B200_ERR_INVALID,
                    "gemv: a column slice of %lld does not fit in shared memory; use more col_splits",
                    (long long)cs);
    const int64_t groups = rows / 16;
    int64_t gx = sms / col_splits;
    if (gx < 1) gx = 1;
    const int64_t rounds = (groups + gx * max_w - 1) / (gx * max_w);
    const int64_t wpc = (groups + gx * rounds - 1) / (gx * rounds);
    gx = (groups + wpc * rounds - 1) / (wpc * rounds);
    const int smem = (int)(fixed + wpc * per_warp);
    const dim3 grid((unsigned)gx, (unsigned)col_splits);
    const dim3 block((unsigned)wpc * 32);
    if (short_slices) {
        rc = set_smem(gemv_kernel<16, kGemvShortWarps>, smem);
        if (!rc) rc = launch_pdl(gemv_kernel<16, kGemvShortWarps>, grid, block, smem, st, "gemv_kernel", args);
        return rc;
    }
    switch (rr) {
        case 16: rc = set_smem(gemv_kernel<16>, smem); if (!rc) rc = launch_pdl(gemv_kernel<16>, grid, block, smem, st, "gemv_kernel", args); break;
        case 32: rc = set_smem(gemv_kernel<32>, smem); if (!rc) rc = launch_pdl(gemv_kernel<32>, grid, block, smem, st, "gemv_kernel", args); break;
        case 64: rc = set_smem(gemv_kernel<64>, smem); if (!rc) rc = launch_pdl(gemv_kernel<64>, grid, block, smem, st, "gemv_kernel", args); break;
        default: rc = set_smem(gemv_kernel<128>, smem); if (!rc) rc = launch_pdl(gemv_kernel<128>, grid, block, smem, st, "gemv_kernel", args); break;
    }
    return rc;
}

extern "C" int tans_b200_gemv(const uint8_t *compressed, int64_t compressed_bytes,
                              const int32_t *offsets, const uint16_t *states,
                              const uint8_t *partial, const uint8_t *sm,
                              const int32_t *decode_table, const float *scale,
                              const uint16_t *x, uint16_t *y, float *partials, int64_t rows,
                              int64_t cols, int64_t batch, int64_t col_splits, int32_t *status,
                              void *stream) {
    tans_b200::clear_error();
    if (rows <= 0 || rows % 16 != 0) return fail(TANS_B200_ERR_INVALID, "gemv: rows must be a positive multiple of 16");
    if (col_splits < 1 || cols <= 0 || cols % (64 * col_splits) != 0)
        return fail(TANS_B200_ERR_INVALID, "gemv: cols must be a positive multiple of 64 * col_splits");
    if (batch < 1 || batch > kGemvMaxBatch) return fail(TANS_B200_ERR_INVALID, "gemv: batch must be 1..8");
    if (!compressed || !offsets || !states || !partial || !sm || !decode_table || !scale || !x || !y ||
        (col_splits > 1 && !partials))
        return fail(TANS_B200_ERR_INVALID, "gemv: null pointer");
    if (!aligned(compressed, 4) || !aligned(offsets, 4) || !aligned(states, 2) || !aligned(sm, 8) ||
        !aligned(decode_table, 4) || !aligned(scale, 4) || !aligned(x, 2) || !aligned(y, 2) ||
        (partials && !aligned(partials, 4)))
        return fail(TANS_B200_ERR_INVALID, "gemv: misaligned buffer");
    if (compressed_bytes < 0 || compressed_bytes % 4 != 0)
        return fail(TANS_B200_ERR_INVALID, "compressed length must be divisible by 4 bytes");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    GemvArgs args{reinterpret_cast<const uint32_t *>(compressed), compressed_bytes, offsets, states,
                  partial, sm, decode_table, scale, x, y, partials, rows, cols, batch, col_splits,
                  status, make_opq(), nullptr, nullptr, 0, (int32_t)(col_splits > 1)};
    cudaStream_t st = (cudaStream_t)stream;
    rc = launch_gemv_kernel(args, sms, st);
    if (rc || col_splits == 1) return rc;
    const int64_t n = rows * batch;
    const int threads = 256;
    const int64_t blocks = (n + threads - 1) / threads;
    return launch_pdl(gemv_reduce_kernel, dim3((unsigned)(blocks < 4 * sms ? blocks : 4 * sms)),
                      dim3(threads), 0, st, "gemv_reduce_kernel", (const float *)partials, scale,
                      (uint16_t *)y, rows, batch, col_splits);
}

extern "C" int tans_b200_gemv_gather(const uint8_t *compressed, int64_t compressed_bytes,
                                     const int32_t *offsets, const uint16_t *states,
                                     const uint8_t *partial, const uint8_t *sm,
                                     const int32_t *decode_table, const float *scale,
                                     const uint16_t *x, float *partials, int64_t rows, int64_t cols,
                                     int64_t batch, int64_t col_splits, const tans_b200_gather *g,
                                     int32_t *status, void *stream) {
    tans_b200::clear_error();
    if (rows <= 0 || rows % 16 != 0) return fail(TANS_B200_ERR_INVALID, "gemv: rows must be a positive multiple of 16");
    if (col_splits < 1 || cols <= 0 || cols % (64 * col_splits) != 0)
        return fail(TANS_B200_ERR_INVALID, "gemv: cols must be a positive multiple of 64 * col_splits");
    if (batch < 1 || batch > kGemvMaxBatch) return fail(TANS_B200_ERR_INVALID, "gemv: batch must be 1..8");
    if (!compressed || !offsets || !states || !partial || !sm || !decode_table || !scale || !x ||
        !partials || !g)
        return fail(TANS_B200_ERR_INVALID, "gemv_gather: null pointer");
    if (g->world < 1 || g->world > kMaxDevices || g->rank < 0 || g->rank >= g->world)
        return fail(TANS_B200_ERR_INVALID, "gemv_gather: rank %d of %d", (int)g->rank, (int)g->world);
    if (!g->y_peers || !g->flag_peers || !g->flags || !g->seq || !g->done)
        return fail(TANS_B200_ERR_INVALID, "gemv_gather: null pointer in the gather descriptor");
    if (g->col0 < 0 || g->col0 % 2 != 0 || g->y_ld % 2 != 0 || g->col0 + rows > g->y_ld)
        return fail(TANS_B200_ERR_INVALID,
                    "gemv_gather: this rank's rows [col0, col0 + rows) must lie in the gathered row "
                    "length y_ld; col0 and y_ld even");
    if (!aligned(compressed, 4) || !aligned(offsets, 4) || !aligned(states, 2) || !aligned(sm, 8) ||
        !aligned(decode_table, 4) || !aligned(scale, 4) || !aligned(x, 2) || !aligned(partials, 4) ||
        !aligned(g->flags, 4) || !aligned(g->seq, 4) || !aligned(g->done, 4))
        return fail(TANS_B200_ERR_INVALID, "gemv_gather: misaligned buffer");
    if (compressed_bytes < 0 || compressed_bytes % 4 != 0)
        return fail(TANS_B200_ERR_INVALID, "compressed length must be divisible by 4 bytes");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    GemvArgs args{reinterpret_cast<const uint32_t *>(compressed), compressed_bytes, offsets, states,
                  partial, sm, decode_table, scale, x, nullptr, partials, rows, cols, batch,
                  col_splits, status, make_opq(), g->flags, g->seq, g->world, 1};
    cudaStream_t st = (cudaStream_t)stream;
    rc = launch_gemv_kernel(args, sms, st);
    if (rc) return rc;
    const PublishArgs pa{partials, scale, rows, batch, col_splits, g->y_peers, g->y_ld, g->col0,
                         g->flag_peers, g->seq, g->done, g->world, g->rank};
    const int64_t n = rows / 2 * batch;
    const int threads = 256;
    const int64_t blocks = (n + threads - 1) / threads;
    return launch_pdl(gemv_publish_kernel, dim3((unsigned)(blocks < 2 * sms ? blocks : 2 * sms)),
                      dim3(threads), 0, st, "gemv_publish_kernel", pa);
}

// y[m][r] = bf16(acc[m][r] * scale[r]): the prefill epilogue after the
// library GEMM (fp32 output), one rounding; 4 columns per thread.
__global__ void scale_rows_bf16_kernel(const float4 *__restrict__ acc, const float *__restrict__ scale,
                                       uint2 *__restrict__ y, int64_t n4, int64_t R4) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float4 a = acc[i];
        const float4 sc = reinterpret_cast<const float4 *>(scale)[i % R4];
        const __nv_bfloat162 lo = __floats2bfloat162_rn(a.x * sc.x, a.y * sc.y);
        const __nv_bfloat162 hi = __floats2bfloat162_rn(a.z * sc.z, a.w * sc.w);
        y[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&lo),
                          *reinterpret_cast<const uint32_t *>(&hi));
    }
}

// Dense decode launch: per warp a slab ring and a 1152-byte staging tile.
template <int R>
int launch_dense(const DenseArgs &args, int64_t chains, int sms, cudaStream_t st) {
    const int per_warp = R * 128 + 1152;
    int max_w = (kSmemMax - kTableBytes - R * 128) / per_warp;
    if (max_w > kMaxWarps) max_w = kMaxWarps;
    const Geometry geo = balance((chains + 31) / 32, sms, max_w);
    const int smem = kTableBytes + R * 128 + geo.warps_per_cta * per_warp;
    int rc = set_smem(gemv_dense_kernel<R>, smem);
    if (rc) return rc;
    gemv_dense_kernel<R><<<geo.grid, geo.warps_per_cta * 32, smem, st>>>(args);
    return launch_status("gemv_dense_kernel");
}

extern "C" int tans_b200_gemv_raw(const uint8_t *w, const float *scale, const uint16_t *x,
                                  uint16_t *y, float *partials, int64_t rows, int64_t cols,
                                  int64_t batch, int64_t col_splits, void *stream) {
    tans_b200::clear_error();
    if (rows <= 0 || rows % 16 != 0)
        return fail(TANS_B200_ERR_INVALID, "gemv_raw: rows must be a positive multiple of 16");
    if (col_splits < 1 || cols <= 0 || cols % (64 * col_splits) != 0)
        return fail(TANS_B200_ERR_INVALID, "gemv_raw: cols must be a positive multiple of 64 * col_splits");
    if (batch < 1 || batch > kGemvMaxBatch) return fail(TANS_B200_ERR_INVALID, "gemv_raw: batch must be 1..8");
    if (!w || !scale || !x || !y || !partials) return fail(TANS_B200_ERR_INVALID, "gemv_raw: null pointer");
    if (!aligned(w, 16) || !aligned(x, 16) || !aligned(y, 2) || !aligned(partials, 4) || !aligned(scale, 4))
        return fail(TANS_B200_ERR_INVALID, "gemv_raw: w and x must be 16-byte aligned");
    const int64_t cs = cols / col_splits;
    const int64_t smem = kGemvMaxBatch * (cs + 8) * 2;
    if (smem > kSmemMax)
        return fail(TANS_B200_ERR_INVALID, "gemv_raw: a column slice of %lld does not fit in shared memory",
                    (long long)cs);
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    rc = set_smem(gemv_raw_kernel, (int)smem);
    if (rc) return rc;
    RawGemvArgs args{w, x, partials, rows, cols, batch, col_splits};
    const int64_t gx = (rows / 16 + kRawGemvWarps - 1) / kRawGemvWarps;
    const dim3 grid((unsigned)gx, (unsigned)col_splits);
    cudaStream_t st = (cudaStream_t)stream;
    gemv_raw_kernel<<<grid, kRawGemvWarps * 32, (int)smem, st>>>(args);
    rc = launch_status("gemv_raw_kernel");
    if (rc) return rc;
    const int64_t n = rows * batch;
    const int64_t blocks = (n + 255) / 256;
    gemv_reduce_kernel<<<(unsigned)(blocks < 4 * sms ? blocks : 4 * sms), 256, 0, st>>>(
        partials, scale, y, rows, batch, col_splits);
    return launch_status("gemv_reduce_kernel");
}

extern "C" int tans_b200_gemv_weight_dense(const uint8_t *compressed, int64_t compressed_bytes,
                                           const int32_t *offsets, const uint16_t *states,
                                           const uint8_t *partial, const uint8_t *sm,
                                           const int32_t *decode_table, uint16_t *w_bf16,
                                           int64_t rows, int64_t cols, int64_t col_splits,
                                           int32_t *status, void *stream) {
    tans_b200::clear_error();
    if (rows <= 0 || rows % 16 != 0)
        return fail(TANS_B200_ERR_INVALID, "gemv: rows must be a positive multiple of 16");
    if (col_splits < 1 || cols <= 0 || cols % (64 * col_splits) != 0)
        return fail(TANS_B200_ERR_INVALID, "gemv: cols must be a positive multiple of 64 * col_splits");
    if (!compressed || !offsets || !states || !partial || !sm || !decode_table || !w_bf16)
        return fail(TANS_B200_ERR_INVALID, "gemv_weight_dense: null pointer");
    if (!aligned(compressed, 4) || !aligned(offsets, 4) || !aligned(states, 2) ||
        !aligned(sm, 8) || !aligned(decode_table, 4) || !aligned(w_bf16, 4))
        return fail(TANS_B200_ERR_INVALID, "gemv_weight_dense: misaligned buffer");
    if (compressed_bytes < 0 || compressed_bytes % 4 != 0)
        return fail(TANS_B200_ERR_INVALID, "compressed length must be divisible by 4 bytes");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    DenseArgs args{reinterpret_cast<const uint32_t *>(compressed), compressed_bytes, offsets,
                   states, partial, sm, decode_table, w_bf16, rows, cols, col_splits, status,
                   make_opq()};
    const int64_t chains = rows * 4 * col_splits;
    cudaStream_t st = (cudaStream_t)stream;
    switch (ring_rows(cols / col_splits / 8)) {
        case 16: return launch_dense<16>(args, chains, sms, st);
        case 32: return launch_dense<32>(args, chains, sms, st);
        case 64: return launch_dense<64>(args, chains, sms, st);
        default: return launch_dense<128>(args, chains, sms, st);
    }
}

extern "C" int tans_b200_scale_rows_bf16(const float *acc, const float *scale, uint16_t *y,
                                         int64_t m, int64_t rows, void *stream) {
    tans_b200::clear_error();
    if (m < 0 || rows <= 0 || rows % 4 != 0)
        return fail(TANS_B200_ERR_INVALID, "scale_rows_bf16: rows must be a positive multiple of 4");
    if (m == 0) return TANS_B200_OK;
    if (!acc || !scale || !y) return fail(TANS_B200_ERR_INVALID, "scale_rows_bf16: null pointer");
    if (!aligned(acc, 16) || !aligned(scale, 16) || !aligned(y, 8))
        return fail(TANS_B200_ERR_INVALID, "scale_rows_bf16: misaligned buffer");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    const int64_t n4 = m * rows / 4;
    const int64_t blocks = (n4 + 255) / 256;
    scale_rows_bf16_kernel<<<(unsigned)(blocks < 8 * sms ? blocks : 8 * sms), 256, 0,
                             (cudaStream_t)stream>>>(reinterpret_cast<const float4 *>(acc), scale,
                                                     reinterpret_cast<uint2 *>(y), n4, rows / 4);
    return launch_status("scale_rows_bf16_kernel");
}

extern "C" int tans_b200_gemm_tc(const uint8_t *compressed, int64_t compressed_bytes,
                                 const int32_t *offsets, const uint16_t *states,
                                 const uint8_t *partial, const uint8_t *sm,
                                 const int32_t *decode_table, const float *scale,
                                 const uint16_t *x, uint16_t *y, int64_t rows, int64_t cols,
                                 int64_t col_splits, int64_t m, int32_t *status, void *stream) {
    tans_b200::clear_error();
    if (rows <= 0 || rows % 128 != 0)
        return fail(TANS_B200_ERR_INVALID, "gemm_tc: rows must be a positive multiple of 128");
    if (col_splits < 1 || cols <= 0 || cols % (64 * col_splits) != 0)
        return fail(TANS_B200_ERR_INVALID, "gemv: cols must be a positive multiple of 64 * col_splits");
    if (m < 1 || m > INT32_MAX - kTcMaxTokens)
        return fail(TANS_B200_ERR_INVALID, "gemm_tc: m must be in [1, 2^31 - 257]");
    if (!compressed || !offsets || !states || !partial || !sm || !decode_table || !scale || !x || !y)
        return fail(TANS_B200_ERR_INVALID, "gemm_tc: null pointer");
    if (!aligned(compressed, 4) || !aligned(offsets, 4) || !aligned(states, 2) || !aligned(sm, 8) ||
        !aligned(decode_table, 4) || !aligned(scale, 4) || !aligned(x, 16) || !aligned(y, 2))
        return fail(TANS_B200_ERR_INVALID, "gemm_tc: misaligned buffer (x needs 16 bytes)");
    if (compressed_bytes < 0 || compressed_bytes % 4 != 0)
        return fail(TANS_B200_ERR_INVALID, "compressed length must be divisible by 4 bytes");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    // Up to 256 tokens: one CTA per 128-row block holds them all (multiple of
    // 16).  Above that, when the row-block count is even, CTA pairs over two
    // row blocks (2-SM MMA, M = 256) with tiles of up to 512 tokens: two MMAs
    // of mma_n tokens per K step (the smallest multiple of 16 that spreads M
    // evenly over the tiles), each CTA holding half of every MMA's x rows.
    // Otherwise 256-token tiles, each decoding W again.
    const int cl = (m > kTcMaxTokens && (rows / 128) % 2 == 0) ? 2 : 1;
    int brows, mma_n, halves, box_rows;
    int64_t ty;
    if (cl == 2) {
        ty = (m + 2 * kTcMaxTokens - 1) / (2 * kTcMaxTokens);
        halves = 2;
        mma_n = (int)(((m + 2 * ty - 1) / (2 * ty) + 15) / 16 * 16);
        box_rows = mma_n / 2;
        brows = mma_n;  // two halves of mma_n / 2 rows
    } else {
        mma_n = (int)((m + 15) / 16 * 16);
        if (mma_n > kTcMaxTokens) mma_n = kTcMaxTokens;
        ty = (m + mma_n - 1) / mma_n;
        halves = 1;
        box_rows = brows = mma_n;
    }
    // ring rows by slice length (at most 32), 16 where 32 would leave fewer
    // than two stages; fixed bytes: 1 KiB to align the stages, the rings'
    // own alignment past that, the rings and the table
    const int per_stage = kTcATile + brows * 128;
    auto fixed_bytes = [](int r) { return 1024 + (r * 128 > 1024 ? r * 128 - 1024 : 0) + kTcWarps * r * 128 + kTableBytes; };
    int rr = ring_rows(cols / col_splits / 8) > 16 ? 32 : 16;
    if (rr == 32 && (kSmemMax - 256 - fixed_bytes(32)) / per_stage < 2) rr = 16;
    const int fixed = fixed_bytes(rr);
    int stages = (kSmemMax - 256 - fixed) / per_stage;  // 256 bytes left for static shared memory
    if (stages > kTcMaxStages) stages = kTcMaxStages;
    if (stages < 2) return fail(TANS_B200_ERR_INVALID, "gemm_tc: shared memory");
    const int smem = fixed + stages * per_stage;
    EncodeTiledFn encode;
    rc = encode_tiled_fn(&encode);
    if (rc) return rc;
    TcArgs args{};
    // x [m][cols] bf16: dimension 0 = columns (contiguous), dimension 1 = tokens;
    // one box = 64 columns (128 bytes, the swizzle span) x box_rows tokens;
    // tokens past m read as zeros
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)m};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = encode(&args.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(TANS_B200_ERR_CUDA, "gemm_tc: tensor map encode failed (%d)", (int)cr);
    args.comp = reinterpret_cast<const uint32_t *>(compressed);
    args.comp_bytes = compressed_bytes;
    args.offsets = offsets;
    args.states = states;
    args.partial = partial;
    args.sm = sm;
    args.table = decode_table;
    args.scale = scale;
    args.y = y;
    args.R = rows;
    args.C = cols;
    args.KS = col_splits;
    args.M = m;
    args.brows = brows;
    args.mma_n = mma_n;
    args.halves = halves;
    args.stages = stages;
    args.status = status;
    args.q = make_opq();
    const dim3 grid((unsigned)(rows / 128), (unsigned)ty);
    if (cl == 2) {
        // CTA pairs along x (row blocks 2b, 2b + 1)
        if (rr != 16) return fail(TANS_B200_ERR_INVALID, "gemm_tc: pair layout");
        rc = set_smem(gemm_tc_kernel<16, 2>, smem);
        if (rc) return rc;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kTcThreads);
        cfg.dynamicSmemBytes = (size_t)smem;
        cfg.stream = (cudaStream_t)stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tc_kernel<16, 2>, args);
        if (e != cudaSuccess)
            return fail(TANS_B200_ERR_CUDA, "gemm_tc_kernel launch: %s", cudaGetErrorString(e));
    } else if (rr == 32) {
        rc = set_smem(gemm_tc_kernel<32, 1>, smem);
        if (rc) return rc;
        gemm_tc_kernel<32, 1><<<grid, kTcThreads, smem, (cudaStream_t)stream>>>(args);
    } else {
        rc = set_smem(gemm_tc_kernel<16, 1>, smem);
        if (rc) return rc;
        gemm_tc_kernel<16, 1><<<grid, kTcThreads, smem, (cudaStream_t)stream>>>(args);
    }
    return launch_status("gemm_tc_kernel");
}

// ------------------------------------------------------- allocation-free decode
//
// tans_b200_decode_noalloc: the standalone decode from spread/freqs for
// callers that cannot allocate device memory (a runtime that hands the
// library a fixed set of buffers carved from a pre-sized pool, or a binding
// from a host language with no device allocator).  The only scratch the path
// needs, the 4096-entry decode table, lives in the file-scope array below:
// 16 KiB on every GPU that loads the library, held until the process exits.
// Each call rewrites the whole table before the decode reads it, so nothing
// has to start at zero; because every call shares the one array, calls whose
// GPU work overlaps (on different streams) race on it and must be ordered by
// the caller.
namespace {

constexpr int kNoAllocTableEntries = kL;  // the maximum (and only) scratch: one table
static __device__ __align__(256) int32_t g_noalloc_table[kNoAllocTableEntries];
int32_t *g_noalloc_table_ptr[kMaxDevices];

// Device address of this device's table, resolved once per device with that
// device current (the first call on a device does this; make that first call
// outside any stream capture).
int noalloc_table(int32_t **ptr) {
    int dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_noalloc_table_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_table);
        if (e != cudaSuccess || !p)
            return fail(TANS_B200_ERR_CUDA, "decode_noalloc: cudaGetSymbolAddress: %s",
                        cudaGetErrorString(e));
        g_noalloc_table_ptr[dev] = static_cast<int32_t *>(p);
    }
    *ptr = g_noalloc_table_ptr[dev];
    return TANS_B200_OK;
}

}  // namespace

extern "C" int tans_b200_decode_noalloc(const uint8_t *compressed, int64_t compressed_bytes,
                                        const int32_t *offsets, const uint16_t *states,
                                        const uint8_t *partial, const uint8_t *sign_mantissa,
                                        const int32_t *spread, const int32_t *freqs,
                                        int64_t n_syms, uint8_t *out, int64_t n_streams,
                                        int64_t n_fp8_per_stream, int32_t *status, void *stream) {
    tans_b200::clear_error();
    if (n_syms <= 0 || n_syms > 256)
        return fail(TANS_B200_ERR_INVALID,
                    "decode_noalloc: alphabet must be 1..256 symbols (got %lld)",
                    (long long)n_syms);
    if (n_fp8_per_stream < 0 || n_fp8_per_stream % 2 != 0)
        return fail(TANS_B200_ERR_INVALID, "n_fp8_per_stream must be even");
    if (compressed_bytes < 0 || compressed_bytes % 4 != 0)
        return fail(TANS_B200_ERR_INVALID, "compressed length must be divisible by 4 bytes");
    if (n_streams < 0) return fail(TANS_B200_ERR_INVALID, "n_streams must be >= 0");
    if (n_streams == 0 || n_fp8_per_stream == 0) return TANS_B200_OK;
    if (!compressed || !offsets || !states || !partial || !sign_mantissa || !spread || !freqs ||
        !out)
        return fail(TANS_B200_ERR_INVALID, "decode_noalloc: null pointer");
    if (!aligned(compressed, 4) || !aligned(offsets, 4) || !aligned(states, 2) ||
        !aligned(spread, 4) || !aligned(freqs, 4))
        return fail(TANS_B200_ERR_INVALID, "decode_noalloc: misaligned input");
    int sms;
    int rc = device_setup(&sms);
    if (rc) return rc;
    int32_t *table = nullptr;
    rc = noalloc_table(&table);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    build_table_kernel<<<1, kBuildWarps * 32, 0, st>>>(spread, freqs, (int)n_syms, table, status);
    rc = launch_status("build_table_kernel");
    if (rc) return rc;
    DecodeArgs args{reinterpret_cast<const uint32_t *>(compressed), compressed_bytes, offsets,
                    states, partial, sign_mantissa, table, out, n_streams,
                    n_fp8_per_stream, n_streams, n_fp8_per_stream / 2, status, make_opq(),
                    (int32_t)(n_streams % 4 == 0 && aligned(sign_mantissa, 4) && aligned(out, 4))};
    switch (ring_rows(n_fp8_per_stream / 2)) {
        case 16: return launch_decode<16>(args, n_streams, sms, st);
        case 32: return launch_decode<32>(args, n_streams, sms, st);
        case 64: return launch_decode<64>(args, n_streams, sms, st);
        default: return launch_decode<128>(args, n_streams, sms, st);
    }
}
