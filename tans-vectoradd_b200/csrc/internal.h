// internal.h — declarations shared by the translation units of libtans_b200
// (not part of the C ABI).
#pragma once

#include <stdint.h>

#include "../../include/tans_b200.h"

namespace tans_b200 {

// log2 L: the largest number of bits one step reads or writes, and
// log2(2L) = kTableLog + 1 bounds every state.
constexpr int kTableLog = TANS_B200_TABLE_SIZE == 4096 ? 12 : (TANS_B200_TABLE_SIZE == 2048 ? 11 : -1);
static_assert(kTableLog > 0, "TANS_B200_TABLE_SIZE must be 4096 or 2048");

// Record a formatted message for tans_b200_last_error() and return `code`.
int fail(int code, const char *fmt, ...);
void clear_error();

// Per-alphabet tables of the slab encoder in the form the device encoder
// uses (shown for L = 4096, log2 L = 12).  For a symbol s with frequency
// f = freqs[s] > 0, k1 = 12 - floor(log2 f):
//   delta[s] = (k1 << 13) - (f << k1)  so that (x + delta) >> 13 is the
//            number of bits x emits before s (k1 - 1 below f << k1, else k1;
//            the threshold rule of csrc/tans_codec.cpp:38-47 in one add and
//            one shift: x and f << k1 both lie in [4096, 8192));
//   base[s]  = cum[s] - f              so that next[base + (x >> k)] is the
//            successor state (x >> k lies in [f, 2f));
//   next[cum[s] + r] = 4096 + (slot of the r-th occurrence of s in spread).
// A symbol outside the alphabet or with f = 0 gets delta = 13 << 13 and base
// 0: the encoder then reads 13 bits (more than any codable symbol, which is
// how it notices) and next[0], which stays in bounds.
struct EncoderTables {
    int32_t delta[256];
    int32_t base[256];
    uint16_t next[TANS_B200_TABLE_SIZE];
};

constexpr int kEncoderBadBits = 13;  // above log2 L for both table sizes

// Validate (freqs sum to L, spread consistent with freqs) and fill `t`.
// Same checks and messages as the CPU encoder; returns a status code.
int encoder_tables(const int32_t *freqs, int64_t n_syms, const int32_t *spread,
                   EncoderTables *t);

}  // namespace tans_b200
