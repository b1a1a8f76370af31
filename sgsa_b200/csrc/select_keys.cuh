// Order-preserving keys and the indexer's first-pass digit.  Plain C++ apart from
// the __host__ __device__ qualifiers, so that a host program can check the
// invariants the exact selection relies on (tests/select_keys_check.cpp).
#pragma once

#include <stdint.h>
#ifndef __CUDACC__
#include <string.h>
#endif

#ifdef __CUDACC__
#define SGSA_HD __host__ __device__ __forceinline__
#else
#define SGSA_HD inline
#endif

namespace sgsa {

SGSA_HD uint32_t float_bits(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, sizeof(u));
    return u;
#endif
}

// Orderable 32-bit key of a float: a > b  <=>  key(a) > key(b) (no NaNs);
// -0.0 and +0.0 compare equal, as they do as floats.
SGSA_HD uint32_t float_key(float f) {
    uint32_t u = float_bits(f);
    if ((u << 1) == 0u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Key of a score for a row whose k-th score is a positive float: the raw bits
// with the sign flipped order every positive score correctly and put every
// negative one (and -0.0) below any positive prefix, which is all the
// comparisons against such a prefix need.
SGSA_HD uint32_t fast_key(float f) { return float_bits(f) ^ 0x80000000u; }

SGSA_HD int imin_(int a, int b) { return a < b ? a : b; }
SGSA_HD int imax_(int a, int b) { return a > b ? a : b; }

// First-pass (fast) digit, placed per CTA and row from a sample of the first key
// tile (the window's top is 4-8x the sample's largest |score|: exponent field etop):
//   mode 0 (rows whose sample says the k-th score is positive): 1/32-octave bins of
//          the positive scores in the 8 octaves below the top: bin = code(v) - pb with
//          code = raw bits >> 18 (14 bits: sign, exponent, 5 mantissa bits) and
//          pb = (etop - 8) << 5 the code of the window's bottom;
//   mode 1 (k-th negative): the same bins of -v, in reverse order;
//   mode 2 (sign unclear): 1/8-octave bins over 16 octaves of each sign (pb =
//          (etop - 16) << 3): negative scores in bins 0..127, positive ones in
//          128..255, the small |v| of both signs meet in 127.
// The kernel picks the mode per warp (fast_digit_m<MODE>), so a warp never mixes
// the formulas.  Bins 0 and 255 (and 127 in mode 2) are the clamp bins: a k-th score
// there makes the row retry in mode 2 (mode 0/1, towards zero) or fall back to plain
// radix.  etop >= 17 keeps zero and the denormals below every window.
constexpr int kDefaultEtop = 127 + 8;  // top 2^8 without a sample

SGSA_HD int fast_base(int mode, int etop) { return mode == 2 ? (etop - 16) << 3 : (etop - 8) << 5; }
SGSA_HD uint32_t fast_mask(int mode) { return mode == 2 ? 0xfff00000u : 0xfffc0000u; }
SGSA_HD int fast_top(int mode) { return mode == 2 ? 20 : 18; }

template <int MODE>
SGSA_HD uint32_t fast_digit_m(float f, int pb) {
    const uint32_t u = float_bits(f);
    if (MODE == 0) return (uint32_t)imin_(imax_((int)u >> 18, pb) - pb, 255);  // (int)u < 0: bin 0
    if (MODE == 1) return (uint32_t)imin_(imax_((int)(u ^ 0x80000000u) >> 18, pb) - pb, 255) ^ 255u;
    const int sg = (int)u >> 31;                               // 0 or -1
    const int c = (int)((u & 0x7fffffffu) >> 20) - pb;         // 1/8-octave code above bottom
    return (uint32_t)(128 + imin_(imax_(c, -1 - sg), 127)) ^ (uint32_t)(sg & 255);
}

SGSA_HD uint32_t fast_digit(float f, int mode, int pb) {
    return mode == 0 ? fast_digit_m<0>(f, pb) : mode == 1 ? fast_digit_m<1>(f, pb) : fast_digit_m<2>(f, pb);
}

// Key prefix (under fast_mask(mode)) of fast bin d, which is interior.
SGSA_HD uint32_t fast_prefix(int d, int mode, int pb) {
    if (mode == 0) return (uint32_t)(0x2000 + pb + d) << 18;
    if (mode == 1) return (uint32_t)(0x1f00 - pb + d) << 18;
    return d >= 128 ? (uint32_t)(0x800 + pb + d - 128) << 20 : (uint32_t)(0x7ff - pb - 127 + d) << 20;
}

}  // namespace sgsa
