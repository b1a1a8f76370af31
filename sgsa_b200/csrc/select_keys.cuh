// Order-preserving keys and the indexer's linear-window bins.  Plain C++ apart
// from the __host__ __device__ qualifiers, so that a host program can check the
// invariants the exact selection relies on (tests/select_keys_check.cpp).
#pragma once

#include <stdint.h>
#ifndef __CUDACC__
#include <string.h>

#include <cmath>
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

// ---- Linear window bins (the tensor-core indexer's first pass) ---------------
//
// A row's window is [lo, lo + W), given as a = 1/W, b = -lo/W.  The bin of a score is
//   lin_bin(v) = round(kLinTop * sat(v * a + b))  in 0 .. kLinTop = 127,
// computed with two fused multiply-adds (the second adds 2^23, so the rounded
// integer is the low byte of the result's bits).  Every step is monotone
// non-decreasing in v (correctly rounded fma, saturation to [0, 1]), so the bin is a
// monotone function of the score: a bin is an interval of scores, and "bin >= c" is
// "key(v) >= min_key_where(bin >= c)".  Bins 0 and kLinTop also hold the scores below
// and above the window.  NaN scores land in bin 0.
constexpr int kLinTop = 127;
SGSA_HD float sat01(float x) {
#ifdef __CUDA_ARCH__
    return __saturatef(x);
#else
    return x > 0.f ? (x < 1.f ? x : 1.f) : 0.f;  // NaN -> 0, as the device saturation
#endif
}

SGSA_HD float fma_rn(float a, float b, float c) {
#ifdef __CUDA_ARCH__
    return __fmaf_rn(a, b, c);
#else
    return std::fma(a, b, c);
#endif
}

SGSA_HD uint32_t lin_bin(float v, float a, float b) {
    const float y = sat01(fma_rn(v, a, b));
    return float_bits(fma_rn(y, (float)kLinTop, 8388608.f)) - 0x4B000000u;
}

// The float whose order-preserving key is k (the inverse of float_key, -0.0 as +0.0).
SGSA_HD float key_float(uint32_t k) {
    const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, sizeof(f));
    return f;
#endif
}

constexpr uint32_t kKeyNegInf = 0x007fffffu;  // float_key(-inf)
constexpr uint32_t kKeyPosInf = 0xff800000u;  // float_key(+inf)

// Smallest key k in (key(-inf), key(+inf)] with pred(key_float(k)) true, for a
// predicate that is monotone in the key, false at -inf and true at +inf (the keys
// between hold no NaN).  32 bisection steps.
template <typename Pred>
SGSA_HD uint32_t min_key_where(Pred pred) {
    uint32_t lo = kKeyNegInf, hi = kKeyPosInf;  // pred(lo) false, pred(hi) true
    while (hi - lo > 1u) {
        const uint32_t mid = lo + ((hi - lo) >> 1);
        if (pred(key_float(mid))) hi = mid;
        else lo = mid;
    }
    return hi;
}

// min_key_where(pred), searched from a guess key0: gallop away from key0 until the
// edge is bracketed, then bisect.  A good guess (a few ulps off) takes a few steps.
template <typename Pred>
SGSA_HD uint32_t min_key_near(Pred pred, uint32_t key0) {
    key0 = key0 <= kKeyNegInf ? kKeyNegInf + 1u : key0 > kKeyPosInf ? kKeyPosInf : key0;
    uint32_t lo, hi;  // pred(lo) false, pred(hi) true
    uint32_t step = 1u;
    if (pred(key_float(key0))) {
        hi = key0;
        for (;;) {
            const uint32_t c = hi - kKeyNegInf > step ? hi - step : kKeyNegInf;
            if (c == kKeyNegInf || !pred(key_float(c))) { lo = c; break; }
            hi = c;
            step <<= 1;
        }
    } else {
        lo = key0;
        for (;;) {
            const uint32_t c = kKeyPosInf - lo > step ? lo + step : kKeyPosInf;
            if (c == kKeyPosInf || pred(key_float(c))) { hi = c; break; }
            lo = c;
            step <<= 1;
        }
    }
    while (hi - lo > 1u) {
        const uint32_t mid = lo + ((hi - lo) >> 1);
        if (pred(key_float(mid))) hi = mid;
        else lo = mid;
    }
    return hi;
}

// Guess of the lower edge of bin c of the window (a, b): the score where
// c_real * (v a + b) crosses c - 1/2.
SGSA_HD uint32_t lin_edge_guess(int c, float a, float b) {
    return float_key(((c - 0.5f) / (float)kLinTop - b) / a);
}

// (prefix, top) of the keys in [lo, hi]: they all agree on the bits above `top`.
SGSA_HD void key_range_prefix(uint32_t lo, uint32_t hi, uint32_t &prefix, int &top) {
    const uint32_t d = lo ^ hi;
    int t = 0;
    while (t < 32 && (d >> t)) ++t;
    top = t;
    prefix = t >= 32 ? 0u : (lo & ~((1u << t) - 1u));
}

}  // namespace sgsa
