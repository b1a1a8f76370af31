// Host check of the invariants the indexer's exact selection relies on
// (sgsa_b200/csrc/select_keys.cuh), over random windows and score ranges:
//   * lin_bin is monotone non-decreasing in the score (-0.0 == +0.0) and in 0..kLinTop;
//   * min_key_where(bin >= c) is the exact lower edge of bin c: its float is in a
//     bin >= c and the float of the key below it in a bin < c; min_key_near finds
//     the same key from the analytic guess or from any key;
//   * the same for the two-level (window bin, refine bin) order of the refine pass;
//   * key_float inverts float_key, and key_range_prefix gives bits all keys of the
//     range share.
// Prints "ok <checks>" and exits 0, or the first failures and exits 1.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "select_keys.cuh"

using namespace sgsa;

static long bad = 0, n = 0;
#define CHECK(cond, ...)                               \
    do {                                               \
        ++n;                                           \
        if (!(cond) && ++bad < 8) printf(__VA_ARGS__); \
    } while (0)

int main() {
    std::mt19937 g(1);
    std::uniform_real_distribution<float> U(-1.f, 1.f);
    for (int trial = 0; trial < 3000; ++trial) {
        // a window of random scale and placement, as the kernel builds it
        const float scale = std::ldexp(1.0f, (int)(g() % 60) - 30);
        const float W = scale * (0.5f + (g() % 1000) / 500.f);
        const int side = g() % 3;
        const float lo = side == 0 ? 0.f : side == 1 ? -W : -0.5f * W;
        const float a = 1.0f / W, b = -lo * a;
        std::vector<float> vals = {0.f, -0.f, lo, lo + W, INFINITY, -INFINITY};
        for (int i = 0; i < 400; ++i) vals.push_back(std::ldexp(U(g), (int)(g() % 8)) * W + lo);
        std::sort(vals.begin(), vals.end());
        uint32_t prev = 0;
        for (size_t i = 0; i < vals.size(); ++i) {
            const uint32_t d = lin_bin(vals[i], a, b);
            CHECK(d <= (uint32_t)kLinTop, "bin out of range %u\n", d);
            CHECK(i == 0 || d >= prev || vals[i] == vals[i - 1], "not monotone at %g\n", vals[i]);
            prev = d;
            CHECK(key_float(float_key(vals[i])) == vals[i], "key_float(float_key(%g))\n", vals[i]);
        }
        CHECK(lin_bin(-INFINITY, a, b) == 0u && lin_bin(INFINITY, a, b) == (uint32_t)kLinTop, "clamp bins\n");
        for (int r = 0; r < 4; ++r) {
            const int c = 1 + (int)(g() % (kLinTop - 1));
            const uint32_t k = min_key_where([&](float x) { return (int)lin_bin(x, a, b) >= c; });
            CHECK((int)lin_bin(key_float(k), a, b) >= c, "edge %d not in bin >= c\n", c);
            CHECK((int)lin_bin(key_float(k - 1u), a, b) < c, "key below edge %d in bin >= c\n", c);
            const uint32_t kn = min_key_near([&](float x) { return (int)lin_bin(x, a, b) >= c; },
                                             lin_edge_guess(c, a, b));
            CHECK(kn == k, "min_key_near from the guess: %u vs %u\n", kn, k);
            const uint32_t kr = min_key_near([&](float x) { return (int)lin_bin(x, a, b) >= c; },
                                             (uint32_t)g());
            CHECK(kr == k, "min_key_near from a random key: %u vs %u\n", kr, k);
            const uint32_t k2 = min_key_where([&](float x) { return (int)lin_bin(x, a, b) >= c + 1; });
            CHECK(k2 >= k, "edges out of order\n");
            // every key in [k, k2) is in bin c
            for (int j = 0; j < 16 && k2 > k; ++j) {
                const uint32_t kk = k + (uint32_t)(((uint64_t)g() * (k2 - k)) >> 32);
                CHECK((int)lin_bin(key_float(kk), a, b) == c, "key inside bin %d elsewhere\n", c);
            }
            if (k2 <= k) continue;
            uint32_t pre;
            int top;
            key_range_prefix(k, k2 - 1u, pre, top);
            const uint32_t m = top >= 32 ? 0u : ~((1u << top) - 1u);
            CHECK((k & m) == pre && ((k2 - 1u) & m) == pre, "range prefix\n");
            if (k2 - k < 2u) continue;
            // the refine window over bin c, and its lexicographic order
            const float xlo = key_float(k), xhi = key_float(k2);
            const float a1 = 1.0f / (xhi - xlo), b1 = -xlo * a1;
            const int c1 = (int)(g() % (kLinTop + 1));
            auto at_least = [&](float x) {
                const int d0 = (int)lin_bin(x, a, b);
                return d0 > c || (d0 == c && (int)lin_bin(x, a1, b1) >= c1);
            };
            const uint32_t e = min_key_where(at_least);
            CHECK(min_key_near(at_least, lin_edge_guess(c1, a1, b1)) == e, "refine edge near guess\n");
            CHECK(at_least(key_float(e)) && !at_least(key_float(e - 1u)), "refine edge\n");
            CHECK(e >= k && e <= k2, "refine edge outside bin\n");
            uint32_t pv = 0;
            for (uint32_t kk = k; kk < k2; kk += std::max(1u, (k2 - k) / 64u)) {
                const uint32_t d1 = lin_bin(key_float(kk), a1, b1);
                CHECK(d1 >= pv, "refine bins not monotone\n");
                pv = d1;
            }
        }
    }
    if (bad) {
        printf("%ld failures in %ld checks\n", bad, n);
        return 1;
    }
    printf("ok %ld\n", n);
    return 0;
}
