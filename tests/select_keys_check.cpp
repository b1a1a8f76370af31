// Host check of the invariants the indexer's exact selection relies on
// (sgsa_b200/csrc/select_keys.cuh), over every window position and mode:
//   * fast_digit is monotone in the score (ties: -0.0 == +0.0);
//   * an interior bin d holds exactly the scores whose order-preserving key has
//     the prefix fast_prefix(d) under the bin's mask (both directions).
// Prints "ok <checks>" and exits 0, or the first failures and exits 1.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "select_keys.cuh"

using namespace sgsa;

int main() {
    std::mt19937 g(1);
    long bad = 0, n = 0;
    for (int etop = 17; etop <= 255; ++etop)
        for (int mode = 0; mode < 3; ++mode) {
            const int pb = fast_base(mode, etop);
            const uint32_t mask = fast_mask(mode);
            auto clamp_bin = [&](uint32_t d) { return d == 0 || d == 255 || (mode == 2 && d == 127); };
            std::vector<float> vals = {0.f, -0.f};
            for (int i = 0; i < 4000; ++i) {
                const float sc = std::ldexp(1.0f, (int)(g() % 48) - 24 + (etop - 127 - 8));
                const float v = sc * (float)(g() % 100000) / 100000.f * ((g() & 1) ? 1.f : -1.f);
                if (std::isfinite(v)) vals.push_back(v);
            }
            std::sort(vals.begin(), vals.end());
            uint32_t prev = 0;
            for (size_t i = 0; i < vals.size(); ++i) {
                const uint32_t d = fast_digit(vals[i], mode, pb);
                ++n;
                if (i && d < prev && !(vals[i] == vals[i - 1])) {
                    if (++bad < 5) printf("not monotone: mode %d etop %d v %g\n", mode, etop, vals[i]);
                }
                prev = d;
                if (!clamp_bin(d) && (float_key(vals[i]) & mask) != fast_prefix((int)d, mode, pb)) {
                    if (++bad < 5) printf("prefix: mode %d etop %d v %g bin %u\n", mode, etop, vals[i], d);
                }
            }
            for (int i = 0; i < 2000; ++i) {  // every key with an interior bin's prefix lands there
                const int d = (int)(g() % 256);
                if (clamp_bin((uint32_t)d)) continue;
                const uint32_t key = fast_prefix(d, mode, pb) | (g() & ~mask);
                const uint32_t u = (key & 0x80000000u) ? (key & 0x7fffffffu) : ~key;
                float v;
                memcpy(&v, &u, sizeof(v));
                if (!std::isfinite(v)) continue;
                ++n;
                if (fast_digit(v, mode, pb) != (uint32_t)d) {
                    if (++bad < 5) printf("reverse: mode %d etop %d bin %d v %g\n", mode, etop, d, v);
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
