// Causal top-k indexer and row top-k select.
//
// Selection rule (the contract of modelings/modeling_sgsa.py:144-165 and
// modelings/hybrid_dense_delta_topk.py:344-349, with a stated tie-break):
// row t keeps the min(K, t+1) largest scores among columns j <= t, equal
// scores ordered by the lower j first.  Output indices are ascending, the
// remaining slots are -1.
//
// Algorithm: an MSB-first radix select over the 32-bit order-preserving key of
// the fp32 score (the CUDA-core path: one thread per query row, up to four 8-bit
// digit passes; the tensor-core path below: a sampled first digit and a candidate
// pass); each pass counts, in a per-row 256-bin histogram held in shared memory as
// hist[bin][row] (bank = row, so conflict free), the scores whose higher digits
// match the prefix chosen so far.  A row is
// resolved as soon as the chosen bin holds exactly the number of elements
// still needed.  A final pass emits, in index order, every column whose masked
// key is above the prefix plus the first `need` columns equal to it -- which
// is exactly the lowest-index tie-break.  Scores are recomputed in every pass
// (bit-identical, same code and order), so nothing of size T^2 is stored.
#include <stdlib.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace sgsa {

// SGSA_INDEXER_SIMT=1 forces the CUDA-core score path for bf16 (A/B checks).
static bool indexer_use_tc() {
    const char *e = getenv("SGSA_INDEXER_SIMT");
    return !(e && e[0] == '1');
}

namespace {

static __device__ unsigned int g_check;  // bounds-checked build only

constexpr int kRows = 128;       // query rows per CTA (one per thread)
constexpr int kKeyTile = 64;     // keys per shared-memory tile

struct SelState {
    uint32_t prefix, mask;
    int need;
    bool done;
};

// Per-row bookkeeping after a histogram pass; returns true once resolved.
__device__ __forceinline__ void sel_choose(SelState &s, const uint32_t *hist, int col,
                                           int shift) {
    int cum = 0, chosen = 0, cnt = 0;
    for (int bin = 255; bin >= 0; --bin) {
        cnt = (int)hist[bin * kRows + col];
        if (cum + cnt >= s.need) { chosen = bin; break; }
        cum += cnt;
    }
    s.need -= cum;
    s.prefix |= (uint32_t)chosen << shift;
    s.mask |= 0xffu << shift;
    if (cnt == s.need || shift == 0) s.done = true;
}

// Generic select driver.  ScoreFn(tileStart, rowScores[kKeyTile]) computes the
// scores of this thread's row for keys [tileStart, tileStart + kKeyTile); it
// may use __syncthreads and must be called by all threads of the CTA.
template <typename TileFn>
__device__ void select_rows(TileFn &&tiles, int nvalid, int K, int32_t *out_row,
                            uint32_t *hist, int max_valid_cta) {
    const int tid = threadIdx.x;
    SelState s{0u, 0u, K, false};
    if (nvalid <= K) {  // every valid column is selected
        if (out_row) {
            for (int i = 0; i < K; ++i) out_row[i] = (i < nvalid) ? i : -1;
        }
        s.done = true;
    }
    float sc[kKeyTile];
    for (int shift = 24; shift >= 0; shift -= 8) {
        if (!__syncthreads_or(!s.done)) break;
        for (int b = 0; b < 256; ++b) hist[b * kRows + tid] = 0u;
        const bool active = !s.done;
        for (int j0 = 0; j0 < max_valid_cta; j0 += kKeyTile) {
            tiles(j0, sc);
            if (active && j0 < nvalid) {
#pragma unroll
                for (int jj = 0; jj < kKeyTile; ++jj) {
                    if (j0 + jj < nvalid) {
                        const uint32_t u = float_key(sc[jj]);
                        if ((u & s.mask) == s.prefix) ++hist[((u >> shift) & 0xffu) * kRows + tid];
                    }
                }
            }
        }
        if (active) sel_choose(s, hist, tid, shift);
    }
    // collect pass
    const bool collect = (out_row != nullptr) && nvalid > K;
    if (!__syncthreads_or(collect)) return;
    int pos = 0, taken = 0;
    for (int j0 = 0; j0 < max_valid_cta; j0 += kKeyTile) {
        tiles(j0, sc);
        if (collect && j0 < nvalid) {
#pragma unroll
            for (int jj = 0; jj < kKeyTile; ++jj) {
                const int j = j0 + jj;
                if (j < nvalid) {
                    const uint32_t m = float_key(sc[jj]) & s.mask;
                    if (m > s.prefix || (m == s.prefix && taken < s.need)) {
                        if (m == s.prefix) ++taken;
                        if (pos < K) out_row[pos] = j;
                        ++pos;
                    }
                }
            }
        }
    }
    if (collect)
        for (int i = pos; i < K; ++i) out_row[i] = -1;
}

// ---- CUDA-core indexer: scores in fp32 FFMA from shared-memory tiles. ------
template <typename Tin, int DI>
__global__ void __launch_bounds__(kRows) indexer_topk_simt_kernel(const Tin *__restrict__ iq,
                                                                  const Tin *__restrict__ ik,
                                                                  int32_t *__restrict__ idx,
                                                                  int B, int T, int H, int K,
                                                                  int n_qtiles) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint32_t *hist = (uint32_t *)smem_raw;                            // 256 x kRows
    float *sq = (float *)(hist + 256 * kRows);                        // kRows x (DI+1)
    float *sk = sq + kRows * (DI + 1);                                // kKeyTile x DI
    const int tid = threadIdx.x;
    const int qt = n_qtiles - 1 - (int)blockIdx.x;  // heaviest tiles first
    const int bh = blockIdx.y, b = bh / H, h = bh % H;
    const int q0 = qt * kRows;
    const int t = q0 + tid;
    const int q_end = min(T, q0 + kRows);
    for (int e = tid; e < kRows * DI; e += kRows) {
        const int r = e / DI, d = e % DI;
        sq[r * (DI + 1) + d] = (q0 + r < T) ? to_f32(iq[(((size_t)b * T + q0 + r) * H + h) * DI + d]) : 0.f;
    }
    __syncthreads();
    auto tiles = [&](int j0, float *sc) {
        __syncthreads();
        for (int e = tid; e < kKeyTile * DI; e += kRows) {
            const int r = e / DI, d = e % DI;
            const int j = j0 + r;
            sk[e] = (j < T) ? to_f32(ik[(((size_t)b * T + j) * H + h) * DI + d]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int jj = 0; jj < kKeyTile; ++jj) sc[jj] = 0.f;
        const float *myq = sq + tid * (DI + 1);
        for (int d = 0; d < DI; ++d) {
            const float x = myq[d];
#pragma unroll
            for (int jj = 0; jj < kKeyTile; ++jj) sc[jj] = fmaf(x, sk[jj * DI + d], sc[jj]);
        }
    };
    const int nvalid = (t < T) ? t + 1 : 0;
    int32_t *out_row = (t < T) ? idx + (((size_t)bh) * T + t) * K : nullptr;
    select_rows(tiles, nvalid, K, out_row, hist, q_end);
}

// ---- select over a given score matrix (exact-parity helper). --------------
__global__ void __launch_bounds__(kRows) topk_select_kernel(const float *__restrict__ scores,
                                                            const int32_t *__restrict__ valid,
                                                            int32_t *__restrict__ idx, int R,
                                                            int S, int K) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint32_t *hist = (uint32_t *)smem_raw;
    const int tid = threadIdx.x;
    const int r = blockIdx.x * kRows + tid;
    const int nvalid = (r < R) ? min(max(valid[r], 0), S) : 0;
    int maxv = nvalid;
    // block-wide max of nvalid
    __shared__ int smax;
    if (tid == 0) smax = 0;
    __syncthreads();
    atomicMax(&smax, maxv);
    __syncthreads();
    maxv = smax;
    const float *row = scores + (size_t)(r < R ? r : 0) * S;
    auto tiles = [&](int j0, float *sc) {
#pragma unroll
        for (int jj = 0; jj < kKeyTile; ++jj) {
            const int j = j0 + jj;
            sc[jj] = (j < nvalid) ? row[j] : 0.f;
        }
    };
    select_rows(tiles, nvalid, K, (r < R) ? idx + (size_t)r * K : nullptr, hist, maxv);
}


// ---- tcgen05 indexer: bf16 scores on the tensor cores, fp32 in TMEM. --------
//
// Warp roles of the 320-thread CTA (one CTA per 128-query tile of one (b, h)):
//   warp 0  TMA producer: key tiles into a ring of shared-memory stages;
//   warp 1  TMEM owner and MMA issuer: S_tile = Q K^T, M=128 (queries) x
//           N=kN (keys) x K=DI with the query tile Q in tensor memory (written
//           once by the epilogue threads), into the TMEM accumulator;
//   warps 2-9  two threads per query row (warps w and w+4 read the same TMEM
//           lane quarter and take alternate 32-column chunks of the tile):
//           tcgen05.ld of their part of the row and the selection work of the
//           pass; the first thread of each row also runs the collect pass, which
//           must walk the row in order.
// The key stream is replayed once per pass; the tensor cores recompute the
// identical fp32 scores each time.
//
// Passes of a row (each row decides its own; a pass serves every kind at once):
//   window   a 128-bin histogram of lin_bin(v) over a linear window placed from a
//            sample (the row's scores against the first key tile: the window is
//            2 max|s| wide, starting at 0, -W/2 or -W by the sample's sign
//            balance).  The bin function is two fused multiply-adds and the
//            counter address one integer multiply-add, all on the FMA pipe, then
//            one shared-memory reduction.  The bin holding the need-th largest
//            score is interior (else: plain radix restart) and its edges are
//            exact keys found by bisection (lin_bin is monotone);
//   refine   if that bin holds more than kCap keys: the same histogram over the
//            bin's own interval, counting only its members;
//   candidate  the members of the chosen bin (at most kCap) are stored (raw float
//            bits) in the row's histogram column, from both ends by the row's two
//            threads, and the k-th is found among them (cand_resolve); a chunk of
//            32 scores is tested for members with FMA-pipe arithmetic only;
//   plain    fallback radix select over the order-preserving key, 7-bit digits,
//            with the same candidate step once a digit bin holds <= kCap keys.
// A row whose chosen bin holds exactly the keys still needed is done at once: its
// selection is "key >= the bin's lower edge".  Every path is exact; ties at the
// k-th score go to the lowest index (collect pass).  The histogram is hist[bin][row]
// in 32-bit counters (64 KB), so two CTAs share an SM.
static __device__ unsigned int g_index_watchdog;
// Test support: rows that took the refine pass, the plain restart, a plain
// candidate pass, a tie cut (counted by the first thread of a row).
static __device__ unsigned long long g_index_stats[4];

constexpr int kEpiThreads = 256;
constexpr int kBins = kLinTop + 1;  // histogram bins per row (32-bit counters)
constexpr int kDigit = 7;           // bits per digit of the plain radix fallback
constexpr int kCap = kBins;         // candidate slots of a row: its whole histogram column
constexpr int kLongRow = 16384;     // rows this long get the narrower first window
constexpr int kSampleFrom = 8192;   // query tiles from here on start with a sampled pass
constexpr int kSampleStride = 8;    // ... over every 8th key tile
constexpr int kSmallGridWaves = 4;  // grids of at most this many CTAs per SM: one CTA per SM
constexpr int kMaxPasses = 8;

struct RowSel {
    uint32_t prefix, mask;  // the k-th key agrees with prefix on the bits of mask
    int need;               // keys still to take at or below the prefix
    int top;                // bits [top-1 : 0] of the k-th key are still unknown
    bool done;
    bool plain;             // radix fallback on the order-preserving keys
    bool exact;             // resolved with every key at the prefix selected (no tie cut)
    bool cand;              // the next pass gathers candidates
    int lvl;                // linear mode: 0 window pass next/done, 1 refine pass next/done
    int cnt;                // keys in the bin chosen by the last histogram pass
    float a0, b0, a1, b1;   // the two linear windows
    int c0, c1;             // their chosen bins
};

__device__ __forceinline__ uint32_t hist_count(const uint32_t *hist, int bin, int col) {
    return hist[bin * kRows + col];
}

// Radix step of the plain fallback: choose the next 8-bit digit among keys matching
// the prefix.
__device__ __forceinline__ void row_choose_plain(RowSel &s, const uint32_t *hist, int col) {
    const int w = min(kDigit, s.top);
    int cum = 0, chosen = 0, cnt = 0;
    for (int bin = (1 << w) - 1; bin >= 0; --bin) {
        cnt = (int)hist_count(hist, bin, col);
        if (cum + cnt >= s.need) { chosen = bin; break; }
        cum += cnt;
    }
    const int shift = s.top - w;
    s.need -= cum;
    s.prefix |= (uint32_t)chosen << shift;
    s.mask |= ((1u << w) - 1u) << shift;
    s.top = shift;
    s.cnt = cnt;
    if (cnt == s.need) s.exact = true;
    if (cnt == s.need || s.top == 0) s.done = true;
}

__device__ __forceinline__ void epi_bar() {
    asm volatile("bar.sync 1, %0;" ::"r"(kEpiThreads) : "memory");
}

__device__ __forceinline__ void st_shared_if(uint32_t addr, uint32_t v, bool pred) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t@p st.shared.u32 [%0], %1;\n\t}" ::"r"(addr),
                 "r"(v), "r"((uint32_t)pred)
                 : "memory");
}

// Shared-memory counter increments.  No memory clobber: the counters are read only
// after the epilogue barrier (epi_bar, which has one), and volatile asm keeps its order.
__device__ __forceinline__ void red_shared(uint32_t addr) {
    asm volatile("red.shared.add.u32 [%0], 1;" ::"r"(addr));
}

__device__ __forceinline__ void red_shared_if(uint32_t addr, bool pred) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %1, 0;\n\t@p red.shared.add.u32 [%0], 1;\n\t}" ::"r"(
                     addr),
                 "r"((uint32_t)pred));
}

// Bits of the bin computation: 0x4B000000 + lin_bin(v).  0x4B000000 * 512 is 0 mod
// 2^32, so bits * 512 + (address of hist[0][row]) is the address of hist[bin][row].
__device__ __forceinline__ uint32_t lin_bits(float v, float a, float b) {
    return __float_as_uint(__fmaf_rn(__saturatef(__fmaf_rn(v, a, b)), (float)kLinTop, 8388608.f));
}

// Window-pass histogram of one 32-column chunk.
template <bool FULL>
__device__ __forceinline__ void lin_hist0(const float (&v)[32], uint32_t cbase, int jb, int nvalid,
                                          float a, float b) {
    uint32_t addr[32];  // all 32 addresses first: independent chains, then the reductions
#pragma unroll
    for (int i = 0; i < 32; ++i) addr[i] = lin_bits(v[i], a, b) * 512u + cbase;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        if (FULL) red_shared(addr[i]);
        else red_shared_if(addr[i], jb + i < nvalid);
    }
}

// Refine-pass histogram: members of window bin c0 only, binned in window 1.
template <bool FULL>
__device__ __forceinline__ void lin_hist1(const float (&v)[32], uint32_t cbase, int jb, int nvalid,
                                          const RowSel &s) {
    const uint32_t want = 0x4B000000u + (uint32_t)s.c0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const bool in = (FULL || jb + i < nvalid) && lin_bits(v[i], s.a0, s.b0) == want;
        red_shared_if(lin_bits(v[i], s.a1, s.b1) * 512u + cbase, in);
    }
}

// Candidate gathering of one 32-column chunk (linear mode): a member of the chosen
// bin(s) is stored (raw float bits) at this thread's slot, which then advances by
// `step` bytes -- a compare, a predicated store and a predicated add per score, no
// branches.  The two threads of a row fill the row's column from its two ends; the
// histogram bounds their total by the chosen bin's count (<= kCap), and the
// membership test is the same bit-identical computation.
template <bool FULL, bool LVL1>
__device__ __forceinline__ void lin_cand(const float (&v)[32], uint32_t &slot, int step, int jb,
                                         int nvalid, const RowSel &s) {
    const uint32_t w0 = 0x4B000000u + (uint32_t)s.c0, w1 = 0x4B000000u + (uint32_t)s.c1;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const uint32_t b0 = lin_bits(v[i], s.a0, s.b0);
        if (FULL && !LVL1) {
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.eq.u32 p, %2, %3;\n\t@p st.shared.u32 [%0], %1;\n\t"
                "@p add.u32 %0, %0, %4;\n\t}"
                : "+r"(slot)
                : "r"(__float_as_uint(v[i])), "r"(b0), "r"(w0), "r"(step));
        } else {
            bool in = b0 == w0 && (FULL || jb + i < nvalid);
            if (LVL1) in = in && lin_bits(v[i], s.a1, s.b1) == w1;
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t@p st.shared.u32 [%0], %1;\n\t"
                "@p add.u32 %0, %0, %3;\n\t}"
                : "+r"(slot)
                : "r"(__float_as_uint(v[i])), "r"((uint32_t)in), "r"(step));
        }
    }
}

// Plain fallback: histogram of the next 8-bit digit among keys matching the prefix.
template <bool FULL>
__device__ __forceinline__ void plain_hist(const float (&v)[32], uint32_t *hcol, int jb, int nvalid,
                                           const RowSel &s) {
    const int w = min(kDigit, s.top);
    const int shift = s.top - w;
    const uint32_t mul = shift ? (1u << (32 - shift)) : 0u;  // u >> shift as a high multiply
    const uint32_t dmask = (1u << w) - 1u;
    const uint32_t cbase = (uint32_t)__cvta_generic_to_shared(hcol);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const uint32_t u = float_key(v[i]);
        const uint32_t d = (shift ? __umulhi(u, mul) : u) & dmask;
        red_shared_if(cbase + d * (kRows * 4), (FULL || jb + i < nvalid) && (u & s.mask) == s.prefix);
    }
}

// Plain fallback: candidates are the scores whose key matches the prefix.
template <bool FULL>
__device__ __forceinline__ void plain_cand(const float (&v)[32], uint32_t &slot, int step, int jb,
                                           int nvalid, const RowSel &s) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const bool in = (FULL || jb + i < nvalid) && (float_key(v[i]) & s.mask) == s.prefix;
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t@p st.shared.u32 [%0], %1;\n\t"
            "@p add.u32 %0, %0, %3;\n\t}"
            : "+r"(slot)
            : "r"(__float_as_uint(v[i])), "r"((uint32_t)in), "r"(step));
    }
}

// The need-th largest of a row's candidates.  The row's two threads stored their
// scores (raw bits) from the two ends of the row's histogram column; after one exchange of the
// list lengths the first thread resolves the row alone, two bits at a time from the
// top unknown bit: count the candidates at or above the three extensions of the
// prefix and keep the largest extension that still has `need` keys.  Called by
// every epilogue thread (one barrier); the second thread of a row just marks it done.
__device__ __forceinline__ void cand_resolve(RowSel &s, bool act_row, const uint32_t *col, int n,
                                             int half, uint32_t (*xch)[2][kRows], int row) {
    if (act_row && half == 1) xch[0][1][row] = (uint32_t)n;
    epi_bar();
    if (!act_row) return;
    s.done = true;
    s.cand = false;
    if (half == 1) return;
    int n1 = (int)xch[0][1][row];
    if (kCheckBuild && (n < 0 || n1 < 0 || n + n1 > kCap)) {  // the two lists overlap
        SGSA_CHECK_FAIL(g_check, kChkCandCap);
        n = min(max(n, 0), kCap);
        n1 = min(max(n1, 0), kCap - n);
    }
    const uint32_t *back = col + (kCap - 1) * kRows;
    uint32_t x = s.prefix;
    const int need = s.need;
    for (int lo = s.top - 2; lo >= -1; lo -= 2) {
        // bits [lo, lo + 2) (lo = -1: only bit 0 is left)
        const int gb = max(lo, 0);
        const uint32_t one = lo < 0 ? 0u : 1u;
        const uint32_t c1 = x | (one << gb), c2 = x | (2u << gb >> (1 - one)),
                       c3 = x | (3u << gb >> (1 - one));
        int k1 = 0, k2 = 0, k3 = 0;
#pragma unroll 4
        for (int i = 0; i < n; ++i) {
            const uint32_t v = float_key(__uint_as_float(col[i * kRows]));
            k1 += v >= c1;
            k2 += v >= c2;
            k3 += v >= c3;
        }
#pragma unroll 4
        for (int i = 0; i < n1; ++i) {
            const uint32_t v = float_key(__uint_as_float(back[-i * kRows]));
            k1 += v >= c1;
            k2 += v >= c2;
            k3 += v >= c3;
        }
        if (one)
            x |= (k3 >= need ? 3u : k2 >= need ? 2u : k1 >= need ? 1u : 0u) << gb;
        else
            x |= k2 >= need ? 1u : 0u;
    }
    int gt = 0, eq = 0;
    for (int i = 0; i < n; ++i) {
        const uint32_t v = float_key(__uint_as_float(col[i * kRows]));
        gt += v > x;
        eq += v == x;
    }
    for (int i = 0; i < n1; ++i) {
        const uint32_t v = float_key(__uint_as_float(back[-i * kRows]));
        gt += v > x;
        eq += v == x;
    }
    s.need -= gt;
    s.prefix = x;
    s.mask = 0xffffffffu;
    s.top = 0;
    s.exact = eq == s.need;
}

// Sets up candidate mode for keys in [klo, khi] (they share the bits above `top`).
__device__ __forceinline__ void to_cand(RowSel &s, uint32_t klo, uint32_t khi) {
    key_range_prefix(klo, khi, s.prefix, s.top);
    s.mask = s.top >= 32 ? 0u : ~((1u << s.top) - 1u);
    s.cand = true;
}

__device__ __forceinline__ void to_plain(RowSel &s, int K) {
    s.plain = true;
    s.cand = false;
    s.prefix = 0u;
    s.mask = 0u;
    s.need = K;
    s.top = 32;
}

// Choose the bin holding the need-th largest counted key: (bin, keys above it, its
// count).  Group sums of 8 bins first (independent loads), then the crossing group.
__device__ __forceinline__ void lin_choose(const uint32_t *hist, int col, int need, int &chosen,
                                           int &cum, int &cnt) {
    constexpr int kG = kBins / 8;
    int gs[kG];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
        int t = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) t += (int)hist_count(hist, g * 8 + i, col);
        gs[g] = t;
    }
    cum = 0;
    int g0 = 0;
#pragma unroll
    for (int g = kG - 1; g >= 0; --g) {
        if (cum + gs[g] >= need) { g0 = g; break; }
        cum += gs[g];
    }
    int c[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = (int)hist_count(hist, g0 * 8 + i, col);
    chosen = g0 * 8;
    cnt = c[0];
#pragma unroll
    for (int i = 7; i >= 0; --i) {
        if (cum + c[i] >= need) { chosen = g0 * 8 + i; cnt = c[i]; break; }
        cum += c[i];
    }
}

// After a sampled window pass (every kSampleStride-th key tile, nsamp of the row's keys):
// the window of the full pass, placed on the sample's own counts.  In a sample of nsamp
// keys the k-th key of the row has rank about need_s = need nsamp / nvalid, within a few
// sqrt(need_s); the window spans the bins holding the sample ranks need_s -+ R, R =
// 6 sqrt(need_s) + 8, so the full pass's chosen bin holds few keys and goes straight to
// the candidate pass.  The window only steers the work: a k-th key outside it restarts the
// row with the plain digits, exactly.
__device__ __forceinline__ void lin_resample(RowSel &s, const uint32_t *hist, int col, int nvalid,
                                             int nsamp) {
    if (nsamp <= 0 || nvalid <= 0) return;
    const float need_s = (float)s.need * (float)nsamp / (float)nvalid;
    const float R = 6.f * sqrtf(need_s) + 8.f;
    const int r_top = (int)(need_s - R), r_bot = (int)ceilf(need_s + R);
    const float a = s.a0, b = s.b0;
    float lo = -b / a, hi = lo + 1.f / a;  // the sampled pass's window
    int c, cum, cnt;
    if (r_bot <= nsamp) {
        lin_choose(hist, col, r_bot, c, cum, cnt);
        if (c > 0) lo = ((c - 0.5f) / (float)kLinTop - b) / a;  // lower edge of bin c
    }
    if (r_top >= 1) {
        lin_choose(hist, col, r_top, c, cum, cnt);
        if (c < kLinTop) hi = ((c + 0.5f) / (float)kLinTop - b) / a;  // upper edge of bin c
    }
    if (hi > lo && hi - lo < INFINITY) {
        s.a0 = 1.0f / (hi - lo);
        s.b0 = -lo * s.a0;
    }
}

// After the window pass: the chosen bin, with exact key edges by bisection.
__device__ __forceinline__ void lin_after0(RowSel &s, const uint32_t *hist, int col, int K,
                                           unsigned long long *stats, bool count) {
    int c, cum, cnt;
    lin_choose(hist, col, s.need, c, cum, cnt);
    if (c == 0 || c == kLinTop) {  // the k-th score is outside the window
        to_plain(s, K);
        if (count) atomicAdd(&stats[1], 1ull);
        return;
    }
    s.need -= cum;
    s.c0 = c;
    s.cnt = cnt;
    const float a = s.a0, b = s.b0;
    const uint32_t klo = min_key_near([&](float x) { return (int)lin_bin(x, a, b) >= c; },
                                      lin_edge_guess(c, a, b));
    if (cnt == s.need) {  // every key of the bin is taken: key >= its lower edge
        s.prefix = klo;
        s.mask = 0xffffffffu;
        s.top = 0;
        s.done = s.exact = true;
        return;
    }
    const uint32_t khi = min_key_near([&](float x) { return (int)lin_bin(x, a, b) >= c + 1; },
                                      lin_edge_guess(c + 1, a, b));
    if (cnt <= kCap) {
        to_cand(s, klo, khi - 1u);
        return;
    }
    // too many keys in the bin: a second window over its interval
    s.lvl = 1;
    const float xlo = key_float(klo), xhi = key_float(khi);
    const float inv = 1.0f / (xhi - xlo);
    s.a1 = inv;
    s.b1 = -xlo * inv;
    if (count) atomicAdd(&stats[0], 1ull);
}

__device__ __forceinline__ void lin_after1(RowSel &s, const uint32_t *hist, int col, int K,
                                           unsigned long long *stats, bool count) {
    int c, cum, cnt;
    lin_choose(hist, col, s.need, c, cum, cnt);
    s.need -= cum;
    s.c1 = c;
    s.cnt = cnt;
    const float a0 = s.a0, b0 = s.b0, a1 = s.a1, b1 = s.b1;
    const int c0 = s.c0;
    // (bin0, bin1) is lexicographically monotone in the score
    auto at_least = [&](int cc) {
        return [=](float x) {
            const int d0 = (int)lin_bin(x, a0, b0);
            return d0 > c0 || (d0 == c0 && (int)lin_bin(x, a1, b1) >= cc);
        };
    };
    const uint32_t klo = min_key_near(at_least(c), lin_edge_guess(c, a1, b1));
    if (cnt == s.need) {
        s.prefix = klo;
        s.mask = 0xffffffffu;
        s.top = 0;
        s.done = s.exact = true;
        return;
    }
    if (cnt <= kCap) {
        const uint32_t khi =
            c < kLinTop ? min_key_near(at_least(c + 1), lin_edge_guess(c + 1, a1, b1))
                        : min_key_near([=](float x) { return (int)lin_bin(x, a0, b0) > c0; },
                                       lin_edge_guess(c0 + 1, a0, b0));
        to_cand(s, klo, khi - 1u);
        return;
    }
    to_plain(s, K);
    if (count) atomicAdd(&stats[1], 1ull);
}

// Collect of one 32-column chunk: selected column indices go, branch-free,
// into this row's 32-slot ring in shared memory (ring[slot * kRows + row]),
// which the caller then flushes in order to the output row.
template <bool FULL>
__device__ __forceinline__ void collect_chunk(const float (&v)[32], uint32_t *ring, int jb,
                                              int nvalid, const RowSel &s, int &pos,
                                              int &taken, int &lastj) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const uint32_t m = float_key(v[i]) & s.mask;
        const bool ok = FULL || jb + i < nvalid;
        const bool eq = ok && m == s.prefix && taken < s.need;
        const bool sel = eq || (ok && m > s.prefix);
        ring[(pos & 31) * kRows] = (uint32_t)(jb + i);
        pos += sel;
        taken += eq;
        lastj = eq ? jb + i : lastj;
    }
}

// ACC = 1: one 128-column accumulator, 256 TMEM columns, two CTAs per SM (the pipeline's
// MMA and epilogue alternate within a CTA; the other CTA fills the gaps).  ACC = 2: two
// accumulators, 512 columns, one CTA per SM whose next tile's MMA overlaps the epilogue of
// the current one: faster per CTA, for grids too small to fill the SMs twice over.
template <int DI, int ACC = 1>
struct TcCfg {
    static constexpr int kKB = DI / 64;                // 128-byte K blocks
    // 128-key tiles: the tensor-core attention recomputes these scores with the
    // same instruction shapes (M=128, N=128, K=16 steps), which keeps them
    // bit-identical
    static constexpr int kN = 128;                     // keys per tile
    static constexpr int kKBytes = kN * DI * 2;
    static constexpr int kStages = 2;
    static constexpr int kHistBytes = kBins * kRows * 4;
    static constexpr int kAcc = ACC;                   // TMEM accumulator buffers
    static constexpr int kBars = 2 * kStages + 2 * kAcc;
    static constexpr size_t kSmem = 1024 + kStages * kKBytes + kHistBytes + kBars * 8;
    // TMEM: the accumulators, then the query tile (the MMA's A operand: row = lane,
    // two bf16 per 32-bit column)
    static constexpr int kTIQ = kAcc * kN;
    static constexpr int kTmemCols = ACC == 1 ? 256 : 512;
    static_assert(kTIQ + DI / 2 <= kTmemCols, "tensor memory");
    static constexpr int kThreads = 64 + kEpiThreads;
};

template <int DI, int ACC>
__global__ void __launch_bounds__(TcCfg<DI, ACC>::kThreads, ACC == 1 ? 2 : 1)
indexer_topk_tc_kernel(const __nv_bfloat16 *__restrict__ iq,
                       const __grid_constant__ CUtensorMap tm_k, int32_t *__restrict__ idx,
                       uint4 *__restrict__ thr, int B, int T, int H, int K, int nqt,
                       const int32_t *__restrict__ q_tiles, float *__restrict__ dbg_scores) {
    using C = TcCfg<DI, ACC>;
    using namespace sm100;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *base = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char *sK = base;
    uint32_t *hist = (uint32_t *)(sK + C::kStages * C::kKBytes);
    uint64_t *bars = (uint64_t *)((unsigned char *)hist + C::kHistBytes);
    uint64_t *full = bars, *empty = bars + C::kStages, *tfull = bars + 2 * C::kStages,
             *tempty = tfull + C::kAcc;
    __shared__ uint32_t s_tmem;
    __shared__ uint32_t s_xch[2][2][kRows];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int BH = B * H;
    // query tile: an explicit list (heaviest first) or all tiles, heaviest first
    const int qt = q_tiles ? q_tiles[blockIdx.x / BH] : nqt - 1 - (int)(blockIdx.x / BH);
    const int bh = (int)(blockIdx.x % BH), b = bh / H, h = bh % H;
    const int q0 = qt * kRows;
    const int q_last = min(T - 1, q0 + kRows - 1);
    const int nkt = q_last / C::kN + 1;
    unsigned int *wd = &g_index_watchdog;

    const bool epi = warp >= 2;
    const int half = epi ? (warp - 2) >> 2 : 0;  // which half of the tile's columns
    const int quad = warp & 3;                    // TMEM lane quarter this warp may access
    const int row = quad * 32 + lane;
    const int t = q0 + row;
    const int nvalid = (epi && t < T) ? t + 1 : 0;
    // long query tiles: pass 0 bins a sample (every kSampleStride-th key tile) to place the
    // window of the full pass (CTA-uniform: every role strides its tile loop the same way)
    const bool sampled = q0 >= kSampleFrom;
    const bool has_row = epi && t < T;
    const bool stat_thread = has_row && half == 0;
    int32_t *out_row = (has_row && idx) ? idx + ((size_t)bh * T + t) * K : nullptr;
    uint4 *thr_row = (has_row && thr) ? thr + (size_t)bh * T + t : nullptr;
    RowSel s{0u, 0u, K, 32, true, false, true, false, 0, 0, 0.f, 0.f, 0.f, 0.f, 0, 0};
    if (epi && nvalid > K) {
        s.done = false;
        s.exact = false;
    }
    if (epi && half == 0 && has_row && nvalid <= K) {
        if (out_row)
            for (int i = 0; i < K; ++i) out_row[i] = (i < nvalid) ? i : -1;
        if (thr_row) *thr_row = make_uint4(0u, 0u, 0x7fffffffu, 1u);  // every column j <= t
    }
    if (q_last + 1 <= K) return;  // every row of the tile keeps all its columns

    if (warp == 0 && lane == 0) {
        for (int i = 0; i < C::kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < C::kAcc; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpiThreads / 32);
        }
        fence_barrier_init();
        prefetch_tmap(&tm_k);
    }
    if (warp == 1) tmem_alloc(&s_tmem, C::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    if (epi) {
        // the query tile into tensor memory: this thread's half of its row, DI/4 values
        // (rows past T as zeros), as bf16 pairs in DI/4 columns
        constexpr int kW = DI / 4;  // 32-bit columns per thread
        uint32_t w[kW];
        const uint4 *src = reinterpret_cast<const uint4 *>(iq + (((size_t)b * T + t) * H + h) * DI + half * (DI / 2));
#pragma unroll
        for (int i = 0; i < kW / 4; ++i) {
            const uint4 u = has_row ? src[i] : make_uint4(0u, 0u, 0u, 0u);
            w[4 * i] = u.x; w[4 * i + 1] = u.y; w[4 * i + 2] = u.z; w[4 * i + 3] = u.w;
        }
        const uint32_t ta = tmem + ((uint32_t)(quad * 32) << 16) + C::kTIQ + half * kW;
#pragma unroll
        for (int c = 0; c < kW / 8; ++c) {
            uint32_t w8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w8[i] = w[8 * c + i];
            tmem_st8u(ta + 8 * c, w8);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    uint32_t it_p = 0, it_m = 0, it_e = 0;
    bool collecting = false;
    bool cand_pass = false;  // CTA-uniform: some row gathers candidates in this pass
    uint32_t *hcol = hist + row;
    const uint32_t cbase = (uint32_t)__cvta_generic_to_shared(hcol);
    for (int pass = 0;; ++pass) {
        if (warp == 0) {
            if (lane == 0) {
                const int kstep = (sampled && pass == 0) ? kSampleStride : 1;
                for (int kt = 0; kt < nkt; kt += kstep, ++it_p) {
                    const uint32_t st = it_p % C::kStages, ph = (it_p / C::kStages) & 1;
                    mbar_wait(&empty[st], ph ^ 1, wd, 1u);
                    mbar_arrive_expect_tx(&full[st], C::kKBytes);
                    unsigned char *dst = sK + st * C::kKBytes;
                    for (int kb = 0; kb < C::kKB; ++kb)
                        tma_load_3d(dst + kb * (C::kN * 128), &tm_k, &full[st], kb * 64, h,
                                    b * T + kt * C::kN);
                }
            }
            __syncwarp();
        } else if (warp == 1) {
            if (lane == 0) {
                constexpr uint32_t idesc = idesc_bf16_f32(128, C::kN);
                const uint32_t tq = tmem + C::kTIQ;  // A operand in tensor memory
                const int kstep = (sampled && pass == 0) ? kSampleStride : 1;
                for (int kt = 0; kt < nkt; kt += kstep, ++it_m) {
                    const uint32_t st = it_m % C::kStages, ph = (it_m / C::kStages) & 1;
                    const uint32_t buf = it_m % C::kAcc, bph = (it_m / C::kAcc) & 1;
                    mbar_wait(&tempty[buf], bph ^ 1, wd, 4u);
                    mbar_wait(&full[st], ph, wd, 8u);
                    tc_fence_after();
                    const uint32_t ka = smem_u32(sK + st * C::kKBytes);
#pragma unroll
                    for (int kb = 0; kb < C::kKB; ++kb) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint64_t bd = sdesc_kmajor_sw128(ka + kb * (C::kN * 128) + kk * 32);
                            mma_bf16_ts(tmem + buf * C::kN, tq + kb * 32 + kk * 8, bd, idesc,
                                        (kb | kk) ? 1u : 0u);
                        }
                    }
                    mma_commit(&empty[st]);
                    mma_commit(&tfull[buf]);
                }
            }
            __syncwarp();
        } else {
            const bool active = !s.done;
            // what this row does in this pass
            const bool do_cand = active && s.cand;
            const bool do_hist = active && !s.cand;
            const bool collect = collecting && half == 0 && has_row && nvalid > K;
            if (!collecting) {
                if (do_hist)
                    for (int w = half * (kBins / 2); w < (half + 1) * (kBins / 2); ++w) hcol[w * kRows] = 0u;
                epi_bar();
            }
            uint32_t *ring = hist + row;  // the histogram is idle during the collect pass
            int pos = 0, taken = 0, flushed = 0, lastj = -1;
            // candidate slots: half 0 from the front of the row's column, half 1 from the back
            uint32_t cslot = (uint32_t)__cvta_generic_to_shared(hcol + (half ? (kCap - 1) * kRows : 0));
            const int cstep = half ? -(int)(kRows * 4) : (int)(kRows * 4);
            const int kstep = (sampled && pass == 0) ? kSampleStride : 1;
            for (int kt = 0; kt < nkt; kt += kstep, ++it_e) {
                const uint32_t buf = it_e % C::kAcc, bph = (it_e / C::kAcc) & 1;
                mbar_wait(&tfull[buf], bph, wd, 16u);
                tc_fence_after();
                const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + buf * C::kN;
                if (!collecting && pass == 0 && kt == 0) {
                    // sample of the first key tile (the row's 128 scores: this thread's two
                    // chunks, 16 columns at a time): place every row's window
                    uint32_t amax = 0u;
                    int np = 0, nv = 0;
#pragma unroll 1
                    for (int q4 = 0; q4 < C::kN / 32; ++q4) {
                        const int c = half + 2 * (q4 >> 1);
                        float w2[16];
                        tmem_ld16(taddr + c * 32 + (q4 & 1) * 16, w2);
                        const int jb2 = c * 32 + (q4 & 1) * 16;
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const bool ok = active && jb2 + i < nvalid;
                            amax = max(amax, ok ? (__float_as_uint(w2[i]) & 0x7fffffffu) : 0u);
                            np += ok && w2[i] > 0.f;
                            nv += ok;
                        }
                    }
                    s_xch[0][half][row] = (uint32_t)np | ((uint32_t)nv << 16);
                    s_xch[1][half][row] = amax;
                    epi_bar();
                    const uint32_t o = s_xch[0][half ^ 1][row];
                    amax = max(amax, s_xch[1][half ^ 1][row]);
                    const int npos = np + (int)(o & 0xffffu), nval = nv + (int)(o >> 16);
                    // window 2 max|s| wide; by the sample's share of positive scores
                    // against the share to select: [0, W), [-W/2, W/2) or [-W, 0)
                    float W = 2.0f * __uint_as_float(min(amax, 0x7f000000u));
                    W = W > 1e-30f ? W : 1.0f;
                    const float p = nval ? (float)npos / (float)nval : 0.5f;
                    const float q = (float)s.need / (float)max(nvalid, 1);
                    const float lo = p > q + 0.15f ? 0.f : p < q - 0.15f ? -W : -0.5f * W;
                    // Long rows selecting from the upper tail: the k-th score lies well
                    // inside [0, max|s| of the sample), and a window of about that width
                    // keeps its bin under the candidate capacity where 2 max|s| would
                    // need the refine pass (a k-th score beyond the window restarts the
                    // row exactly, with the plain digits, so this only trades passes).
                    if (lo == 0.f && nvalid >= kLongRow) W *= 0.525f;
                    s.a0 = 1.0f / W;
                    s.b0 = -lo * s.a0;
                }
                if (!collecting) {
#pragma unroll 1
                  for (int ci = 0; ci < C::kN / 64; ++ci) {  // chunks half, half + 2 of the tile
                    const int c = half + 2 * ci;
                    float v[32];
                    tmem_ld32(taddr + c * 32, v);
                    const int jb = kt * C::kN + c * 32;
                    const bool full_tile = jb + 32 <= nvalid;
                    if (dbg_scores && pass == 0 && has_row) {
                        // test support: the fp32 scores this pass selects from
                        float *dr = dbg_scores + ((size_t)bh * T + t) * T;
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (jb + i < nvalid) dr[jb + i] = v[i];
                    }
                    if (active && jb < nvalid) {
                        if (do_cand) {
                            if (s.plain) {
                                if (full_tile) plain_cand<true>(v, cslot, cstep, jb, nvalid, s);
                                else plain_cand<false>(v, cslot, cstep, jb, nvalid, s);
                            } else if (s.lvl == 0) {
                                if (full_tile) lin_cand<true, false>(v, cslot, cstep, jb, nvalid, s);
                                else lin_cand<false, false>(v, cslot, cstep, jb, nvalid, s);
                            } else {
                                if (full_tile) lin_cand<true, true>(v, cslot, cstep, jb, nvalid, s);
                                else lin_cand<false, true>(v, cslot, cstep, jb, nvalid, s);
                            }
                        } else if (s.plain) {
                            if (full_tile) plain_hist<true>(v, hcol, jb, nvalid, s);
                            else plain_hist<false>(v, hcol, jb, nvalid, s);
                        } else if (s.lvl == 0) {
                            if (full_tile) lin_hist0<true>(v, cbase, jb, nvalid, s.a0, s.b0);
                            else lin_hist0<false>(v, cbase, jb, nvalid, s.a0, s.b0);
                        } else {
                            if (full_tile) lin_hist1<true>(v, cbase, jb, nvalid, s);
                            else lin_hist1<false>(v, cbase, jb, nvalid, s);
                        }
                    }
                  }
                } else if (half == 0) {
#pragma unroll 1
                    for (int c = 0; c < C::kN / 32; ++c) {
                        float v[32];
                        tmem_ld32(taddr + c * 32, v);
                        const int jb = kt * C::kN + c * 32;
                        if (!collect || jb >= nvalid) continue;
                        const bool full_tile = jb + 32 <= nvalid;
                        if (full_tile) collect_chunk<true>(v, ring, jb, nvalid, s, pos, taken, lastj);
                        else collect_chunk<false>(v, ring, jb, nvalid, s, pos, taken, lastj);
                        if (out_row) {
                            for (; flushed < pos; ++flushed)
                                if (flushed < K) {
                                    const uint32_t jv = ring[(flushed & 31) * kRows];
                                    if (kCheckBuild && jv >= (uint32_t)nvalid)
                                        SGSA_CHECK_FAIL(g_check, kChkCollectIndex);
                                    out_row[flushed] = (int32_t)jv;
                                }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
            }
            if (!collecting) {
                epi_bar();  // every reduction / candidate of the pass has landed
                if (cand_pass) {
                    const uint32_t c0 = (uint32_t)__cvta_generic_to_shared(hcol + (half ? (kCap - 1) * kRows : 0));
                    const int ncand = (int)((half ? c0 - cslot : cslot - c0) / (kRows * 4));
                    cand_resolve(s, do_cand, hcol, ncand, half, s_xch, row);
                }
                if (do_hist) {
                    if (s.plain) {
                        row_choose_plain(s, hist, row);
                        if (!s.done && s.cnt <= kCap) {
                            s.cand = true;
                            if (stat_thread) atomicAdd(&g_index_stats[2], 1ull);
                        }
                    } else if (s.lvl == 0 && sampled && pass == 0) {
                        int nsamp = 0;  // this row's keys in the sampled tiles
                        for (int kt = 0; kt < nkt; kt += kSampleStride)
                            nsamp += max(0, min(C::kN, nvalid - kt * C::kN));
                        lin_resample(s, hist, row, nvalid, nsamp);
                    } else if (s.lvl == 0) {
                        lin_after0(s, hist, row, K, g_index_stats, stat_thread);
                    } else {
                        lin_after1(s, hist, row, K, g_index_stats, stat_thread);
                    }
                }
            } else if (collect) {
                if (kCheckBuild && pos != K) SGSA_CHECK_FAIL(g_check, kChkCollectCount);
                if (out_row)
                    for (int i = min(pos, K); i < K; ++i) out_row[i] = -1;
                // the exact selection as a threshold: key & mask > prefix, or equal and j <= cut
                if (thr_row) *thr_row = make_uint4(s.prefix, s.mask, (uint32_t)lastj, 1u);
            }
        }
        const int more = __syncthreads_or(epi && !s.done);
        cand_pass = __syncthreads_or(epi && !s.done && s.cand);
        if (collecting) break;
        if (more && pass + 1 >= kMaxPasses) {
            // cannot happen (the plain radix ends after 4 digits); flag it rather than spin
            if (threadIdx.x == 0) atomicOr(wd, 0x40u);
        }
        if (!more || pass + 1 >= kMaxPasses) {
            // Without index rows to write, the collect pass only finds the tie cut of
            // rows whose k-th key is an exact tie; if there is none, it is skipped.
            const bool tie_row = epi && half == 0 && has_row && nvalid > K && !s.exact;
            if (tie_row) atomicAdd(&g_index_stats[3], 1ull);
            if (!idx) {
                const bool ties = __syncthreads_or(tie_row);
                if (!ties) {
                    if (epi && half == 0 && thr_row && nvalid > K)
                        *thr_row = make_uint4(s.prefix, s.mask, 0x7fffffffu, 1u);
                    break;
                }
            }
            collecting = true;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

template <int DI>
cudaError_t run_tc(const void *iq, const void *ik, int32_t *idx, uint4 *thr, int B, int T, int H,
                   int K, const int32_t *q_tiles, int n_tiles, cudaStream_t st,
                   float *dbg_scores = nullptr, bool shares_sms = false) {
    CUtensorMap mk;
    if (!make_tmap_rows_bf16(&mk, ik, B, T, H, DI, TcCfg<DI>::kN)) return cudaErrorInvalidValue;
    const int nqt = ceil_div(T, kRows);
    const int ntiles = q_tiles ? n_tiles : nqt;
    if (ntiles <= 0) return cudaSuccess;
    const long long ctas = (long long)ntiles * B * H;
    int dev = 0, nsm = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    // Grids that do not fill the SMs several times over: one CTA per SM with two accumulators
    auto go = [&](auto kern, size_t smem, int threads) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        kern<<<(unsigned)ctas, threads, smem, st>>>((const __nv_bfloat16 *)iq, mk, idx, thr, B, T, H, K,
                                                    nqt, q_tiles, dbg_scores);
        return launched();
    };
    // (not while other kernels run beside it: its 512 TMEM columns would keep them off the SM)
    if (!shares_sms && ctas <= (long long)kSmallGridWaves * nsm)
        return go(indexer_topk_tc_kernel<DI, 2>, TcCfg<DI, 2>::kSmem, TcCfg<DI, 2>::kThreads);
    return go(indexer_topk_tc_kernel<DI, 1>, TcCfg<DI, 1>::kSmem, TcCfg<DI, 1>::kThreads);
}

template <int DI>
cudaError_t run_tc_t(const void *iq, const void *ik, int32_t *idx, uint4 *thr, int B, int T,
                     int H, int K, const int32_t *q_tiles, int n_tiles, cudaStream_t st,
                     bool shares_sms = false) {
    return run_tc<DI>(iq, ik, idx, thr, B, T, H, K, q_tiles, n_tiles, st, nullptr, shares_sms);
}

template <typename Tin, int DI>
cudaError_t run_simt(const void *iq, const void *ik, int32_t *idx, int B, int T, int H, int K,
                     cudaStream_t st) {
    const size_t smem = 256 * kRows * sizeof(uint32_t) + (size_t)kRows * (DI + 1) * sizeof(float) +
                        (size_t)kKeyTile * DI * sizeof(float);
    auto kern = indexer_topk_simt_kernel<Tin, DI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int nqt = ceil_div(T, kRows);
    kern<<<dim3(nqt, B * H), kRows, smem, st>>>((const Tin *)iq, (const Tin *)ik, idx, B, T, H, K, nqt);
    return launched();
}

template <typename Tin>
cudaError_t run_simt_d(int DI, const void *iq, const void *ik, int32_t *idx, int B, int T, int H,
                       int K, cudaStream_t st) {
    switch (DI) {
        case 32: return run_simt<Tin, 32>(iq, ik, idx, B, T, H, K, st);
        case 64: return run_simt<Tin, 64>(iq, ik, idx, B, T, H, K, st);
        case 128: return run_simt<Tin, 128>(iq, ik, idx, B, T, H, K, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool indexer_tc_eligible(int DI, int dtype) {
    return dtype == SGSA_DTYPE_BF16 && (DI == 64 || DI == 128) && indexer_use_tc();
}

cudaError_t launch_indexer_topk_thr(const void *iq, const void *ik, int32_t *idx, uint32_t *thr,
                                    int B, int T, int H, int DI, int K, const int32_t *q_tiles,
                                    int n_tiles, cudaStream_t st, bool shares_sms) {
    if (DI == 64)
        return run_tc_t<64>(iq, ik, idx, (uint4 *)thr, B, T, H, K, q_tiles, n_tiles, st, shares_sms);
    if (DI == 128)
        return run_tc_t<128>(iq, ik, idx, (uint4 *)thr, B, T, H, K, q_tiles, n_tiles, st, shares_sms);
    return cudaErrorInvalidValue;
}

cudaError_t launch_indexer_topk(const void *iq, const void *ik, int32_t *idx, int B, int T, int H,
                                int DI, int K, int dtype, cudaStream_t st) {
    if (dtype == SGSA_DTYPE_F32) return run_simt_d<float>(DI, iq, ik, idx, B, T, H, K, st);
    if (indexer_use_tc()) {
        if (DI == 64) return run_tc_t<64>(iq, ik, idx, nullptr, B, T, H, K, nullptr, 0, st);
        if (DI == 128) return run_tc_t<128>(iq, ik, idx, nullptr, B, T, H, K, nullptr, 0, st);
    }
    return run_simt_d<__nv_bfloat16>(DI, iq, ik, idx, B, T, H, K, st);
}

unsigned int read_index_watchdog(cudaStream_t st) {
    unsigned int v = 0, z = 0;
    if (cudaStreamSynchronize(st) != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyFromSymbol(&v, g_index_watchdog, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (v) cudaMemcpyToSymbol(g_index_watchdog, &z, sizeof(z));
    return v;
}

// Watchdog self-test: one thread waits, with a short spin limit, on an mbarrier that
// nothing ever arrives at.  The wait gives up, records `code` in the indexer's
// watchdog word and the kernel returns -- the path a stalled pipeline takes.
namespace {
__global__ void watchdog_selftest_kernel(uint32_t limit, unsigned int code) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);
        sm100::fence_barrier_init();
        sm100::mbar_wait(&bar, 0, &g_index_watchdog, code, limit);
    }
}
}  // namespace

cudaError_t launch_watchdog_selftest(uint32_t limit, cudaStream_t st) {
    watchdog_selftest_kernel<<<1, 32, 0, st>>>(limit, 0x80u);
    return launched();
}

cudaError_t launch_indexer_topk_debug(const void *iq, const void *ik, int32_t *idx,
                                     float *scores, int B, int T, int H, int DI, int K,
                                     cudaStream_t st) {
    if (T >= 65536) return cudaErrorInvalidValue;
    if (DI == 64) return run_tc<64>(iq, ik, idx, nullptr, B, T, H, K, nullptr, 0, st, scores);
    if (DI == 128) return run_tc<128>(iq, ik, idx, nullptr, B, T, H, K, nullptr, 0, st, scores);
    return cudaErrorInvalidValue;
}

int read_index_stats(unsigned long long *out, bool reset) {
    if (cudaMemcpyFromSymbol(out, g_index_stats, 4 * sizeof(unsigned long long)) != cudaSuccess)
        return -1;
    if (reset) {
        const unsigned long long z[4] = {0, 0, 0, 0};
        if (cudaMemcpyToSymbol(g_index_stats, z, sizeof(z)) != cudaSuccess) return -1;
    }
    return 0;
}

cudaError_t launch_topk_select(const float *scores, const int32_t *valid, int32_t *idx, int R,
                               int S, int K, cudaStream_t st) {
    const size_t smem = 256 * kRows * sizeof(uint32_t);
    cudaError_t e = cudaFuncSetAttribute(topk_select_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    topk_select_kernel<<<ceil_div(R, kRows), kRows, smem, st>>>(scores, valid, idx, R, S, K);
    return launched();
}

unsigned int check_word_indexer(bool reset) {
    unsigned int v = 0, z = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyFromSymbol(&v, g_check, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (reset && v) cudaMemcpyToSymbol(g_check, &z, sizeof(z));
    return v;
}

}  // namespace sgsa
