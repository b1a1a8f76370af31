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
//   warp 0  TMA producer: the query tile once, then key tiles into a ring of
//           shared-memory stages;
//   warp 1  TMEM owner and MMA issuer: S_tile = Q K^T, M=128 (queries) x
//           N=kN (keys) x K=DI, into one of two TMEM accumulators;
//   warps 2-9  two threads per query row (warps w and w+4 read the same TMEM
//           lane quarter and split the tile's columns): tcgen05.ld of their
//           part of the row, radix histogram; the first thread of each row
//           also runs the collect pass, which must walk the row in order.
// The key stream is replayed once per pass; the tensor cores recompute the
// identical fp32 scores each time.
//
// Digits.  The first pass bins a fast digit of each score over a window placed
// from a sample of the first key tile (select_keys.cuh: 1/32-octave bins of one
// sign, or 1/8-octave bins of both signs when the sample leaves the k-th score's
// sign unclear).  A row whose k-th score lands in an interior bin knows the top
// 13-14 bits of its key; if the bin then holds at most 128 keys for every row of
// the warp, the next pass stores those keys (candidate mode) and the k-th is found
// among them in shared memory; otherwise 8-bit digits follow.  A k-th score in a
// clamp bin retries the other window once or restarts with plain 8-bit digits
// from the top.  Every path is exact.  Rows shorter than 65536 use 16-bit
// counters packed two per 32-bit word (64 KB), so the CTA needs ~105 KB and two
// CTAs share an SM.  Counters are bumped with predicated shared-memory
// reductions: no branches, no returned values, and the two threads of a row may
// share a counter.
static __device__ unsigned int g_index_watchdog;

constexpr int kEpiThreads = 256;

struct RowSel {
    uint32_t prefix, mask;
    int need;
    int top;     // bits [top-1 : 0] of the k-th key are still unknown
    bool done;
    bool plain;  // the row left the fast window: full order-preserving keys
    bool exact;  // resolved with every key of the final group selected (no tie cut)
    int cnt;     // keys in the bin chosen by the last pass
    bool cand;   // this pass gathers the row's remaining candidate keys instead of counting
    bool fast;   // this pass bins the fast digit (mode, pb)
    int mode;
    int pb;
    int etop;
};

// Key of a score for a row whose k-th score is a positive float: the raw bits
// with the sign flipped order every positive score correctly and put every
// negative one (and -0.0) below any positive prefix, which is all the
// comparisons against such a prefix need.

template <bool PACKED>
__device__ __forceinline__ uint32_t hist_count(const uint32_t *hist, int bin, int col) {
    if (PACKED) return (hist[(bin >> 1) * kRows + col] >> ((bin & 1) << 4)) & 0xffffu;
    return hist[bin * kRows + col];
}

// Choose the bin holding the need-th largest remaining key.  FAST: the
// fast-digit pass of the row's window.
template <bool PACKED, bool FAST>
__device__ __forceinline__ void row_choose(RowSel &s, const uint32_t *hist, int col, int K) {
    const int w = FAST ? 8 : min(8, s.top);
    int cum = 0, chosen = 0, cnt = 0;
    for (int bin = (1 << w) - 1; bin >= 0; --bin) {
        cnt = (int)hist_count<PACKED>(hist, bin, col);
        if (cum + cnt >= s.need) { chosen = bin; break; }
        cum += cnt;
    }
    if (FAST) {
        if (chosen == 0 || chosen == 255 || (s.mode == 2 && chosen == 127)) {
            // outside the window: towards zero, retry with both signs; else plain radix
            const bool toward_zero = s.mode == 0 ? chosen == 0 : s.mode == 1 ? chosen == 255 : false;
            if (toward_zero) {
                s.mode = 2;
                s.pb = fast_base(2, s.etop);
                s.fast = true;
            } else {
                s.prefix = 0u; s.mask = 0u; s.need = K; s.top = 32; s.plain = true;
                s.fast = false;
            }
            s.cnt = 0x7fffffff;
            return;
        }
        s.need -= cum;
        s.prefix = fast_prefix(chosen, s.mode, s.pb);
        const bool two = s.mode == 2;
        s.mask = fast_mask(s.mode);
        s.top = fast_top(s.mode);
        // negative k-th: continue on the order-preserving keys
        s.plain = s.mode == 1 || (two && chosen < 128);
        s.fast = false;
    } else {
        const int shift = s.top - w;
        s.need -= cum;
        s.prefix |= (uint32_t)chosen << shift;
        s.mask |= ((1u << w) - 1u) << shift;
        s.top = shift;
    }
    s.cnt = cnt;
    if (cnt == s.need) s.exact = true;
    if (cnt == s.need || s.top == 0) s.done = true;
}

// Candidate mode.  Once the chosen bin of a row holds at most kCandCap keys, the
// next pass stores those keys (the row's two threads from the two ends of the
// row's histogram column) instead of counting a digit, and the row's k-th key is
// then found among them: bit by bit from the highest unknown bit, keep a bit if at
// least `need` candidates are >= the prefix with it set.  Exact, and it replaces
// the remaining digit passes (usually two or three) by one.
__device__ __forceinline__ void epi_bar() {
    asm volatile("bar.sync 1, %0;" ::"r"(kEpiThreads) : "memory");
}

template <bool PACKED>
struct Cand {
    static constexpr int kCap = PACKED ? 128 : 256;  // 32-bit slots of a histogram column
};

__device__ __forceinline__ void st_shared_if(uint32_t addr, uint32_t v, bool pred) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t@p st.shared.u32 [%0], %1;\n\t}" ::"r"(addr),
                 "r"(v), "r"((uint32_t)pred)
                 : "memory");
}

// Candidate gathering of one 32-column chunk: predicated stores, no branches.
// `slot` is the shared-memory address of this thread's next slot and `step` the
// byte step between slots (+/- one histogram row); n counts the stored keys.
template <bool PLAIN, bool FULL, int CAP>
__device__ __forceinline__ void cand_chunk(const float (&v)[32], uint32_t &slot, int step, int jb,
                                           int nvalid, const RowSel &s, int &n) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const uint32_t u = PLAIN ? float_key(v[i]) : fast_key(v[i]);
        const bool in = (FULL || jb + i < nvalid) && (u & s.mask) == s.prefix && n < CAP;
        st_shared_if(slot, u, in);
        slot += in ? step : 0;
        n += in;
    }
}

// The need-th largest of a row's candidates, found two bits at a time from the top
// unknown bit: both threads of the row count their own list against the three
// extensions of the prefix, swap the counts through shared memory and take the
// largest extension that still has `need` keys at or above it.  All epilogue
// threads run every step (the barriers are CTA-wide); rows not in candidate mode
// only take part in the barriers.
template <int CAP>
__device__ __forceinline__ void cand_resolve(RowSel &s, bool act_row, const uint32_t *col, int n,
                                             int half, uint32_t (*xch)[2][kRows], int row) {
    const int cstep = half ? -kRows : kRows;
    const uint32_t *first = col + (half ? (CAP - 1) * kRows : 0);
    uint32_t x = s.prefix;
    int it = 0;
    for (; it < 16; ++it) {
        // bits [lo, lo + 2) of this row (lo = -1: only bit 0 is left)
        const int lo = s.top - 2 * (it + 1);
        const bool act = act_row && lo >= -1;
        const int gb = max(lo, 0);
        const uint32_t one = lo < 0 ? 0u : 1u;  // a single bit: only c2 (= bit 0) counts
        uint32_t pk = 0;
        if (act) {
            const uint32_t c1 = x | (one << gb), c2 = x | (2u << gb >> (1 - one)),
                           c3 = x | (3u << gb >> (1 - one));
            int k1 = 0, k2 = 0, k3 = 0;
            for (int i = 0; i < n; ++i) {
                const uint32_t v = first[i * cstep];
                k1 += v >= c1;
                k2 += v >= c2;
                k3 += v >= c3;
            }
            pk = (uint32_t)k1 | ((uint32_t)k2 << 10) | ((uint32_t)k3 << 20);
            xch[it & 1][half][row] = pk;
        }
        epi_bar();
        if (act) {
            const uint32_t o = xch[it & 1][half ^ 1][row];
            const int need = s.need;
            const int k3 = (int)((pk >> 20) + (o >> 20));
            const int k2 = (int)(((pk >> 10) & 1023u) + ((o >> 10) & 1023u));
            const int k1 = (int)((pk & 1023u) + (o & 1023u));
            if (one)
                x |= (k3 >= need ? 3u : k2 >= need ? 2u : k1 >= need ? 1u : 0u) << gb;
            else
                x |= k2 >= need ? 1u : 0u;
        }
    }
    uint32_t pk = 0;
    if (act_row) {
        int gt = 0, eq = 0;
        for (int i = 0; i < n; ++i) {
            const uint32_t v = first[i * cstep];
            gt += v > x;
            eq += v == x;
        }
        pk = (uint32_t)gt | ((uint32_t)eq << 10);
        xch[it & 1][half][row] = pk;
    }
    epi_bar();
    if (act_row) {
        const uint32_t o = xch[it & 1][half ^ 1][row];
        const int gt = (int)((pk & 1023u) + (o & 1023u));
        const int eq = (int)((pk >> 10) + (o >> 10));
        s.need -= gt;
        s.prefix = x;
        s.mask = 0xffffffffu;
        s.top = 0;
        s.done = true;
        s.exact = eq == s.need;
    }
}

template <int DI, bool PACKED>
struct TcCfg {
    static constexpr int kKB = DI / 64;                // 128-byte K blocks
    // 64-key tiles in both modes: the tensor-core attention recomputes these
    // scores with the same instruction shapes, which keeps them bit-identical
    static constexpr int kN = 64;                      // keys per tile
    static constexpr int kStages = 3;
    static constexpr int kQBytes = 128 * DI * 2;
    static constexpr int kKBytes = kN * DI * 2;
    static constexpr int kHistBytes = (PACKED ? 128 : 256) * kRows * 4;
    static constexpr int kAcc = 4;                     // TMEM accumulator buffers
    static constexpr int kBars = 2 * kStages + 2 * kAcc + 1;
    static constexpr size_t kSmem = 1024 + kQBytes + kStages * kKBytes + kHistBytes + kBars * 8;
    static constexpr int kMinBlocks = (kSmem * 2 + 2048 <= 233472) ? 2 : 1;
    static constexpr int kTmemCols = kAcc * kN;
    static constexpr int kThreads = 64 + kEpiThreads;
};

__device__ __forceinline__ void red_shared_if(uint32_t *addr, uint32_t inc, bool pred) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t@p red.shared.add.u32 [%0], %1;\n\t}" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(addr)),
                 "r"(inc), "r"((uint32_t)pred)
                 : "memory");
}


// Histogram update of one 32-column chunk.  FAST: the fast digit of the row's
// window (fast_digit); else the row's next digit among keys
// matching its prefix, with keys from float_key (PLAIN) or fast_key.  FULL skips
// the causal bound check.
template <bool FAST, bool PLAIN, bool FULL, bool PACKED, int MODE = 0>
__device__ __forceinline__ void hist_chunk(const float (&v)[32], uint32_t *hcol, int jb,
                                           int nvalid, const RowSel &s) {
    // u >> shift as a high multiply (no variable-amount shift in the loop)
    const int w = min(8, s.top);
    const int shift = s.top - w;
    const uint32_t mul = shift ? (1u << (32 - shift)) : 0u;
    const uint32_t dmask = (1u << w) - 1u;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const bool ok = FULL || jb + i < nvalid;
        uint32_t d;
        bool in;
        if (FAST) {
            d = fast_digit_m<MODE>(v[i], s.pb);
            in = ok;
        } else {
            const uint32_t u = PLAIN ? float_key(v[i]) : fast_key(v[i]);
            d = (shift ? __umulhi(u, mul) : u) & dmask;
            in = ok && (u & s.mask) == s.prefix;
        }
        if (PACKED) red_shared_if(hcol + (d >> 1) * kRows, (d & 1u) * 0xffffu + 1u, in);
        else red_shared_if(hcol + d * kRows, 1u, in);
    }
}

// Collect of one 32-column chunk: selected column indices go, branch-free,
// into this row's 32-slot ring in shared memory (ring[slot * kRows + row]),
// which the caller then flushes in order to the output row.
template <bool PLAIN, bool FULL>
__device__ __forceinline__ void collect_chunk(const float (&v)[32], uint32_t *ring, int jb,
                                              int nvalid, const RowSel &s, int &pos,
                                              int &taken, int &lastj) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const uint32_t m = (PLAIN ? float_key(v[i]) : fast_key(v[i])) & s.mask;
        const bool ok = FULL || jb + i < nvalid;
        const bool eq = ok && m == s.prefix && taken < s.need;
        const bool sel = eq || (ok && m > s.prefix);
        ring[(pos & 31) * kRows] = (uint32_t)(jb + i);
        pos += sel;
        taken += eq;
        lastj = eq ? jb + i : lastj;
    }
}

template <int DI, bool PACKED>
__global__ void __launch_bounds__(TcCfg<DI, PACKED>::kThreads, (TcCfg<DI, PACKED>::kMinBlocks))
indexer_topk_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k, int32_t *__restrict__ idx,
                       uint4 *__restrict__ thr, int B, int T, int H, int K, int nqt,
                       const int32_t *__restrict__ q_tiles, float *__restrict__ dbg_scores) {
    using C = TcCfg<DI, PACKED>;
    using namespace sm100;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *base = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char *sQ = base;
    unsigned char *sK = sQ + C::kQBytes;
    uint32_t *hist = (uint32_t *)(sK + C::kStages * C::kKBytes);
    uint64_t *bars = (uint64_t *)((unsigned char *)hist + C::kHistBytes);
    uint64_t *full = bars, *empty = bars + C::kStages, *tfull = bars + 2 * C::kStages,
             *tempty = tfull + C::kAcc, *qbar = tempty + C::kAcc;
    __shared__ uint32_t s_tmem;
    __shared__ uint32_t s_xch[2][2][kRows];
    __shared__ uint32_t s_amax;  // largest |score| bits of the first key tile's sample
    constexpr int kCap = Cand<PACKED>::kCap;

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
    const bool has_row = epi && t < T;
    int32_t *out_row = (has_row && idx) ? idx + ((size_t)bh * T + t) * K : nullptr;
    uint4 *thr_row = (has_row && thr) ? thr + (size_t)bh * T + t : nullptr;
    RowSel s{0u, 0u, K, 32, true, false, true, 0, false, false, 0, fast_base(0, kDefaultEtop),
             kDefaultEtop};
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
        s_amax = 0u;
        for (int i = 0; i < C::kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < C::kAcc; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpiThreads / 32);
        }
        mbar_init(qbar, 1);
        fence_barrier_init();
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
    }
    if (warp == 1) tmem_alloc(&s_tmem, C::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    // fast digit, the other-sign retry, 4 plain digits after a fallback, spare
    constexpr int kMaxDigitPasses = 7;
    constexpr int kChunksPerHalf = C::kN / 64;
    static_assert(kChunksPerHalf == 1, "the first-tile sample assumes one chunk per thread and tile");
    uint32_t it_p = 0, it_m = 0, it_e = 0;
    bool collecting = false;
    bool cand_pass = false;  // CTA-uniform: some row gathers candidates in this pass
    for (int pass = 0;; ++pass) {
        if (warp == 0) {
            if (lane == 0) {
                if (pass == 0) {
                    mbar_arrive_expect_tx(qbar, C::kQBytes);
                    for (int kb = 0; kb < C::kKB; ++kb)
                        tma_load_3d(sQ + kb * (128 * 128), &tm_q, qbar, kb * 64, h, b * T + q0);
                }
                for (int kt = 0; kt < nkt; ++kt, ++it_p) {
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
                if (pass == 0) mbar_wait(qbar, 0, wd, 2u);
                constexpr uint32_t idesc = idesc_bf16_f32(128, C::kN);
                const uint32_t qa = smem_u32(sQ);
                for (int kt = 0; kt < nkt; ++kt, ++it_m) {
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
                            const uint64_t ad = sdesc_kmajor_sw128(qa + kb * (128 * 128) + kk * 32);
                            const uint64_t bd = sdesc_kmajor_sw128(ka + kb * (C::kN * 128) + kk * 32);
                            mma_bf16(tmem + buf * C::kN, ad, bd, idesc, (kb | kk) ? 1u : 0u);
                        }
                    }
                    mma_commit(&empty[st]);
                    mma_commit(&tfull[buf]);
                }
            }
            __syncwarp();
        } else {
            const bool active = !s.done;
            uint32_t *hcol = hist + row;
            const bool collect = collecting && half == 0 && has_row && nvalid > K;
            if (!collecting) {
                if (half == 0 && active && !s.cand)
                    for (int w = 0; w < (PACKED ? 128 : 256); ++w) hcol[w * kRows] = 0u;
                epi_bar();
            }
            uint32_t *ring = hist + row;  // the histogram is idle during the collect pass
            int pos = 0, taken = 0, flushed = 0, lastj = -1, ncand = 0;
            // candidate slots: half 0 from the front of the row's column, half 1 from the back
            uint32_t cslot = (uint32_t)__cvta_generic_to_shared(hcol + (half ? (kCap - 1) * kRows : 0));
            const int cstep = half ? -(int)(kRows * 4) : (int)(kRows * 4);
            for (int kt = 0; kt < nkt; ++kt, ++it_e) {
                const uint32_t buf = it_e % C::kAcc, bph = (it_e / C::kAcc) & 1;
                mbar_wait(&tfull[buf], bph, wd, 16u);
                tc_fence_after();
                const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + buf * C::kN;
                const bool full_tile = (kt + 1) * C::kN <= nvalid;
                if (!collecting) {
#pragma unroll 1
                    for (int c = half * kChunksPerHalf; c < (half + 1) * kChunksPerHalf; ++c) {
                        float v[32];
                        tmem_ld32(taddr + c * 32, v);
                        const int jb = kt * C::kN + c * 32;
                        if (dbg_scores && pass == 0 && has_row) {
                            // test support: the fp32 scores this pass selects from
                            float *dr = dbg_scores + ((size_t)bh * T + t) * T;
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (jb + i < nvalid) dr[jb + i] = v[i];
                        }
                        if (pass == 0 && kt == 0) {
                            // sample of the first key tile: place every row's fast window
                            uint32_t amax = 0u;
                            int np = 0, nv = 0;
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                const bool ok = active && jb + i < nvalid;
                                amax = max(amax, ok ? (__float_as_uint(v[i]) & 0x7fffffffu) : 0u);
                                np += ok && v[i] > 0.f;
                                nv += ok;
                            }
                            amax = __reduce_max_sync(0xffffffffu, amax);
                            if (lane == 0) atomicMax(&s_amax, amax);
                            s_xch[0][half][row] = (uint32_t)np | ((uint32_t)nv << 16);
                            epi_bar();
                            const uint32_t o = s_xch[0][half ^ 1][row];
                            const int npos = np + (int)(o & 0xffffu), nval = nv + (int)(o >> 16);
                            const int etop = min(max((int)(s_amax >> 23) + 3, 17), 255);  // bottom above 0 and denormals
                            s.etop = etop;
                            // estimated positives p*(t+1) against need: clear margins pick a sign
                            const float p = nval ? (float)npos / (float)nval : 0.5f;
                            const float q = (float)s.need / (float)nvalid;
                            const int m = p > q + 0.15f ? 0 : p < q - 0.15f ? 1 : 2;
                            // one formula per warp: a sign only if every active row agrees
                            const bool all0 = __all_sync(0xffffffffu, !active || m == 0);
                            const bool all1 = __all_sync(0xffffffffu, !active || m == 1);
                            s.mode = all0 ? 0 : all1 ? 1 : 2;
                            s.pb = fast_base(s.mode, etop);
                            s.fast = true;
                        }
                        if (!active || jb >= nvalid) continue;
                        if (s.cand) {
                            if (!s.plain) {
                                if (full_tile) cand_chunk<false, true, kCap>(v, cslot, cstep, jb, nvalid, s, ncand);
                                else cand_chunk<false, false, kCap>(v, cslot, cstep, jb, nvalid, s, ncand);
                            } else {
                                if (full_tile) cand_chunk<true, true, kCap>(v, cslot, cstep, jb, nvalid, s, ncand);
                                else cand_chunk<true, false, kCap>(v, cslot, cstep, jb, nvalid, s, ncand);
                            }
                        } else if (s.fast) {
                            if (s.mode == 0) {
                                if (full_tile) hist_chunk<true, false, true, PACKED, 0>(v, hcol, jb, nvalid, s);
                                else hist_chunk<true, false, false, PACKED, 0>(v, hcol, jb, nvalid, s);
                            } else if (s.mode == 1) {
                                if (full_tile) hist_chunk<true, false, true, PACKED, 1>(v, hcol, jb, nvalid, s);
                                else hist_chunk<true, false, false, PACKED, 1>(v, hcol, jb, nvalid, s);
                            } else {
                                if (full_tile) hist_chunk<true, false, true, PACKED, 2>(v, hcol, jb, nvalid, s);
                                else hist_chunk<true, false, false, PACKED, 2>(v, hcol, jb, nvalid, s);
                            }
                        } else if (!s.plain) {
                            if (full_tile) hist_chunk<false, false, true, PACKED>(v, hcol, jb, nvalid, s);
                            else hist_chunk<false, false, false, PACKED>(v, hcol, jb, nvalid, s);
                        } else {
                            if (full_tile) hist_chunk<false, true, true, PACKED>(v, hcol, jb, nvalid, s);
                            else hist_chunk<false, true, false, PACKED>(v, hcol, jb, nvalid, s);
                        }
                    }
                } else if (half == 0) {
#pragma unroll 1
                    for (int c = 0; c < C::kN / 32; ++c) {
                        float v[32];
                        tmem_ld32(taddr + c * 32, v);
                        const int jb = kt * C::kN + c * 32;
                        if (!collect || jb >= nvalid) continue;
                        if (!s.plain) {
                            if (full_tile) collect_chunk<false, true>(v, ring, jb, nvalid, s, pos, taken, lastj);
                            else collect_chunk<false, false>(v, ring, jb, nvalid, s, pos, taken, lastj);
                        } else {
                            if (full_tile) collect_chunk<true, true>(v, ring, jb, nvalid, s, pos, taken, lastj);
                            else collect_chunk<true, false>(v, ring, jb, nvalid, s, pos, taken, lastj);
                        }
                        if (out_row) {
                            for (; flushed < pos; ++flushed)
                                if (flushed < K) out_row[flushed] = (int32_t)ring[(flushed & 31) * kRows];
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
            }
            if (!collecting) {
                epi_bar();  // every reduction / candidate of the pass has landed
                if (cand_pass) cand_resolve<kCap>(s, active && s.cand, hcol, ncand, half, s_xch, row);
                if (active && !s.cand) {
                    if (s.fast) row_choose<PACKED, true>(s, hist, row, K);
                    else row_choose<PACKED, false>(s, hist, row, K);
                }
                // candidate mode only for whole warps: a warp mixing the two kinds of
                // pass would run both code paths
                const bool fits = __all_sync(0xffffffffu, s.done || s.cnt <= kCap);
                if (!s.done && fits) s.cand = true;
            } else if (collect) {
                if (out_row)
                    for (int i = min(pos, K); i < K; ++i) out_row[i] = -1;
                // the exact selection as a threshold: key & mask > prefix, or equal and j <= cut
                if (thr_row) *thr_row = make_uint4(s.prefix, s.mask, (uint32_t)lastj, 1u);
            }
        }
        const int more = __syncthreads_or(epi && !s.done);
        cand_pass = __syncthreads_or(epi && !s.done && s.cand);
        if (collecting) break;
        if (!more || pass + 1 >= kMaxDigitPasses) {
            // Without index rows to write, the collect pass only finds the tie cut of
            // rows whose k-th key is an exact tie; if there is none, it is skipped.
            if (!idx) {
                const bool ties = __syncthreads_or(epi && half == 0 && has_row && nvalid > K && !s.exact);
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

template <int DI, bool PACKED>
cudaError_t run_tc(const void *iq, const void *ik, int32_t *idx, uint4 *thr, int B, int T, int H,
                   int K, const int32_t *q_tiles, int n_tiles, cudaStream_t st,
                   float *dbg_scores = nullptr) {
    using C = TcCfg<DI, PACKED>;
    CUtensorMap mq, mk;
    if (!make_tmap_rows_bf16(&mq, iq, B, T, H, DI, 128) ||
        !make_tmap_rows_bf16(&mk, ik, B, T, H, DI, C::kN))
        return cudaErrorInvalidValue;
    auto kern = indexer_topk_tc_kernel<DI, PACKED>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)C::kSmem);
    if (e != cudaSuccess) return e;
    const int nqt = ceil_div(T, kRows);
    const int ntiles = q_tiles ? n_tiles : nqt;
    if (ntiles <= 0) return cudaSuccess;
    kern<<<ntiles * B * H, C::kThreads, C::kSmem, st>>>(mq, mk, idx, thr, B, T, H, K, nqt, q_tiles,
                                                      dbg_scores);
    return launched();
}

template <int DI>
cudaError_t run_tc_t(const void *iq, const void *ik, int32_t *idx, uint4 *thr, int B, int T,
                     int H, int K, const int32_t *q_tiles, int n_tiles, cudaStream_t st) {
    // 16-bit counters hold any count below 65536, the longest row they can see.
    if (T < 65536) return run_tc<DI, true>(iq, ik, idx, thr, B, T, H, K, q_tiles, n_tiles, st);
    return run_tc<DI, false>(iq, ik, idx, thr, B, T, H, K, q_tiles, n_tiles, st);
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
                                    int n_tiles, cudaStream_t st) {
    if (DI == 64) return run_tc_t<64>(iq, ik, idx, (uint4 *)thr, B, T, H, K, q_tiles, n_tiles, st);
    if (DI == 128) return run_tc_t<128>(iq, ik, idx, (uint4 *)thr, B, T, H, K, q_tiles, n_tiles, st);
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
    if (DI == 64) return run_tc<64, true>(iq, ik, idx, nullptr, B, T, H, K, nullptr, 0, st, scores);
    if (DI == 128) return run_tc<128, true>(iq, ik, idx, nullptr, B, T, H, K, nullptr, 0, st, scores);
    return cudaErrorInvalidValue;
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

}  // namespace sgsa
