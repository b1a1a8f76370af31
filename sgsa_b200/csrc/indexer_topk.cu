// Causal top-k indexer and row top-k select.
//
// Selection rule (the contract of modelings/modeling_sgsa.py:144-165 and
// modelings/hybrid_dense_delta_topk.py:344-349, with a stated tie-break):
// row t keeps the min(K, t+1) largest scores among columns j <= t, equal
// scores ordered by the lower j first.  Output indices are ascending, the
// remaining slots are -1.
//
// Algorithm: one thread owns one query row.  An MSB-first radix select over
// the 32-bit order-preserving key of the fp32 score runs in up to four 8-bit
// digit passes; pass p counts, in a per-thread 256-bin histogram held in
// shared memory as hist[bin][thread] (bank = thread, so conflict free), the
// scores whose higher digits match the prefix chosen so far.  A row is
// resolved as soon as the chosen bin holds exactly the number of elements
// still needed.  A final pass emits, in index order, every column whose masked
// key is above the prefix plus the first `need` columns equal to it -- which
// is exactly the lowest-index tie-break.  Scores are recomputed in every pass
// (bit-identical, same code and order), so nothing of size T^2 is stored.
#include "common.cuh"

namespace sgsa {
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
    return cudaGetLastError();
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

cudaError_t launch_indexer_topk(const void *iq, const void *ik, int32_t *idx, int B, int T, int H,
                                int DI, int K, int dtype, cudaStream_t st) {
    if (dtype == SGSA_DTYPE_F32) return run_simt_d<float>(DI, iq, ik, idx, B, T, H, K, st);
    return run_simt_d<__nv_bfloat16>(DI, iq, ik, idx, B, T, H, K, st);
}

cudaError_t launch_topk_select(const float *scores, const int32_t *valid, int32_t *idx, int R,
                               int S, int K, cudaStream_t st) {
    const size_t smem = 256 * kRows * sizeof(uint32_t);
    cudaError_t e = cudaFuncSetAttribute(topk_select_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    topk_select_kernel<<<ceil_div(R, kRows), kRows, smem, st>>>(scores, valid, idx, R, S, K);
    return cudaGetLastError();
}

}  // namespace sgsa
