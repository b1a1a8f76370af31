// Recurrent SGSA and the decode-time pieces of the layer.
//
// * recurrent_sgsa_kernel: the token-by-token recurrence of
//   modelings/sgsa_ops/naive.py:39-55 (the semantics of fused_recurrent_sgsa,
//   modelings/sgsa_ops/recurrent.py:138-175, whose Triton forward is
//   recurrent_fwd_triton.py:19-87).  One CTA per (b, h), one thread per state
//   column v: the column S[:, v] (D fp32 values) lives in registers for the
//   whole sequence; each token's k / q / sparse_k are staged in shared memory
//   and read as broadcasts.  A decode step is the T = 1 case.
// * decode_topk_kernel: top-k of one query row against an indexer key cache,
//   the decode form of the causal indexer (one CTA per (b, h); the row's scores
//   live in shared memory; block-wide radix select; ordered compaction with the
//   lowest-index tie-break).
// * decode_attn_kernel: softmax attention of one query over its selected cache
//   rows plus the gate (one CTA per (b, h), 8 warps split the rows, online
//   softmax states merged through shared memory).
#include <algorithm>

#include "common.cuh"

namespace sgsa {
namespace {

static __device__ unsigned int g_check;  // bounds-checked build only

// Load 8 consecutive elements (16 bytes of bf16, 32 of fp32) as floats.
__device__ __forceinline__ void load8(const __nv_bfloat16 *p, float *x) {
    const uint4 r = __ldg(reinterpret_cast<const uint4 *>(p));
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void load8(const float *p, float *x) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

// ---------------------------------------------------------------- recurrence
template <typename Tin, typename Tout, int D>
__global__ void __launch_bounds__(D) recurrent_sgsa_kernel(
    const Tin *__restrict__ q, const Tin *__restrict__ k, const Tin *__restrict__ v,
    const Tin *__restrict__ beta, const Tin *__restrict__ gamma, const Tin *__restrict__ sk,
    const Tin *__restrict__ sv, const Tin *__restrict__ alpha, const float *__restrict__ s0,
    Tout *__restrict__ o, float *__restrict__ sT, int T, int H) {
    __shared__ __align__(16) float sh[2][3][D];  // [buffer][k | q | sparse_k][d]
    __shared__ float sc[2][3];                   // [buffer][gamma | beta | alpha]
    const int e = threadIdx.x, bh = blockIdx.x, b = bh / H, h = bh % H;
    const bool sparse = sk != nullptr;
    float col[D];
#pragma unroll
    for (int d = 0; d < D; ++d) col[d] = s0 ? s0[((size_t)bh * D + d) * D + e] : 0.f;
    auto stage = [&](int t, int buf) {
        const size_t row = ((size_t)b * T + t) * H + h;
        sh[buf][0][e] = to_f32(k[row * D + e]);
        sh[buf][1][e] = to_f32(q[row * D + e]);
        if (sparse) sh[buf][2][e] = to_f32(sk[row * D + e]);
        if (e == 0) {
            sc[buf][0] = to_f32(gamma[row]);
            sc[buf][1] = to_f32(beta[row]);
            sc[buf][2] = sparse ? to_f32(alpha[row]) : 0.f;
        }
    };
    if (T > 0) stage(0, 0);
    __syncthreads();
    for (int t = 0; t < T; ++t) {
        const int buf = t & 1;
        const size_t row = ((size_t)b * T + t) * H + h;
        const float vv = to_f32(v[row * D + e]);
        const float svv = sparse ? to_f32(sv[row * D + e]) : 0.f;
        if (t + 1 < T) stage(t + 1, buf ^ 1);
        const float g = sc[buf][0], bt = sc[buf][1], al = sc[buf][2];
        const float *kk = sh[buf][0], *qq = sh[buf][1], *ss = sh[buf][2];
        // predictions read the decayed base state gamma * S (both writes read the same base)
        float pl = 0.f, ps = 0.f;
#pragma unroll
        for (int d = 0; d < D; ++d) pl = fmaf(col[d], kk[d], pl);
        if (sparse) {
#pragma unroll
            for (int d = 0; d < D; ++d) ps = fmaf(col[d], ss[d], ps);
        }
        const float dl = (vv - g * pl) * bt;
        const float ds = sparse ? (svv - g * ps) * al : 0.f;
        float out = 0.f;
#pragma unroll
        for (int d = 0; d < D; ++d) {
            float x = fmaf(kk[d], dl, g * col[d]);
            if (sparse) x = fmaf(ss[d], ds, x);
            col[d] = x;
            out = fmaf(x, qq[d], out);
        }
        o[row * D + e] = from_f32<Tout>(out);
        __syncthreads();
    }
    if (sT) {
#pragma unroll
        for (int d = 0; d < D; ++d) sT[((size_t)bh * D + d) * D + e] = col[d];
    }
}

// ------------------------------------------------------------- decode top-k
constexpr int kTopkThreads = 1024;

template <typename Tin, int DI>
__global__ void __launch_bounds__(kTopkThreads) decode_topk_kernel(
    const Tin *__restrict__ iq, const Tin *__restrict__ ikc, int32_t *__restrict__ idx, int H,
    int Tc, int n, int K) {
    extern __shared__ __align__(16) uint32_t keys[];  // n order-preserving score keys
    __shared__ uint32_t hist[256];
    __shared__ int s_scan[kTopkThreads];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_need, s_done;
    __shared__ float s_q[DI];
    const int tid = threadIdx.x, bh = blockIdx.x, b = bh / H, h = bh % H;
    int32_t *out = idx + (size_t)bh * K;
    if (n <= K) {  // every cached key is selected
        for (int i = tid; i < K; i += kTopkThreads) out[i] = (i < n) ? i : -1;
        return;
    }
    if (tid < DI) s_q[tid] = to_f32(iq[(size_t)bh * DI + tid]);
    __syncthreads();
    {
        // Scores: DI / 8 lanes per cached row, one 16-byte load each (a row's DI values
        // in one coalesced request; rows of one head are H * DI elements apart), the
        // partial dots summed by xor shuffles; kU rows per lane group in flight.
        constexpr int G = DI / 8, RPW = 32 / G, kU = 4;
        const int warp = tid >> 5, lane = tid & 31, sub = lane % G, r0 = lane / G;
        constexpr int step = (kTopkThreads / 32) * RPW;
        float qv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) qv[i] = s_q[sub * 8 + i];
        const Tin *base = ikc + ((size_t)b * Tc * H + h) * DI + sub * 8;
        for (int jb = warp * RPW; jb < n; jb += step * kU) {  // warp-uniform
            float x[kU][8];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int j = jb + u * step + r0;
                if (j < n) {
                    load8(base + (size_t)j * H * DI, x[u]);
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) x[u][i] = 0.f;
                }
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                float s = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) s = fmaf(qv[i], x[u][i], s);
#pragma unroll
                for (int off = G / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
                const int j = jb + u * step + r0;
                if (sub == 0 && j < n) keys[j] = float_key(s);
            }
        }
    }
    if (tid == 0) { s_prefix = 0u; s_mask = 0u; s_need = K; s_done = 0; }
    __syncthreads();
    for (int shift = 24; shift >= 0 && !s_done; shift -= 8) {
        for (int i = tid; i < 256; i += kTopkThreads) hist[i] = 0u;
        __syncthreads();
        const uint32_t pre = s_prefix, msk = s_mask;
        for (int j = tid; j < n; j += kTopkThreads) {
            const uint32_t u = keys[j];
            if ((u & msk) == pre) atomicAdd(&hist[(u >> shift) & 0xffu], 1u);
        }
        __syncthreads();
        if (tid < 32) {
            const int lane = tid;
            // the bin that holds the need-th largest key: lane l sums bins 255-8l .. 248-8l,
            // an inclusive scan over lanes from the top, the first lane that reaches
            // `need` walks its eight bins
            const int need = s_need;
            uint32_t c[8];
            int tot = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) { c[i] = hist[255 - 8 * lane - i]; tot += (int)c[i]; }
            int incl = tot;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += y;
            }
            const uint32_t hit = __ballot_sync(0xffffffffu, incl >= need);
            const int total = __shfl_sync(0xffffffffu, incl, 31);
            const int L = hit ? __ffs(hit) - 1 : -1;
            if (L < 0) {  // not reached (the active keys number at least `need`): bin 0
                if (lane == 0) {
                    s_need = need - total;
                    s_mask |= 0xffu << shift;
                    if ((int)hist[0] == s_need) s_done = 1;
                }
            } else if (lane == L) {
                int cum = incl - tot, chosen = 0, cnt = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (cum + (int)c[i] >= need) { chosen = 255 - 8 * lane - i; cnt = (int)c[i]; break; }
                    cum += (int)c[i];
                }
                s_need = need - cum;
                s_prefix |= (uint32_t)chosen << shift;
                s_mask |= 0xffu << shift;
                if (cnt == s_need) s_done = 1;
            }
        }
        __syncthreads();
    }
    // Ordered compaction: warp w owns the contiguous index segment [lo, hi) and reads it
    // 32 consecutive keys at a time (lane i the i-th: no bank conflicts).  Pass 1 counts the
    // keys above the threshold prefix (gt) and equal to it (eq) per warp; after one exchange
    // of the warp totals, pass 2 emits in index order, the equal keys by rank (lowest
    // indices first) while fewer than `need` have been taken.
    {
        constexpr int kWarps = kTopkThreads / 32;
        const uint32_t pre = s_prefix, msk = s_mask;
        const int need = s_need;
        const int warp = tid >> 5, lane = tid & 31;
        const uint32_t lt = (1u << lane) - 1u;
        const int seg = (n + kWarps - 1) / kWarps;
        const int lo = min(n, warp * seg), hi = min(n, lo + seg);
        int gt = 0, eq = 0;
        for (int j0 = lo; j0 < hi; j0 += 32) {
            const int j = j0 + lane;
            const uint32_t m = j < hi ? (keys[j] & msk) : 0u;
            gt += __popc(__ballot_sync(0xffffffffu, j < hi && m > pre));
            eq += __popc(__ballot_sync(0xffffffffu, j < hi && m == pre));
        }
        if (lane == 0) { s_scan[2 * warp] = gt; s_scan[2 * warp + 1] = eq; }
        __syncthreads();
        int eq_before = 0, out_before = 0;
        for (int w = 0; w < warp; ++w) {
            const int g = s_scan[2 * w], e = s_scan[2 * w + 1];
            out_before += g + max(0, min(e, need - eq_before));
            eq_before += e;
        }
        int pos = out_before, eq_rank = eq_before;
        for (int j0 = lo; j0 < hi; j0 += 32) {
            const int j = j0 + lane;
            const uint32_t m = j < hi ? (keys[j] & msk) : 0u;
            const bool is_gt = j < hi && m > pre, is_eq = j < hi && m == pre;
            const uint32_t eqb = __ballot_sync(0xffffffffu, is_eq);
            const bool take = is_gt || (is_eq && eq_rank + __popc(eqb & lt) < need);
            const uint32_t tb = __ballot_sync(0xffffffffu, take);
            if (take) out[pos + __popc(tb & lt)] = j;
            pos += __popc(tb);
            eq_rank += __popc(eqb);
        }
    }
}

// ------------------------------------------------------------ cache append
// Row `pos` of the k, v and indexer-key caches from this token's k, v and ik, every batch
// row, in one launch: 16-byte vectors, 64-bit row offsets (a [B, Tc, H, D] cache passes 2^31
// elements at configs[4] sizes).
__global__ void __launch_bounds__(256)
decode_append_kernel(uint4 *__restrict__ kc, uint4 *__restrict__ vc, uint4 *__restrict__ ikc,
                     const uint4 *__restrict__ k, const uint4 *__restrict__ v,
                     const uint4 *__restrict__ ik, int B, long long Tc, int nkv, int nik,
                     long long pos) {
    const long long per = 2LL * nkv + nik, n = (long long)B * per;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (long long)gridDim.x * blockDim.x) {
        const long long b = e / per, x = e - b * per, row = b * Tc + pos;
        if (x < nkv) kc[row * nkv + x] = k[b * nkv + x];
        else if (x < 2 * nkv) vc[row * nkv + x - nkv] = v[b * nkv + x - nkv];
        else ikc[row * nik + x - 2 * nkv] = ik[b * nik + x - 2 * nkv];
    }
}

// ------------------------------------------------------- decode attention
constexpr int kAttnWarps = 4;  // 4 measured faster than 8 or 16 at configs[4]
static_assert(kAttnWarps * 32 >= 128, "the merge writes output column c from thread c (D <= 128)");

template <typename T, int D>
__global__ void __launch_bounds__(kAttnWarps * 32) decode_attn_kernel(
    const T *__restrict__ q, const T *__restrict__ kc, const T *__restrict__ vc,
    const int32_t *__restrict__ idx, const float *__restrict__ od, const T *__restrict__ mix,
    T *__restrict__ out, int H, int Tc, int K, float scale_log2, int mix_pc) {
    constexpr int EPL = D / 16;
    __shared__ float s_m[kAttnWarps * 2], s_l[kAttnWarps * 2];
    __shared__ float s_acc[kAttnWarps * 2][D];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = lane >> 4, hl = lane & 15;
    const int bh = blockIdx.x, b = bh / H, h = bh % H;
    const size_t stride = (size_t)H * D;
    const T *kb = kc + ((size_t)b * Tc * H + h) * D + hl * EPL;
    const T *vb = vc + ((size_t)b * Tc * H + h) * D + hl * EPL;
    float qv[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) qv[e] = to_f32(q[(size_t)bh * D + hl * EPL + e]) * scale_log2;
    const int32_t *ix = idx + (size_t)bh * K;
    float m = -INFINITY, l = 0.f, acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
    // slot s is handled by warp (s / 2) % kAttnWarps, half s % 2, in increasing order; each
    // iteration takes kRowsU of a half's slots, their index loads first, then all their k and
    // v rows, so that the gathers of kRowsU rows are in flight together.  Both halves of a
    // warp run the same number of iterations (the shuffles need the whole warp).
    constexpr int kRowsU = 2, kStep = 2 * kAttnWarps;
    for (int base = 2 * warp; base < K; base += kStep * kRowsU) {
        int js[kRowsU];
#pragma unroll
        for (int u = 0; u < kRowsU; ++u) {
            const int s = base + u * kStep + half;
            int j = (s < K) ? ix[s] : -1;
            if (kCheckBuild && s < K && (j < -1 || j >= Tc)) SGSA_CHECK_FAIL(g_check, kChkDecodeIndex);
            if ((unsigned)j >= (unsigned)Tc) j = -1;  // out-of-range rows count as padding
            js[u] = j;
        }
        float kr[kRowsU][EPL], vr[kRowsU][EPL];
#pragma unroll
        for (int u = 0; u < kRowsU; ++u) {
            const int j = js[u];
            if (j >= 0) {
                if constexpr (EPL == 8) {
                    load8(kb + (size_t)j * stride, kr[u]);
                    load8(vb + (size_t)j * stride, vr[u]);
                } else {
#pragma unroll
                    for (int e = 0; e < EPL; ++e) {
                        kr[u][e] = to_f32(kb[(size_t)j * stride + e]);
                        vr[u][e] = to_f32(vb[(size_t)j * stride + e]);
                    }
                }
            } else {
#pragma unroll
                for (int e = 0; e < EPL; ++e) kr[u][e] = vr[u][e] = 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < kRowsU; ++u) {
            float d0 = 0.f;
#pragma unroll
            for (int e = 0; e < EPL; ++e) d0 = fmaf(qv[e], kr[u][e], d0);
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) d0 += __shfl_xor_sync(0xffffffffu, d0, off);
            if (js[u] >= 0) {
                const float mn = fmaxf(m, d0);
                const float c = (m == -INFINITY) ? 0.f : exp2f(m - mn);
                const float p = exp2f(d0 - mn);
                l = l * c + p;
#pragma unroll
                for (int e = 0; e < EPL; ++e) acc[e] = fmaf(p, vr[u][e], acc[e] * c);
                m = mn;
            }
        }
    }
    const int slot = warp * 2 + half;
    if (hl == 0) {
        s_m[slot] = m;
        s_l[slot] = l;
    }
#pragma unroll
    for (int e = 0; e < EPL; ++e) s_acc[slot][hl * EPL + e] = acc[e];
    __syncthreads();
    if (threadIdx.x < D) {
        const int c = threadIdx.x;
        float mt = -INFINITY;
        for (int i = 0; i < 2 * kAttnWarps; ++i) mt = fmaxf(mt, s_m[i]);
        float lt = 0.f, o = 0.f;
        for (int i = 0; i < 2 * kAttnWarps; ++i) {
            if (s_m[i] == -INFINITY) continue;
            const float f = exp2f(s_m[i] - mt);
            lt += s_l[i] * f;
            o += s_acc[i][c] * f;
        }
        float r = (lt > 0.f) ? o / lt : 0.f;
        if (od) {
            const float mm = mix ? to_f32(mix_pc ? mix[(size_t)bh * D + c] : mix[bh]) : 1.f;
            r = mm * r + (1.f - mm) * od[(size_t)bh * D + c];
        }
        out[(size_t)bh * D + c] = from_f32<T>(r);
    }
}

template <typename Tin, typename Tout, int D>
cudaError_t run_rec(const void *q, const void *k, const void *v, const void *beta,
                    const void *gamma, const void *sk, const void *sv, const void *alpha,
                    const float *s0, void *o, float *sT, int B, int T, int H, cudaStream_t st) {
    recurrent_sgsa_kernel<Tin, Tout, D><<<B * H, D, 0, st>>>(
        (const Tin *)q, (const Tin *)k, (const Tin *)v, (const Tin *)beta, (const Tin *)gamma,
        (const Tin *)sk, (const Tin *)sv, (const Tin *)alpha, s0, (Tout *)o, sT, T, H);
    return launched();
}

template <typename Tin, typename Tout>
cudaError_t run_rec_d(int D, const void *q, const void *k, const void *v, const void *beta,
                      const void *gamma, const void *sk, const void *sv, const void *alpha,
                      const float *s0, void *o, float *sT, int B, int T, int H,
                      cudaStream_t st) {
    switch (D) {
        case 32: return run_rec<Tin, Tout, 32>(q, k, v, beta, gamma, sk, sv, alpha, s0, o, sT, B, T, H, st);
        case 64: return run_rec<Tin, Tout, 64>(q, k, v, beta, gamma, sk, sv, alpha, s0, o, sT, B, T, H, st);
        case 128: return run_rec<Tin, Tout, 128>(q, k, v, beta, gamma, sk, sv, alpha, s0, o, sT, B, T, H, st);
        default: return cudaErrorInvalidValue;
    }
}

template <typename Tin, int DI>
cudaError_t run_topk(const void *iq, const void *ikc, int32_t *idx, int B, int H, int Tc, int n,
                     int K, cudaStream_t st) {
    const size_t smem = (size_t)max(n, 1) * 4;
    auto kern = decode_topk_kernel<Tin, DI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<B * H, kTopkThreads, smem, st>>>((const Tin *)iq, (const Tin *)ikc, idx, H, Tc, n, K);
    return launched();
}

template <typename T, int D>
cudaError_t run_dattn(const void *q, const void *kc, const void *vc, const int32_t *idx,
                      const float *od, const void *mix, void *out, int B, int H, int Tc, int K,
                      float scale, int mix_pc, cudaStream_t st) {
    decode_attn_kernel<T, D><<<B * H, kAttnWarps * 32, 0, st>>>(
        (const T *)q, (const T *)kc, (const T *)vc, idx, od, (const T *)mix, (T *)out, H, Tc, K,
        scale * 1.4426950408889634f, mix_pc);
    return launched();
}

}  // namespace

constexpr int kDecodeMaxCache = 54 * 1024;  // scores of one row in shared memory (+ static, <= 227 KB)

int decode_max_cache() { return kDecodeMaxCache; }

cudaError_t launch_recurrent(const void *q, const void *k, const void *v, const void *beta,
                             const void *gamma, const void *sk, const void *sv, const void *alpha,
                             const float *s0, void *o, float *sT, int B, int T, int H, int D,
                             int dtype, bool out_f32, cudaStream_t st) {
    if (dtype == SGSA_DTYPE_F32)
        return run_rec_d<float, float>(D, q, k, v, beta, gamma, sk, sv, alpha, s0, o, sT, B, T, H, st);
    if (out_f32)
        return run_rec_d<__nv_bfloat16, float>(D, q, k, v, beta, gamma, sk, sv, alpha, s0, o, sT, B, T, H, st);
    return run_rec_d<__nv_bfloat16, __nv_bfloat16>(D, q, k, v, beta, gamma, sk, sv, alpha, s0, o, sT, B, T, H, st);
}

cudaError_t launch_decode_topk(const void *iq, const void *ikc, int32_t *idx, int B, int H,
                               int Tc, int n, int DI, int K, int dtype, cudaStream_t st) {
    if (dtype == SGSA_DTYPE_F32) {
        if (DI == 32) return run_topk<float, 32>(iq, ikc, idx, B, H, Tc, n, K, st);
        if (DI == 64) return run_topk<float, 64>(iq, ikc, idx, B, H, Tc, n, K, st);
        if (DI == 128) return run_topk<float, 128>(iq, ikc, idx, B, H, Tc, n, K, st);
    } else {
        if (DI == 32) return run_topk<__nv_bfloat16, 32>(iq, ikc, idx, B, H, Tc, n, K, st);
        if (DI == 64) return run_topk<__nv_bfloat16, 64>(iq, ikc, idx, B, H, Tc, n, K, st);
        if (DI == 128) return run_topk<__nv_bfloat16, 128>(iq, ikc, idx, B, H, Tc, n, K, st);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_decode_attn(const void *q, const void *kc, const void *vc, const int32_t *idx,
                               const float *od, const void *mix, void *out, int B, int H, int Tc,
                               int D, int K, float scale, int mix_pc, int dtype, cudaStream_t st) {
    if (dtype == SGSA_DTYPE_F32) {
        if (D == 32) return run_dattn<float, 32>(q, kc, vc, idx, od, mix, out, B, H, Tc, K, scale, mix_pc, st);
        if (D == 64) return run_dattn<float, 64>(q, kc, vc, idx, od, mix, out, B, H, Tc, K, scale, mix_pc, st);
        if (D == 128) return run_dattn<float, 128>(q, kc, vc, idx, od, mix, out, B, H, Tc, K, scale, mix_pc, st);
    } else {
        if (D == 32) return run_dattn<__nv_bfloat16, 32>(q, kc, vc, idx, od, mix, out, B, H, Tc, K, scale, mix_pc, st);
        if (D == 64) return run_dattn<__nv_bfloat16, 64>(q, kc, vc, idx, od, mix, out, B, H, Tc, K, scale, mix_pc, st);
        if (D == 128) return run_dattn<__nv_bfloat16, 128>(q, kc, vc, idx, od, mix, out, B, H, Tc, K, scale, mix_pc, st);
    }
    return cudaErrorInvalidValue;
}

unsigned int check_word_decode(bool reset) {
    unsigned int v = 0, z = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyFromSymbol(&v, g_check, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (reset && v) cudaMemcpyToSymbol(g_check, &z, sizeof(z));
    return v;
}

cudaError_t launch_decode_append(void *kc, void *vc, void *ikc, const void *k, const void *v,
                                 const void *ik, int B, int Tc, int H, int D, int DI, int pos,
                                 int elem_bytes, cudaStream_t st) {
    const int nkv = H * D * elem_bytes / 16, nik = H * DI * elem_bytes / 16;
    const long long n = (long long)B * (2LL * nkv + nik);
    const int grid = (int)std::min<long long>((n + 255) / 256, 148LL * 8);
    decode_append_kernel<<<grid, 256, 0, st>>>((uint4 *)kc, (uint4 *)vc, (uint4 *)ikc,
                                                (const uint4 *)k, (const uint4 *)v,
                                                (const uint4 *)ik, B, Tc, nkv, nik, pos);
    return launched();
}

}  // namespace sgsa
