// Sparse attention over the top-k rows of each query, fused with the gate.
//
//   o_s,t = sum_{j in I_t} softmax_j(q_t . k_j * scale) v_j        (fp32)
//   out_t = m_t * o_s,t + (1 - m_t) * o_delta,t
// as in modelings/hybrid_dense_delta_topk.py:343-356 (top-k softmax in fp32,
// row gather, weighted sum) and :389-390 (sigmoid gate mix), without
// materialising the [B,H,T,K,D] gather of the reference.
//
// One warp per (b, h, t).  Each half-warp gathers one selected row per step
// with 16-byte vector loads (a 128-wide bf16 row is 16 lanes x 16 B), so one
// warp keeps up to 16 k rows and 16 v rows in flight; the score is reduced over the
// half-warp with shuffles, and each half keeps its own online-softmax state
// (running max, sum, accumulator) that the two halves merge at the end.
#include <algorithm>

#include "common.cuh"

namespace sgsa {
namespace {

static __device__ unsigned int g_check;  // bounds-checked build only

constexpr int kWarps = 8;

template <typename T, int N>
struct VecLoad;
template <int N>
struct VecLoad<__nv_bfloat16, N> {  // N bf16 values (N in {2,4,8})
    __device__ __forceinline__ static void load(const __nv_bfloat16 *p, float *x) {
        if constexpr (N == 8) {
            uint4 r = __ldg(reinterpret_cast<const uint4 *>(p));
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&r);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float2 f = __bfloat1622float2(h[i]);
                x[2 * i] = f.x;
                x[2 * i + 1] = f.y;
            }
        } else if constexpr (N == 4) {
            uint2 r = __ldg(reinterpret_cast<const uint2 *>(p));
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&r);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                float2 f = __bfloat1622float2(h[i]);
                x[2 * i] = f.x;
                x[2 * i + 1] = f.y;
            }
        } else {
            uint32_t r = __ldg(reinterpret_cast<const unsigned int *>(p));
            float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&r));
            x[0] = f.x;
            x[1] = f.y;
        }
    }
};
template <int N>
struct VecLoad<float, N> {  // N floats (N in {2,4,8})
    __device__ __forceinline__ static void load(const float *p, float *x) {
        if constexpr (N % 4 == 0) {
#pragma unroll
            for (int i = 0; i < N / 4; ++i) {
                float4 r = __ldg(reinterpret_cast<const float4 *>(p) + i);
                x[4 * i] = r.x; x[4 * i + 1] = r.y; x[4 * i + 2] = r.z; x[4 * i + 3] = r.w;
            }
        } else {
            float2 r = __ldg(reinterpret_cast<const float2 *>(p));
            x[0] = r.x;
            x[1] = r.y;
        }
    }
};

// A row segment of one lane kept packed (as loaded) until it is used.
template <typename T, int EPL>
struct RawSeg {
    static constexpr int W = EPL * (int)sizeof(T) / 4;  // 32-bit words
    uint32_t w[W];
    __device__ __forceinline__ void load(const T *p) {
        if constexpr (W % 4 == 0) {
#pragma unroll
            for (int i = 0; i < W / 4; ++i) {
                const uint4 r = __ldg(reinterpret_cast<const uint4 *>(p) + i);
                w[4 * i] = r.x; w[4 * i + 1] = r.y; w[4 * i + 2] = r.z; w[4 * i + 3] = r.w;
            }
        } else if constexpr (W == 2) {
            const uint2 r = __ldg(reinterpret_cast<const uint2 *>(p));
            w[0] = r.x; w[1] = r.y;
        } else {
            w[0] = __ldg(reinterpret_cast<const unsigned int *>(p));
        }
    }
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int i = 0; i < W; ++i) w[i] = 0u;
    }
    __device__ __forceinline__ float get(int e) const {
        if constexpr (sizeof(T) == 4) {
            return __uint_as_float(w[e]);
        } else {
            const uint32_t x = w[e >> 1];
            return __uint_as_float((e & 1) ? (x & 0xffff0000u) : (x << 16));
        }
    }
};

// WITH_K: also accumulate the same softmax-weighted sum of the k rows into khat
// (the retrieval k_hat / v_hat of the sparse-write SGSA block).
template <typename T, int D, bool WITH_K = false>
__global__ void __launch_bounds__(kWarps * 32) sparse_attn_mix_kernel(
    const T *__restrict__ q, const T *__restrict__ k, const T *__restrict__ v,
    const int32_t *__restrict__ idx, const float *__restrict__ od, const T *__restrict__ mix,
    T *__restrict__ out, int B, int T_, int H, int K, float scale_log2, int mix_pc, int HI,
    T *__restrict__ khat = nullptr) {
    constexpr int EPL = D / 16;
    // rows per half-warp in flight: up to 8, bounded by ~64 registers of packed rows
    constexpr int kWords = EPL * (int)sizeof(T) / 4;
    constexpr int kU = (32 / kWords) < 8 ? (32 / kWords < 2 ? 2 : 32 / kWords) : 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int half = lane >> 4, hl = lane & 15;
    const long long qi = (long long)blockIdx.x * kWarps + warp;  // over [B*H*T]
    if (qi >= (long long)B * H * T_) return;
    const int t = (int)(qi % T_);
    const int bh = (int)(qi / T_);
    const int b = bh / H, h = bh % H;
    const size_t rowq = ((size_t)b * T_ + t) * H + h;
    const size_t kvstride = (size_t)H * D;
    const T *kb = k + ((size_t)b * T_ * H + h) * D + hl * EPL;
    const T *vb = v + ((size_t)b * T_ * H + h) * D + hl * EPL;

    float qv[EPL];
    VecLoad<T, EPL>::load(q + rowq * D + hl * EPL, qv);
#pragma unroll
    for (int e = 0; e < EPL; ++e) qv[e] *= scale_log2;

    const int32_t *ix = idx + (((size_t)b * HI + (HI == 1 ? 0 : h)) * T_ + t) * K;
    const int nsel = min(K, t + 1);
    float m = -INFINITY, l = 0.f, acc[EPL], acck[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = acck[e] = 0.f;

    for (int base = 0; base < nsel; base += 32) {
        const int cnt = min(32, nsel - base);
        const int my = (lane < cnt) ? __ldg(ix + base + lane) : 0;
        for (int p = 0; p < cnt; p += 2 * kU) {
            // issue every k and v row load of the group before any use
            RawSeg<T, EPL> kr[kU], vr[kU];
            int jr[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int slot = p + 2 * u + half;
                jr[u] = __shfl_sync(0xffffffffu, my, slot & 31);
                // out-of-range rows (caller-supplied indices) count as padding
                if (kCheckBuild && slot < cnt && (jr[u] < -1 || jr[u] >= T_))
                    SGSA_CHECK_FAIL(g_check, kChkGatherIndex);
                if (slot >= cnt || (unsigned)jr[u] >= (unsigned)T_) jr[u] = -1;
                if (jr[u] >= 0) {
                    kr[u].load(kb + (size_t)jr[u] * kvstride);
                    vr[u].load(vb + (size_t)jr[u] * kvstride);
                } else {
                    kr[u].zero();
                    vr[u].zero();
                }
            }
            float s[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                float d0 = 0.f;
#pragma unroll
                for (int e = 0; e < EPL; ++e) d0 = fmaf(qv[e], kr[u].get(e), d0);
#pragma unroll
                for (int off = 8; off > 0; off >>= 1) d0 += __shfl_xor_sync(0xffffffffu, d0, off);
                s[u] = (jr[u] >= 0) ? d0 : -INFINITY;
            }
            float mn = m;
#pragma unroll
            for (int u = 0; u < kU; ++u) mn = fmaxf(mn, s[u]);
            if (mn != -INFINITY) {
                const float corr = exp2f(m - mn);  // m == -inf gives 0
                l *= corr;
#pragma unroll
                for (int e = 0; e < EPL; ++e) {
                    acc[e] *= corr;
                    if (WITH_K) acck[e] *= corr;
                }
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const float pu = exp2f(s[u] - mn);
                    l += pu;
#pragma unroll
                    for (int e = 0; e < EPL; ++e) {
                        acc[e] = fmaf(pu, vr[u].get(e), acc[e]);
                        if (WITH_K) acck[e] = fmaf(pu, kr[u].get(e), acck[e]);
                    }
                }
                m = mn;
            }
        }
    }
    // merge the two half-warp states
    const float m2 = __shfl_xor_sync(0xffffffffu, m, 16);
    const float l2 = __shfl_xor_sync(0xffffffffu, l, 16);
    const float mt = fmaxf(m, m2);
    const float c1 = (m == -INFINITY) ? 0.f : exp2f(m - mt);
    const float c2 = (m2 == -INFINITY) ? 0.f : exp2f(m2 - mt);
    const float lt = l * c1 + l2 * c2;
    const float inv = (lt > 0.f) ? 1.f / lt : 0.f;
    float o[EPL], ok[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const float a2 = __shfl_xor_sync(0xffffffffu, acc[e], 16);
        o[e] = (acc[e] * c1 + a2 * c2) * inv;
        if (WITH_K) {
            const float b2 = __shfl_xor_sync(0xffffffffu, acck[e], 16);
            ok[e] = (acck[e] * c1 + b2 * c2) * inv;
        }
    }
    if (WITH_K && half == 0) {
        T *dk = khat + rowq * D + hl * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) dk[e] = from_f32<T>(ok[e]);
    }
    if (half == 0) {
        T *dst = out + rowq * D + hl * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
            float r = o[e];
            if (od) {
                const float mm = mix ? to_f32(mix_pc ? mix[rowq * D + hl * EPL + e] : mix[rowq]) : 1.f;
                r = mm * r + (1.f - mm) * od[rowq * D + hl * EPL + e];
            }
            dst[e] = from_f32<T>(r);
        }
    }
}

template <typename T, int D>
cudaError_t run(const void *q, const void *k, const void *v, const int32_t *idx, const float *od,
                const void *mix, void *out, int B, int T_, int H, int K, float scale, int mix_pc,
                int HI, cudaStream_t st) {
    const long long nq = (long long)B * H * T_;
    const unsigned grid = (unsigned)((nq + kWarps - 1) / kWarps);
    sparse_attn_mix_kernel<T, D><<<grid, kWarps * 32, 0, st>>>(
        (const T *)q, (const T *)k, (const T *)v, idx, od, (const T *)mix, (T *)out, B, T_, H, K,
        scale * 1.4426950408889634f, mix_pc, HI);
    return launched();
}

template <typename T>
cudaError_t run_d(int D, const void *q, const void *k, const void *v, const int32_t *idx,
                  const float *od, const void *mix, void *out, int B, int T_, int H, int K,
                  float scale, int mix_pc, int HI, cudaStream_t st) {
    switch (D) {
        case 32: return run<T, 32>(q, k, v, idx, od, mix, out, B, T_, H, K, scale, mix_pc, HI, st);
        case 64: return run<T, 64>(q, k, v, idx, od, mix, out, B, T_, H, K, scale, mix_pc, HI, st);
        case 128: return run<T, 128>(q, k, v, idx, od, mix, out, B, T_, H, K, scale, mix_pc, HI, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_sparse_attn_mix(const void *q, const void *k, const void *v,
                                   const int32_t *idx, const float *od, const void *mix,
                                   void *out, int B, int T, int H, int D, int K, float scale,
                                   int mix_pc, int dtype, int HI, cudaStream_t st) {
    if (dtype == SGSA_DTYPE_F32)
        return run_d<float>(D, q, k, v, idx, od, mix, out, B, T, H, K, scale, mix_pc, HI, st);
    return run_d<__nv_bfloat16>(D, q, k, v, idx, od, mix, out, B, T, H, K, scale, mix_pc, HI, st);
}

namespace {
template <typename T>
__global__ void gate_mix_kernel(const float *__restrict__ os, const float *__restrict__ od,
                                const T *__restrict__ mix, T *__restrict__ out, long long n, int D,
                                int mix_pc) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const float m = to_f32(mix_pc ? mix[i] : mix[i / D]);
        out[i] = from_f32<T>(m * os[i] + (1.f - m) * od[i]);
    }
}
}  // namespace

namespace {
template <typename T, int D>
cudaError_t run_retrieve(const void *q, const void *k, const void *v, const int32_t *idx,
                         void *khat, void *vhat, int B, int T_, int H, int K, float scale, int HI,
                         cudaStream_t st) {
    const long long nq = (long long)B * H * T_;
    const unsigned grid = (unsigned)((nq + kWarps - 1) / kWarps);
    sparse_attn_mix_kernel<T, D, true><<<grid, kWarps * 32, 0, st>>>(
        (const T *)q, (const T *)k, (const T *)v, idx, nullptr, nullptr, (T *)vhat, B, T_, H, K,
        scale * 1.4426950408889634f, 0, HI, (T *)khat);
    return launched();
}
}  // namespace

cudaError_t launch_sparse_retrieve(const void *q, const void *k, const void *v, const int32_t *idx,
                                   void *khat, void *vhat, int B, int T, int H, int D, int K,
                                   float scale, int HI, int dtype, cudaStream_t st) {
    if (dtype == SGSA_DTYPE_F32) {
        if (D == 32) return run_retrieve<float, 32>(q, k, v, idx, khat, vhat, B, T, H, K, scale, HI, st);
        if (D == 64) return run_retrieve<float, 64>(q, k, v, idx, khat, vhat, B, T, H, K, scale, HI, st);
        if (D == 128) return run_retrieve<float, 128>(q, k, v, idx, khat, vhat, B, T, H, K, scale, HI, st);
    } else {
        if (D == 32) return run_retrieve<__nv_bfloat16, 32>(q, k, v, idx, khat, vhat, B, T, H, K, scale, HI, st);
        if (D == 64) return run_retrieve<__nv_bfloat16, 64>(q, k, v, idx, khat, vhat, B, T, H, K, scale, HI, st);
        if (D == 128) return run_retrieve<__nv_bfloat16, 128>(q, k, v, idx, khat, vhat, B, T, H, K, scale, HI, st);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_gate_mix(const float *os, const float *od, const void *mix, void *out,
                            long long rows, int D, int mix_pc, int dtype, cudaStream_t st) {
    const long long n = rows * D;
    const int grid = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
    if (dtype == SGSA_DTYPE_F32)
        gate_mix_kernel<float><<<grid, 256, 0, st>>>(os, od, (const float *)mix, (float *)out, n, D, mix_pc);
    else
        gate_mix_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(os, od, (const __nv_bfloat16 *)mix,
                                                             (__nv_bfloat16 *)out, n, D, mix_pc);
    return launched();
}

unsigned int check_word_gather(bool reset) {
    unsigned int v = 0, z = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyFromSymbol(&v, g_check, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (reset && v) cudaMemcpyToSymbol(g_check, &z, sizeof(z));
    return v;
}

}  // namespace sgsa
