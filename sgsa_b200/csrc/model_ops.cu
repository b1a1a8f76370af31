// Elementwise kernels of the hybrid model around the SGSA layer: embedding rows,
// RMSNorm, the SwiGLU activation, RoPE of the dense layers' q/k, and the epilogue of
// the SGSA layer's fused input projection.  All are HBM-bound (one read and one write
// of each element); they move 16-byte vectors and compute in fp32 with one rounding.
//
// Reference modules (modelings/hybrid_dense_delta_topk.py): RMSNorm :97-106,
// SwiGLUMLP :109-119, _build_rope_cache / _apply_rope :127-151, embedding :447;
// SGSA layer projections follow SGSAStateLayer (modelings/modeling_sgsa.py:538-539)
// and HybridDeltaTopKAttention's mix gate (modelings/hybrid_dense_delta_topk.py:389).
#include "common.cuh"

namespace sgsa {
namespace {

__device__ __forceinline__ void ld8(const __nv_bfloat16 *p, float *x) {
    const uint4 u = *reinterpret_cast<const uint4 *>(p);
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void ld8(const float *p, float *x) {
    const float4 a = *reinterpret_cast<const float4 *>(p);
    const float4 b = *reinterpret_cast<const float4 *>(p + 4);
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
}
__device__ __forceinline__ void st8(__nv_bfloat16 *p, const float *x) {
    uint4 u;
    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    *reinterpret_cast<uint4 *>(p) = u;
}
__device__ __forceinline__ void st8(float *p, const float *x) {
    *reinterpret_cast<float4 *>(p) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4 *>(p + 4) = make_float4(x[4], x[5], x[6], x[7]);
}

__device__ __forceinline__ float warp_sum(float s) {
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

constexpr int kRowWarps = 8;

// out[r] = w * x[r] / sqrt(mean(x[r]^2) + eps); one warp per row, N % 8 == 0.
template <typename T>
__global__ void __launch_bounds__(kRowWarps * 32)
rmsnorm_kernel(const T *__restrict__ x, const T *__restrict__ w, T *__restrict__ out,
               long long rows, int N, float eps) {
    const int lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const T *xr = x + row * N;
    float ss = 0.f;
    for (int c = lane * 8; c < N; c += 256) {
        float v[8];
        ld8(xr + c, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
    }
    const float r = rsqrtf(warp_sum(ss) / (float)N + eps);
    T *orow = out + row * N;
    for (int c = lane * 8; c < N; c += 256) {
        float v[8], g[8];
        ld8(xr + c, v);
        ld8(w + c, g);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = g[e] * (v[e] * r);
        st8(orow + c, v);
    }
}

// out[r, i] = silu(gu[r, i]) * gu[r, I + i]   (gate and up projections side by side)
template <typename T>
__global__ void swiglu_kernel(const T *__restrict__ gu, T *__restrict__ out, long long rows,
                              int I) {
    const long long nv = rows * (I / 8);
    for (long long u = blockIdx.x * (long long)blockDim.x + threadIdx.x; u < nv;
         u += (long long)gridDim.x * blockDim.x) {
        const long long r = u / (I / 8);
        const int c = (int)(u - r * (I / 8)) * 8;
        float g[8], p[8];
        ld8(gu + r * 2 * I + c, g);
        ld8(gu + r * 2 * I + I + c, p);
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] = g[e] * sigmoidf_(g[e]) * p[e];
        st8(out + r * I + c, g);
    }
}

// qkv [B*T, 3*H*D] -> q, k (rotated) and v in [B, T, H, D].  cs[t][j] = (cos, sin) of
// position t and frequency j < D/2; each thread rotates 4 pairs (j, j + D/2).
template <typename T>
__global__ void rope_qkv_kernel(const T *__restrict__ qkv, const float2 *__restrict__ cs,
                                T *__restrict__ q, T *__restrict__ k, T *__restrict__ v,
                                long long rows, int T_, int H, int D, int pos0) {
    const int half = D / 2, per_head = half / 4;
    const long long n = rows * H * per_head;
    const int HD = H * D;
    for (long long u = blockIdx.x * (long long)blockDim.x + threadIdx.x; u < n;
         u += (long long)gridDim.x * blockDim.x) {
        const long long r = u / (H * per_head);
        const int rem = (int)(u - r * (H * per_head));
        const int h = rem / per_head, j = (rem - h * per_head) * 4;
        const int t = (int)(r % T_) + pos0;
        const T *src = qkv + r * 3 * HD + h * D;
        const long long o = r * HD + h * D;
        float c[4], s[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = cs[(long long)t * half + j + e];
            c[e] = f.x, s[e] = f.y;
        }
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const T *x = src + m * HD;
            T *y = m == 0 ? q : k;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float a = to_f32(x[j + e]), b = to_f32(x[j + half + e]);
                y[o + j + e] = from_f32<T>(a * c[e] - b * s[e]);
                y[o + j + half + e] = from_f32<T>(b * c[e] + a * s[e]);
            }
        }
        const T *xv = src + 2 * HD;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            v[o + j + e] = xv[j + e];
            v[o + j + half + e] = xv[j + half + e];
        }
    }
}

// The fused projection P [rows, ld] of an SGSA layer has the column blocks
// q | k | v | mix (H*D each) | iq | ik (H*DI each) | beta | gamma (H each):
// q, k -> l2-normalised per head, mix -> sigmoid, beta -> max(sigmoid, 1e-4),
// gamma -> sigmoid; v, iq, ik are copied.  One block of 8 warps per row.
template <typename T>
__global__ void __launch_bounds__(256)
sgsa_proj_kernel(const T *__restrict__ P, int ld, T *__restrict__ q, T *__restrict__ k,
                 T *__restrict__ v, T *__restrict__ mix, T *__restrict__ iq,
                 T *__restrict__ ik, T *__restrict__ beta, T *__restrict__ gamma, int H, int D,
                 int DI) {
    const long long r = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int HD = H * D, HI = H * DI;
    const T *p = P + r * ld;
    for (int u = warp; u < 2 * H; u += 8) {
        const int h = u % H;
        const T *src = p + (u < H ? 0 : HD) + h * D;
        T *dst = (u < H ? q : k) + r * HD + h * D;
        float ss = 0.f;
        for (int c = lane; c < D; c += 32) {
            const float x = to_f32(src[c]);
            ss = fmaf(x, x, ss);
        }
        const float inv = 1.f / fmaxf(sqrtf(warp_sum(ss)), 1e-12f);
        for (int c = lane; c < D; c += 32) dst[c] = from_f32<T>(to_f32(src[c]) * inv);
    }
    for (int c = threadIdx.x * 8; c < HD; c += 256 * 8) {
        float x[8];
        ld8(p + 2 * HD + c, x);
        st8(v + r * HD + c, x);
        ld8(p + 3 * HD + c, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = sigmoidf_(x[e]);
        st8(mix + r * HD + c, x);
    }
    for (int c = threadIdx.x * 8; c < HI; c += 256 * 8) {
        float x[8];
        ld8(p + 4 * HD + c, x);
        st8(iq + r * HI + c, x);
        ld8(p + 4 * HD + HI + c, x);
        st8(ik + r * HI + c, x);
    }
    if (threadIdx.x < H) {
        const int h = threadIdx.x;
        beta[r * H + h] = from_f32<T>(fmaxf(sigmoidf_(to_f32(p[4 * HD + 2 * HI + h])), 1e-4f));
        gamma[r * H + h] = from_f32<T>(sigmoidf_(to_f32(p[4 * HD + 2 * HI + H + h])));
    }
}

// out[r] = table[ids[r]]; ids outside [0, vocab) give a zero row.
template <typename T>
__global__ void embed_kernel(const int64_t *__restrict__ ids, const T *__restrict__ table,
                             T *__restrict__ out, long long rows, int N, int vocab) {
    const int per = N / 8;
    const long long n = rows * per;
    for (long long u = blockIdx.x * (long long)blockDim.x + threadIdx.x; u < n;
         u += (long long)gridDim.x * blockDim.x) {
        const long long r = u / per;
        const int c = (int)(u - r * per) * 8;
        const int64_t id = ids[r];
        float x[8];
        if (id >= 0 && id < vocab) {
            ld8(table + id * N + c, x);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = 0.f;
        }
        st8(out + r * N + c, x);
    }
}

unsigned grid_for(long long n, int threads) {
    long long g = (n + threads - 1) / threads;
    const long long cap = 148LL * 16;  // a few waves of resident blocks per SM
    return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

cudaError_t launch_rmsnorm(const void *x, const void *w, void *out, long long rows, int N,
                           float eps, int dtype, cudaStream_t st) {
    const unsigned grid = (unsigned)((rows + kRowWarps - 1) / kRowWarps);
    if (dtype == SGSA_DTYPE_F32)
        rmsnorm_kernel<float><<<grid, kRowWarps * 32, 0, st>>>((const float *)x, (const float *)w,
                                                               (float *)out, rows, N, eps);
    else
        rmsnorm_kernel<__nv_bfloat16><<<grid, kRowWarps * 32, 0, st>>>(
            (const __nv_bfloat16 *)x, (const __nv_bfloat16 *)w, (__nv_bfloat16 *)out, rows, N, eps);
    return launched();
}

cudaError_t launch_swiglu(const void *gu, void *out, long long rows, int I, int dtype,
                          cudaStream_t st) {
    const unsigned grid = grid_for(rows * (I / 8), 256);
    if (dtype == SGSA_DTYPE_F32)
        swiglu_kernel<float><<<grid, 256, 0, st>>>((const float *)gu, (float *)out, rows, I);
    else
        swiglu_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16 *)gu,
                                                           (__nv_bfloat16 *)out, rows, I);
    return launched();
}

cudaError_t launch_rope_qkv(const void *qkv, const float *cs, void *q, void *k, void *v, int B,
                            int T, int H, int D, int pos0, int dtype, cudaStream_t st) {
    const long long rows = (long long)B * T;
    const unsigned grid = grid_for(rows * H * (D / 8), 256);
    if (dtype == SGSA_DTYPE_F32)
        rope_qkv_kernel<float><<<grid, 256, 0, st>>>((const float *)qkv, (const float2 *)cs,
                                                     (float *)q, (float *)k, (float *)v, rows, T,
                                                     H, D, pos0);
    else
        rope_qkv_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
            (const __nv_bfloat16 *)qkv, (const float2 *)cs, (__nv_bfloat16 *)q,
            (__nv_bfloat16 *)k, (__nv_bfloat16 *)v, rows, T, H, D, pos0);
    return launched();
}

cudaError_t launch_sgsa_proj(const void *P, int ld, void *q, void *k, void *v, void *mix,
                             void *iq, void *ik, void *beta, void *gamma, long long rows, int H,
                             int D, int DI, int dtype, cudaStream_t st) {
    if (rows > 0x7fffffffLL) return cudaErrorInvalidValue;
    if (dtype == SGSA_DTYPE_F32)
        sgsa_proj_kernel<float><<<(unsigned)rows, 256, 0, st>>>(
            (const float *)P, ld, (float *)q, (float *)k, (float *)v, (float *)mix, (float *)iq,
            (float *)ik, (float *)beta, (float *)gamma, H, D, DI);
    else
        sgsa_proj_kernel<__nv_bfloat16><<<(unsigned)rows, 256, 0, st>>>(
            (const __nv_bfloat16 *)P, ld, (__nv_bfloat16 *)q, (__nv_bfloat16 *)k,
            (__nv_bfloat16 *)v, (__nv_bfloat16 *)mix, (__nv_bfloat16 *)iq, (__nv_bfloat16 *)ik,
            (__nv_bfloat16 *)beta, (__nv_bfloat16 *)gamma, H, D, DI);
    return launched();
}

cudaError_t launch_embed(const int64_t *ids, const void *table, void *out, long long rows, int N,
                         int vocab, int dtype, cudaStream_t st) {
    const unsigned grid = grid_for(rows * (N / 8), 256);
    if (dtype == SGSA_DTYPE_F32)
        embed_kernel<float><<<grid, 256, 0, st>>>(ids, (const float *)table, (float *)out, rows,
                                                  N, vocab);
    else
        embed_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
            ids, (const __nv_bfloat16 *)table, (__nv_bfloat16 *)out, rows, N, vocab);
    return launched();
}

}  // namespace sgsa
