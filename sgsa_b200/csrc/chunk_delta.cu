// Chunked SGSA / gated-delta-rule forward (CUDA-core fp32 path).
//
// Chunk algebra (chunk of C=64 tokens, M virtual samples: M = C, or 2C when a
// sparse write interleaves (k_t, sparse_k_t) as in
// modelings/sgsa_ops/chunk_fwd.py:49-56).  With G_t the inclusive cumulative
// sum of log(gamma) inside the chunk and tau_m the token of sample m:
//   A[i][j]  = [tau_j < tau_i] lam_i exp(G_tau_i - G_tau_j) <kap_i, kap_j>
//   W        = (I + A)^-1 diag(lam exp(G_tau)) Kap       [M x D]
//   Uh       = (I + A)^-1 diag(lam) Nu                   [M x D]
//   Aqk[t,m] = [tau_m <= t] exp(G_t - G_tau_m) <q_t, kap_m>
// and, carried across chunks with the state S [D x D]:
//   U   = Uh - W S
//   O   = diag(exp(G)) Q S + Aqk U
//   S'  = exp(G_last) S + Kap~^T U,   Kap~_m = exp(G_last - G_tau_m) kap_m
// This is the residual system (I+T)R = B of chunk_fwd.py:73-89 written with
// U = lam R and log-space decay differences (never a ratio of cumprods, so the
// clamp_min(1e-6) of chunk_fwd.py:86,110,121 is not needed), and the WY form of
// modelings/gated_delta_rule/chunk.py:32-117.  Semantics are those of
// naive_recurrent_sgsa (modelings/sgsa_ops/naive.py:39-55).
//
// Kernel 1 (chunk_prep) runs every chunk in parallel and writes W, Uh, Aqk and G
// to the workspace; kernel 2 (chunk_scan) walks the chunks of one (b, h) in
// order, one CTA per 32-column slice of the state, the slice held in shared
// memory in fp32.
#include "common.cuh"

namespace sgsa {
namespace {

constexpr int kC = 64;
constexpr int kThreads = 256;
constexpr int kBV = 32;

struct ChunkArgs {
    const void *q, *k, *v, *beta, *gamma, *sk, *sv, *alpha;
    const float *s0;
    void *o;
    float *sT;
    int B, T, H, NC;
    float *W, *U, *Aqk, *G;
};

template <int D, bool SPARSE>
struct Dims {
    static constexpr int M = SPARSE ? 2 * kC : kC;
    static constexpr int LD = D + 1;
    static constexpr size_t prep_smem = (size_t)(2 * M * LD + M * (M + 1)) * sizeof(float);
    static constexpr size_t scan_smem =
        (size_t)(M * D + kC * D + kC * M + D * kBV + M * kBV) * sizeof(float);
};

template <typename Tin, int D, bool SPARSE>
__global__ void __launch_bounds__(kThreads) chunk_prep_kernel(ChunkArgs a) {
    using Dm = Dims<D, SPARSE>;
    constexpr int M = Dm::M, LD = Dm::LD;
    extern __shared__ float smem[];
    float *KW = smem;           // M x LD   kap, then W
    float *VU = KW + M * LD;    // M x LD   q (C rows), then nu, then Uh
    float *A = VU + M * LD;     // M x (M+1)
    __shared__ float sG[kC];
    __shared__ float sLam[M];

    const int c = blockIdx.x, bh = blockIdx.y;
    const int b = bh / a.H, h = bh % a.H;
    const int t0 = c * kC;
    const int L = min(kC, a.T - t0);
    const int tid = threadIdx.x;
    const Tin *q = (const Tin *)a.q, *k = (const Tin *)a.k, *v = (const Tin *)a.v;
    const Tin *beta = (const Tin *)a.beta, *gamma = (const Tin *)a.gamma;
    const Tin *sk = (const Tin *)a.sk, *sv = (const Tin *)a.sv, *alpha = (const Tin *)a.alpha;
    auto row = [&](int t) -> size_t { return ((size_t)b * a.T + t0 + t) * a.H + h; };

    if (tid < kC) sG[tid] = (tid < L) ? logf(to_f32(gamma[row(tid)])) : 0.f;
    for (int m = tid; m < M; m += kThreads) {
        const int tau = SPARSE ? (m >> 1) : m;
        float lam = 0.f;
        if (tau < L) lam = (SPARSE && (m & 1)) ? to_f32(alpha[row(tau)]) : to_f32(beta[row(tau)]);
        sLam[m] = lam;
    }
    for (int e = tid; e < M * D; e += kThreads) {
        const int m = e / D, d = e % D;
        const int tau = SPARSE ? (m >> 1) : m;
        float x = 0.f;
        if (tau < L) x = to_f32(((SPARSE && (m & 1)) ? sk : k)[row(tau) * D + d]);
        KW[m * LD + d] = x;
    }
    for (int e = tid; e < kC * D; e += kThreads) {
        const int t = e / D, d = e % D;
        VU[t * LD + d] = (t < L) ? to_f32(q[row(t) * D + d]) : 0.f;
    }
    __syncthreads();
    if (tid < 32) {  // inclusive prefix sum of log(gamma), two tokens per lane
        const float x0 = sG[2 * tid], x1 = sG[2 * tid + 1];
        float s = x0 + x1;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, s, off);
            if (tid >= off) s += y;
        }
        const float ex = s - (x0 + x1);
        sG[2 * tid] = ex + x0;
        sG[2 * tid + 1] = ex + x0 + x1;
    }
    __syncthreads();

    const int ti = tid & 15, tj = tid >> 4;
    {   // A = strictly-earlier-token transition
        constexpr int R = M / 16;
        float acc[R][R];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int s = 0; s < R; ++s) acc[r][s] = 0.f;
        for (int d = 0; d < D; ++d) {
            float ki[R], kj[R];
#pragma unroll
            for (int r = 0; r < R; ++r) ki[r] = KW[(ti + 16 * r) * LD + d];
#pragma unroll
            for (int s = 0; s < R; ++s) kj[s] = KW[(tj + 16 * s) * LD + d];
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int s = 0; s < R; ++s) acc[r][s] = fmaf(ki[r], kj[s], acc[r][s]);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = ti + 16 * r, taui = SPARSE ? (i >> 1) : i;
#pragma unroll
            for (int s = 0; s < R; ++s) {
                const int j = tj + 16 * s, tauj = SPARSE ? (j >> 1) : j;
                float val = 0.f;
                if (tauj < taui) val = sLam[i] * __expf(sG[taui] - sG[tauj]) * acc[r][s];
                A[i * (M + 1) + j] = val;
            }
        }
    }
    {   // Aqk (query rows are held in VU)
        constexpr int RT = kC / 16, RM = M / 16;
        float acc[RT][RM];
#pragma unroll
        for (int r = 0; r < RT; ++r)
#pragma unroll
            for (int s = 0; s < RM; ++s) acc[r][s] = 0.f;
        for (int d = 0; d < D; ++d) {
            float qi[RT], kj[RM];
#pragma unroll
            for (int r = 0; r < RT; ++r) qi[r] = VU[(ti + 16 * r) * LD + d];
#pragma unroll
            for (int s = 0; s < RM; ++s) kj[s] = KW[(tj + 16 * s) * LD + d];
#pragma unroll
            for (int r = 0; r < RT; ++r)
#pragma unroll
                for (int s = 0; s < RM; ++s) acc[r][s] = fmaf(qi[r], kj[s], acc[r][s]);
        }
        float *aqk = a.Aqk + ((size_t)bh * a.NC + c) * kC * M;
#pragma unroll
        for (int r = 0; r < RT; ++r) {
            const int t = ti + 16 * r;
#pragma unroll
            for (int s = 0; s < RM; ++s) {
                const int m = tj + 16 * s, tau = SPARSE ? (m >> 1) : m;
                float val = 0.f;
                if (tau <= t && t < L) val = __expf(sG[t] - sG[tau]) * acc[r][s];
                aqk[t * M + m] = val;
            }
        }
    }
    __syncthreads();
    // nu into VU, scale the right-hand sides
    for (int e = tid; e < M * D; e += kThreads) {
        const int m = e / D, d = e % D;
        const int tau = SPARSE ? (m >> 1) : m;
        float x = 0.f;
        if (tau < L) x = to_f32(((SPARSE && (m & 1)) ? sv : v)[row(tau) * D + d]);
        VU[m * LD + d] = x * sLam[m];
        KW[m * LD + d] *= sLam[m] * __expf(sG[tau]);
    }
    __syncthreads();
    // Forward substitution (I + A) Y = RHS, one column per thread (columns are independent).
    for (int col = tid; col < 2 * D; col += kThreads) {
        float *Y = (col < D) ? (KW + col) : (VU + (col - D));
        for (int i = 1; i < M; ++i) {
            const float *Ai = A + i * (M + 1);
            float s = 0.f;
            for (int j = 0; j < i; ++j) s = fmaf(Ai[j], Y[j * LD], s);
            Y[i * LD] -= s;
        }
    }
    __syncthreads();
    float *W = a.W + ((size_t)bh * a.NC + c) * M * D;
    float *U = a.U + ((size_t)bh * a.NC + c) * M * D;
    for (int e = tid; e < M * D; e += kThreads) {
        const int m = e / D, d = e % D;
        W[e] = KW[m * LD + d];
        U[e] = VU[m * LD + d];
    }
    if (tid < kC) a.G[((size_t)bh * a.NC + c) * kC + tid] = sG[tid];
}

template <typename Tin, typename Tout, int D, bool SPARSE>
__global__ void __launch_bounds__(kThreads) chunk_scan_kernel(ChunkArgs a) {
    using Dm = Dims<D, SPARSE>;
    constexpr int M = Dm::M;
    extern __shared__ float smem[];
    float *R1 = smem;              // M x D     W, then kap
    float *R2 = R1 + M * D;        // C x D     q
    float *R3 = R2 + kC * D;       // C x M     Aqk
    float *S = R3 + kC * M;        // D x BV    state slice
    float *Us = S + D * kBV;       // M x BV
    __shared__ float sEG[kC];      // exp(G_t)
    __shared__ float sTail[M];     // exp(G_last - G_tau_m)

    const int v0 = blockIdx.x * kBV, bh = blockIdx.y;
    const int b = bh / a.H, h = bh % a.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const Tin *q = (const Tin *)a.q, *k = (const Tin *)a.k, *sk = (const Tin *)a.sk;

    for (int e = tid; e < D * kBV; e += kThreads) {
        const int d = e / kBV, vv = e % kBV;
        S[e] = a.s0 ? a.s0[((size_t)bh * D + d) * D + v0 + vv] : 0.f;
    }
    for (int c = 0; c < a.NC; ++c) {
        const int t0 = c * kC;
        const int L = min(kC, a.T - t0);
        auto row = [&](int t) -> size_t { return ((size_t)b * a.T + t0 + t) * a.H + h; };
        const size_t cix = (size_t)bh * a.NC + c;
        const float *W = a.W + cix * M * D, *Uh = a.U + cix * M * D;
        const float *G = a.G + cix * kC;
        for (int e = tid; e < M * D; e += kThreads) R1[e] = W[e];
        for (int e = tid; e < M * kBV; e += kThreads) Us[e] = Uh[(e / kBV) * D + v0 + e % kBV];
        if (tid < kC) sEG[tid] = __expf(G[tid]);
        for (int m = tid; m < M; m += kThreads)
            sTail[m] = __expf(G[kC - 1] - G[SPARSE ? (m >> 1) : m]);
        __syncthreads();
        // U = Uh - W S     (rows m = warp + 8 r, column = lane)
        for (int m = warp; m < M; m += kThreads / 32) {
            float s = 0.f;
#pragma unroll 8
            for (int d = 0; d < D; ++d) s = fmaf(R1[m * D + d], S[d * kBV + lane], s);
            Us[m * kBV + lane] -= s;
        }
        __syncthreads();
        for (int e = tid; e < M * D; e += kThreads) {
            const int m = e / D, d = e % D;
            const int tau = SPARSE ? (m >> 1) : m;
            R1[e] = (tau < L) ? to_f32(((SPARSE && (m & 1)) ? sk : k)[row(tau) * D + d]) : 0.f;
        }
        for (int e = tid; e < kC * D; e += kThreads) {
            const int t = e / D, d = e % D;
            R2[e] = (t < L) ? to_f32(q[row(t) * D + d]) : 0.f;
        }
        {
            const float *aqk = a.Aqk + cix * kC * M;
            for (int e = tid; e < kC * M; e += kThreads) R3[e] = aqk[e];
        }
        __syncthreads();
        // O = exp(G) Q S + Aqk U
        Tout *o = (Tout *)a.o;
        for (int t = warp; t < L; t += kThreads / 32) {
            float s1 = 0.f, s2 = 0.f;
#pragma unroll 8
            for (int d = 0; d < D; ++d) s1 = fmaf(R2[t * D + d], S[d * kBV + lane], s1);
#pragma unroll 8
            for (int m = 0; m < M; ++m) s2 = fmaf(R3[t * M + m], Us[m * kBV + lane], s2);
            o[row(t) * D + v0 + lane] = from_f32<Tout>(sEG[t] * s1 + s2);
        }
        __syncthreads();
        // S = exp(G_last) S + Kap~^T U
        const float gl = sEG[kC - 1];
        for (int d = warp; d < D; d += kThreads / 32) {
            float s = 0.f;
#pragma unroll 8
            for (int m = 0; m < M; ++m) s = fmaf(sTail[m] * R1[m * D + d], Us[m * kBV + lane], s);
            S[d * kBV + lane] = gl * S[d * kBV + lane] + s;
        }
        __syncthreads();
    }
    if (a.sT) {
        for (int e = tid; e < D * kBV; e += kThreads) {
            const int d = e / kBV, vv = e % kBV;
            a.sT[((size_t)bh * D + d) * D + v0 + vv] = S[e];
        }
    }
}

template <typename Tin, typename Tout, int D, bool SPARSE>
cudaError_t run(const ChunkArgs &a, cudaStream_t st) {
    using Dm = Dims<D, SPARSE>;
    auto prep = chunk_prep_kernel<Tin, D, SPARSE>;
    auto scan = chunk_scan_kernel<Tin, Tout, D, SPARSE>;
    cudaError_t e = cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Dm::prep_smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(scan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Dm::scan_smem);
    if (e != cudaSuccess) return e;
    prep<<<dim3(a.NC, a.B * a.H), kThreads, Dm::prep_smem, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    scan<<<dim3(D / kBV, a.B * a.H), kThreads, Dm::scan_smem, st>>>(a);
    return cudaGetLastError();
}

template <typename Tin, typename Tout, bool SPARSE>
cudaError_t run_d(int D, const ChunkArgs &a, cudaStream_t st) {
    switch (D) {
        case 32: return run<Tin, Tout, 32, SPARSE>(a, st);
        case 64: return run<Tin, Tout, 64, SPARSE>(a, st);
        case 128: return run<Tin, Tout, 128, SPARSE>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

size_t chunk_delta_ws_bytes(int B, int T, int H, int D, int flags) {
    const int M = (flags & SGSA_FLAG_HAS_SPARSE) ? 2 * kC : kC;
    const size_t NC = (size_t)ceil_div(T, kC);
    const size_t per = (size_t)2 * M * D + (size_t)kC * M + kC;
    return (size_t)B * H * NC * per * sizeof(float);
}

cudaError_t launch_chunk_delta(const void *q, const void *k, const void *v, const void *beta,
                               const void *gamma, const void *sk, const void *sv,
                               const void *alpha, const float *s0, void *o, float *sT, int B,
                               int T, int H, int D, int dtype, int flags, void *ws,
                               cudaStream_t st) {
    const bool sparse = flags & SGSA_FLAG_HAS_SPARSE;
    const int M = sparse ? 2 * kC : kC;
    ChunkArgs a;
    a.q = q; a.k = k; a.v = v; a.beta = beta; a.gamma = gamma;
    a.sk = sk; a.sv = sv; a.alpha = alpha;
    a.s0 = (flags & SGSA_FLAG_HAS_INIT) ? s0 : nullptr;
    a.o = o;
    a.sT = (flags & SGSA_FLAG_STORE_FINAL) ? sT : nullptr;
    a.B = B; a.T = T; a.H = H; a.NC = ceil_div(T, kC);
    const size_t nchunk = (size_t)B * H * a.NC;
    a.W = (float *)ws;
    a.U = a.W + nchunk * M * D;
    a.Aqk = a.U + nchunk * M * D;
    a.G = a.Aqk + nchunk * kC * M;
    const bool of32 = (flags & SGSA_FLAG_OUT_F32) || dtype == SGSA_DTYPE_F32;
    if (dtype == SGSA_DTYPE_F32) {
        return sparse ? run_d<float, float, true>(D, a, st) : run_d<float, float, false>(D, a, st);
    }
    if (of32)
        return sparse ? run_d<__nv_bfloat16, float, true>(D, a, st)
                      : run_d<__nv_bfloat16, float, false>(D, a, st);
    return sparse ? run_d<__nv_bfloat16, __nv_bfloat16, true>(D, a, st)
                  : run_d<__nv_bfloat16, __nv_bfloat16, false>(D, a, st);
}

}  // namespace sgsa
