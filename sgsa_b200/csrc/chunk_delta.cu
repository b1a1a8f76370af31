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
#include <stdlib.h>

#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace sgsa {
namespace {

constexpr int kC = 64;
constexpr int kThreads = 256;
constexpr int kBV = 32;

// Internal flag of launch_chunk_delta: the inputs are the sparse write's interleaved virtual
// samples (ChunkArgs::pairs).  Outside the public SGSA_FLAG_* bits.
constexpr int kFlagPairs = 1 << 30;

struct ChunkArgs {
    const void *q, *k, *v, *beta, *gamma, *sk, *sv, *alpha;
    const float *s0;
    void *o;
    float *sT;
    int B, T, H, NC;
    int bh0, nbh;  // this launch's (batch, head) pairs: flattened b*H + h in [bh0, bh0 + nbh)
    float *W, *U, *Aqk, *G;
    float *Qt, *KtT;  // tensor-core scan only: exp(G_t) q_t [C x D] and Kap~^T [D x C]
    int transition;   // tensor-core scan only: v taken as zero, o not written
    // tensor-core kernels only: the rows are the sparse write's virtual samples, two per token
    // (local sample at 2t, sparse sample at 2t + 1, decay 1 on the second); the sparse sample
    // does not see its own token's local sample, and only the odd rows are read out, into
    // row t of an o of a.T / 2 tokens
    int pairs;
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
    const int b = (a.bh0 + bh) / a.H, h = (a.bh0 + bh) % a.H;
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

    if (!SPARSE && a.Qt) {  // operands of the tensor-core scan, in fp32
        const size_t cix = (size_t)bh * a.NC + c;
        float *qt = a.Qt + cix * kC * D, *kt = a.KtT + cix * D * kC;
        const float gl = sG[kC - 1];
        for (int e = tid; e < kC * D; e += kThreads) {
            const int t = e / D, d = e % D;
            qt[e] = __expf(sG[t]) * VU[t * LD + d];
        }
        for (int e = tid; e < kC * D; e += kThreads) {
            const int d = e / kC, m = e % kC;
            kt[e] = __expf(gl - sG[m]) * KW[m * LD + d];
        }
    }
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
    const int gbh = a.bh0 + bh, b = gbh / a.H, h = gbh % a.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const Tin *q = (const Tin *)a.q, *k = (const Tin *)a.k, *sk = (const Tin *)a.sk;

    for (int e = tid; e < D * kBV; e += kThreads) {
        const int d = e / kBV, vv = e % kBV;
        S[e] = a.s0 ? a.s0[((size_t)gbh * D + d) * D + v0 + vv] : 0.f;
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
            a.sT[((size_t)gbh * D + d) * D + v0 + vv] = S[e];
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
    prep<<<dim3(a.NC, a.nbh), kThreads, Dm::prep_smem, st>>>(a);
    e = launched();
    if (e != cudaSuccess) return e;
    scan<<<dim3(D / kBV, a.nbh), kThreads, Dm::scan_smem, st>>>(a);
    return launched();
}

// ---- tensor-core scan (bf16 inputs, D = 128, no sparse write) ---------------
//
// One CTA per (b, h); the 128x128 fp32 state lives transposed (S^T[v][dk], row v = TMEM
// lane v) in tensor memory for the whole scan: it is the A operand of the chunk's first
// MMA and the accumulator of its last, so it never passes through shared memory.  Every
// contraction runs as tcgen05.mma.kind::tf32 with M = 128 (state rows), fp32 in TMEM:
//   [D1 | D2] = S^T [W; Qt]^T     (U^T = Uh^T - D1)        [v x (tok | t)]
//   S^T <- e^{G_last} S^T          (the epilogue, in place in TMEM)
//   S^T += U^T Kt                  (the state update: MMA accumulate)
//   D2 += U^T Aqk^T                -> o^T                   [v x t]
// W, Qt, Aqk and Kt^T come from the prep kernel's workspace through TMA.
// Warp 0: TMA producer; warp 1: TMEM owner + MMA issuer; warps 2-5: one thread per
// state row v, the chain's epilogue (U, the decay); warps 6-9: Uh^T into TMEM ahead of
// its chunk and o^T out to global memory.
static __device__ unsigned int g_scan_watchdog;

namespace tc {
constexpr int kD = 128;
// W and Qt interleaved by 32-column block (block kb at kW + 16 KB kb: 64 rows of W, then
// 64 rows of Qt): one N = 128 K-major operand [W; Qt], so S^T W^T and S^T Qt^T are one MMA
constexpr int kW = 0;                        // [W; Qt] [128 rows][128 dk]  64 KB
constexpr int kQ = kW + 8192;                // Qt rows inside each 16 KB block
constexpr int kA = kW + 65536;               // Aqk  [64 t][64 tok]    16 KB
constexpr int kK = kA + 16384;               // Kt^T [128 dk][64 tok]  32 KB
constexpr int kU = kK + 32768;               // U^T  [128 v][64 tok]   32 KB
constexpr int kBar = kU + 32768;
constexpr int kBytes = kBar + 128;
constexpr size_t kSmem = 1024 + kBytes;
constexpr uint32_t kOpWQ = 32768 * 2;         // W and Qt: the first MMA group's operands
constexpr uint32_t kOpAK = 16384 + 32768;      // Aqk and Kt^T: the second group's
}  // namespace tc

// Byte offset of fp32 element (r, k) in a K-major 128-byte-swizzled operand of
// `rows` rows (32 k per 128-byte row, blocks of 32 k stacked).
__device__ __forceinline__ uint32_t sw128_f32(int rows, int r, int k) {
    return (uint32_t)((k >> 5) * rows * 128 + r * 128 + ((((k & 31) >> 2) ^ (r & 7)) << 4) +
                      ((k & 3) << 2));
}

template <typename Tout>
__global__ void __launch_bounds__(320, 1)
chunk_scan_tc_kernel(ChunkArgs a, const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_k) {
    using namespace sm100;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *sm = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(sm + tc::kBar);
    // opfull / opfull2: W, Qt / Aqk, Kt^T of the chunk landed; d1done: D1 = S^T W^T in TMEM;
    // wqfree: the MMAs reading W and Qt completed; utready: U^T in shared memory (and this
    // chunk's Uh read, S^T decayed); d3done: the state update S^T += U^T Kt; d2done: o^T = D2
    // complete (and U^T, Aqk,
    // Kt^T read); stready: the initial state in TMEM; uhready: the chunk's Uh^T in
    // TMEM; ofree: the chunk's o^T read out of its TMEM buffer.
    uint64_t *opfull = bars + 0, *d1done = bars + 1, *utready = bars + 2, *d3done = bars + 3,
             *stready = bars + 4, *opfull2 = bars + 5, *wqfree = bars + 6, *d2done = bars + 7,
             *uhready = bars + 8, *ofree = bars + 10, *uhfree = bars + 12, *d2out = bars + 14;
    // uhready, ofree, uhfree, d2out: two each, by chunk parity.  A thread never waits on a
    // barrier that may have completed two phases past the one it wants (the parity would
    // read as pending), so the output warps, which may lag the chain by a chunk, wait on
    // per-parity barriers: uhfree (E1 read Uh of that buffer) and d2out (o^T of that buffer
    // complete).
    __shared__ uint32_t s_tmem;
    unsigned int *wd = &g_scan_watchdog;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.x, gbh = a.bh0 + bh, b = gbh / a.H, h = gbh % a.H;
    const int NC = a.NC;

    if (threadIdx.x == 0) {
        mbar_init(opfull, 1);
        mbar_init(d1done, 1);
        mbar_init(utready, 4);
        mbar_init(d3done, 1);
        mbar_init(stready, 4);
        mbar_init(opfull2, 1);
        mbar_init(wqfree, 1);
        mbar_init(d2done, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&uhready[i], 4);
            mbar_init(&ofree[i], 4);
            mbar_init(&uhfree[i], 4);
            mbar_init(&d2out[i], 1);
        }
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(&s_tmem, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    // TMEM columns: S^T [0, 128); D1 | D2 (o^T) [128 + 128 p, 192 + 128 p) |
    // [192 + 128 p, 256 + 128 p) and Uh^T [384 + 64 p, 448 + 64 p) for chunk parity p.
    constexpr uint32_t kTS = 0, kTD12 = 128, kTUh = 384;

    if (warp == 0) {
        if (lane == 0) {
            // Each operand pair is refilled as soon as the MMAs that read it have completed:
            // W and Qt of chunk c once chunk c - 1's D1 and S^T Qt^T are done (wqfree), Aqk and
            // Kt^T once its D3 and U^T Aqk^T are done (d2done).
            auto prefetch = [&](int c) {  // chunk c's operand tiles into L2
                if (c >= NC) return;
                const int cix = bh * NC + c;
                for (int kb = 0; kb < 4; ++kb) {
                    tma_prefetch_2d(&tm_w, kb * 32, cix * 64);
                    tma_prefetch_2d(&tm_q, kb * 32, cix * 64);
                }
                for (int kb = 0; kb < 2; ++kb) {
                    tma_prefetch_2d(&tm_a, kb * 32, cix * 64);
                    tma_prefetch_2d(&tm_k, kb * 32, cix * 128);
                }
            };
            prefetch(1);
            for (int c = 0; c < NC; ++c) {
                const int cix = bh * NC + c;
                prefetch(c + 2);  // two chunks ahead: the loads below then hit L2
                if (c > 0) mbar_wait(wqfree, (c - 1) & 1, wd, 1u);
                mbar_arrive_expect_tx(opfull, tc::kOpWQ);
                for (int kb = 0; kb < 4; ++kb) {
                    tma_load_2d(sm + tc::kW + kb * 16384, &tm_w, opfull, kb * 32, cix * 64);
                    tma_load_2d(sm + tc::kQ + kb * 16384, &tm_q, opfull, kb * 32, cix * 64);
                }
                if (c > 0) mbar_wait(d2done, (c - 1) & 1, wd, 1u);
                mbar_arrive_expect_tx(opfull2, tc::kOpAK);
                for (int kb = 0; kb < 2; ++kb) {
                    tma_load_2d(sm + tc::kA + kb * 8192, &tm_a, opfull2, kb * 32, cix * 64);
                    tma_load_2d(sm + tc::kK + kb * 16384, &tm_k, opfull2, kb * 32, cix * 128);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t wq = smem_u32(sm + tc::kW), aq = smem_u32(sm + tc::kA),
                           kq = smem_u32(sm + tc::kK), uq = smem_u32(sm + tc::kU);
            constexpr uint32_t id64 = idesc_tf32_f32(128, 64), id128 = idesc_tf32_f32(128, 128);
            const uint32_t tS = tmem + kTS;
            // The chain that carries the state is S -> D1 -> U -> D3 -> S; the output's MMAs
            // (S^T Qt^T, U^T Aqk^T) follow the chain's MMA of their group in the in-order
            // tensor pipe, and o^T leaves TMEM through its own warps.
            for (int c = 0; c < NC; ++c) {
                const uint32_t ph = c & 1;
                const uint32_t tD12 = tmem + kTD12 + 128 * ph, tD2 = tD12 + 64;
                // the state: initial (written by the epilogue) or after chunk c - 1's update
                if (c == 0) mbar_wait(stready, 0, wd, 2u);
                else mbar_wait(d3done, (c - 1) & 1, wd, 2u);
                mbar_wait(opfull, ph, wd, 4u);
                // the buffer chunk c - 2's o^T has left
                if (c >= 2) mbar_wait(&ofree[ph], ((c - 2) >> 1) & 1, wd, 4u);
                tc_fence_after();
                // [D1 | D2] = S^T [W; Qt]^T   (N = 128, K = dk = 128: 16 steps of 8)
                for (int kb = 0; kb < 4; ++kb)
                    for (int kk = 0; kk < 4; ++kk)
                        mma_tf32_ts(tD12, tS + kb * 32 + kk * 8,
                                    sdesc_kmajor_sw128(wq + kb * 16384 + kk * 32), id128, (kb | kk) ? 1u : 0u);
                mma_commit(d1done);
                mma_commit(wqfree);
                mbar_wait(utready, ph, wd, 8u);
                mbar_wait(opfull2, ph, wd, 4u);
                tc_fence_after();
                // S^T += U^T Kt   (the epilogue scaled S^T by e^{G_last}; K = tok = 64)
                for (int kb = 0; kb < 2; ++kb)
                    for (int kk = 0; kk < 4; ++kk)
                        mma_tf32(tS, sdesc_kmajor_sw128(uq + kb * 16384 + kk * 32),
                                 sdesc_kmajor_sw128(kq + kb * 16384 + kk * 32), id128, 1u);
                mma_commit(d3done);
                // D2 += U^T Aqk^T
                for (int kb = 0; kb < 2; ++kb)
                    for (int kk = 0; kk < 4; ++kk)
                        mma_tf32(tD2, sdesc_kmajor_sw128(uq + kb * 16384 + kk * 32),
                                 sdesc_kmajor_sw128(aq + kb * 8192 + kk * 32), id64, 1u);
                mma_commit(d2done);
                mma_commit(&d2out[ph]);
            }
        }
        __syncwarp();
    } else if (warp < 6) {
        // the state chain: one thread per state row v (its TMEM lane)
        const int quad = warp & 3, v = quad * 32 + lane;
        const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
        unsigned char *UT = sm + tc::kU;
        // initial state, transposed into TMEM: S^T[v][dk] = S0[dk][v]
#pragma unroll 1
        for (int k0 = 0; k0 < tc::kD; k0 += 32) {
            float x[32];
#pragma unroll
            for (int i = 0; i < 32; ++i)
                x[i] = a.s0 ? a.s0[(size_t)gbh * tc::kD * tc::kD + (size_t)(k0 + i) * tc::kD + v] : 0.f;
            tmem_st32(trow + kTS + k0, x);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(stready);
        for (int c = 0; c < NC; ++c) {
            const uint32_t ph = c & 1;
            const size_t cix = (size_t)bh * NC + c;
            const float gl = __expf(a.G[cix * kC + kC - 1]);
            // ---- U^T = Uh^T - S^T W^T, both from TMEM, into shared memory (the A operand
            // of the last two MMAs)
            mbar_wait(&uhready[ph], (c >> 1) & 1, wd, 16u);
            mbar_wait(d1done, ph, wd, 16u);
            tc_fence_after();
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t d[32], u[32];
                tmem_ld32_issue(trow + kTD12 + 128 * ph + half * 32, d);
                tmem_ld32_issue(trow + kTUh + 64 * ph + half * 32, u);
                tmem_ld_wait(d);
                tmem_ld_wait(u);
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const int t = half * 32 + j;
                    *(float4 *)(UT + sw128_f32(128, v, t)) = make_float4(
                        __uint_as_float(u[j]) - __uint_as_float(d[j]),
                        __uint_as_float(u[j + 1]) - __uint_as_float(d[j + 1]),
                        __uint_as_float(u[j + 2]) - __uint_as_float(d[j + 2]),
                        __uint_as_float(u[j + 3]) - __uint_as_float(d[j + 3]));
                }
            }
            // ---- the decay, in place: S^T <- e^{G_last} S^T (the first MMA of the chunk,
            // which read S^T, has completed)
#pragma unroll
            for (int q = 0; q < 4; q += 2) {
                uint32_t r0[32], r1[32];
                tmem_ld32_issue(trow + kTS + q * 32, r0);
                tmem_ld32_issue(trow + kTS + (q + 1) * 32, r1);
                tmem_ld_wait(r0);
                tmem_ld_wait(r1);
                float x0[32], x1[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    x0[i] = gl * __uint_as_float(r0[i]);
                    x1[i] = gl * __uint_as_float(r1[i]);
                }
                tmem_st32(trow + kTS + q * 32, x0);
                tmem_st32(trow + kTS + (q + 1) * 32, x1);
            }
            fence_proxy_async();  // U^T: generic-proxy stores, read by the tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(utready);
                mbar_arrive(&uhfree[ph]);
            }
        }
        // the final state once the last update has completed
        mbar_wait(d3done, (NC - 1) & 1, wd, 64u);
        tc_fence_after();
        if (a.sT) {
            float *sT = a.sT + (size_t)gbh * tc::kD * tc::kD + v;
#pragma unroll 1
            for (int k0 = 0; k0 < tc::kD; k0 += 32) {
                float x[32];
                tmem_ld32(trow + kTS + k0, x);
#pragma unroll
                for (int i = 0; i < 32; ++i) sT[(size_t)(k0 + i) * tc::kD] = x[i];
            }
        }
    } else {
        // output and prefetch warps (same TMEM lane quarters): Uh^T of chunk c + 2 into the
        // TMEM buffer chunk c has used, and o^T of chunk c out to global memory
        const int quad = warp & 3, v = quad * 32 + lane;
        const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
        Tout *o = (Tout *)a.o;
        const size_t tstride = (size_t)a.H * tc::kD;
        auto put_uh = [&](int c) {  // Uh^T[v][t] of chunk c into buffer c & 1
            if (!a.transition) {
                const float *Uh = a.U + ((size_t)bh * NC + c) * kC * tc::kD + v;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float u[32];
#pragma unroll
                    for (int t = 0; t < 32; ++t) u[t] = Uh[(half * 32 + t) * tc::kD];
                    tmem_st32(trow + kTUh + 64 * (c & 1) + half * 32, u);
                }
            } else {  // the transition scan takes v as zero: Uh = 0
                float u[32];
#pragma unroll
                for (int t = 0; t < 32; ++t) u[t] = 0.f;
                tmem_st32(trow + kTUh + 64 * (c & 1), u);
                tmem_st32(trow + kTUh + 64 * (c & 1) + 32, u);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&uhready[c & 1]);
        };
        put_uh(0);
        if (NC > 1) put_uh(1);
        for (int c = 0; c < NC; ++c) {
            const uint32_t ph = c & 1;
            const int t0 = c * kC, L = min(kC, a.T - t0);
            // E1 of chunk c has read its Uh: chunk c + 2's goes into the same buffer
            mbar_wait(&uhfree[ph], (c >> 1) & 1, wd, 128u);
            tc_fence_after();
            if (c + 2 < NC) put_uh(c + 2);
            mbar_wait(&d2out[ph], (c >> 1) & 1, wd, 64u);
            tc_fence_after();
            if (!a.transition) {
                uint32_t ro0[32], ro1[32];
                tmem_ld32_issue(trow + kTD12 + 128 * ph + 64, ro0);
                tmem_ld32_issue(trow + kTD12 + 128 * ph + 96, ro1);
                tmem_ld_wait(ro0);
                tmem_ld_wait(ro1);
                if (a.pairs) {  // odd virtual rows only: sample 2t+1 holds token t's output
                    Tout *op = o + (((size_t)b * (a.T >> 1) + (t0 >> 1)) * a.H + h) * tc::kD + v;
#pragma unroll
                    for (int t = 1; t < kC; t += 2)
                        if (t < L) op[(t >> 1) * tstride] = from_f32<Tout>(__uint_as_float(t < 32 ? ro0[t] : ro1[t - 32]));
                } else {
                    Tout *op = o + (((size_t)b * a.T + t0) * a.H + h) * tc::kD + v;
#pragma unroll
                    for (int t = 0; t < kC; ++t)
                        if (t < L) op[t * tstride] = from_f32<Tout>(__uint_as_float(t < 32 ? ro0[t] : ro1[t - 32]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ofree[ph]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// ---- tensor-core prep (bf16 inputs, D = 128, no sparse write) --------------
//
// One CTA per pair of consecutive chunks of one (b, h), stacked into 128 rows:
//   KK^T, QK^T   bf16 tcgen05.mma (only the two 64x64 diagonal blocks are used)
//   T = (I + A)^-1 per 64x64 block: one thread per column, the column in
//                registers, forward substitution with broadcast reads of A
//   W  = T diag(lam e^G) K,  Uh = T diag(lam) V   bf16 tcgen05.mma with the
//                scaled T split into bf16 hi + lo parts (fp32-level accuracy;
//                K and V enter exactly, straight from their TMA tiles as
//                MN-major operands)
// plus the operands of the tensor-core scan (Aqk, Qt, Kt^T, G) of both chunks.
namespace ptc {
constexpr int kK = 0;           // K tile bf16 [128 j][128 dk], 2 x 16 KB
constexpr int kV = 32768;       // V tile bf16, 2 x 16 KB
constexpr int kQ = 65536;       // Q tile bf16 (2 x 16 KB), then T''hi (16 KB) | T''lo
constexpr int kA = 98304;       // A blocks fp32 [2][64][64] (32 KB), then (kQ..): T''
constexpr int kX = 131072;      // T'hi | T'lo bf16 [128 i][128 j], 2 x 32 KB
constexpr int kBar = 196608;
constexpr size_t kSmem = 1024 + kBar + 64;
}  // namespace ptc

// Byte offset of bf16 element (r, c) in a K-major 128-byte-swizzled operand of
// 128 rows (64 columns per 16 KB block).
__device__ __forceinline__ uint32_t sw128_bf16(int r, int c) {
    return (uint32_t)((c >> 6) * 16384 + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) +
                      ((c & 7) << 1));
}

__global__ void __launch_bounds__(256, 1)
chunk_prep_tc_kernel(ChunkArgs a, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_v) {
    using namespace sm100;
    constexpr int D = 128;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *sm = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(sm + ptc::kBar);
    uint64_t *ldbar = bars, *mma1 = bars + 1, *mma2 = bars + 2;
    __shared__ uint32_t s_tmem;
    __shared__ float sG[128], sLam[128], sEq[128], sEk[128];
    unsigned int *wd = &g_scan_watchdog;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c0 = blockIdx.x * 2, bh = blockIdx.y, b = (a.bh0 + bh) / a.H, h = (a.bh0 + bh) % a.H;
    const int NC = a.NC, T = a.T;
    const int t0 = c0 * kC;
    const __nv_bfloat16 *beta = (const __nv_bfloat16 *)a.beta,
                        *gamma = (const __nv_bfloat16 *)a.gamma;
    auto valid = [&](int i) { return t0 + i < T && (i < kC || c0 + 1 < NC); };
    auto row = [&](int i) -> size_t { return ((size_t)b * T + t0 + i) * a.H + h; };

    if (tid == 0) {
        mbar_init(ldbar, 1);
        mbar_init(mma1, 1);
        mbar_init(mma2, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(ldbar, 3 * 32768);
        for (int kb = 0; kb < 2; ++kb) {
            tma_load_3d(sm + ptc::kK + kb * 16384, &tm_k, ldbar, kb * 64, h, b * T + t0);
            tma_load_3d(sm + ptc::kV + kb * 16384, &tm_v, ldbar, kb * 64, h, b * T + t0);
            tma_load_3d(sm + ptc::kQ + kb * 16384, &tm_q, ldbar, kb * 64, h, b * T + t0);
        }
    }
    if (warp == 1) tmem_alloc(&s_tmem, 256);
    if (tid < 128) {
        const bool ok = valid(tid);
        sG[tid] = ok ? logf(__bfloat162float(gamma[row(tid)])) : 0.f;
        sLam[tid] = ok ? __bfloat162float(beta[row(tid)]) : 0.f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    if (warp < 2) {  // inclusive cumsum of log(gamma) per 64-token chunk, two tokens per lane
        float *g = sG + warp * kC;
        const float x0 = g[2 * lane], x1 = g[2 * lane + 1];
        float s = x0 + x1;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, s, off);
            if (lane >= off) s += y;
        }
        const float ex = s - (x0 + x1);
        g[2 * lane] = ex + x0;
        g[2 * lane + 1] = ex + x0 + x1;
    }
    if (tid == 0) {  // KK^T -> cols [0,128), QK^T -> cols [128,256)
        mbar_wait(ldbar, 0, wd, 0x100u);
        tc_fence_after();
        constexpr uint32_t id = idesc_bf16_f32(128, 128);
        const uint32_t kq = smem_u32(sm + ptc::kK), qq = smem_u32(sm + ptc::kQ);
        for (int kb = 0; kb < 2; ++kb)
            for (int kk = 0; kk < 4; ++kk) {
                const uint64_t bd = sdesc_kmajor_sw128(kq + kb * 16384 + kk * 32);
                const uint32_t acc = (kb | kk) ? 1u : 0u;
                mma_bf16(tmem, sdesc_kmajor_sw128(kq + kb * 16384 + kk * 32), bd, id, acc);
                mma_bf16(tmem + 128, sdesc_kmajor_sw128(qq + kb * 16384 + kk * 32), bd, id, acc);
            }
        mma_commit(mma1);
    }
    __syncthreads();
    mbar_wait(mma1, 0, wd, 0x200u);
    tc_fence_after();
    // A blocks [2][64 i][64 j], 16-byte column groups XOR-swizzled by (i & 7): the epilogue
    // stores 32 rows at once (conflict-free), the solve reads rows as broadcasts
    float *Ablk = (float *)(sm + ptc::kA);
    auto a_off = [](int i, int j) { return i * 64 + ((((j >> 2) ^ (i & 7))) << 2) + (j & 3); };
    {   // A (warps 0-3) and Aqk (warps 4-7), one row per thread, its own 64-column block
        const int quad = warp & 3, i = quad * 32 + lane, cb = i >> 6, tau = i & 63;
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (warp < 4 ? 0 : 128) + cb * 64;
        const bool vi = valid(i);
        const float lam_i = sLam[i];
        float *aqk = a.Aqk + (((size_t)bh * NC + c0 + cb) * kC + tau) * kC;
        const bool chunk_ok = c0 + cb < NC;
        float *astg = (float *)(sm + ptc::kX) + (warp & 3) * (32 * 68);  // T' area, not yet used
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            float d[32];
            tmem_ld32(taddr + hf * 32, d);
#pragma unroll
            for (int jj = 0; jj < 32; jj += 4) {
                float4 r4;
                float *r = &r4.x;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int m = hf * 32 + jj + u, j = cb * 64 + m;
                    const bool vj = valid(j);
                    // branch-free: the exponent is clamped at 0 (its value only matters where
                    // m <= tau, where G_i <= G_j) and the mask selects
                    const float e = __expf(fminf(sG[i] - sG[j], 0.f)) * d[jj + u];
                    // pairs: sample 2t+1 predicts from the state before token t's local
                    // sample 2t (both samples of a token read the same decayed state)
                    const bool dep = m < tau && !(a.pairs && (tau & 1) && m == tau - 1);
                    if (warp < 4)
                        r[u] = (vi && vj && dep) ? lam_i * e : 0.f;
                    else
                        r[u] = (vi && vj && m <= tau) ? e : 0.f;
                }
                if (warp < 4) *(float4 *)(Ablk + cb * 4096 + a_off(tau, hf * 32 + jj)) = r4;
                else *(float4 *)(astg + lane * 68 + hf * 32 + jj) = r4;
            }
        }
        if (warp >= 4) {  // the warp's 32 Aqk rows are contiguous: whole 256-byte rows per store
            __syncwarp();
            if (chunk_ok) {
                float *dst = aqk - (size_t)lane * kC;  // row of lane 0
                const int cq = lane & 15;
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const int r = (lane >> 4) + 2 * k;
                    *(float4 *)(dst + (size_t)r * kC + cq * 4) = *(const float4 *)(astg + r * 68 + cq * 4);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    float tcol[64];
    if (tid < 128) {
        // column c of T = (I + A)^-1 of block blk: t_i = [i == c] - sum_{j<i} A[i][j] t_j
        const int blk = tid >> 6, c = tid & 63;
        const float *Ab = Ablk + blk * 4096;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            // four partial sums: a chain of i/4 dependent FMAs instead of i
            float s0 = (i == c) ? 1.f : 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
            for (int j = 0; j < i; j += 4) {
                const float4 a4 = *(const float4 *)(Ab + a_off(i, j));  // broadcast
                s0 -= a4.x * tcol[j];
                if (j + 1 < i) s1 -= a4.y * tcol[j + 1];
                if (j + 2 < i) s2 -= a4.z * tcol[j + 2];
                if (j + 3 < i) s3 -= a4.w * tcol[j + 3];
            }
            tcol[i] = (s0 + s1) + (s2 + s3);
        }
    } else {
        // operands of the scan: Qt = e^{G} q (row-major), Kt^T = e^{G_last - G} k ([dk][tok]),
        // read from the swizzled Q and K tiles 16 bytes at a time; G
        const int u = tid - 128;
        const unsigned char *Kt = sm + ptc::kK, *Qt = sm + ptc::kQ;
        {  // the per-token factors, once
            const bool ok = valid(u);
            const float glast = sG[(u >> 6) * 64 + 63];
            sEq[u] = ok ? __expf(sG[u]) : 0.f;
            sEk[u] = ok ? __expf(glast - sG[u]) : 0.f;
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
        for (int cb = 0; cb < 2; ++cb) {
            if (c0 + cb >= NC) break;
            const size_t cix = (size_t)bh * NC + c0 + cb;
            for (int e = u; e < kC * D / 8; e += 128) {  // Qt: 8 consecutive d of one token
                const int m = e >> 4, d0 = (e & 15) * 8, j = cb * 64 + m;
                const uint4 raw = *(const uint4 *)(Qt + sw128_bf16(j, d0));
                const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
                const float f = sEq[j];
                float4 lo, hi;
                float2 x0 = __bfloat1622float2(h2[0]), x1 = __bfloat1622float2(h2[1]),
                       x2 = __bfloat1622float2(h2[2]), x3 = __bfloat1622float2(h2[3]);
                lo = make_float4(f * x0.x, f * x0.y, f * x1.x, f * x1.y);
                hi = make_float4(f * x2.x, f * x2.y, f * x3.x, f * x3.y);
                float *dst = a.Qt + (cix * kC + m) * D + d0;
                *(float4 *)dst = lo;
                *(float4 *)(dst + 4) = hi;
            }
            for (int e = u; e < kC * D / 8; e += 128) {  // Kt^T: 8 consecutive tokens of one d
                // lanes take consecutive d of the same 8 tokens: conflict-free tile reads
                const int d = e & (D - 1), m0 = (e / D) * 8;
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int j = cb * 64 + m0 + i;
                    v[i] = sEk[j] * __bfloat162float(*(const __nv_bfloat16 *)(Kt + sw128_bf16(j, d)));
                }
                float *dst = a.KtT + (cix * D + d) * kC + m0;
                *(float4 *)dst = make_float4(v[0], v[1], v[2], v[3]);
                *(float4 *)(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
            }
            if (u < 64) a.G[cix * kC + u] = sG[cb * 64 + u];
        }
    }
    __syncthreads();  // the Q tile and the A blocks are dead from here
    if (tid < 128) {
        // T' = T diag(lam e^G) into kX (hi | lo), T'' = T diag(lam) into kQ.. (hi | lo):
        // this thread's column over its block's 64 rows
        const int blk = tid >> 6, c = tid & 63, col = blk * 64 + c;
        const float s1 = sLam[col] * __expf(sG[col]), s2 = sLam[col];
        unsigned char *X = sm + ptc::kX, *Y = sm + ptc::kQ;
#pragma unroll
        for (int li = 0; li < 64; ++li) {
            const int i = blk * 64 + li;
            const float v1 = tcol[li] * s1, v2 = tcol[li] * s2;
            const __nv_bfloat16 h1 = __float2bfloat16_rn(v1), h2 = __float2bfloat16_rn(v2);
            const uint32_t off = sw128_bf16(i, col);
            *(__nv_bfloat16 *)(X + off) = h1;
            *(__nv_bfloat16 *)(X + 32768 + off) = __float2bfloat16_rn(v1 - __bfloat162float(h1));
            *(__nv_bfloat16 *)(Y + off) = h2;
            *(__nv_bfloat16 *)(Y + 32768 + off) = __float2bfloat16_rn(v2 - __bfloat162float(h2));
        }
    } else {
        // the off-diagonal blocks of T' and T'' are zero: 16-byte chunks
        unsigned char *X = sm + ptc::kX, *Y = sm + ptc::kQ;
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        for (int e = tid - 128; e < 128 * 8; e += 128) {
            const int i = e >> 3, col0 = ((1 - (i >> 6)) * 8 + (e & 7)) * 8;
            const uint32_t off = sw128_bf16(i, col0);
            *(uint4 *)(X + off) = z;
            *(uint4 *)(X + 32768 + off) = z;
            *(uint4 *)(Y + off) = z;
            *(uint4 *)(Y + 32768 + off) = z;
        }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {  // W -> cols [0,128), Uh -> cols [128,256); B = K / V tiles, MN-major
        constexpr uint32_t id = idesc_bf16_f32_bmn(128, 128);
        const uint32_t xq = smem_u32(sm + ptc::kX), yq = smem_u32(sm + ptc::kQ),
                       kq = smem_u32(sm + ptc::kK), vq = smem_u32(sm + ptc::kV);
        for (int part = 0; part < 2; ++part)
            for (int kb = 0; kb < 2; ++kb)
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t aoff = part * 32768 + kb * 16384 + kk * 32;
                    const uint32_t boff = kb * 8192 + kk * 2048;  // 64 rows of j per block
                    const uint32_t acc = (part | kb | kk) ? 1u : 0u;
                    mma_bf16(tmem, sdesc_kmajor_sw128(xq + aoff),
                             sdesc_mnmajor_sw128(kq + boff, 16384, 1024), id, acc);
                    mma_bf16(tmem + 128, sdesc_kmajor_sw128(yq + aoff),
                             sdesc_mnmajor_sw128(vq + boff, 16384, 1024), id, acc);
                }
        mma_commit(mma2);
    }
    __syncthreads();
    mbar_wait(mma2, 0, wd, 0x400u);
    tc_fence_after();
    {
        // W (warps 0-3) / Uh (warps 4-7): a warp's 32 rows are 32 consecutive rows of the
        // output; 32 x 32 blocks go through shared memory (the dead T' area) so that every
        // store instruction writes whole 128-byte row segments
        const int quad = warp & 3, i0 = quad * 32, cb = i0 >> 6, tau0 = i0 & 63;
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (warp < 4 ? 0 : 128);
        float *dst = (warp < 4 ? a.W : a.U) + (((size_t)bh * NC + c0 + cb) * kC + tau0) * D;
        const bool ok = c0 + cb < NC;
        float *stg = (float *)(sm + ptc::kX) + warp * (32 * 36);
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
            float d[32];
            tmem_ld32(taddr + cc * 32, d);
#pragma unroll
            for (int q = 0; q < 8; ++q)
                *(float4 *)(stg + lane * 36 + q * 4) = make_float4(d[4 * q], d[4 * q + 1], d[4 * q + 2], d[4 * q + 3]);
            __syncwarp();
            if (ok) {
                const int cq = lane & 7;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int r = (lane >> 3) + 4 * k;
                    *(float4 *)(dst + (size_t)r * D + cc * 32 + cq * 4) = *(const float4 *)(stg + r * 36 + cq * 4);
                }
            }
            __syncwarp();
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 256);
}

static bool scan_use_tc() {
    const char *e = getenv("SGSA_SCAN_SIMT");
    return !(e && e[0] == '1');
}

template <typename Tout>
cudaError_t run_tc_scan(const ChunkArgs &a, bool reuse_prep, cudaStream_t st,
                        cudaEvent_t prep_done = nullptr) {
    const long long nch = (long long)a.nbh * a.NC;
    CUtensorMap mw, mq, ma, mk, mkin, mqin, mvin;
    if (!make_tmap_2d_f32(&mw, a.W, 128, nch * 64, 64) ||
        !make_tmap_2d_f32(&mq, a.Qt, 128, nch * 64, 64) ||
        !make_tmap_2d_f32(&ma, a.Aqk, 64, nch * 64, 64) ||
        !make_tmap_2d_f32(&mk, a.KtT, 64, nch * 128, 128) ||
        !make_tmap_rows_bf16(&mkin, a.k, a.B, a.T, a.H, 128, 128) ||
        !make_tmap_rows_bf16(&mqin, a.q, a.B, a.T, a.H, 128, 128) ||
        !make_tmap_rows_bf16(&mvin, a.v, a.B, a.T, a.H, 128, 128))
        return cudaErrorInvalidValue;
    auto prep = chunk_prep_tc_kernel;
    cudaError_t e = cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)ptc::kSmem);
    if (e != cudaSuccess) return e;
    auto scan = chunk_scan_tc_kernel<Tout>;
    e = cudaFuncSetAttribute(scan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::kSmem);
    if (e != cudaSuccess) return e;
    if (!reuse_prep) {
        prep<<<dim3((a.NC + 1) / 2, a.nbh), 256, ptc::kSmem, st>>>(a, mkin, mqin, mvin);
        e = launched();
        if (e != cudaSuccess) return e;
        if (prep_done && (e = cudaEventRecord(prep_done, st)) != cudaSuccess) return e;
    }
    scan<<<a.nbh, 320, tc::kSmem, st>>>(a, mw, mq, ma, mk);
    return launched();
}

// The sparse write's virtual samples as a plain sequence of 2T rows for the tensor-core
// kernels (chunk_fwd.py:49-56 builds the same interleave: kappa = (k_t, sparse_k_t),
// nu = (v_t, sparse_v_t), lam = (beta_t, alpha_t), both samples at token t's decay):
// row 2t = (k, v, beta, gamma, q = 0), row 2t+1 = (sparse_k, sparse_v, alpha, 1, q).
// One thread per 8 bf16 values (16 bytes) of one token row of one head.
__global__ void __launch_bounds__(256)
pair_interleave_kernel(const uint4 *q, const uint4 *k, const uint4 *v, const uint4 *sk,
                       const uint4 *sv, const __nv_bfloat16 *beta, const __nv_bfloat16 *gamma,
                       const __nv_bfloat16 *alpha, uint4 *qv, uint4 *kv, uint4 *vv,
                       __nv_bfloat16 *bv, __nv_bfloat16 *gv, long long rows, int H, int vec) {
    const long long n = rows * vec;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (long long)gridDim.x * blockDim.x) {
        // e = r*vec + x with token row r = (b*T + t)*H + h; the virtual rows of (b, t) are
        // 2(b*T + t) and 2(b*T + t) + 1 of a [B, 2T, H] layout
        const long long r = e / vec, bt = r / H;
        const int h = (int)(r - bt * H), x = (int)(e - r * vec);
        const long long r0 = (2 * bt) * H + h, r1 = r0 + H;
        const long long e0 = r0 * vec + x, e1 = r1 * vec + x;
        kv[e0] = k[e];
        kv[e1] = sk[e];
        vv[e0] = v[e];
        vv[e1] = sv[e];
        qv[e0] = make_uint4(0u, 0u, 0u, 0u);
        qv[e1] = q[e];
        if (x == 0) {
            bv[r0] = beta[r];
            bv[r1] = alpha[r];
            gv[r0] = gamma[r];
            gv[r1] = __float2bfloat16(1.f);
        }
    }
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

bool chunk_tc_eligible(int D, int dtype, int flags) {
    return dtype == SGSA_DTYPE_BF16 && D == 128 && !(flags & SGSA_FLAG_HAS_SPARSE) &&
           scan_use_tc();
}

unsigned int read_scan_watchdog(cudaStream_t st) {
    unsigned int v = 0, z = 0;
    if (cudaStreamSynchronize(st) != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyFromSymbol(&v, g_scan_watchdog, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (v) cudaMemcpyToSymbol(g_scan_watchdog, &z, sizeof(z));
    return v;
}

// The sparse write on the tensor-core kernels: bf16, D = 128, a plain forward (the transition
// and prep-reuse passes of the sequence-parallel path stay on the single-sample layout).
static bool chunk_tc_pairs_eligible(int D, int dtype, int flags) {
    return dtype == SGSA_DTYPE_BF16 && D == 128 && (flags & SGSA_FLAG_HAS_SPARSE) &&
           !(flags & (SGSA_FLAG_TRANSITION | SGSA_FLAG_REUSE_PREP)) && scan_use_tc();
}

static size_t align256z(size_t x) { return (x + 255) & ~(size_t)255; }

// Interleaved virtual inputs of the sparse write (q, k, v rows; beta, gamma scalars), bf16.
static size_t pair_inputs_bytes(int B, int T, int H, int D) {
    const size_t rows = (size_t)B * 2 * T * H;
    return 3 * align256z(rows * D * 2) + 2 * align256z(rows * 2);
}

size_t chunk_delta_ws_bytes_pairs(long long pairs, int T, int D, int flags) {
    const int M = (flags & SGSA_FLAG_HAS_SPARSE) ? 2 * kC : kC;
    const size_t NC = (size_t)ceil_div(T, kC);
    size_t per = (size_t)2 * M * D + (size_t)kC * M + kC;
    size_t extra = 0;
    if (D == 128 && M == kC) {  // Qt and Kt^T of the tensor-core scan (+ alignment pad)
        per += (size_t)2 * kC * D;
        extra = 256;
    }
    return (size_t)pairs * NC * per * sizeof(float) + extra;
}

size_t chunk_delta_ws_bytes(int B, int T, int H, int D, int flags) {
    const size_t simt = chunk_delta_ws_bytes_pairs((long long)B * H, T, D, flags);
    if (!((flags & SGSA_FLAG_HAS_SPARSE) && D == 128 &&
          !(flags & (SGSA_FLAG_TRANSITION | SGSA_FLAG_REUSE_PREP))))
        return simt;
    // the size does not know the dtype: room for either the CUDA-core sparse layout or the
    // tensor-core one (interleaved inputs + the single-sample operands of 2T rows)
    const size_t tc = pair_inputs_bytes(B, T, H, D) +
                      chunk_delta_ws_bytes_pairs((long long)B * H, 2 * T, D,
                                                 flags & ~SGSA_FLAG_HAS_SPARSE);
    return std::max(simt, tc);
}

int chunk_delta_group_pairs(int B, int T, int H, int D, int flags, size_t cap) {
    const long long pairs = (long long)B * H;
    if (cap == 0 || chunk_delta_ws_bytes_pairs(pairs, T, D, flags) <= cap) return (int)pairs;
    const size_t one = chunk_delta_ws_bytes_pairs(1, T, D, flags);
    return (int)std::max<long long>(1, std::min<long long>(pairs, (long long)(cap / one)));
}

cudaError_t launch_chunk_delta(const void *q, const void *k, const void *v, const void *beta,
                               const void *gamma, const void *sk, const void *sv,
                               const void *alpha, const float *s0, void *o, float *sT, int B,
                               int T, int H, int D, int dtype, int flags, void *ws,
                               cudaStream_t st, size_t ws_cap, cudaEvent_t prep_done) {
    if (chunk_tc_pairs_eligible(D, dtype, flags)) {
        // the sparse write as 2T virtual samples on the tensor-core kernels: interleave, then
        // the single-sample prep / scan with the pair mask; the scan writes token rows of o
        const size_t rows = (size_t)B * T * H, vrows = 2 * rows, ib = pair_inputs_bytes(B, T, H, D);
        if (ws_cap && ws_cap <= ib) return cudaErrorInvalidValue;
        unsigned char *p = (unsigned char *)ws;
        __nv_bfloat16 *qv = (__nv_bfloat16 *)p;
        __nv_bfloat16 *kv = (__nv_bfloat16 *)(p += align256z(vrows * D * 2));
        __nv_bfloat16 *vv = (__nv_bfloat16 *)(p += align256z(vrows * D * 2));
        __nv_bfloat16 *bv = (__nv_bfloat16 *)(p += align256z(vrows * D * 2));
        __nv_bfloat16 *gv = (__nv_bfloat16 *)(p += align256z(vrows * 2));
        p += align256z(vrows * 2);
        const int vec = D / 8;
        const long long n = (long long)rows * vec;
        const int grid = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
        pair_interleave_kernel<<<grid, 256, 0, st>>>(
            (const uint4 *)q, (const uint4 *)k, (const uint4 *)v, (const uint4 *)sk,
            (const uint4 *)sv, (const __nv_bfloat16 *)beta, (const __nv_bfloat16 *)gamma,
            (const __nv_bfloat16 *)alpha, (uint4 *)qv, (uint4 *)kv, (uint4 *)vv, bv, gv,
            (long long)rows, H, vec);
        cudaError_t e = launched();
        if (e != cudaSuccess) return e;
        return launch_chunk_delta(qv, kv, vv, bv, gv, nullptr, nullptr, nullptr, s0, o, sT, B,
                                  2 * T, H, D, dtype, (flags & ~SGSA_FLAG_HAS_SPARSE) | kFlagPairs,
                                  p, st, ws_cap ? ws_cap - ib : 0, prep_done);
    }
    const bool pairs = flags & kFlagPairs;
    flags &= ~kFlagPairs;
    const bool sparse = flags & SGSA_FLAG_HAS_SPARSE;
    const int M = sparse ? 2 * kC : kC;
    const int group = chunk_delta_group_pairs(B, T, H, D, flags, ws_cap);
    ChunkArgs a;
    a.q = q; a.k = k; a.v = v; a.beta = beta; a.gamma = gamma;
    a.sk = sk; a.sv = sv; a.alpha = alpha;
    a.s0 = (flags & SGSA_FLAG_HAS_INIT) ? s0 : nullptr;
    a.o = o;
    a.sT = (flags & SGSA_FLAG_STORE_FINAL) ? sT : nullptr;
    a.B = B; a.T = T; a.H = H; a.NC = ceil_div(T, kC);
    a.transition = (flags & SGSA_FLAG_TRANSITION) ? 1 : 0;
    a.pairs = pairs ? 1 : 0;
    const bool tc = chunk_tc_eligible(D, dtype, flags);
    const bool of32 = (flags & SGSA_FLAG_OUT_F32) || dtype == SGSA_DTYPE_F32;
    // The (batch, head) pairs in groups whose per-chunk operands fit the workspace cap; the
    // groups run one after the other on `st` and reuse the same workspace.
    for (int g0 = 0; g0 < B * H; g0 += group) {
        a.bh0 = g0;
        a.nbh = std::min(group, B * H - g0);
        const size_t nchunk = (size_t)a.nbh * a.NC;
        a.W = (float *)ws;
        a.U = a.W + nchunk * M * D;
        a.Aqk = a.U + nchunk * M * D;
        a.G = a.Aqk + nchunk * kC * M;
        a.Qt = nullptr;
        a.KtT = nullptr;
        cudaError_t e;
        if (tc) {
            float *tail = a.G + nchunk * kC;
            // keep the fp32 operand arrays 16-byte aligned for TMA
            tail = (float *)(((uintptr_t)tail + 255) & ~(uintptr_t)255);
            a.Qt = tail;
            a.KtT = a.Qt + nchunk * kC * D;
            const bool reuse = (flags & SGSA_FLAG_REUSE_PREP);
            cudaEvent_t pd = g0 == 0 ? prep_done : nullptr;  // after the first group's prep
            e = (flags & SGSA_FLAG_OUT_F32) ? run_tc_scan<float>(a, reuse, st, pd)
                                            : run_tc_scan<__nv_bfloat16>(a, reuse, st, pd);
        } else if (dtype == SGSA_DTYPE_F32) {
            e = sparse ? run_d<float, float, true>(D, a, st) : run_d<float, float, false>(D, a, st);
        } else if (of32) {
            e = sparse ? run_d<__nv_bfloat16, float, true>(D, a, st)
                       : run_d<__nv_bfloat16, float, false>(D, a, st);
        } else {
            e = sparse ? run_d<__nv_bfloat16, __nv_bfloat16, true>(D, a, st)
                       : run_d<__nv_bfloat16, __nv_bfloat16, false>(D, a, st);
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace sgsa
