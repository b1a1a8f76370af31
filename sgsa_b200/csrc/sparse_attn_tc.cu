// Fused sparse attention + gate on the tensor cores (bf16, D = 128, DI = 64).
//
// The top-k selection of each query row is an exact threshold on its indexer
// scores (written by the tensor-core indexer): column j <= t is selected iff
// (key(s_tj) & mask) > prefix, or == prefix and j <= cut.  This kernel
// recomputes the indexer scores with the very same tcgen05 instruction
// sequence the indexer used (M=128 query rows, N=64 keys, K=64 in four K=16
// steps, tiles at the same offsets), so the scores -- and the selection -- are
// bit-identical, and evaluates
//     o_s,t = sum_{j selected} softmax_j(q_t . k_j * scale) v_j
//     out_t = mix_t * o_s,t + (1 - mix_t) * o_delta,t
// (modelings/hybrid_dense_delta_topk.py:343-356 and :389-390) over 64-key
// tiles of the causal prefix: S = Q K^T and O += P V on the tensor cores, the
// softmax in fp32 with an online maximum.  Work grows with the causal prefix
// instead of the number of selected rows, but runs at tensor-core rate and
// reads each K/V tile once per 128 queries instead of once per query.
//
// P is fed to the PV MMA as bf16 hi + lo parts (p = hi + lo to ~2^-16), so the
// result keeps fp32-level accuracy with V in bf16.  The running maximum is
// updated lazily: O and the row sum are rescaled only when a tile's maximum
// exceeds the one in use by more than 2^8, which keeps p <= 256 and is exact.
//
// With HI == 1 (a shared-across-heads indexer, one index set per token as in
// the DeepSeek indexer of modelings/deepseek_v3_2.py:435-487) every head reads
// indexer head 0's vectors and thresholds.
//
// Warp roles (96 + 128 kParts threads, one CTA per (b, h, 128-query tile)): warp 0 TMA,
// warp 1 TMEM owner + MMA issuer, warp 2 TMA of the values, warps 3.. kParts
// threads per query row.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace sgsa {
namespace {

static __device__ unsigned int g_attn_watchdog;

constexpr int kRowsA = 128;
constexpr int kNk = 64;  // keys per tile
constexpr int kParts = 4;              // softmax threads per query row
constexpr int kCP = kNk / kParts;      // key columns per thread
constexpr int kOP = 128 / kParts;      // O columns per thread
constexpr int kAttnThreads = 96 + 128 * kParts;
constexpr int kKS = 3;                 // stages of the (indexer key, key) ring
constexpr int kVS = 2;                 // stages of the value ring
namespace L {
constexpr int kQ = 0;                    // Q tile, 2 x 16 KB (K-major, 64-col blocks)
constexpr int kIQ = kQ + 32768;          // IQ tile 16 KB
constexpr int kKStage = kIQ + 16384;     // kKS stages x 24 KB: IK 8 KB | K 2 x 8 KB
constexpr int kKBytes = 24576;
constexpr int kVStage = kKStage + kKS * kKBytes;  // kVS stages x 16 KB: V 2 x 8 KB
constexpr int kVBytes = 16384;
constexpr int kP = kVStage + kVS * kVBytes;  // 2 buffers x (hi 16 KB | lo 16 KB)
constexpr int kBar = kP + 2 * 32768;
constexpr int kBytes = kBar + 256 + 2 * kParts * 128 * 4;  // barriers | tile maxima
constexpr size_t kSmem = 1024 + kBytes;
}  // namespace L

template <typename Tmix, typename Tout>
__global__ void __launch_bounds__(kAttnThreads, 1)
sparse_attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_iq,
                      const __grid_constant__ CUtensorMap tm_ik, const uint4 *__restrict__ thr,
                      const float *__restrict__ od, const Tmix *__restrict__ mix,
                      Tout *__restrict__ out, int B, int T, int H, float scale_log2,
                      int mix_pc, int nqt, const int32_t *__restrict__ q_tiles, int HI) {
    using namespace sm100;
    constexpr int D = 128;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *sm = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(sm + L::kBar);
    uint64_t *qfull = bars, *kfull = bars + 1, *kempty = bars + 4, *vfull = bars + 7,
             *vempty = bars + 9, *sfull = bars + 11, *sfree = bars + 13, *pfull = bars + 15,
             *pfree = bars + 17;
    __shared__ uint32_t s_tmem;
    unsigned int *wd = &g_attn_watchdog;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int BH = B * H;
    const int qt = q_tiles ? q_tiles[blockIdx.x / BH] : nqt - 1 - (int)(blockIdx.x / BH);
    const int bh = (int)(blockIdx.x % BH), b = bh / H, h = bh % H;
    const int hi = (HI == 1) ? 0 : h;  // indexer head: shared by all heads when HI == 1
    const int q0 = qt * kRowsA;
    const int q_last = min(T - 1, q0 + kRowsA - 1);
    const int nkt = q_last / kNk + 1;

    if (threadIdx.x == 0) {
        mbar_init(qfull, 1);
        for (int i = 0; i < kKS; ++i) {
            mbar_init(&kfull[i], 1);
            mbar_init(&kempty[i], 1);
        }
        for (int i = 0; i < kVS; ++i) {
            mbar_init(&vfull[i], 1);
            mbar_init(&vempty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sfull[i], 1);
            mbar_init(&sfree[i], 4 * kParts);
            mbar_init(&pfull[i], 4 * kParts);
            mbar_init(&pfree[i], 1);
        }
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(&s_tmem, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    // TMEM columns: Sidx[2] at 0/64, S[2] at 128/192, O at 256..383
    const uint32_t tSidx = tmem, tS = tmem + 128, tO = tmem + 256;

    if (warp == 0) {  // producer of the query tiles and the (indexer key, key) ring
        if (lane == 0) {
            mbar_arrive_expect_tx(qfull, 32768 + 16384);
            tma_load_3d(sm + L::kQ, &tm_q, qfull, 0, h, b * T + q0);
            tma_load_3d(sm + L::kQ + 16384, &tm_q, qfull, 64, h, b * T + q0);
            tma_load_3d(sm + L::kIQ, &tm_iq, qfull, 0, hi, b * T + q0);
            for (int j = 0; j < nkt; ++j) {
                const int st = j % kKS;
                mbar_wait(&kempty[st], ((j / kKS) & 1) ^ 1, wd, 1u);
                unsigned char *stg = sm + L::kKStage + st * L::kKBytes;
                mbar_arrive_expect_tx(&kfull[st], L::kKBytes);
                const int row = b * T + j * kNk;
                tma_load_3d(stg, &tm_ik, &kfull[st], 0, hi, row);
                tma_load_3d(stg + 8192, &tm_k, &kfull[st], 0, h, row);
                tma_load_3d(stg + 16384, &tm_k, &kfull[st], 64, h, row);
            }
        }
        __syncwarp();
    } else if (warp == 2) {  // producer of the value ring
        if (lane == 0) {
            for (int j = 0; j < nkt; ++j) {
                const int st = j % kVS;
                mbar_wait(&vempty[st], ((j / kVS) & 1) ^ 1, wd, 1u);
                unsigned char *stg = sm + L::kVStage + st * L::kVBytes;
                mbar_arrive_expect_tx(&vfull[st], L::kVBytes);
                const int row = b * T + j * kNk;
                tma_load_3d(stg, &tm_v, &vfull[st], 0, h, row);
                tma_load_3d(stg + 8192, &tm_v, &vfull[st], 64, h, row);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_bf16_f32(128, kNk);
            constexpr uint32_t id_pv = idesc_bf16_f32_bmn(128, D);
            const uint32_t aq = smem_u32(sm + L::kQ), aiq = smem_u32(sm + L::kIQ);
            mbar_wait(qfull, 0, wd, 2u);
            auto issue_pv = [&](int jj) {
                const int pb = jj & 1;
                const int vs = jj % kVS;
                mbar_wait(&vfull[vs], (jj / kVS) & 1, wd, 4u);
                mbar_wait(&pfull[pb], (jj >> 1) & 1, wd, 4u);
                tc_fence_after();
                const uint32_t ph = smem_u32(sm + L::kP + pb * 32768);
                const uint32_t vq = smem_u32(sm + L::kVStage + vs * L::kVBytes);
#pragma unroll
                for (int part = 0; part < 2; ++part)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = sdesc_kmajor_sw128(ph + part * 16384 + kk * 32);
                        const uint64_t bd = sdesc_mnmajor_sw128(vq + kk * 2048, 8192, 1024);
                        mma_bf16(tO, ad, bd, id_pv, (jj | part | kk) ? 1u : 0u);
                    }
                mma_commit(&pfree[pb]);
                mma_commit(&vempty[vs]);
            };
            for (int j = 0; j < nkt; ++j) {
                const int st = j % kKS, buf = j & 1;
                mbar_wait(&kfull[st], (j / kKS) & 1, wd, 8u);
                mbar_wait(&sfree[buf], ((j >> 1) & 1) ^ 1, wd, 16u);
                tc_fence_after();
                const uint32_t stg = smem_u32(sm + L::kKStage + st * L::kKBytes);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)  // indexer scores: same sequence as the indexer
                    mma_bf16(tSidx + buf * kNk, sdesc_kmajor_sw128(aiq + kk * 32),
                             sdesc_kmajor_sw128(stg + kk * 32), id_s, kk ? 1u : 0u);
#pragma unroll
                for (int kb = 0; kb < 2; ++kb)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_bf16(tS + buf * kNk, sdesc_kmajor_sw128(aq + kb * 16384 + kk * 32),
                                 sdesc_kmajor_sw128(stg + 8192 + kb * 8192 + kk * 32), id_s,
                                 (kb | kk) ? 1u : 0u);
                mma_commit(&sfull[buf]);
                mma_commit(&kempty[st]);
                if (j > 0) issue_pv(j - 1);
            }
            issue_pv(nkt - 1);
        }
        __syncwarp();
    } else {
        // kParts threads per query row: warps w, w+4, w+8, ... share a TMEM lane
        // quarter; `part` picks kCP of the tile's 64 key columns (and kOP of O's).
        const int quad = warp & 3, r = quad * 32 + lane, part = (warp - 3) >> 2;
        const int t = q0 + r;
        const bool valid_row = t < T;
        const uint32_t lrow = (uint32_t)(quad * 32) << 16;
        float *xmax = (float *)(sm + L::kBar + 256);  // [2 tiles][kParts][128 rows]
        uint4 th = make_uint4(0u, 0xffffffffu, 0u, 0u);  // selects nothing
        if (valid_row) th = thr[((size_t)b * HI + hi) * T + t];
        // The threshold as a float: key(s) & mask > prefix, or == prefix and j <= cut, is
        // s > a || (s == a && j <= cut) with a the float whose key is the prefix (its
        // unmasked bits are zero; a partial mask always comes with cut = max, which makes
        // both forms "key(s) >= prefix").  mask 0 selects every column (a = -inf).
        const uint32_t prefix = th.x, mask = th.y;
        const int cut = (int)th.z;
        const float a_thr = mask == 0u ? -INFINITY
                                       : __uint_as_float((prefix & 0x80000000u) ? (prefix & 0x7fffffffu) : ~prefix);
        float m_used = -INFINITY, l = 0.f;
        for (int j = 0; j < nkt; ++j) {
            const int buf = j & 1;
            mbar_wait(&sfull[buf], (j >> 1) & 1, wd, 32u);
            tc_fence_after();
            float x[kCP], si[kCP], sv[kCP];
            float mt = -INFINITY;
            tmem_ld16(tSidx + lrow + buf * kNk + part * kCP, si);
            tmem_ld16(tS + lrow + buf * kNk + part * kCP, sv);
            const int jb = j * kNk + part * kCP;
            const bool full = jb + kCP - 1 <= q0;  // every row of the tile sees all columns
#pragma unroll
            for (int i = 0; i < kCP; ++i) {
                const int jj = jb + i;
                const bool sel = (full || jj <= t) && (si[i] > a_thr || (si[i] == a_thr && jj <= cut));
                const float xv = sel ? sv[i] * scale_log2 : -INFINITY;
                x[i] = xv;
                mt = fmaxf(mt, xv);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sfree[buf]);
            xmax[(buf * kParts + part) * 128 + r] = mt;
            asm volatile("bar.sync 1, %0;" ::"r"(kParts * 128) : "memory");
#pragma unroll
            for (int p2 = 0; p2 < kParts; ++p2) mt = fmaxf(mt, xmax[(buf * kParts + p2) * 128 + r]);
            // lazy maximum: rescale only when this tile's maximum is > m_used + 8
            const bool grow = mt > m_used + 8.f || (m_used == -INFINITY && mt != -INFINITY);
            if (__any_sync(0xffffffffu, grow)) {
                const float m_new = grow ? mt : m_used;
                const float f = (m_used == -INFINITY) ? 0.f : exp2f(m_used - m_new);
                l *= (grow ? f : 1.f);
                if (j > 0) {  // O holds tiles < j: wait for the last PV into it
                    mbar_wait(&pfree[(j - 1) & 1], ((j - 1) >> 1) & 1, wd, 64u);
                    tc_fence_after();
                    float o[32];
                    tmem_ld32(tO + lrow + part * kOP, o);
                    const float g = grow ? f : 1.f;
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= g;
                    tmem_st32(tO + lrow + part * kOP, o);
                    tc_fence_before();
                }
                if (grow) m_used = m_new;
            }
            // P = exp2(x - m_used) as bf16 hi + lo, K-major rows of 64 keys
            const float mref = (m_used == -INFINITY) ? 0.f : m_used;  // x = -inf -> p = 0
            if (j >= 2) mbar_wait(&pfree[buf], ((j >> 1) & 1) ^ 1, wd, 128u);
            unsigned char *ph = sm + L::kP + buf * 32768;
#pragma unroll
            for (int c8 = 0; c8 < kCP / 8; ++c8) {
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float p0 = exp2f(x[c8 * 8 + 2 * u] - mref);
                    const float p1 = exp2f(x[c8 * 8 + 2 * u + 1] - mref);
                    l += p0 + p1;
                    const __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
                    const float2 hf = __bfloat1622float2(h2);
                    const __nv_bfloat162 l2 = __floats2bfloat162_rn(p0 - hf.x, p1 - hf.y);
                    hi[u] = *reinterpret_cast<const uint32_t *>(&h2);
                    lo[u] = *reinterpret_cast<const uint32_t *>(&l2);
                }
                const int chunk = part * (kCP / 8) + c8;
                const uint32_t off = (uint32_t)r * 128 + (uint32_t)((chunk ^ (r & 7)) << 4);
                *(uint4 *)(ph + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *(uint4 *)(ph + 16384 + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&pfull[buf]);
        }
        // epilogue: out = mix * O / l + (1 - mix) * o_delta, l summed over the parts
        xmax[part * 128 + r] = l;
        asm volatile("bar.sync 1, %0;" ::"r"(kParts * 128) : "memory");
        l = 0.f;
#pragma unroll
        for (int p2 = 0; p2 < kParts; ++p2) l += xmax[p2 * 128 + r];
        mbar_wait(&pfree[(nkt - 1) & 1], ((nkt - 1) >> 1) & 1, wd, 256u);
        tc_fence_after();
        const float inv = (l > 0.f) ? 1.f / l : 0.f;
        const size_t rowq = ((size_t)b * T + t) * H + h;
        {
            float o[32];
            const int c0 = part * kOP;
            tmem_ld32(tO + lrow + c0, o);
            if (valid_row) {
                Tout *dst = out + rowq * D + c0;
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    float r0 = o[i] * inv, r1 = o[i + 1] * inv;
                    if (od) {
                        const size_t e = rowq * D + c0 + i;
                        const float m0 = mix ? to_f32(mix_pc ? mix[e] : mix[rowq]) : 1.f;
                        const float m1 = mix ? to_f32(mix_pc ? mix[e + 1] : mix[rowq]) : 1.f;
                        r0 = m0 * r0 + (1.f - m0) * od[e];
                        r1 = m1 * r1 + (1.f - m1) * od[e + 1];
                    }
                    if constexpr (sizeof(Tout) == 2) {
                        *reinterpret_cast<__nv_bfloat162 *>(dst + i) = __floats2bfloat162_rn(r0, r1);
                    } else {
                        *reinterpret_cast<float2 *>(dst + i) = make_float2(r0, r1);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace

bool sparse_attn_tc_eligible(int T, int D, int DI, int dtype) {
    (void)T;
    return dtype == SGSA_DTYPE_BF16 && D == 128 && DI == 64;
}

cudaError_t launch_sparse_attn_tc(const void *q, const void *k, const void *v, const void *iq,
                                  const void *ik, const uint32_t *thr, const float *od,
                                  const void *mix, void *out, int B, int T, int H, float scale,
                                  int mix_pc, const int32_t *q_tiles, int n_tiles, bool out_f32,
                                  int HI, cudaStream_t st) {
    CUtensorMap mq, mk, mv, miq, mik;
    if (!make_tmap_rows_bf16(&mq, q, B, T, H, 128, 128) ||
        !make_tmap_rows_bf16(&mk, k, B, T, H, 128, kNk) ||
        !make_tmap_rows_bf16(&mv, v, B, T, H, 128, kNk) ||
        !make_tmap_rows_bf16(&miq, iq, B, T, HI, 64, 128) ||
        !make_tmap_rows_bf16(&mik, ik, B, T, HI, 64, kNk))
        return cudaErrorInvalidValue;
    const int nqt = ceil_div(T, kRowsA);
    const int ntiles = q_tiles ? n_tiles : nqt;
    if (ntiles <= 0) return cudaSuccess;
    const float sl = scale * 1.4426950408889634f;
    if (out_f32) {
        auto kern = sparse_attn_tc_kernel<__nv_bfloat16, float>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)L::kSmem);
        if (e != cudaSuccess) return e;
        kern<<<ntiles * B * H, kAttnThreads, L::kSmem, st>>>(
            mq, mk, mv, miq, mik, (const uint4 *)thr, od, (const __nv_bfloat16 *)mix,
            (float *)out, B, T, H, sl, mix_pc, nqt, q_tiles, HI);
    } else {
        auto kern = sparse_attn_tc_kernel<__nv_bfloat16, __nv_bfloat16>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)L::kSmem);
        if (e != cudaSuccess) return e;
        kern<<<ntiles * B * H, kAttnThreads, L::kSmem, st>>>(
            mq, mk, mv, miq, mik, (const uint4 *)thr, od, (const __nv_bfloat16 *)mix,
            (__nv_bfloat16 *)out, B, T, H, sl, mix_pc, nqt, q_tiles, HI);
    }
    return cudaGetLastError();
}

unsigned int read_attn_watchdog(cudaStream_t st) {
    unsigned int v = 0, z = 0;
    if (cudaStreamSynchronize(st) != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyFromSymbol(&v, g_attn_watchdog, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (v) cudaMemcpyToSymbol(g_attn_watchdog, &z, sizeof(z));
    return v;
}

}  // namespace sgsa
