// Fused sparse attention + gate on the tensor cores (bf16, D = 128, DI = 64).
//
// The top-k selection of each query row is an exact threshold on its indexer
// scores (written by the tensor-core indexer): column j <= t is selected iff
// (key(s_tj) & mask) > prefix, or == prefix and j <= cut.  This kernel
// recomputes the indexer scores with the very same tcgen05 instruction
// sequence the indexer used (M=128 query rows from tensor memory, N=128 keys,
// K=64 in four K=16 steps, tiles at the same offsets), so the scores -- and the
// selection -- are bit-identical, and evaluates
//     o_s,t = sum_{j selected} softmax_j(q_t . k_j * scale) v_j
//     out_t = mix_t * o_s,t + (1 - mix_t) * o_delta,t
// (modelings/hybrid_dense_delta_topk.py:343-356 and :389-390) over 128-key
// tiles of the causal prefix: S = Q K^T and O += P V on the tensor cores, the
// softmax in fp32.  Work grows with the causal prefix instead of the number of
// selected rows, but runs at tensor-core rate and reads each K/V tile once per
// 128 queries instead of once per query.
//
// Operands: the query tiles (q and the indexer's iq) sit in tensor memory as the
// A operand of the score MMAs, so those MMAs read only the key tile from shared
// memory; P is fed to the PV MMA from shared memory as bf16 hi + lo parts
// (p = hi + lo to ~2^-16), so the result keeps fp32-level accuracy with V in
// bf16.  The score MMAs use N = 128 (two 64-key TMA stages): with N = 64 an MMA
// instruction took about as long as one with N = 128.  The scores of the next
// tile are computed as soon as the softmax has read the current ones; P has its
// own shared-memory tiles.
//
// The softmax reference is a fixed bound (max|q| max|k| scale, from a norm
// pre-pass) when that keeps p within 2^-120.  Otherwise (no norm pass, or large
// norms) a lazy running maximum is kept per row (the row's threads exchange
// their tile maxima): O and the row sum are rescaled only when a tile's maximum
// exceeds the one in use by more than 2^8, which keeps p <= 256 and is exact.
//
// With HI == 1 (a shared-across-heads indexer, one index set per token as in
// the DeepSeek indexer of modelings/deepseek_v3_2.py:435-487) every head reads
// indexer head 0's vectors and thresholds.
//
// Warp roles (96 + 128 kParts threads, one CTA per (b, h, 128-query tile)): warp 0
// TMA of the indexer-key and key rings, warp 1 TMEM owner + MMA issuer, warp 2 TMA
// of the value ring, warps 3.. softmax: kParts threads per query row, 32 keys of
// each tile each.  The MMA warp issues event-driven: the scores of a tile once its
// keys have landed and the previous scores have been read, PV in order once P and
// V are there.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace sgsa {
namespace {

static __device__ unsigned int g_check;  // bounds-checked build only

static __device__ unsigned int g_attn_watchdog;

constexpr int kRowsA = 128;
constexpr int kNk = 128;               // keys per tile (the N of the score MMAs)
constexpr int kBlk = 64;               // keys per TMA stage (two stages form a tile)
constexpr int kParts = 4;              // threads per query row
constexpr int kCP = kNk / kParts;      // key columns per thread
constexpr int kSoftThreads = 128 * kParts;
constexpr int kAttnThreads = 96 + kSoftThreads;
constexpr int kKS = 4;                 // 64-key stages of the indexer-key and key rings (even)
constexpr int kVS = 3;                 // 64-key stages of the value ring
namespace L {
// Three rings of 64-key stages: IK (8 KB), K columns 0-63 (8 KB), K columns 64-127
// (8 KB); stages 2i and 2i+1 are adjacent, so a 128-key tile is one K-major operand
// (128 rows, 128-byte swizzle) in each ring.
constexpr int kIK = 0;
constexpr int kK0 = kIK + kKS * 8192;
constexpr int kK1 = kK0 + kKS * 8192;
constexpr int kVStage = kK1 + kKS * 8192;         // kVS stages x 16 KB: V columns 0-63 | 64-127
constexpr int kVBytes = 16384;
constexpr int kP = kVStage + kVS * kVBytes;       // P hi 2 x 16 KB | P lo 2 x 16 KB (64-key blocks)
constexpr int kPBytes = 65536;
constexpr int kBar = kP + kPBytes;
constexpr int kXmax = kBar + 256;                 // [slot][part][row] floats
constexpr int kLrow = kXmax + 2 * kParts * 128 * 4;  // [part][row]
constexpr int kBytes = kLrow + kParts * 128 * 4;
constexpr size_t kSmem = 1024 + kBytes;
}  // namespace L
static_assert(L::kSmem <= 232448, "shared memory");
static_assert(kKS % 2 == 0, "a tile takes two adjacent key stages");

// TMEM columns (512): O, the query tiles (bf16 pairs), the indexer scores and the
// scores of the current tile.
constexpr uint32_t kTO = 0, kTQ = 128, kTIQ = 192, kTSidx = 256, kTS = 384;

template <typename Tmix, typename Tout>
__global__ void __launch_bounds__(kAttnThreads, 1)
sparse_attn_tc_kernel(const __nv_bfloat16 *__restrict__ q,
                      const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v,
                      const __nv_bfloat16 *__restrict__ iq,
                      const __grid_constant__ CUtensorMap tm_ik, const uint4 *__restrict__ thr,
                      const float *__restrict__ od, const Tmix *__restrict__ mix,
                      Tout *__restrict__ out, int B, int T, int H, float scale_log2,
                      int mix_pc, int nqt, const int32_t *__restrict__ q_tiles, int HI,
                      const uint32_t *__restrict__ qkmax, float *__restrict__ dbg_scores) {
    using namespace sm100;
    constexpr int D = 128;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *sm = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(sm + L::kBar);
    uint64_t *kfull = bars, *kempty = bars + kKS, *vfull = bars + 2 * kKS,
             *vempty = vfull + kVS, *sfull = vempty + kVS, *sfree = sfull + 1, *pfull = sfree + 1,
             *pfree = pfull + 1;
    __shared__ uint32_t s_tmem;
    unsigned int *wd = &g_attn_watchdog;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int BH = B * H;
    const int qt = q_tiles ? q_tiles[blockIdx.x / BH] : nqt - 1 - (int)(blockIdx.x / BH);
    const int bh = (int)(blockIdx.x % BH), b = bh / H, h = bh % H;
    const int hi = (HI == 1) ? 0 : h;  // indexer head: shared by all heads when HI == 1
    const int q0 = qt * kRowsA;
    const int q_last = min(T - 1, q0 + kRowsA - 1);
    const int nkt = q_last / kNk + 1;  // 128-key tiles
    const int nblk = 2 * nkt;          // 64-key stages

    if (threadIdx.x == 0) {
        for (int i = 0; i < kKS; ++i) {
            mbar_init(&kfull[i], 1);
            mbar_init(&kempty[i], 1);
        }
        for (int i = 0; i < kVS; ++i) {
            mbar_init(&vfull[i], 1);
            mbar_init(&vempty[i], 1);
        }
        mbar_init(sfull, 1);
        mbar_init(sfree, kSoftThreads / 32);
        mbar_init(pfull, kSoftThreads / 32);
        mbar_init(pfree, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(&s_tmem, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    if (warp >= 3) {
        // The query tiles into tensor memory (A operand: row = lane, bf16 pairs in 32-bit
        // columns): the four warps of a lane quarter take a quarter of each row each.
        const int w4 = (warp - 3) >> 2, quad = warp & 3;
        const int t = q0 + quad * 32 + lane;
        const bool ok = t < T;
        const uint32_t lq = (uint32_t)(quad * 32) << 16;
        const uint4 *sq = reinterpret_cast<const uint4 *>(q + (((size_t)b * T + t) * H + h) * D + 32 * w4);
        const uint4 *si = reinterpret_cast<const uint4 *>(iq + (((size_t)b * T + t) * HI + hi) * 64 + 16 * w4);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const uint4 u0 = ok ? sq[2 * c] : make_uint4(0u, 0u, 0u, 0u);
            const uint4 u1 = ok ? sq[2 * c + 1] : make_uint4(0u, 0u, 0u, 0u);
            const uint32_t w8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
            tmem_st8u(tmem + lq + kTQ + 16 * w4 + 8 * c, w8);
        }
        {
            const uint4 u0 = ok ? si[0] : make_uint4(0u, 0u, 0u, 0u);
            const uint4 u1 = ok ? si[1] : make_uint4(0u, 0u, 0u, 0u);
            const uint32_t w8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
            tmem_st8u(tmem + lq + kTIQ + 8 * w4, w8);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == 0) {  // producer of the indexer-key and key rings, 64 keys per stage
        if (lane == 0) {
            for (int j = 0; j < nblk; ++j) {
                const int st = j % kKS;
                mbar_wait(&kempty[st], ((j / kKS) & 1) ^ 1, wd, 1u);
                mbar_arrive_expect_tx(&kfull[st], 3 * 8192);
                const int row = b * T + j * kBlk;
                tma_load_3d(sm + L::kIK + st * 8192, &tm_ik, &kfull[st], 0, hi, row);
                tma_load_3d(sm + L::kK0 + st * 8192, &tm_k, &kfull[st], 0, h, row);
                tma_load_3d(sm + L::kK1 + st * 8192, &tm_k, &kfull[st], 64, h, row);
            }
        }
        __syncwarp();
    } else if (warp == 2) {  // producer of the value ring
        if (lane == 0) {
            for (int j = 0; j < nblk; ++j) {
                const int st = j % kVS;
                mbar_wait(&vempty[st], ((j / kVS) & 1) ^ 1, wd, 1u);
                unsigned char *stg = sm + L::kVStage + st * L::kVBytes;
                mbar_arrive_expect_tx(&vfull[st], L::kVBytes);
                const int row = b * T + j * kBlk;
                tma_load_3d(stg, &tm_v, &vfull[st], 0, h, row);
                tma_load_3d(stg + 8192, &tm_v, &vfull[st], 64, h, row);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_bf16_f32(128, kNk);
            constexpr uint32_t id_pv = idesc_bf16_f32_bmn(128, D);
            const uint32_t tq = tmem + kTQ, tiq = tmem + kTIQ;
            // Event-driven issue: S(js) once its two key stages have landed and the scores
            // of tile js - 1 have been read; PV(jp), in order, once P(jp) and its two value
            // stages are there.
            int js = 0, jp = 0;
            uint32_t idle = 0;
            while (jp < nkt) {
                bool progress = false;
                if (js < nkt) {
                    const int st = (2 * js) % kKS;  // and st + 1
                    const uint32_t kph = ((2 * js) / kKS) & 1;
                    if (mbar_test_wait(&kfull[st], kph) && mbar_test_wait(&kfull[st + 1], kph) &&
                        mbar_test_wait(sfree, (js & 1) ^ 1)) {
                        tc_fence_after();
                        const uint32_t aik = smem_u32(sm + L::kIK + st * 8192);
                        const uint32_t ak0 = smem_u32(sm + L::kK0 + st * 8192);
                        const uint32_t ak1 = smem_u32(sm + L::kK1 + st * 8192);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)  // indexer scores: same sequence as the indexer
                            mma_bf16_ts(tmem + kTSidx, tiq + kk * 8, sdesc_kmajor_sw128(aik + kk * 32),
                                        id_s, kk ? 1u : 0u);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_bf16_ts(tmem + kTS, tq + kk * 8, sdesc_kmajor_sw128(ak0 + kk * 32), id_s,
                                        kk ? 1u : 0u);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_bf16_ts(tmem + kTS, tq + 32 + kk * 8, sdesc_kmajor_sw128(ak1 + kk * 32),
                                        id_s, 1u);
                        mma_commit(sfull);
                        mma_commit(&kempty[st]);
                        mma_commit(&kempty[st + 1]);
                        ++js;
                        progress = true;
                    }
                }
                if (jp < js) {  // PV of tile jp into O
                    const int v0 = (2 * jp) % kVS, v1 = (2 * jp + 1) % kVS;
                    if (mbar_test_wait(&vfull[v0], ((2 * jp) / kVS) & 1) &&
                        mbar_test_wait(&vfull[v1], ((2 * jp + 1) / kVS) & 1) &&
                        mbar_test_wait(pfull, jp & 1)) {
                        tc_fence_after();
                        // P from shared memory (K-major, 128-byte swizzle, 64-key blocks): the hi
                        // parts at +0, the lo parts at +32 KB
                        const uint32_t pq = smem_u32(sm + L::kP);
#pragma unroll
                        for (int blk = 0; blk < 2; ++blk) {
                            const uint32_t vq = smem_u32(sm + L::kVStage + (blk ? v1 : v0) * L::kVBytes);
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) {
                                const uint64_t bd = sdesc_mnmajor_sw128(vq + kk * 2048, 8192, 1024);
                                mma_bf16(tmem + kTO, sdesc_kmajor_sw128(pq + blk * 16384 + kk * 32), bd,
                                         id_pv, (jp | blk | kk) ? 1u : 0u);
                                mma_bf16(tmem + kTO, sdesc_kmajor_sw128(pq + 32768 + blk * 16384 + kk * 32),
                                         bd, id_pv, 1u);
                            }
                        }
                        mma_commit(pfree);
                        mma_commit(&vempty[v0]);
                        mma_commit(&vempty[v1]);
                        ++jp;
                        progress = true;
                    }
                }
                if (progress) {
                    idle = 0;
                } else if (++idle > kSpinLimit) {  // nothing moved for a long time: give up
                    atomicOr(wd, 8u);
                    break;
                } else if ((idle & 1023u) == 1023u && *(volatile unsigned int *)wd) {
                    break;
                }
            }
        }
        __syncwarp();
    } else {
        // kParts threads per query row, every key tile: warps 3 + 4 p + i take TMEM lane
        // quarter (warp & 3) and keys [32 p, 32 p + 32) of the tile.
        const int sw = warp - 3, part = sw >> 2;
        const int quad = warp & 3, r = quad * 32 + lane;
        const int t = q0 + r;
        const bool valid_row = t < T;
        const uint32_t lrow = (uint32_t)(quad * 32) << 16;
        float *xmax = (float *)(sm + L::kXmax);
        float *lrow_s = (float *)(sm + L::kLrow);
        uint4 th = make_uint4(0u, 0xffffffffu, 0u, 0u);  // selects nothing
        if (valid_row) th = thr[((size_t)b * HI + hi) * T + t];
        if (kCheckBuild && valid_row && th.w != 1u) SGSA_CHECK_FAIL(g_check, kChkThresholdRecord);
        // The threshold as a float: key(s) & mask > prefix, or == prefix and j <= cut, is
        // s > a || (s == a && j <= cut) with a the float whose key is the prefix (its
        // unmasked bits are zero; a partial mask always comes with cut = max, which makes
        // both forms "key(s) >= prefix").  mask 0 selects every column (a = -inf).
        const uint32_t prefix = th.x, mask = th.y;
        const int cut = (int)th.z;
        const float a_thr = mask == 0u ? -INFINITY
                                       : __uint_as_float((prefix & 0x80000000u) ? (prefix & 0x7fffffffu) : ~prefix);
        // Fixed reference maximum: with |s| <= max|q| max|k| (Cauchy-Schwarz, per head),
        // bound = max|q| max|k| * scale * log2(e) is >= every x, and when it is <= 60,
        // p = 2^(x - bound) stays in [2^-120, ~1]: no running maximum, no exchange
        // between the row's threads, no rescaling of O.
        bool use_bound = false;
        float m_used = -INFINITY, l = 0.f;
        if (qkmax) {
            const float qm2 = __uint_as_float(qkmax[2 * bh]), km2 = __uint_as_float(qkmax[2 * bh + 1]);
            const float bound = sqrtf(qm2) * sqrtf(km2) * scale_log2;
            if (bound <= 60.f) {
                use_bound = true;
                m_used = bound;
            }
        }
        // no row of this warp has a tie cut (the common case): selection is s >= a
        const bool tie_free = __all_sync(0xffffffffu, cut == 0x7fffffff);
        for (int j = 0; j < nkt; ++j) {
            mbar_wait(sfull, j & 1, wd, 32u);
            tc_fence_after();
            float x[kCP];
            float mt = -INFINITY;
            const int jb0 = j * kNk + part * kCP;
            const bool full = jb0 + kCP - 1 <= q0;  // every row of the tile sees all columns
            // x = the raw score where selected, -inf elsewhere (scaled inside the exponent);
            // off the diagonal and without tie cuts in the warp the test is one compare
            const bool simple = full && tie_free;
            {
                // both 32-column loads in flight before one wait
                uint32_t rsi[32], rsv[32];
                tmem_ld32_issue(tmem + kTSidx + lrow + part * kCP, rsi);
                tmem_ld32_issue(tmem + kTS + lrow + part * kCP, rsv);
                tmem_ld_wait(rsi);
                tmem_ld_wait(rsv);
                if (dbg_scores && valid_row) {  // test support: the recomputed indexer scores
                    float *dr = dbg_scores + ((size_t)bh * T + t) * T;
#pragma unroll
                    for (int i = 0; i < kCP; ++i)
                        if (jb0 + i <= t) dr[jb0 + i] = __uint_as_float(rsi[i]);
                }
                if (simple) {
#pragma unroll
                    for (int i = 0; i < kCP; ++i)
                        x[i] = __uint_as_float(rsi[i]) >= a_thr ? __uint_as_float(rsv[i]) : -INFINITY;
                } else {
#pragma unroll
                    for (int i = 0; i < kCP; ++i) {
                        const int jj = jb0 + i;
                        const float si = __uint_as_float(rsi[i]);
                        const bool sel = (full || jj <= t) && (si > a_thr || (si == a_thr && jj <= cut));
                        x[i] = sel ? __uint_as_float(rsv[i]) : -INFINITY;
                    }
                }
            }
            if (!use_bound) {
#pragma unroll
                for (int i = 0; i < kCP; ++i) mt = fmaxf(mt, x[i]);
                mt *= scale_log2;  // scale > 0: the maximum of the scaled scores
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sfree);
            if (!use_bound) {  // lazy running maximum, shared by the row's threads
                const int slot = j & 1;
                xmax[(slot * kParts + part) * 128 + r] = mt;
                asm volatile("bar.sync 1, %0;" ::"r"(kSoftThreads) : "memory");
#pragma unroll
                for (int p2 = 0; p2 < kParts; ++p2)
                    mt = fmaxf(mt, xmax[(slot * kParts + p2) * 128 + r]);
                // lazy maximum: rescale only when this tile's maximum is > m_used + 8
                const bool grow = mt > m_used + 8.f || (m_used == -INFINITY && mt != -INFINITY);
                if (__any_sync(0xffffffffu, grow)) {
                    const float m_new = grow ? mt : m_used;
                    const float f = (m_used == -INFINITY) ? 0.f : exp2f(m_used - m_new);
                    l *= (grow ? f : 1.f);
                    if (j > 0) {  // O holds the earlier tiles
                        mbar_wait(pfree, (j - 1) & 1, wd, 64u);
                        tc_fence_after();
                        const float gsc = grow ? f : 1.f;
#pragma unroll 1
                        for (int c = 0; c < 2; ++c) {
                            float o[16];
                            const uint32_t oa = tmem + kTO + lrow + part * 32 + c * 16;
                            tmem_ld16(oa, o);
#pragma unroll
                            for (int i = 0; i < 16; ++i) o[i] *= gsc;
                            tmem_st16(oa, o);
                        }
                        tc_fence_before();
                    }
                    if (grow) m_used = m_new;
                }
            }
            // P = exp2(x - m_used) as bf16 hi + lo parts into the P tiles in shared memory
            // (K-major, 128-byte swizzle, 64-key blocks): the A operand of PV
            const float mref = (m_used == -INFINITY) ? 0.f : m_used;  // x = -inf -> p = 0
            {
                uint32_t hw[16], lw[16];
                const float2 sc2 = make_float2(scale_log2, scale_log2), nm2 = make_float2(-mref, -mref);
                float2 l2s = make_float2(0.f, 0.f);
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const float2 e2 = fma2(make_float2(x[2 * u], x[2 * u + 1]), sc2, nm2);
                    const float2 p2 = make_float2(ex2_approx(e2.x), ex2_approx(e2.y));
                    l2s = add2(l2s, p2);
                    const __nv_bfloat162 h2 = __floats2bfloat162_rn(p2.x, p2.y);
                    const float2 lo = sub2(p2, __bfloat1622float2(h2));
                    const __nv_bfloat162 l2 = __floats2bfloat162_rn(lo.x, lo.y);
                    hw[u] = *reinterpret_cast<const uint32_t *>(&h2);
                    lw[u] = *reinterpret_cast<const uint32_t *>(&l2);
                }
                l += l2s.x + l2s.y;
                // the previous PV must have read the P tiles before they are rewritten
                if (j > 0) mbar_wait(pfree, (j - 1) & 1, wd, 128u);
                unsigned char *ph = sm + L::kP + (part >> 1) * 16384;
                const uint32_t rbase = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4) {  // 16-byte chunk c holds keys 8c .. 8c + 7 of the block
                    const uint32_t off = rbase + ((uint32_t)(((part & 1) * 4 + c4) ^ (r & 7)) << 4);
                    *reinterpret_cast<uint4 *>(ph + off) =
                        make_uint4(hw[4 * c4], hw[4 * c4 + 1], hw[4 * c4 + 2], hw[4 * c4 + 3]);
                    *reinterpret_cast<uint4 *>(ph + 32768 + off) =
                        make_uint4(lw[4 * c4], lw[4 * c4 + 1], lw[4 * c4 + 2], lw[4 * c4 + 3]);
                }
                fence_proxy_async();  // the generic-proxy stores, before the tensor core reads them
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(pfull);
        }
        // out = mix * O / l + (1 - mix) * o_delta
        lrow_s[part * 128 + r] = l;
        asm volatile("bar.sync 1, %0;" ::"r"(kSoftThreads) : "memory");
        float lsum = 0.f;
#pragma unroll
        for (int p2 = 0; p2 < kParts; ++p2) lsum += lrow_s[p2 * 128 + r];
        const float inv = (lsum > 0.f) ? 1.f / lsum : 0.f;
        // wait for the last PV (the tensor pipe completes them in order)
        mbar_wait(pfree, (nkt - 1) & 1, wd, 256u);
        tc_fence_after();
        const size_t rowq = ((size_t)b * T + t) * H + h;
        const int c0 = part * 32;  // this thread's 32 output columns
        // the row's mix when it is one value per row
        const float mrow_v = (od && mix && !mix_pc && valid_row) ? to_f32(mix[rowq]) : 1.f;
#pragma unroll 1
        for (int hc = 0; hc < 2; ++hc) {
            const int cc = c0 + hc * 16;
            float o[16];
            tmem_ld16(tmem + kTO + lrow + cc, o);
            if (valid_row) {
                const size_t e = rowq * D + cc;  // 16 consecutive columns: 16-byte vectors
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] *= inv;
                if (od) {
                    float dv[16], mv[16];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 f = reinterpret_cast<const float4 *>(od + e)[i];
                        dv[4 * i] = f.x; dv[4 * i + 1] = f.y; dv[4 * i + 2] = f.z; dv[4 * i + 3] = f.w;
                    }
                    if (mix && mix_pc) {
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            const uint4 u = reinterpret_cast<const uint4 *>(mix + e)[i];
                            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[j]));
                                mv[8 * i + 2 * j] = f.x;
                                mv[8 * i + 2 * j + 1] = f.y;
                            }
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) mv[i] = mrow_v;
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[i] = mv[i] * o[i] + (1.f - mv[i]) * dv[i];
                }
                if constexpr (sizeof(Tout) == 2) {
                    uint32_t w[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const __nv_bfloat162 h2 = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
                        w[i] = *reinterpret_cast<const uint32_t *>(&h2);
                    }
                    uint4 *dst = reinterpret_cast<uint4 *>(out + e);
                    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                } else {
                    float4 *dst = reinterpret_cast<float4 *>(out + e);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// max_t |q_t|^2 and max_t |k_t|^2 of each (b, h) (D = 128, bf16) into out[2 (b H + h) + {0, 1}]
// as float bits (non-negative floats order as unsigned integers).  One block per
// (kNormRows tokens, b h), a warp per token row.
constexpr int kNormRows = 256;
__global__ void __launch_bounds__(256) qk_norm_max_kernel(const __nv_bfloat16 *__restrict__ q,
                                                          const __nv_bfloat16 *__restrict__ k,
                                                          uint32_t *__restrict__ out, int T, int H) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, bh = blockIdx.y;
    const int b = bh / H, h = bh % H;
    float mq = 0.f, mk = 0.f;
    for (int t = blockIdx.x * kNormRows + warp; t < min(T, (blockIdx.x + 1) * kNormRows); t += 8) {
        const size_t off = (((size_t)b * T + t) * H + h) * 128 + lane * 4;
        const uint2 uq = *reinterpret_cast<const uint2 *>(q + off);
        const uint2 uk = *reinterpret_cast<const uint2 *>(k + off);
        const float2 q0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&uq.x));
        const float2 q1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&uq.y));
        const float2 k0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&uk.x));
        const float2 k1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&uk.y));
        float sq = q0.x * q0.x + q0.y * q0.y + q1.x * q1.x + q1.y * q1.y;
        float sk = k0.x * k0.x + k0.y * k0.y + k1.x * k1.x + k1.y * k1.y;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
            sk += __shfl_xor_sync(0xffffffffu, sk, o);
        }
        mq = fmaxf(mq, sq);
        mk = fmaxf(mk, sk);
    }
    __shared__ float red[2][8];
    if (lane == 0) {
        red[0][warp] = mq;
        red[1][warp] = mk;
    }
    __syncthreads();
    if (threadIdx.x < 2) {
        float m = 0.f;
        for (int w = 0; w < 8; ++w) m = fmaxf(m, red[threadIdx.x][w]);
        // a little headroom over the fp32 sums of squares
        atomicMax(&out[2 * bh + threadIdx.x], __float_as_uint(m * 1.0001f));
    }
}

}  // namespace

cudaError_t launch_qk_norm_max(const void *q, const void *k, uint32_t *qkmax, int B, int T, int H,
                               cudaStream_t st) {
    if (B * H > 65535) return cudaSuccess;  // the attention then keeps a running maximum
    cudaError_t e = cudaMemsetAsync(qkmax, 0, (size_t)B * H * 2 * sizeof(uint32_t), st);
    if (e != cudaSuccess) return e;
    qk_norm_max_kernel<<<dim3(ceil_div(T, kNormRows), B * H), 256, 0, st>>>(
        (const __nv_bfloat16 *)q, (const __nv_bfloat16 *)k, qkmax, T, H);
    return launched();
}

bool sparse_attn_tc_eligible(int T, int D, int DI, int dtype) {
    (void)T;
    return dtype == SGSA_DTYPE_BF16 && D == 128 && DI == 64;
}

cudaError_t launch_sparse_attn_tc(const void *q, const void *k, const void *v, const void *iq,
                                  const void *ik, const uint32_t *thr, const float *od,
                                  const void *mix, void *out, int B, int T, int H, float scale,
                                  int mix_pc, const int32_t *q_tiles, int n_tiles, bool out_f32,
                                  int HI, uint32_t *qkmax, cudaStream_t st, float *dbg_scores,
                                  bool norms_ready) {
    CUtensorMap mk, mv, mik;
    if (!make_tmap_rows_bf16(&mk, k, B, T, H, 128, kBlk) ||
        !make_tmap_rows_bf16(&mv, v, B, T, H, 128, kBlk) ||
        !make_tmap_rows_bf16(&mik, ik, B, T, HI, 64, kBlk))
        return cudaErrorInvalidValue;
    const int nqt = ceil_div(T, kRowsA);
    const int ntiles = q_tiles ? n_tiles : nqt;
    if (ntiles <= 0) return cudaSuccess;
    const float sl = scale * 1.4426950408889634f;
    if (B * H > 65535) qkmax = nullptr;  // grid limit of the norm pass: running maximum instead
    if (qkmax && !norms_ready) {
        cudaError_t e = launch_qk_norm_max(q, k, qkmax, B, T, H, st);
        if (e != cudaSuccess) return e;
    }
    if (out_f32) {
        auto kern = sparse_attn_tc_kernel<__nv_bfloat16, float>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)L::kSmem);
        if (e != cudaSuccess) return e;
        kern<<<ntiles * B * H, kAttnThreads, L::kSmem, st>>>(
            (const __nv_bfloat16 *)q, mk, mv, (const __nv_bfloat16 *)iq, mik, (const uint4 *)thr, od,
            (const __nv_bfloat16 *)mix, (float *)out, B, T, H, sl, mix_pc, nqt, q_tiles, HI, qkmax, dbg_scores);
    } else {
        auto kern = sparse_attn_tc_kernel<__nv_bfloat16, __nv_bfloat16>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)L::kSmem);
        if (e != cudaSuccess) return e;
        kern<<<ntiles * B * H, kAttnThreads, L::kSmem, st>>>(
            (const __nv_bfloat16 *)q, mk, mv, (const __nv_bfloat16 *)iq, mik, (const uint4 *)thr, od,
            (const __nv_bfloat16 *)mix, (__nv_bfloat16 *)out, B, T, H, sl, mix_pc, nqt, q_tiles, HI,
            qkmax, dbg_scores);
    }
    return launched();
}

unsigned int read_attn_watchdog(cudaStream_t st) {
    unsigned int v = 0, z = 0;
    if (cudaStreamSynchronize(st) != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyFromSymbol(&v, g_attn_watchdog, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (v) cudaMemcpyToSymbol(g_attn_watchdog, &z, sizeof(z));
    return v;
}

unsigned int check_word_attn(bool reset) {
    unsigned int v = 0, z = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyFromSymbol(&v, g_check, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (reset && v) cudaMemcpyToSymbol(g_check, &z, sizeof(z));
    return v;
}

}  // namespace sgsa
