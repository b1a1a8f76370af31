// extern "C" boundary of libsgsa_b200.so: argument checks, workspace carving,
// status codes.  No entry point allocates, frees, aborts or traps.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "common.cuh"

namespace {
std::atomic<unsigned long long> g_launches{0};
}  // namespace

cudaError_t sgsa::launched() {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

namespace {

thread_local char g_last_error[256] = "";

int fail_cuda(cudaError_t e) {
    snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(e),
             cudaGetErrorString(e));
    return SGSA_ERR_LAUNCH;
}

int check_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return SGSA_ERR_DEVICE;
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return SGSA_ERR_DEVICE;
    return major == 10 ? SGSA_OK : SGSA_ERR_DEVICE;
}

bool head_dim_ok(int D) { return D == 32 || D == 64 || D == 128; }
bool dtype_ok(int dt) { return dt == SGSA_DTYPE_F32 || dt == SGSA_DTYPE_BF16; }
size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// The layer's concurrent delta stage runs on a non-blocking side stream (the highest
// priority, so that its few long-lived scan CTAs find SMs first) with a fork and a join
// event, and an event after its prep kernel.  They are created once per (host thread,
// device) and reused, so callers on different host threads never share them and a call
// creates or destroys nothing after the first on its thread.
struct SideStream {
    cudaStream_t stream = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr, prep = nullptr;
    bool ok = false;
};

SideStream *side_stream() {
    thread_local SideStream per_dev[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    SideStream &s = per_dev[dev];
    if (!s.ok) {
        int lo = 0, hi = 0;
        if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess) hi = 0;
        if (!s.stream &&
            cudaStreamCreateWithPriority(&s.stream, cudaStreamNonBlocking, hi) != cudaSuccess)
            s.stream = nullptr;
        if (!s.fork && cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming) != cudaSuccess)
            s.fork = nullptr;
        if (!s.join && cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming) != cudaSuccess)
            s.join = nullptr;
        if (!s.prep && cudaEventCreateWithFlags(&s.prep, cudaEventDisableTiming) != cudaSuccess)
            s.prep = nullptr;
        s.ok = s.stream && s.fork && s.join && s.prep;
        if (!s.ok) cudaGetLastError();
    }
    return s.ok ? &s : nullptr;
}

// SGSA_ATTN_GATHER=1 makes the layer use the row-gather attention (A/B checks).
bool fused_attn_enabled() {
    const char *e = getenv("SGSA_ATTN_GATHER");
    return !(e && e[0] == '1');
}

}  // namespace

extern "C" {

const char *sgsa_status_string(int s) {
    switch (s) {
        case SGSA_OK: return "ok";
        case SGSA_ERR_SHAPE: return "bad or unsupported shape";
        case SGSA_ERR_DTYPE: return "unsupported dtype";
        case SGSA_ERR_NULL: return "required pointer is NULL";
        case SGSA_ERR_WORKSPACE: return "workspace too small or misaligned";
        case SGSA_ERR_LAUNCH: return "CUDA launch or runtime error";
        case SGSA_ERR_UNSUPPORTED: return "unsupported request";
        case SGSA_ERR_DEVICE: return "current CUDA device is not an sm_100 (B200) part";
        default: return "unknown status";
    }
}

const char *sgsa_last_error(void) { return g_last_error; }

int sgsa_version(void) { return 1000; }

unsigned long long sgsa_kernel_launches(void) {
    return g_launches.load(std::memory_order_relaxed);
}

int sgsa_watchdog_status(void *stream) {
    const cudaStream_t st = (cudaStream_t)stream;
    const unsigned int a = sgsa::read_index_watchdog(st), b = sgsa::read_scan_watchdog(st),
                       c = sgsa::read_attn_watchdog(st);
    if (a == 0xffffffffu || b == 0xffffffffu || c == 0xffffffffu) return -1;
    return (int)(a | (b << 8) | (c << 16));
}

int sgsa_watchdog_selftest(unsigned int spin_limit, void *stream) {
    if (spin_limit == 0 || spin_limit > (1u << 20)) return SGSA_ERR_SHAPE;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_watchdog_selftest(spin_limit, (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_check_status(unsigned int *word, int reset) {
    if (!word) return SGSA_ERR_NULL;
    *word = 0;
    if (!sgsa::kCheckBuild) return SGSA_ERR_UNSUPPORTED;
    if (int s = check_device()) return s;
    const unsigned int w[4] = {sgsa::check_word_gather(reset != 0), sgsa::check_word_decode(reset != 0),
                               sgsa::check_word_indexer(reset != 0), sgsa::check_word_attn(reset != 0)};
    unsigned int all = 0;
    for (unsigned int x : w) {
        if (x == 0xffffffffu) return fail_cuda(cudaGetLastError());
        all |= x;
    }
    *word = all;
    return SGSA_OK;
}

size_t sgsa_chunk_fwd_workspace_size(int B, int T, int H, int D, int flags) {
    if (B <= 0 || T <= 0 || H <= 0 || !head_dim_ok(D)) return 0;
    return sgsa::chunk_delta_ws_bytes(B, T, H, D, flags);
}

int sgsa_chunk_fwd(const void *q, const void *k, const void *v, const void *beta,
                   const void *gamma, const void *sparse_k, const void *sparse_v,
                   const void *alpha, const float *initial_state, void *o, float *final_state,
                   int B, int T, int H, int D, int dtype, int chunk_size, int flags,
                   void *workspace, size_t workspace_bytes, void *stream) {
    if (B < 0 || T < 0 || H < 0) return SGSA_ERR_SHAPE;
    if (!head_dim_ok(D) || chunk_size != 64) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if (B == 0 || T == 0 || H == 0) {
        // Empty sequence: the final state is the initial state (or zero).
        if ((flags & SGSA_FLAG_STORE_FINAL) && final_state && B > 0 && H > 0) {
            const size_t n = (size_t)B * H * D * D * sizeof(float);
            cudaError_t e = (flags & SGSA_FLAG_HAS_INIT) && initial_state
                                ? cudaMemcpyAsync(final_state, initial_state, n,
                                                  cudaMemcpyDeviceToDevice, (cudaStream_t)stream)
                                : cudaMemsetAsync(final_state, 0, n, (cudaStream_t)stream);
            if (e != cudaSuccess) return fail_cuda(e);
        }
        return SGSA_OK;
    }
    if (!q || !k || !v || !beta || !gamma || !o) return SGSA_ERR_NULL;
    flags &= 63;  // the public SGSA_FLAG_* bits; the rest are internal to the kernels
    if ((flags & SGSA_FLAG_HAS_SPARSE) && (!sparse_k || !sparse_v || !alpha)) return SGSA_ERR_NULL;
    if ((flags & SGSA_FLAG_HAS_INIT) && !initial_state) return SGSA_ERR_NULL;
    if ((flags & SGSA_FLAG_STORE_FINAL) && !final_state) return SGSA_ERR_NULL;
    if ((flags & (SGSA_FLAG_TRANSITION | SGSA_FLAG_REUSE_PREP)) &&
        !sgsa::chunk_tc_eligible(D, dtype, flags))
        return SGSA_ERR_UNSUPPORTED;
    if (int s = check_device()) return s;
    const size_t need = sgsa::chunk_delta_ws_bytes(B, T, H, D, flags);
    if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255)) return SGSA_ERR_WORKSPACE;
    cudaError_t e = sgsa::launch_chunk_delta(q, k, v, beta, gamma, sparse_k, sparse_v, alpha,
                                             initial_state, o, final_state, B, T, H, D, dtype,
                                             flags, workspace, (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_indexer_topk(const void *iq, const void *ik, int32_t *indices, int B, int T, int H,
                      int DI, int top_k, int dtype, void *stream) {
    if (B < 0 || T < 0 || H < 0 || top_k <= 0) return SGSA_ERR_SHAPE;
    if (DI != 32 && DI != 64 && DI != 128) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if ((size_t)B * T * H == 0) return SGSA_OK;
    if (!iq || !ik || !indices) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_indexer_topk(iq, ik, indices, B, T, H, DI, top_k, dtype,
                                              (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_indexer_topk_scores(const void *iq, const void *ik, int32_t *indices, float *scores,
                             int B, int T, int H, int DI, int top_k, void *stream) {
    if (B < 0 || T < 0 || H < 0 || top_k <= 0 || T > 4096) return SGSA_ERR_SHAPE;
    if (!sgsa::indexer_tc_eligible(DI, SGSA_DTYPE_BF16)) return SGSA_ERR_UNSUPPORTED;
    if ((size_t)B * T * H == 0) return SGSA_OK;
    if (!iq || !ik || !indices || !scores) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_indexer_topk_debug(iq, ik, indices, scores, B, T, H, DI, top_k,
                                                    (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_indexer_stats(unsigned long long *counts, int reset) {
    if (!counts) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    if (cudaDeviceSynchronize() != cudaSuccess) return SGSA_ERR_LAUNCH;
    return sgsa::read_index_stats(counts, reset != 0) == 0 ? SGSA_OK : SGSA_ERR_LAUNCH;
}

int sgsa_topk_select(const float *scores, const int32_t *valid, int32_t *indices, int R, int S,
                     int top_k, void *stream) {
    if (R < 0 || S < 0 || top_k <= 0) return SGSA_ERR_SHAPE;
    if (R == 0) return SGSA_OK;
    if (!scores || !valid || !indices) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_topk_select(scores, valid, indices, R, S, top_k,
                                             (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_sparse_attn_mix(const void *q, const void *k, const void *v, const int32_t *indices,
                         const float *o_delta, const void *mix, void *out, int B, int T, int H,
                         int D, int top_k, int idx_heads, float scale, int mix_per_channel,
                         int dtype, void *stream) {
    if (B < 0 || T < 0 || H < 0 || top_k <= 0 || !head_dim_ok(D)) return SGSA_ERR_SHAPE;
    if (idx_heads != 1 && idx_heads != H) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if ((size_t)B * T * H == 0) return SGSA_OK;
    if (!q || !k || !v || !indices || !out) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_sparse_attn_mix(q, k, v, indices, o_delta, mix, out, B, T, H, D,
                                                 top_k, scale, mix_per_channel, dtype, idx_heads,
                                                 (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_indexer_thresholds(const void *iq, const void *ik, int32_t *indices,
                            uint32_t *thresholds, const int32_t *q_tiles, int n_tiles, int B,
                            int T, int H, int DI, int top_k, void *stream) {
    if (B < 0 || T < 0 || H < 0 || top_k <= 0 || n_tiles < 0) return SGSA_ERR_SHAPE;
    if (!sgsa::indexer_tc_eligible(DI, SGSA_DTYPE_BF16)) return SGSA_ERR_UNSUPPORTED;
    if ((size_t)B * T * H == 0) return SGSA_OK;
    if (!iq || !ik || !thresholds) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_indexer_topk_thr(iq, ik, indices, thresholds, B, T, H, DI, top_k,
                                                  q_tiles, n_tiles, (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_sparse_attn_thresholds(const void *q, const void *k, const void *v, const void *iq,
                                const void *ik, const uint32_t *thresholds,
                                const int32_t *q_tiles, int n_tiles, const float *o_delta,
                                const void *mix, void *out, int B, int T, int H, int D, int DI,
                                int idx_heads, float scale, int mix_per_channel, int out_f32,
                                void *norm_scratch, void *stream) {
    if (B < 0 || T < 0 || H < 0 || n_tiles < 0) return SGSA_ERR_SHAPE;
    if (idx_heads != 1 && idx_heads != H) return SGSA_ERR_SHAPE;
    if (!sgsa::sparse_attn_tc_eligible(T, D, DI, SGSA_DTYPE_BF16)) return SGSA_ERR_UNSUPPORTED;
    if ((size_t)B * T * H == 0) return SGSA_OK;
    if (!q || !k || !v || !iq || !ik || !thresholds || !out) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_sparse_attn_tc(q, k, v, iq, ik, thresholds, o_delta, mix, out,
                                                B, T, H, scale, mix_per_channel, q_tiles, n_tiles,
                                                out_f32 != 0, idx_heads, (uint32_t *)norm_scratch,
                                                (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_sparse_attn_index_scores(const void *q, const void *k, const void *v, const void *iq,
                                  const void *ik, const uint32_t *thresholds, float *out,
                                  float *scores, int B, int T, int H, void *stream) {
    if (B < 0 || T < 0 || H < 0 || T > 4096) return SGSA_ERR_SHAPE;
    if (!sgsa::sparse_attn_tc_eligible(T, 128, 64, SGSA_DTYPE_BF16)) return SGSA_ERR_UNSUPPORTED;
    if ((size_t)B * T * H == 0) return SGSA_OK;
    if (!q || !k || !v || !iq || !ik || !thresholds || !out || !scores) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_sparse_attn_tc(q, k, v, iq, ik, thresholds, nullptr, nullptr, out,
                                                B, T, H, 1.0f / sqrtf(128.0f), 0, nullptr, 0, true,
                                                H, nullptr, (cudaStream_t)stream, scores);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_sparse_retrieve(const void *q, const void *k, const void *v, const int32_t *indices,
                         void *k_hat, void *v_hat, int B, int T, int H, int D, int top_k,
                         int idx_heads, float scale, int dtype, void *stream) {
    if (B < 0 || T < 0 || H < 0 || top_k <= 0 || !head_dim_ok(D)) return SGSA_ERR_SHAPE;
    if (idx_heads != 1 && idx_heads != H) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if ((size_t)B * T * H == 0) return SGSA_OK;
    if (!q || !k || !v || !indices || !k_hat || !v_hat) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_sparse_retrieve(q, k, v, indices, k_hat, v_hat, B, T, H, D,
                                                 top_k, scale, idx_heads, dtype,
                                                 (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_gate_mix(const float *o_s, const float *o_delta, const void *mix, void *out,
                  long long rows, int D, int mix_per_channel, int dtype, void *stream) {
    if (rows < 0 || D <= 0) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if (rows == 0) return SGSA_OK;
    if (!o_s || !o_delta || !mix || !out) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_gate_mix(o_s, o_delta, mix, out, rows, D, mix_per_channel, dtype,
                                          (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

}  // extern "C"

namespace {

// Workspace carving of sgsa_layer_fwd.  The delta stage's per-chunk operands are
// bounded by kLayerDeltaCap: larger problems run the delta stage in groups of
// (batch, head) pairs that reuse one region.  The fused path (tensor-core indexer
// and attention) keeps 16-byte threshold records per row and never an index
// buffer; the gather path keeps the B*idx_heads*T*K int32 index rows.
constexpr size_t kLayerDeltaCap = (size_t)5 << 28;  // 1.25 GiB

// SGSA_LAYER_DELTA_CAP=<bytes> lowers the cap (tests exercise the grouping on small problems).
size_t layer_delta_cap() {
    const char *e = getenv("SGSA_LAYER_DELTA_CAP");
    if (e && e[0]) {
        const unsigned long long v = strtoull(e, nullptr, 10);
        if (v > 0 && v < kLayerDeltaCap) return (size_t)v;
    }
    return kLayerDeltaCap;
}

struct LayerPlan {
    bool fused;
    size_t chunk, od, idx, thr, qkmax, total;
};

bool layer_fused(int T, int D, int DI, int dtype) {
    return sgsa::indexer_tc_eligible(DI, dtype) && sgsa::sparse_attn_tc_eligible(T, D, DI, dtype) &&
           fused_attn_enabled();
}

LayerPlan layer_plan(int B, int T, int H, int D, int DI, int idx_heads, int top_k, int dtype) {
    LayerPlan p{};
    p.fused = layer_fused(T, D, DI, dtype);
    const size_t bthd = (size_t)B * T * H * D;
    const int pairs = sgsa::chunk_delta_group_pairs(B, T, H, D, 0, layer_delta_cap());
    p.chunk = align256(sgsa::chunk_delta_ws_bytes_pairs(pairs, T, D, 0));
    p.od = align256(bthd * sizeof(float));
    p.idx = p.fused ? 0 : align256((size_t)B * idx_heads * T * top_k * sizeof(int32_t));
    p.thr = p.fused ? align256((size_t)B * idx_heads * T * 16) : 0;
    p.qkmax = p.fused ? align256((size_t)B * H * 2 * sizeof(uint32_t)) : 0;
    p.total = p.chunk + p.od + p.idx + p.thr + p.qkmax;
    return p;
}

}  // namespace

extern "C" {

size_t sgsa_layer_fwd_workspace_size(int B, int T, int H, int D, int DI, int idx_heads,
                                     int top_k, int dtype) {
    if (B <= 0 || T <= 0 || H <= 0 || !head_dim_ok(D) || top_k <= 0) return 0;
    if (idx_heads != 1 && idx_heads != H) return 0;
    if ((DI != 32 && DI != 64 && DI != 128) || !dtype_ok(dtype)) return 0;
    return layer_plan(B, T, H, D, DI, idx_heads, top_k, dtype).total;
}

int sgsa_layer_fwd(const void *q, const void *k, const void *v, const void *beta,
                   const void *gamma, const void *iq, const void *ik, const void *mix,
                   const float *initial_state, void *out, float *final_state, int32_t *indices,
                   int B, int T, int H, int D, int DI, int idx_heads, int top_k,
                   int mix_per_channel, int dtype, void *workspace, size_t workspace_bytes,
                   void *stream) {
    if (B <= 0 || T <= 0 || H <= 0 || !head_dim_ok(D) || top_k <= 0) return SGSA_ERR_SHAPE;
    if (idx_heads != 1 && idx_heads != H) return SGSA_ERR_SHAPE;
    if (DI != 32 && DI != 64 && DI != 128) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if (!q || !k || !v || !beta || !gamma || !iq || !ik || !mix || !out) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    const LayerPlan p = layer_plan(B, T, H, D, DI, idx_heads, top_k, dtype);
    if (!workspace || workspace_bytes < p.total || ((uintptr_t)workspace & 255))
        return SGSA_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    char *w = (char *)workspace;
    float *od = (float *)(w + p.chunk);
    int32_t *ix = (int32_t *)(w + p.chunk + p.od);
    uint32_t *thr = (uint32_t *)((char *)ix + p.idx);
    uint32_t *qkmax = (uint32_t *)((char *)thr + p.thr);
    if (indices) ix = indices;
    int flags = SGSA_FLAG_OUT_F32 | (initial_state ? SGSA_FLAG_HAS_INIT : 0) |
                (final_state ? SGSA_FLAG_STORE_FINAL : 0);
    const float scale = 1.0f / sqrtf((float)D);
    cudaError_t e;
    if (p.fused) {
        // The delta stage runs on a side stream beside the indexer (which does not read its
        // output); the streams join before the attention, whose epilogue applies the gate
        // with the delta output.
        SideStream *ss = side_stream();
        cudaStream_t side = ss ? ss->stream : st;  // without one: in order on the caller's stream
        if (side != st) {
            if ((e = cudaEventRecord(ss->fork, st)) != cudaSuccess) return fail_cuda(e);
            if ((e = cudaStreamWaitEvent(side, ss->fork, 0)) != cudaSuccess) return fail_cuda(e);
        }
        // A small indexer grid runs one CTA per SM (faster per CTA, but its tensor memory
        // keeps other kernels off the SM): it then starts after the delta stage's prep and
        // beside its few scan CTAs, which the side stream's priority places first.
        int dev = 0, nsm = 148;
        if (cudaGetDevice(&dev) == cudaSuccess)
            cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        const bool small_idx = side != st &&
                               (long long)((T + 127) / 128) * B * idx_heads <= 4LL * nsm;
        e = sgsa::launch_chunk_delta(q, k, v, beta, gamma, nullptr, nullptr, nullptr,
                                     initial_state, od, final_state, B, T, H, D, dtype, flags, w,
                                     side, layer_delta_cap(), small_idx ? ss->prep : nullptr);
        // the attention's per-head norm bound, memory-bound, also beside the indexer
        if (e == cudaSuccess) e = sgsa::launch_qk_norm_max(q, k, qkmax, B, T, H, side);
        cudaError_t ej = cudaSuccess;
        if (side != st) ej = cudaEventRecord(ss->join, side);
        if (e == cudaSuccess && small_idx) e = cudaStreamWaitEvent(st, ss->prep, 0);
        if (e == cudaSuccess)  // selection as per-row thresholds; indices only if asked for
            e = sgsa::launch_indexer_topk_thr(iq, ik, indices, thr, B, T, idx_heads, DI, top_k,
                                              nullptr, 0, st,
                                              /*shares_sms=*/side != st && !small_idx);
        // always join, so that the caller's stream never runs ahead of the side stream
        if (side != st && ej == cudaSuccess) ej = cudaStreamWaitEvent(st, ss->join, 0);
        if (e != cudaSuccess) return fail_cuda(e);
        if (ej != cudaSuccess) return fail_cuda(ej);
        e = sgsa::launch_sparse_attn_tc(q, k, v, iq, ik, thr, od, mix, out, B, T, H, scale,
                                        mix_per_channel, nullptr, 0, dtype == SGSA_DTYPE_F32,
                                        idx_heads, qkmax, st, nullptr, /*norms_ready=*/true);
        return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
    }
    e = sgsa::launch_chunk_delta(q, k, v, beta, gamma, nullptr, nullptr, nullptr, initial_state,
                                 od, final_state, B, T, H, D, dtype, flags, w, st, layer_delta_cap());
    if (e != cudaSuccess) return fail_cuda(e);
    e = sgsa::launch_indexer_topk(iq, ik, ix, B, T, idx_heads, DI, top_k, dtype, st);
    if (e != cudaSuccess) return fail_cuda(e);
    e = sgsa::launch_sparse_attn_mix(q, k, v, ix, od, mix, out, B, T, H, D, top_k, scale,
                                     mix_per_channel, dtype, idx_heads, st);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_recurrent_fwd(const void *q, const void *k, const void *v, const void *beta,
                       const void *gamma, const void *sparse_k, const void *sparse_v,
                       const void *alpha, const float *initial_state, void *o,
                       float *final_state, int B, int T, int H, int D, int dtype, int flags,
                       void *stream) {
    if (B < 0 || T < 0 || H < 0 || !head_dim_ok(D)) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if ((size_t)B * H == 0) return SGSA_OK;
    if (T > 0 && (!q || !k || !v || !beta || !gamma || !o)) return SGSA_ERR_NULL;
    const bool sparse = flags & SGSA_FLAG_HAS_SPARSE;
    if (sparse && (!sparse_k || !sparse_v || !alpha)) return SGSA_ERR_NULL;
    if ((flags & SGSA_FLAG_HAS_INIT) && !initial_state) return SGSA_ERR_NULL;
    if ((flags & SGSA_FLAG_STORE_FINAL) && !final_state) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_recurrent(
        q, k, v, beta, gamma, sparse ? sparse_k : nullptr, sparse ? sparse_v : nullptr,
        sparse ? alpha : nullptr, (flags & SGSA_FLAG_HAS_INIT) ? initial_state : nullptr, o,
        (flags & SGSA_FLAG_STORE_FINAL) ? final_state : nullptr, B, T, H, D, dtype,
        (flags & SGSA_FLAG_OUT_F32) != 0, (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_decode_append(void *k_cache, void *v_cache, void *ik_cache, const void *k,
                       const void *v, const void *ik, int B, int Tc, int H, int D, int DI,
                       int pos, int dtype, void *stream) {
    if (B < 0 || H < 0 || Tc <= 0 || pos < 0 || pos >= Tc) return SGSA_ERR_SHAPE;
    if (!head_dim_ok(D) || (DI != 32 && DI != 64 && DI != 128)) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if ((size_t)B * H == 0) return SGSA_OK;
    if (!k_cache || !v_cache || !ik_cache || !k || !v || !ik) return SGSA_ERR_NULL;
    const uintptr_t any = (uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)ik_cache |
                          (uintptr_t)k | (uintptr_t)v | (uintptr_t)ik;
    if (any & 15) return SGSA_ERR_SHAPE;  // 16-byte vectors
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_decode_append(k_cache, v_cache, ik_cache, k, v, ik, B, Tc, H, D,
                                               DI, pos, dtype == SGSA_DTYPE_F32 ? 4 : 2,
                                               (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_decode_topk(const void *iq, const void *ik_cache, int32_t *indices, int B, int H,
                     int Tc, int n, int DI, int top_k, int dtype, void *stream) {
    if (B < 0 || H < 0 || Tc < 0 || n < 0 || n > Tc || top_k <= 0) return SGSA_ERR_SHAPE;
    if (DI != 32 && DI != 64 && DI != 128) return SGSA_ERR_SHAPE;
    if (n > sgsa::decode_max_cache()) return SGSA_ERR_UNSUPPORTED;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if ((size_t)B * H == 0) return SGSA_OK;
    if (!iq || !ik_cache || !indices) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_decode_topk(iq, ik_cache, indices, B, H, Tc, n, DI, top_k,
                                             dtype, (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_decode_attn_mix(const void *q, const void *k_cache, const void *v_cache,
                         const int32_t *indices, const float *o_delta, const void *mix, void *out,
                         int B, int H, int Tc, int D, int top_k, float scale, int mix_per_channel,
                         int dtype, void *stream) {
    if (B < 0 || H < 0 || Tc < 0 || top_k <= 0 || !head_dim_ok(D)) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if ((size_t)B * H == 0) return SGSA_OK;
    if (!q || !k_cache || !v_cache || !indices || !out) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_decode_attn(q, k_cache, v_cache, indices, o_delta, mix, out, B,
                                             H, Tc, D, top_k, scale, mix_per_channel, dtype,
                                             (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

// ---- hybrid model kernels ----

int sgsa_rmsnorm(const void *x, const void *weight, void *out, long long rows, int N, float eps,
                 int dtype, void *stream) {
    if (rows < 0 || N <= 0 || N % 8) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if (rows == 0) return SGSA_OK;
    if (!x || !weight || !out) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_rmsnorm(x, weight, out, rows, N, eps, dtype, (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_swiglu(const void *gate_up, void *out, long long rows, int I, int dtype, void *stream) {
    if (rows < 0 || I <= 0 || I % 8) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if (rows == 0) return SGSA_OK;
    if (!gate_up || !out) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_swiglu(gate_up, out, rows, I, dtype, (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_rope_qkv(const void *qkv, const float *cos_sin, void *q, void *k, void *v, int B, int T,
                  int H, int D, int pos0, int dtype, void *stream) {
    if (B < 0 || T < 0 || H < 0 || pos0 < 0 || D <= 0 || D % 8) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if ((size_t)B * T * H == 0) return SGSA_OK;
    if (!qkv || !cos_sin || !q || !k || !v) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_rope_qkv(qkv, cos_sin, q, k, v, B, T, H, D, pos0, dtype,
                                          (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_layer_proj(const void *proj, int ld, void *q, void *k, void *v, void *mix, void *iq,
                    void *ik, void *beta, void *gamma, long long rows, int H, int D, int DI,
                    int dtype, void *stream) {
    if (rows < 0 || H <= 0 || H > 256 || D <= 0 || DI <= 0) return SGSA_ERR_SHAPE;
    if ((H * D) % 8 || (H * DI) % 8 || ld % 8 || ld < 4 * H * D + 2 * H * DI + 2 * H)
        return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if (rows == 0) return SGSA_OK;
    if (!proj || !q || !k || !v || !mix || !iq || !ik || !beta || !gamma) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_sgsa_proj(proj, ld, q, k, v, mix, iq, ik, beta, gamma, rows, H,
                                           D, DI, dtype, (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

int sgsa_embed(const int64_t *ids, const void *table, void *out, long long rows, int N, int vocab,
               int dtype, void *stream) {
    if (rows < 0 || N <= 0 || N % 8 || vocab <= 0) return SGSA_ERR_SHAPE;
    if (!dtype_ok(dtype)) return SGSA_ERR_DTYPE;
    if (rows == 0) return SGSA_OK;
    if (!ids || !table || !out) return SGSA_ERR_NULL;
    if (int s = check_device()) return s;
    cudaError_t e = sgsa::launch_embed(ids, table, out, rows, N, vocab, dtype, (cudaStream_t)stream);
    return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
}

}  // extern "C"
