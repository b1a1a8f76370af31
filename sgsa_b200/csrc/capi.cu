// extern "C" boundary of libsgsa_b200.so: argument checks, workspace carving,
// status codes.  No entry point allocates, frees, aborts or traps.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "common.cuh"

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

// One non-blocking side stream per device for the layer's concurrent delta stage.
cudaStream_t side_stream() {
    static std::mutex mu;
    static cudaStream_t streams[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!streams[dev] && cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking) != cudaSuccess)
        streams[dev] = nullptr;
    return streams[dev];
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

int sgsa_watchdog_status(void *stream) {
    const cudaStream_t st = (cudaStream_t)stream;
    const unsigned int a = sgsa::read_index_watchdog(st), b = sgsa::read_scan_watchdog(st),
                       c = sgsa::read_attn_watchdog(st);
    if (a == 0xffffffffu || b == 0xffffffffu || c == 0xffffffffu) return -1;
    return (int)(a | (b << 8) | (c << 16));
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

size_t sgsa_layer_fwd_workspace_size(int B, int T, int H, int D, int DI, int top_k) {
    if (B <= 0 || T <= 0 || H <= 0 || !head_dim_ok(D) || top_k <= 0) return 0;
    (void)DI;
    size_t n = align256(sgsa::chunk_delta_ws_bytes(B, T, H, D, 0));
    n += align256((size_t)B * T * H * D * sizeof(float));       // o_delta
    n += align256((size_t)B * H * T * top_k * sizeof(int32_t));  // indices
    n += align256((size_t)B * H * T * 16);                       // per-row selection thresholds
    n += align256((size_t)B * H * 2 * sizeof(uint32_t));         // max |q|^2, |k|^2 per head
    n += align256((size_t)B * T * H * D * sizeof(float));       // o_s (attention before the gate)
    return n;
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
    const size_t need = sgsa_layer_fwd_workspace_size(B, T, H, D, DI, top_k);
    if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255)) return SGSA_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    char *w = (char *)workspace;
    const size_t cws = align256(sgsa::chunk_delta_ws_bytes(B, T, H, D, 0));
    float *od = (float *)(w + cws);
    int32_t *ix = (int32_t *)(w + cws + align256((size_t)B * T * H * D * sizeof(float)));
    uint32_t *thr = (uint32_t *)((char *)ix + align256((size_t)B * H * T * top_k * sizeof(int32_t)));
    uint32_t *qkmax = (uint32_t *)((char *)thr + align256((size_t)B * H * T * 16));
    float *os_ws = (float *)((char *)qkmax + align256((size_t)B * H * 2 * sizeof(uint32_t)));
    const bool fused = sgsa::indexer_tc_eligible(DI, dtype) &&
                       sgsa::sparse_attn_tc_eligible(T, D, DI, dtype) && fused_attn_enabled();
    if (indices) ix = indices;
    int flags = SGSA_FLAG_OUT_F32 | (initial_state ? SGSA_FLAG_HAS_INIT : 0) |
                (final_state ? SGSA_FLAG_STORE_FINAL : 0);
    const float scale = 1.0f / sqrtf((float)D);
    cudaError_t e;
    if (fused) {
        // The delta stage runs on a side stream beside the indexer and the attention
        // (neither reads its output); the attention writes o_s in fp32 and the gate,
        // which needs the delta output, joins the two streams.
        cudaStream_t side = side_stream();
        cudaEvent_t fork = nullptr, join = nullptr;
        if (!side || cudaEventCreateWithFlags(&fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&join, cudaEventDisableTiming) != cudaSuccess) {
            if (fork) cudaEventDestroy(fork);
            side = st;  // run in order on the caller's stream
        }
        if (side != st) {
            cudaEventRecord(fork, st);
            cudaStreamWaitEvent(side, fork, 0);
        }
        e = sgsa::launch_chunk_delta(q, k, v, beta, gamma, nullptr, nullptr, nullptr,
                                     initial_state, od, final_state, B, T, H, D, dtype, flags, w,
                                     side);
        if (side != st) {
            cudaEventRecord(join, side);
            cudaEventDestroy(fork);
        }
        if (e == cudaSuccess)  // selection as per-row thresholds; indices only if asked for
            e = sgsa::launch_indexer_topk_thr(iq, ik, indices, thr, B, T, idx_heads, DI, top_k,
                                              nullptr, 0, st);
        if (e == cudaSuccess)
            e = sgsa::launch_sparse_attn_tc(q, k, v, iq, ik, thr, nullptr, nullptr, os_ws, B, T, H,
                                            scale, mix_per_channel, nullptr, 0, true, idx_heads,
                                            qkmax, st);
        if (side != st) {
            cudaStreamWaitEvent(st, join, 0);
            cudaEventDestroy(join);
        }
        if (e != cudaSuccess) return fail_cuda(e);
        e = sgsa::launch_gate_mix(os_ws, od, mix, out, (long long)B * T * H, D, mix_per_channel,
                                  dtype, st);
        return e == cudaSuccess ? SGSA_OK : fail_cuda(e);
    }
    e = sgsa::launch_chunk_delta(q, k, v, beta, gamma, nullptr, nullptr, nullptr, initial_state,
                                 od, final_state, B, T, H, D, dtype, flags, w, st);
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
