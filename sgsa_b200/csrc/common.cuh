// Shared helpers of the sgsa_b200 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sgsa_b200.h"
#include "select_keys.cuh"

namespace sgsa {

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}


__host__ __device__ constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Counts one kernel launch of this library (sgsa_kernel_launches) and returns
// cudaGetLastError(); every launch site calls it right after its <<<...>>>.
cudaError_t launched();

// Bounds-checked debug build (compiled with -DSGSA_CHECK into libsgsa_b200_check.so):
// kernels test the invariants below, record a violated one as a bit of their source
// file's check word and skip the access it guards; sgsa_check_status() reads the words.
// In the release build the tests compile away.
#ifdef SGSA_CHECK
#define SGSA_CHECK_FAIL(word, code) atomicOr(&(word), (unsigned int)(code))
constexpr bool kCheckBuild = true;
#else
#define SGSA_CHECK_FAIL(word, code) ((void)0)
constexpr bool kCheckBuild = false;
#endif
constexpr unsigned int kChkGatherIndex = 0x1u;     // gather: index outside [-1, T) (or > t)
constexpr unsigned int kChkDecodeIndex = 0x2u;     // decode: index outside [-1, cache length)
constexpr unsigned int kChkCandCap = 0x10u;        // indexer: candidate list over capacity
constexpr unsigned int kChkCollectCount = 0x20u;   // indexer: collect selected != top_k
constexpr unsigned int kChkCollectIndex = 0x40u;   // indexer: collected index outside the row
constexpr unsigned int kChkThresholdRecord = 0x100u;  // attention: no threshold record for a row
unsigned int check_word_gather(bool reset);
unsigned int check_word_decode(bool reset);
unsigned int check_word_indexer(bool reset);
unsigned int check_word_attn(bool reset);

// Launch wrappers implemented in the .cu files (all return cudaError_t of the launch).
// ws_cap > 0: run the (batch, head) pairs in groups whose per-chunk operands fit
// ws_cap bytes (chunk_delta_group_pairs), one after the other in the same workspace.
cudaError_t launch_chunk_delta(const void *q, const void *k, const void *v, const void *beta,
                               const void *gamma, const void *sk, const void *sv,
                               const void *alpha, const float *s0, void *o, float *sT, int B,
                               int T, int H, int D, int dtype, int flags, void *ws,
                               cudaStream_t st, size_t ws_cap = 0,
                               cudaEvent_t prep_done = nullptr);
// prep_done (optional): recorded on st after the first tensor-core prep launch (a
// scheduling point for work that should follow it; nothing depends on it for correctness)
size_t chunk_delta_ws_bytes(int B, int T, int H, int D, int flags);
size_t chunk_delta_ws_bytes_pairs(long long pairs, int T, int D, int flags);
int chunk_delta_group_pairs(int B, int T, int H, int D, int flags, size_t cap);
bool chunk_tc_eligible(int D, int dtype, int flags);

cudaError_t launch_indexer_topk(const void *iq, const void *ik, int32_t *idx, int B, int T,
                                int H, int DI, int K, int dtype, cudaStream_t st);
unsigned int read_index_watchdog(cudaStream_t st);
cudaError_t launch_watchdog_selftest(uint32_t limit, cudaStream_t st);
int read_index_stats(unsigned long long *out, bool reset);
cudaError_t launch_indexer_topk_debug(const void *iq, const void *ik, int32_t *idx,
                                     float *scores, int B, int T, int H, int DI, int K,
                                     cudaStream_t st);
// Tensor-core indexer that also writes, per query row, the exact selection as a
// threshold {prefix, mask, cut, 1}: column j <= t is selected iff
// (key(s_tj) & mask) > prefix, or == prefix and j <= cut.  idx may be NULL.
bool indexer_tc_eligible(int DI, int dtype);
cudaError_t launch_indexer_topk_thr(const void *iq, const void *ik, int32_t *idx, uint32_t *thr,
                                    int B, int T, int H, int DI, int K, const int32_t *q_tiles,
                                    int n_tiles, cudaStream_t st, bool shares_sms = false);
cudaError_t launch_topk_select(const float *scores, const int32_t *valid, int32_t *idx, int R,
                               int S, int K, cudaStream_t st);
cudaError_t launch_sparse_attn_mix(const void *q, const void *k, const void *v,
                                   const int32_t *idx, const float *od, const void *mix,
                                   void *out, int B, int T, int H, int D, int K, float scale,
                                   int mix_pc, int dtype, int HI, cudaStream_t st);
bool sparse_attn_tc_eligible(int T, int D, int DI, int dtype);
cudaError_t launch_sparse_attn_tc(const void *q, const void *k, const void *v, const void *iq,
                                  const void *ik, const uint32_t *thr, const float *od,
                                  const void *mix, void *out, int B, int T, int H, float scale,
                                  int mix_pc, const int32_t *q_tiles, int n_tiles, bool out_f32,
                                  int HI, uint32_t *qkmax, cudaStream_t st,
                                  float *dbg_scores = nullptr, bool norms_ready = false);
// max|q|^2, max|k|^2 per (b, h) into qkmax[2 (b H + h) + {0, 1}] (bf16, D = 128): the bound the
// tensor-core attention's softmax uses (launch_sparse_attn_tc runs it unless norms_ready).
cudaError_t launch_qk_norm_max(const void *q, const void *k, uint32_t *qkmax, int B, int T, int H,
                               cudaStream_t st);
cudaError_t launch_sparse_retrieve(const void *q, const void *k, const void *v, const int32_t *idx,
                                   void *khat, void *vhat, int B, int T, int H, int D, int K,
                                   float scale, int HI, int dtype, cudaStream_t st);
cudaError_t launch_gate_mix(const float *os, const float *od, const void *mix, void *out,
                            long long rows, int D, int mix_pc, int dtype, cudaStream_t st);
unsigned int read_attn_watchdog(cudaStream_t st);
int decode_max_cache();
cudaError_t launch_recurrent(const void *q, const void *k, const void *v, const void *beta,
                             const void *gamma, const void *sk, const void *sv, const void *alpha,
                             const float *s0, void *o, float *sT, int B, int T, int H, int D,
                             int dtype, bool out_f32, cudaStream_t st);
cudaError_t launch_decode_append(void *kc, void *vc, void *ikc, const void *k, const void *v,
                                 const void *ik, int B, int Tc, int H, int D, int DI, int pos,
                                 int elem_bytes, cudaStream_t st);
cudaError_t launch_decode_topk(const void *iq, const void *ikc, int32_t *idx, int B, int H,
                               int Tc, int n, int DI, int K, int dtype, cudaStream_t st);
cudaError_t launch_decode_attn(const void *q, const void *kc, const void *vc, const int32_t *idx,
                               const float *od, const void *mix, void *out, int B, int H, int Tc,
                               int D, int K, float scale, int mix_pc, int dtype, cudaStream_t st);
cudaError_t launch_rmsnorm(const void *x, const void *w, void *out, long long rows, int N,
                           float eps, int dtype, cudaStream_t st);
cudaError_t launch_swiglu(const void *gu, void *out, long long rows, int I, int dtype,
                          cudaStream_t st);
cudaError_t launch_rope_qkv(const void *qkv, const float *cs, void *q, void *k, void *v, int B,
                            int T, int H, int D, int pos0, int dtype, cudaStream_t st);
cudaError_t launch_sgsa_proj(const void *P, int ld, void *q, void *k, void *v, void *mix,
                             void *iq, void *ik, void *beta, void *gamma, long long rows, int H,
                             int D, int DI, int dtype, cudaStream_t st);
cudaError_t launch_embed(const int64_t *ids, const void *table, void *out, long long rows, int N,
                         int vocab, int dtype, cudaStream_t st);
unsigned int read_scan_watchdog(cudaStream_t st);
}  // namespace sgsa
