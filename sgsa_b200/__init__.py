"""B200 (sm_100a) SGSA layer forward: chunked delta rule, top-k indexer,
sparse attention + gate, behind the C ABI of include/sgsa_b200.h."""
from .ops import (DecodeCache, decode_attn_mix, decode_topk, fused_recurrent_sgsa, chunk_sgsa, chunk_sgsa_fp32_state, indexer_thresholds, indexer_topk,
                  sgsa_layer_fwd, sgsa_layer_fwd_from_host, sparse_attn_mix,
                  sparse_attn_thresholds, sgsa_sparse_write_fwd, sparse_retrieve,
                  topk_select)

__all__ = ["DecodeCache", "decode_attn_mix", "decode_topk", "fused_recurrent_sgsa", "chunk_sgsa", "chunk_sgsa_fp32_state", "indexer_topk", "topk_select",
           "sparse_attn_mix", "sgsa_layer_fwd", "sgsa_layer_fwd_from_host",
           "indexer_thresholds", "sparse_attn_thresholds", "sparse_retrieve",
           "sgsa_sparse_write_fwd"]
