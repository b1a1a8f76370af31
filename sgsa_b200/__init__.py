"""B200 (sm_100a) SGSA layer forward: chunked delta rule, top-k indexer,
sparse attention + gate, behind the C ABI of include/sgsa_b200.h."""
from .ops import (chunk_sgsa, chunk_sgsa_fp32_state, indexer_topk, sgsa_layer_fwd,
                  sparse_attn_mix, topk_select)

__all__ = ["chunk_sgsa", "chunk_sgsa_fp32_state", "indexer_topk", "topk_select",
           "sparse_attn_mix", "sgsa_layer_fwd"]
