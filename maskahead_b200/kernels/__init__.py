"""sm_100a operators of the select + attend path (reference: src/maskahead/kernels)."""

from .ops import (KernelUnavailableError, SelectorResult, SelectorScratch, dense_packed_attention,
                  gather_packed_kv, quantize_key_groups_into, quantize_values_into, sdpa_compact,
                  select_topk_indices, selector_topk)
from .splitk import Prefix, dequantize_prefix, prefix_scores, splitk_attention

__all__ = ["KernelUnavailableError", "SelectorResult", "SelectorScratch", "dense_packed_attention",
           "gather_packed_kv", "quantize_key_groups_into", "quantize_values_into", "sdpa_compact",
           "select_topk_indices", "selector_topk", "Prefix", "dequantize_prefix", "prefix_scores",
           "splitk_attention"]
