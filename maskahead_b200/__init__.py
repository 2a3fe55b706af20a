"""maskahead_b200 -- the MaskAhead select + attend hot path on B200 (sm_100a).

Hand-written CUDA kernels behind a C ABI (include/maskahead_b200.h,
maskahead_b200/_lib/libmaskahead_b200.so), with the reference package's operator API
on top:

  maskahead_b200.kernels   selector_topk, gather_packed_kv, dense_packed_attention,
                           splitk_attention, prefix_scores, Prefix
  maskahead_b200.hotpath   fast_step0, compact_attention, probe_attention,
                           value_score, lookahead_survivors
  maskahead_b200.layouts   LayerCacheView, Prefix, the ma_kv descriptor

Kernel waits are bounded; ``device_status()`` raises ``MaError`` (MA_ERR_TIMEOUT) when one
gave up since the last check. There is no CPU path: the operators need the built library
and a CUDA device.
"""

from ._lib import (EXPORTED, KernelUnavailableError, LIB_PATH, MaError, device_status, load_library,
                   set_peer_wait_ns)

__version__ = "0.2.0"

__all__ = ["EXPORTED", "KernelUnavailableError", "LIB_PATH", "MaError", "device_status", "load_library",
           "set_peer_wait_ns", "__version__"]
