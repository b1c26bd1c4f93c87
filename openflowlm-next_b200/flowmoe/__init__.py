"""flowmoe -- the Qwen3.6-MoE expert FFN block of OpenFlowLM on B200 (sm_100a).

Router (softmax top-k, renormalised), token dispatch (count, scan, permute), grouped Q4_1
dequantise-and-multiply for gate/up/down with SwiGLU, and the routing-weighted combine plus the
sigmoid-gated shared expert, as hand-written CUDA behind the C ABI of ``libflowmoe.so``
(``include/flowmoe.h``). Importing this package loads that library; there is no CPU fallback.
"""
from . import _lib  # noqa: F401  (loads libflowmoe.so or raises)
from .layer import (MoEConfig, MoELayer, experts_from_pool, gate_up_to_tiles, pool_to_q4_1, q4_1_to_tiles,  # noqa: F401
                    router_block, tiles_to_q4_1)
from .linear import Q4Linear  # noqa: F401
from .pipeline import HostPipeline  # noqa: F401
from .quant import dequantize_q4_1, quantize_q4_1  # noqa: F401

__all__ = ["MoEConfig", "MoELayer", "Q4Linear", "HostPipeline", "router_block", "q4_1_to_tiles", "tiles_to_q4_1", "pool_to_q4_1", "experts_from_pool",
           "quantize_q4_1", "dequantize_q4_1"]
