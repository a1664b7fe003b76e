"""B200-native (sm_100a) per-denoising-step attention path for diffusion LLM
serving: non-causal varlen attention, paged KV-cache store/load, and the
SparseConfig-driven importance scoring / top-k selection.

Public surface mirrors the reference package's (chosen-ox/dLLM-Serve):
  dllmserve_b200.layers.attention.Attention / store_kvcache / load_kvcache
  dllmserve_b200.sparse.state.SparseConfig / PerRequestSparseState
  dllmserve_b200.utils.context.set_context / get_context / reset_context
"""
from .sparse.state import SparseConfig, PerRequestSparseState
from .utils.context import Context, get_context, set_context, reset_context

__all__ = [
    "SparseConfig",
    "PerRequestSparseState",
    "Context",
    "get_context",
    "set_context",
    "reset_context",
]
__version__ = "0.1.0"
