"""Route an existing dLLM-Serve installation through this package.

``install()`` replaces the attention layer of the reference package
(``dllmserve.layers.attention.Attention`` together with its module-level
``store_kvcache`` / ``load_kvcache``) and its rotary embedding
(``dllmserve.layers.rotary_embedding.RotaryEmbedding`` / ``get_rope``) by this
package's drop-in versions, in every already-imported module that bound them
by name (the model files import ``Attention`` and ``get_rope`` at import time:
dllmserve/models/llada.py, dllmserve/models/dream.py),
and points the layer at the reference's ``get_context`` so the reference's
``ModelRunner._run_diffusion`` (model_runner.py:310-321) drives it unchanged.
Call it before the model is constructed (``LLM(...)``).
"""
from __future__ import annotations

import importlib
import sys

from .layers import attention as _attn
from .layers import rotary_embedding as _rope

_PATCHED: list[tuple[object, str, object]] = []


def install(package: str = "dllmserve") -> list[str]:
    """Patch ``package``'s attention path; returns the patched module names."""
    ref_attn = importlib.import_module(f"{package}.layers.attention")
    ref_ctx = importlib.import_module(f"{package}.utils.context")
    patched = []

    def swap(mod, name, value):
        if hasattr(mod, name):
            _PATCHED.append((mod, name, getattr(mod, name)))
            setattr(mod, name, value)

    swap(ref_attn, "Attention", _attn.Attention)
    swap(ref_attn, "store_kvcache", _attn.store_kvcache)
    swap(ref_attn, "load_kvcache", _attn.load_kvcache)
    patched.append(ref_attn.__name__)
    try:
        ref_rope = importlib.import_module(f"{package}.layers.rotary_embedding")
    except ImportError:
        ref_rope = None
    if ref_rope is not None:
        swap(ref_rope, "RotaryEmbedding", _rope.RotaryEmbedding)
        swap(ref_rope, "get_rope", _rope.get_rope)
        patched.append(ref_rope.__name__)
    for name, mod in list(sys.modules.items()):
        if mod is None or mod is ref_attn or not name.startswith(package + "."):
            continue
        hit = False
        orig = mod.__dict__.get("Attention")
        if orig is not None and orig is not _attn.Attention and getattr(orig, "__module__", "") == ref_attn.__name__:
            swap(mod, "Attention", _attn.Attention)
            hit = True
        orig = mod.__dict__.get("get_rope")
        if (ref_rope is not None and mod is not ref_rope and orig is not None and orig is not _rope.get_rope
                and getattr(orig, "__module__", "") == ref_rope.__name__):
            swap(mod, "get_rope", _rope.get_rope)
            hit = True
        if hit:
            patched.append(name)
    # the layer reads the context the reference's model runner writes
    _PATCHED.append((_attn, "get_context", _attn.get_context))
    _attn.get_context = ref_ctx.get_context
    return patched


def uninstall() -> None:
    """Undo ``install()`` (restores every replaced attribute)."""
    while _PATCHED:
        mod, name, value = _PATCHED.pop()
        setattr(mod, name, value)
