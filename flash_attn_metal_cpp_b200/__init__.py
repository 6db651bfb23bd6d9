"""FlashAttention-2 forward for NVIDIA B200 (sm_100a).

Drop-in for the `_flash_attn_metal` module of harvestingmoon/flash_attn_metal_cpp:
importing this package loads the prebuilt extension and registers it as the
top-level module `_flash_attn_metal`, so unchanged scripts that do
`import _flash_attn_metal` get the CUDA implementation.

`metal_attention` mirrors the reference package wrapper (__init__.py:48-89):
it casts inputs to float16, defaults softmax_scale to 1/sqrt(head_dim) and
calls `_flash_attn_metal.forward`.

There is no CPU fallback: if the extension is missing, importing raises.
"""
from __future__ import annotations

import os
import sys

__version__ = "0.1.0"

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libfa_b200.so")

try:
    from . import _flash_attn_metal  # noqa: F401  (built by flash_attn_metal_cpp_b200.build)
except ImportError as exc:  # pragma: no cover - exercised only without a build
    raise ImportError(
        "flash_attn_metal_cpp_b200: the CUDA extension is not built "
        f"({exc}). Build it with `python flash_attn_metal_cpp_b200/build.py`."
    ) from exc

sys.modules.setdefault("_flash_attn_metal", _flash_attn_metal)

initialize = _flash_attn_metal.initialize
get_device_info = _flash_attn_metal.get_device_info
forward = _flash_attn_metal.forward


def metal_attention(q, k, v, causal=False, softmax_scale=None, dropout_p=0.0):
    """Attention forward with the reference wrapper's conventions.

    q: (batch, seqlen_q, num_heads, head_dim); k, v: (batch, seqlen_k,
    num_heads_k, head_dim). Inputs are cast to float16 (NumPy arrays) or
    kept as torch tensors cast to float16; softmax_scale defaults to
    1/sqrt(head_dim). Returns float16 output of q's shape.
    """
    import numpy as np

    if hasattr(q, "data_ptr") and hasattr(q, "is_cuda"):
        import torch

        q, k, v = (t.to(torch.float16) for t in (q, k, v))
    else:
        q, k, v = (np.asarray(t).astype(np.float16) for t in (q, k, v))
    if softmax_scale is None:
        softmax_scale = 1.0 / float(np.sqrt(q.shape[-1]))
    return _flash_attn_metal.forward(
        q, k, v, softmax_scale=float(softmax_scale), is_causal=bool(causal), dropout_p=float(dropout_p)
    )


__all__ = ["metal_attention", "initialize", "get_device_info", "forward", "LIB_PATH"]
