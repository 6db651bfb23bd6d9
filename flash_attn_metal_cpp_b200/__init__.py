"""FlashAttention-2 forward for NVIDIA B200 (sm_100a).

Drop-in for the `_flash_attn_metal` module of harvestingmoon/flash_attn_metal_cpp:
importing this package loads the prebuilt extension and registers it as the
top-level module `_flash_attn_metal`, so unchanged scripts that do
`import _flash_attn_metal` get the CUDA implementation.

`metal_attention` mirrors the reference package wrapper (__init__.py:48-89):
it converts inputs to NumPy float16 arrays, defaults softmax_scale to
1/sqrt(head_dim) and calls `_flash_attn_metal.forward`, returning a NumPy
float16 array.

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


def _to_numpy(x):
    """np.array(x) of the reference wrapper (__init__.py:63-68); torch
    tensors (also CUDA ones, which np.array cannot read) via .cpu().numpy()."""
    import numpy as np

    if isinstance(x, np.ndarray):
        return x
    if hasattr(x, "detach") and hasattr(x, "cpu"):
        x = x.detach().cpu()
        if str(x.dtype) == "torch.bfloat16":
            x = x.float()  # NumPy has no bfloat16; the cast below goes to float16 anyway
        return x.numpy()
    return np.array(x)


def metal_attention(q, k, v, causal=False, softmax_scale=None, dropout_p=0.0):
    """Attention forward with the reference wrapper's conventions
    (__init__.py:48-89).

    q: (batch, seqlen_q, num_heads, head_dim); k, v: (batch, seqlen_k,
    num_heads_k, head_dim), as NumPy arrays, torch tensors or nested
    sequences. Inputs are converted to NumPy and cast to float16;
    softmax_scale defaults to 1/sqrt(head_dim). Returns a NumPy float16
    array of q's shape (computed on the GPU through the host-pointer path).
    """
    import numpy as np

    q, k, v = (_to_numpy(t).astype(np.float16) for t in (q, k, v))
    if softmax_scale is None:
        softmax_scale = 1.0 / np.sqrt(q.shape[-1])
    return _flash_attn_metal.forward(
        q, k, v, softmax_scale=float(softmax_scale), is_causal=bool(causal), dropout_p=float(dropout_p)
    )


__all__ = ["metal_attention", "initialize", "get_device_info", "forward", "LIB_PATH"]
