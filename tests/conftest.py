"""Shared test helpers: the `gpu` marker, golden-fixture loading, tolerances."""
from __future__ import annotations

import glob
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# Tolerances of the attention path against an fp32 oracle on the same inputs:
# fp16/bf16 inputs with fp32 accumulation, checked on a float32 output.
TOL_MAX_ABS_16 = 2e-3
TOL_MEAN_ABS_16 = 2e-4
# fp32 inputs: max |err| / max |ref| (relative to the output scale).
TOL_REL_32 = 1e-5


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device (sm_100a)")


def golden_names():
    return sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def load_golden(name: str) -> dict:
    """Load one fixture; inputs come back as float32 arrays holding the exact
    input values, plus `dtype` (the input format) and the metadata."""
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    meta = json.loads(str(z["meta"]))
    dt = meta["dtype"]

    def native_to_f32(a):
        if dt == "bfloat16":
            return (a.astype(np.uint32) << 16).view(np.float32)
        return a.astype(np.float32)

    q = native_to_f32(z["q"])
    if meta.get("kv_is_q"):
        k = v = q
    else:
        k = native_to_f32(z["k"])
        v = native_to_f32(z["v"])
    out = dict(meta=meta, q=q, k=k, v=v, out=z["out"].astype(np.float32))
    if "out_f16" in z:
        out["out_f16"] = z["out_f16"]
    return out


def err_stats(got, ref):
    d = np.abs(np.asarray(got, dtype=np.float64) - np.asarray(ref, dtype=np.float64))
    return float(d.max()) if d.size else 0.0, float(d.mean()) if d.size else 0.0


def assert_close_16(got, ref, what=""):
    """fp16/bf16 path bar: max-abs <= 2e-3 and mean-abs <= 2e-4, no NaN/Inf."""
    got = np.asarray(got, dtype=np.float64)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    mx, mean = err_stats(got, ref)
    assert mx <= TOL_MAX_ABS_16 and mean <= TOL_MEAN_ABS_16, f"{what}: max_abs={mx:.3e} mean_abs={mean:.3e}"
    return mx, mean


def assert_close_32(got, ref, what=""):
    """fp32 path bar: max |err| <= 1e-5 * max |ref|."""
    got = np.asarray(got, dtype=np.float64)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    mx, _ = err_stats(got, ref)
    scale = float(np.abs(ref).max()) or 1.0
    assert mx <= TOL_REL_32 * scale, f"{what}: max_abs={mx:.3e} (scale {scale:.3e})"
    return mx


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def fa(cuda_device):
    """The `_flash_attn_metal` extension (must be the in-tree CUDA build)."""
    import flash_attn_metal_cpp_b200 as pkg

    mod = pkg._flash_attn_metal
    assert mod.__file__.startswith(os.path.join(ROOT, "flash_attn_metal_cpp_b200")), mod.__file__
    assert mod.initialize(), "initialize() failed on a GPU box"
    return mod
