"""The `_flash_attn_metal` module surface matches the reference's
(python/bindings.cpp:239-269): names, defaults and error behaviour (CPU)."""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def fam():
    import flash_attn_metal_cpp_b200 as pkg
    import sys

    mod = pkg._flash_attn_metal
    assert sys.modules["_flash_attn_metal"] is mod
    assert mod.__file__.startswith(os.path.join(ROOT, "flash_attn_metal_cpp_b200"))
    return mod


def test_surface_names(fam):
    for n in ("initialize", "load_shaders", "compile_shaders", "get_device_info", "forward"):
        assert callable(getattr(fam, n))


def test_forward_signature_defaults(fam):
    import re

    doc = fam.forward.__doc__.splitlines()[0]
    names = re.findall(r"(\w+): [^=,]+?(?: = ([^,)]+))?(?=,|\))", doc)
    args = dict(names)
    order = [n for n, _ in names]
    assert order[:10] == ["Q", "K", "V", "softmax_scale", "is_causal", "dropout_p", "alibi_slopes",
                          "window_size", "cos", "sin"]
    assert args["softmax_scale"] == "0.0" and args["is_causal"] == "False" and args["dropout_p"] == "0.0"
    for n in ("alibi_slopes", "window_size", "cos", "sin"):
        assert args[n] == "None"


def test_device_info_keys(fam):
    info = fam.get_device_info()
    assert set(info) >= {"device_name", "max_buffer_length", "initialized"}


def test_shader_calls_are_accepted(fam):
    import torch

    expect = torch.cuda.is_available()
    assert fam.compile_shaders("kernel void f() {}") is expect
    assert fam.load_shaders("/nonexistent.metallib") is expect
    assert fam.initialize() is expect


def test_forward_validation_errors(fam):
    x = np.zeros((1, 4, 2, 64), np.float16)
    with pytest.raises(RuntimeError, match="Forward pass error: Input arrays must be 4D"):
        fam.forward(x[0], x[0], x[0])
    with pytest.raises(RuntimeError, match="Forward pass error: K and V shapes must match"):
        fam.forward(x, x, np.zeros((1, 5, 2, 64), np.float16))
    with pytest.raises(RuntimeError, match="Forward pass error"):
        fam.forward(x.astype(np.int16), x.astype(np.int16), x.astype(np.int16))
    with pytest.raises(RuntimeError, match="dropout"):
        fam.forward(x, x, x, 0.1, False, 0.5)
    with pytest.raises(RuntimeError, match="alibi_slopes must hold one"):
        fam.forward(x, x, x, 0.1, False, 0.0, np.ones(3, np.float32))  # 2 query heads


def test_package_wrapper(fam):
    import torch

    import flash_attn_metal_cpp_b200 as pkg

    assert callable(pkg.metal_attention)
    assert pkg.forward is fam.forward
    # Inputs become NumPy arrays as in the reference wrapper (np.array(x)).
    x = np.arange(24, dtype=np.float32).reshape(1, 2, 3, 4)
    assert pkg._to_numpy(x) is x
    assert np.array_equal(pkg._to_numpy(torch.from_numpy(x)), x)
    assert np.array_equal(pkg._to_numpy(x.tolist()), x)
    assert pkg._to_numpy(torch.from_numpy(x).to(torch.bfloat16)).dtype == np.float32
    assert set(fam.get_wait_limit.__doc__.split()) & {"wait", "limit"}
