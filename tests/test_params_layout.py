"""The C layout of fa_params (include/fa_b200.h) against the ctypes mirror
the tests bind the library with (tests/fa_ctypes.py). A drifted mirror
would make fa_params_init write past the end of the Python structure, so the
size and every field offset must agree. Compiles a small C program with gcc;
runs on CPU."""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FIELDS = ["batch_size", "seqlen_q", "seqlen_k", "num_heads_q", "num_heads_k", "head_dim", "softmax_scale",
          "is_causal", "window_left", "window_right", "dropout_p", "has_alibi", "has_rotary", "gqa_group_size",
          "dtype", "out_dtype", "rope_theta", "q_stride", "k_stride", "v_stride", "o_stride", "alibi_slopes"]


@pytest.fixture(scope="module")
def c_layout(tmp_path_factory):
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    d = tmp_path_factory.mktemp("layout")
    src = d / "layout.c"
    lines = ['#include "fa_b200.h"', "#include <stdio.h>", "#include <stddef.h>", "int main(void) {",
             '  printf("size %zu\\n", sizeof(fa_params));']
    lines += [f'  printf("{f} %zu\\n", offsetof(fa_params, {f}));' for f in FIELDS]
    lines += ["  return 0;", "}"]
    src.write_text("\n".join(lines) + "\n")
    exe = d / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return {k: int(v) for k, v in (ln.split() for ln in out.splitlines())}


def _check(struct_cls, layout):
    names = [f[0] for f in struct_cls._fields_]
    assert names == FIELDS
    assert ctypes.sizeof(struct_cls) == layout["size"]
    for f in FIELDS:
        assert getattr(struct_cls, f).offset == layout[f], f


def test_ctypes_mirror_matches_header(c_layout):
    from fa_ctypes import FaParams

    _check(FaParams, c_layout)
