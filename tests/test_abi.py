"""CPU checks of the drop-in boundary: the library loads, exports every symbol include/flux_b200.h
declares, and the ctypes mirror of fb_linear matches the C struct byte for byte. No compute calls."""

from __future__ import annotations

import ctypes
import re
import subprocess
import sys

import pytest

from selas_b200 import _lib

from .conftest import ROOT

HEADER = ROOT / "include" / "flux_b200.h"


def _declared() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"\b(fb_[a-z0-9_]+)\s*\(", text))


@pytest.fixture(scope="module")
def built():
    from selas_b200 import build

    build.build()
    return _lib.LIB_PATH


def test_header_declares_the_api():
    names = _declared()
    assert {"fb_init", "fb_nf4_dequant", "fb_ln_mod", "fb_linear_grouped", "fb_attention", "fb_attention_split",
            "fb_gated_add", "fb_gelu_tanh", "fb_qk_norm_rope", "fb_last_error", "fb_device_status"} <= names


def test_library_exports_every_declared_symbol(built):
    out = subprocess.run(["nm", "-D", "--defined-only", str(built)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (fb_[a-z0-9_]+)\b", out))
    missing = _declared() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_ctypes_signatures_cover_the_header(built):
    assert _declared() == set(_lib.SIGNATURES)
    lib = _lib.load(built)  # loads and binds every signature; no CUDA call is made
    for name in _declared():
        assert getattr(lib, name).restype is not None or name == "fb_version"


def test_fb_linear_layout_matches_c(tmp_path):
    fields = [f[0] for f in _lib.FbLinear._fields_]
    src = tmp_path / "layout.c"
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {",
             '  printf("size %zu\\n", sizeof(fb_linear));']
    lines += [f'  printf("{f} %zu\\n", offsetof(fb_linear, {f}));' for f in fields]
    lines += ["  return 0;", "}"]
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-o", str(exe), str(src)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines())
    assert int(got["size"]) == ctypes.sizeof(_lib.FbLinear)
    for f in fields:
        assert int(got[f]) == getattr(_lib.FbLinear, f).offset, f


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(_lib.FluxB200Error, match="no CPU fallback"):
        _lib.load(tmp_path / "nope.so")


def test_ops_refuse_cpu_tensors():
    import torch

    from selas_b200 import ops

    with pytest.raises(_lib.FluxB200Error, match="CUDA"):
        ops.gelu_tanh(torch.zeros(8, dtype=torch.bfloat16))


def test_product_path_does_not_import_the_oracle():
    code = ("import sys; import selas_b200, selas_b200.flux, selas_b200.model, selas_b200.ops, selas_b200.codec; "
            "bad = [m for m in sys.modules if m == 'oracle' or m.startswith('oracle.')]; assert not bad, bad")
    subprocess.run([sys.executable, "-c", code], cwd=ROOT, check=True)
