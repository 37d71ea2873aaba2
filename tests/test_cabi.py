"""The C-ABI library loads and exports every entry point include/*.h declares.

No compute is issued (no GPU is needed): this checks the boundary itself.
"""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from laprune_b200 import _lib, ops

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(lp_[A-Za-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_functions()
    assert "lp_sparse_decode" in names and "lp_last_error" in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports(name):
    lib = _lib.load()
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert name in _lib.SIGNATURES, f"{name} has no Python binding signature"


def test_struct_layout_matches():
    lib = _lib.load()
    assert lib.lp_sizeof_sparse_decode_args() == ctypes.sizeof(_lib.SparseDecodeArgs)


def test_workspace_size_is_host_only():
    # the workspace query runs without touching a GPU
    a = _lib.SparseDecodeArgs()
    a.B, a.Hkv, a.G, a.D, a.M, a.K = 1, 8, 4, 128, 32, 256
    a.T_codes = a.T_total = 131072
    a.sink, a.local, a.topk = 4, 64, 2048
    n = _lib.load().lp_sparse_decode_workspace_size(ctypes.byref(a))
    assert n > 8 * 131072 * 4  # at least the selection scores
    a.topk = 10 ** 7  # more than the candidates -> invalid -> 0
    assert _lib.load().lp_sparse_decode_workspace_size(ctypes.byref(a)) == 0
    assert "topk" in _lib.load().lp_last_error().decode()


def test_no_cpu_fallback():
    q = torch.zeros(32, 128, dtype=torch.bfloat16)
    C = torch.zeros(8, 32, 256, 128)
    codes = torch.zeros(8, 100, 32, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.sparse_decode(q, C, codes, topk=4, attention=False)
