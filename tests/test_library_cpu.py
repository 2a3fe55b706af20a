"""CPU checks of the C-ABI library and the host layer (no compute calls).

The library must load without a GPU and export every entry point that
include/maskahead_b200.h declares; the ctypes signatures must cover exactly those; the
host layer must refuse to run (no silent CPU fallback) when CUDA is unavailable.
"""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "maskahead_b200.h"


def _declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"MA_API\s+[\w\s\*]+?\b(ma_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    from maskahead_b200.build import build

    build()
    import maskahead_b200

    return maskahead_b200.load_library()


def test_header_declares_entry_points():
    names = _declared()
    assert {"ma_prefix_attention", "ma_prefix_scores", "ma_value_score", "ma_select_topk", "ma_retain",
            "ma_sparse_attention", "ma_gather_kv"} <= names


def test_library_exports_every_declared_symbol(lib):
    from maskahead_b200._lib import EXPORTED, LIB_PATH

    for name in _declared():
        assert hasattr(lib, name), f"{name} declared but not exported"
    assert set(EXPORTED) == _declared(), "ctypes signatures and header disagree"
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == _declared(), f"unexpected exports: {exported ^ _declared()}"


def test_status_strings_and_sizing(lib):
    assert lib.ma_version() >= 1
    assert lib.ma_status_string(0) == b"ok"
    assert lib.ma_status_string(-3) == b"workspace missing or too small"
    assert lib.ma_prefix_attention_workspace(1, 4, 224, 8192, 128, 32) > 0
    assert lib.ma_prefix_attention_workspace(0, 4, 224, 8192, 128, 32) == 0
    assert lib.ma_value_score_workspace(1, 4, 8192, 128) > 0


def test_argument_validation_without_gpu(lib):
    """Rejected calls return an error before touching the device."""
    from maskahead_b200._lib import MaKV, MaRows, MaBlock, i64

    rows = MaRows()
    assert lib.ma_prefix_attention(rows, MaKV(), 4, MaBlock(), 1.0, 0, 0, 0, None, i64(0, 0, 0), None,
                                   None, None, None, 0, None) == -1
    assert lib.ma_select_topk(None, 1, 1, 8, i64(8, 8), None, None, 3, None, None, i64(3, 3), None) == -1
    assert lib.ma_retain(None, None, 0, None, 1, 8, 4, 2, 0, None, None) == -1


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_silent_cpu_fallback():
    from maskahead_b200 import KernelUnavailableError
    from maskahead_b200.kernels import select_topk_indices

    with pytest.raises(KernelUnavailableError):
        select_topk_indices(torch.zeros(1, 1, 8), 2)
