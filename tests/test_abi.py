"""The C-ABI library: it loads, exports every symbol include/modelc_cuda.h
declares, and fails loudly (no CPU fallback) when no sm_100 device exists."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

import modelc_b200 as mb
from modelc_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "modelc_cuda.h")).read()
    return sorted(set(re.findall(r"^MC_API\s+[\w\s\*]+?\b(mc_\w+)\(", txt, re.M)))


def test_header_declares_expected_api():
    syms = declared_symbols()
    assert sorted(_lib.EXPORTS) == syms


def test_library_exports_every_declared_symbol():
    lib = mb.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (mc_\w+)$", out, re.M))
    for s in declared_symbols():
        assert s in exported, s
        assert hasattr(lib, s)


def test_version_string():
    assert b"sm_100a" in mb.lib().mc_version()


def test_library_is_built_for_sm100a_only():
    from modelc_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device error path")
def test_no_device_fails_loudly():
    w = {"model.embed_tokens.weight": mb.QTensor("i8_row", np.zeros((4, 8), np.int8),
                                                  np.ones(4, np.float32))}
    cfg = mb.LlamaConfig(0, 8, 1, 1, 8, 8, 4)
    with pytest.raises(mb.McError) as e:
        mb.Weights(w, cfg)
    assert e.value.status == -5 and "no CUDA device" in str(e.value)
