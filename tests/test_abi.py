"""CPU checks of the C-ABI boundary: the library loads, exports exactly what
include/*.h declares, and rejects bad calls before touching a device."""
import ctypes
import re
from pathlib import Path

import pytest

import ouroboros_b200 as oq

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = set()
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(ouroq_\w+)\s*\(", text))
    return names


def test_library_built_and_loads():
    assert oq.LIB_PATH.exists(), "run python -m ouroboros_b200.build"
    lib = ctypes.CDLL(str(oq.LIB_PATH))
    assert lib is not None


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(oq.LIB_PATH))
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_mirror_covers_the_header():
    assert declared_functions() == set(oq.ABI_FUNCTIONS)


def test_abi_version_and_status_strings():
    lib = oq.load_library()
    assert lib.ouroq_abi_version() == 1
    assert lib.ouroq_status_string(0) == b"ok"
    assert lib.ouroq_status_string(1) == b"bad shape"
    assert lib.ouroq_status_string(5) == b"timeout"


def test_null_handles_are_rejected_without_a_device():
    lib = oq.load_library()
    assert lib.ouroq_ctx_destroy(None) == 7
    assert lib.ouroq_gemm(None, None, None, None, 1, None, None, None) == 7
    assert lib.ouroq_weight_info(None, None, None, None, None) == 7
    assert lib.ouroq_ctx_create(0, None) == 7
    assert lib.ouroq_last_error(None) == b""


def test_no_device_is_an_error_not_a_fallback():
    import torch
    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    with pytest.raises(oq.OuroqError) as e:
        oq.Context(0)
    assert e.value.status == 8  # OUROQ_ERR_NO_DEVICE


def test_product_package_does_not_load_the_oracle():
    pat = re.compile(r"import\s+oracle|from\s+oracle|pyoracle|liboracle|oracle\.c\b")
    for p in (ROOT / "ouroboros_b200").rglob("*"):
        if p.suffix in (".py", ".cpp", ".cu", ".cuh", ".h"):
            assert not pat.search(p.read_text()), p


def test_ptr_kind_of_pageable_host_memory_without_a_device():
    # cudaPointerGetAttributes answers for plain host memory even when the
    # runtime finds no device; a caller on a CPU-only host gets PTR_HOST, -1
    import numpy as np
    a = np.empty(16, np.float32)
    assert oq.ptr_kind(a.ctypes.data) == (oq.PTR_HOST, -1)
