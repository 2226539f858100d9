"""The C-ABI library builds for sm_100a, loads, and exports every entry point include/lastro_b200.h declares.

No compute call is made here (no GPU in this suite); with no CUDA device the context constructor must fail with a
status code instead of falling back to anything.
"""
import ctypes
import os
import re

import pytest

import lastro_b200 as LB

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions(header):
    src = open(header).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(lastro_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_reference_boundary():
    names = declared_functions(os.path.join(ROOT, "include", "lastro_b200.h"))
    for must in ("lastro_layer_create", "lastro_layer_forward", "lastro_layer_add_into", "lastro_model_create",
                 "lastro_model_load_tensor", "lastro_model_step", "lastro_model_generate", "lastro_model_reset"):
        assert must in names


def test_library_exports_every_declared_symbol():
    if not os.path.exists(LB.LIB_PATH):
        LB.build()
    lib = ctypes.CDLL(LB.LIB_PATH)
    missing = [n for n in declared_functions(os.path.join(ROOT, "include", "lastro_b200.h")) if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding declares exactly the same set
    assert sorted(LB.EXPORTS) == declared_functions(os.path.join(ROOT, "include", "lastro_b200.h"))


def test_version_string_names_the_target():
    assert b"sm_100a" in LB.lib().lastro_version()


def test_no_cuda_device_fails_loudly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(LB.LastroError):
        LB.Context(0)
