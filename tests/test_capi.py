"""CPU checks of the C ABI: the library loads, exports every symbol the header
declares, and reports errors the way the reference does (no GPU calls)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hachiue_cuda.h")


@pytest.fixture(scope="module")
def lib():
    from hachiue_b200 import build, _lib
    build.build()
    return _lib.load()


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hcu_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_binding_table():
    from hachiue_b200 import _lib
    assert declared_symbols() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_version_and_no_error(lib):
    assert lib.hcu_version() == 3
    assert lib.hcu_last_error() == b""


def test_unknown_pipeline_message(lib):
    words = (ctypes.c_uint32 * 8)()
    st = lib.hcu_dispatch(None, b"gemv_q4_k", words, None, 0)
    assert st == 1  # HCU_EINVAL
    assert lib.hcu_last_error() == b"hachiue: missing pipeline gemv_q4_k"


def test_dispatch_checks_buffer_count(lib):
    words = (ctypes.c_uint32 * 8)(1, 16, 8, 128, 0, 0, 0, 0)
    bufs = (ctypes.c_void_p * 2)(None, None)
    assert lib.hcu_dispatch(None, b"attention_q8", words, bufs, 2) == 1
    assert b"expected 6 storage buffers" in lib.hcu_last_error()


def test_null_handle_is_rejected(lib):
    from hachiue_b200 import _lib
    p = _lib.hcu_attention_params()
    st = lib.hcu_attention(None, ctypes.byref(p), None, None, None)
    assert st == 1 and lib.hcu_last_error().startswith(b"hachiue: hcu_attention")


def test_create_without_gpu_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = lib.hcu_create(0, 0, ctypes.byref(h))
    assert st != 0 and not h.value
    assert lib.hcu_last_error().startswith(b"hachiue: hcu_create")


def test_backend_refuses_cpu_tensors():
    import torch
    from hachiue_b200.backend import _ptr
    from hachiue_b200 import HachiueError
    with pytest.raises(HachiueError):
        _ptr(torch.zeros(4))
