"""CPU tests of the C ABI boundary: libhymoe.so loads, exports every function that
include/hymoe.h declares, and rejects bad configurations with a status (no crash), all
without a GPU."""
import ctypes as C
import os
import re

import pytest

import hymoe


def declared_functions() -> list[str]:
    src = open(hymoe.HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(hymoe_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_what_bindings_expect():
    assert declared_functions() == sorted(hymoe.EXPORTS)


def test_library_exports_every_declared_symbol():
    L = hymoe.lib()
    for name in declared_functions():
        assert hasattr(L, name), name


def test_version_string():
    assert b"sm_100a" in hymoe.lib().hymoe_version()


def test_invalid_config_is_rejected_without_a_device():
    L = hymoe.lib()
    bad = hymoe.Config(4000, 3072, 64, 8, 1, 16, 0, 0, 1, None)  # H % 128 != 0
    h = C.c_void_p()
    st = L.hymoe_create(C.byref(bad), C.byref(h))
    assert st == 1 and not h.value
    assert b"unsupported shape" in L.hymoe_last_error(None)


def test_null_arguments_are_rejected():
    L = hymoe.lib()
    assert L.hymoe_create(None, None) == 1
    assert L.hymoe_synchronize(None) == 1
    assert L.hymoe_forward(None, 0, None, None, None, 0, None, None, 0) == 1
    assert L.hymoe_set_routing(None, None) == 1
    assert L.hymoe_set_norm(None, 0, None, 1e-5, 0) == 1
    assert L.hymoe_set_placement(None, 0, None) == 1
    assert L.hymoe_load_layer_gguf(None, 0, None, 0) == 1
    L.hymoe_destroy(None)


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="a GPU is present")
def test_create_without_gpu_reports_cuda_error():
    L = hymoe.lib()
    cfg = hymoe.Config(256, 128, 16, 8, 1, 16, 0, 0, 1, None)
    h = C.c_void_p()
    st = L.hymoe_create(C.byref(cfg), C.byref(h))
    assert st in (2, 4) and not h.value
