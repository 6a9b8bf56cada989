"""CPU checks of the C-ABI library: it loads, exports every entry point that
include/detgpu.h declares, and reports the absence of a GPU as an error
instead of computing anything on the host."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "detgpu.h")).read()
    return sorted(set(re.findall(r"^\s*(?:det_status|void|const char\*)\s+(det_\w+)\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    import detllm_b200 as D

    if not os.path.exists(D.LIB_PATH):
        import __graft_entry__

        __graft_entry__.build()
    return D.lib()


def test_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n


def test_status_strings(lib):
    assert lib.det_status_string(0) == b"ok"
    assert lib.det_status_string(35) == b"cdf: symbol out of range"


def test_no_silent_cpu_path_without_gpu(lib):
    import ctypes as C

    import detllm_b200 as D

    n = C.c_int(-1)
    assert lib.det_device_count(C.byref(n)) == 0
    if n.value > 0:
        pytest.skip("a GPU is visible")
    from oracle import oracle as O

    with pytest.raises(D.DetError) as e:
        D.Model(O.fixture_gguf("tiny-f32"))
    assert e.value.code == D.ERR_NO_DEVICE


def test_q8_kernel_choice_round_trips(lib):
    import detllm_b200 as D

    prev = D.set_q8_tensor_cores(True)
    try:
        assert D.set_q8_tensor_cores(False) is True
        assert D.set_q8_tensor_cores(False) is False
    finally:
        D.set_q8_tensor_cores(prev)


def test_add_latency_needs_a_gpu(lib):
    import ctypes as C

    import detllm_b200 as D

    n = C.c_int(-1)
    assert lib.det_device_count(C.byref(n)) == 0
    if n.value > 0:
        pytest.skip("a GPU is visible")
    with pytest.raises(D.DetError) as e:
        D.add_latency_cycles(0)
    assert e.value.code == D.ERR_NO_DEVICE
