"""C-ABI boundary checks that need no GPU: the libraries load, every entry
point declared in include/evkcu.h is exported and bound, and a call without a
device fails with a status and a message instead of crashing."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT, has_gpu

HEADER = os.path.join(ROOT, "include", "evkcu.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|uint64_t|void)\s+(evkcu_\w+)\s*\(", text, re.M)))


def test_header_declares_the_operator_set():
    names = declared()
    for op in ["matmul", "flash_attention", "single_query_attention", "rms_norm", "rope", "gelu", "softmax", "add",
               "greedy_sample", "embed", "causal_mask", "scale", "zero"]:
        assert f"evkcu_{op}" in names


def test_library_exports_every_declared_symbol():
    import evk_b200

    lib = ctypes.CDLL(evk_b200.LIB_PATH)
    for name in declared():
        assert hasattr(lib, name), f"{name} declared in evkcu.h but not exported"
    assert set(declared()) <= set(evk_b200.SIGNATURES), "Python binding misses a declared entry point"


def test_python_binding_loads():
    import evk_b200

    lib = evk_b200.lib()
    assert lib.evkcu_version().decode().startswith("evkcu")


def test_cpp_layer_exports_operator_api():
    import evk_b200

    out = subprocess.run(["nm", "-DC", evk_b200.AI_LIB_PATH], capture_output=True, text=True, check=True).stdout
    for sym in ["evk::ai::matmul(Tensor&, Tensor&, Tensor&, bool, bool, bool, unsigned char, unsigned char)",
                "evk::ai::flash_attention(Tensor&, Tensor&, Tensor&, Tensor&)",
                "evk::ai::greedy_sample(Tensor&, Tensor&, unsigned int, unsigned short, unsigned short)",
                "evk::ai::rms_norm(Tensor&, Tensor&, float)", "evk::CreateBuffer(evk::BufferDesc const&)",
                "evk::CmdWait(unsigned long)"]:
        assert sym in out, sym


@pytest.mark.skipif(has_gpu(), reason="checks the no-device error path")
def test_call_without_device_reports_status():
    import evk_b200

    lib = evk_b200.lib()
    st = lib.evkcu_init(0)
    assert st != 0
    assert lib.evkcu_last_error().decode() != ""


def test_argument_validation_needs_no_device():
    """Bad arguments are rejected before any CUDA call."""
    import evk_b200

    lib = evk_b200.lib()
    # null pointers
    assert lib.evkcu_add(None, None, None, 16, 0, None) == 7
    # bad dtype on a zero-size call still succeeds (nothing to do)
    assert lib.evkcu_add(None, None, None, 0, 0, None) == 0
    # flash: H not a multiple of Hkv
    assert lib.evkcu_flash_attention(8, 8, 8, 8, 1, 16, 3, 2, 64, 0.0, 0, 0, None) == 1
    # flash: Dh not a multiple of 16
    assert lib.evkcu_flash_attention(8, 8, 8, 8, 1, 16, 2, 1, 40, 0.0, 0, 0, None) == 1
    # greedy: out_bytes must be 2 or 4
    assert lib.evkcu_greedy_sample(8, 8, 1, 1, 10, 0, 0, 10, 3, 0, None) == 7
