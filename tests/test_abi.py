"""CPU: the C-ABI library loads, exports every entry point the header declares,
and rejects bad arguments before touching the GPU."""
import ctypes
import os
import re
import subprocess

import pytest

from megaqwen_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"^\s*int\s+(\w+)\s*\(", src, flags=re.M)
    return names


def test_header_declares_expected_set():
    assert set(header_functions()) == set(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    for name in header_functions():
        assert name in exported, name
        assert getattr(lib, name) is not None


@pytest.mark.gpu
def test_library_is_built_for_sm100a():
    """The decode kernel loads as an sm_100 binary (cudaFuncGetAttributes().binaryVersion)."""
    import torch
    torch.cuda.init()
    assert _lib.library_info()["binary_version"] == 100


def test_argument_validation_without_gpu():
    lib = _lib.load()
    n = ctypes.c_void_p(0)
    rc = lib.launch_a10_int8_decode(0, *([n] * 21), 28, 0, 1, 2048, ctypes.c_float(0.088), n, n)
    assert rc == -1
    assert lib.mq_quantize_per_channel(n, 4, 4, n, n, n) == -1
    assert lib.mq_matvec(0, n, n, n, n, 4, 1024, n) == -1
    assert lib.mq_set_wait_budget_ns(0) == -1
    assert lib.mq_decode_multi(2, 0, n, n, 1, *([n] * 13), 28, 0, 2048, ctypes.c_float(0.1), 16, n) == -1


def test_check_raises_on_error_codes():
    with pytest.raises(_lib.MQError):
        _lib.check(-3, "x")
    with pytest.raises(_lib.MQError):
        _lib.check(700, "x")
    _lib.check(0, "x")
