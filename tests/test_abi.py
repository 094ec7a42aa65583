"""The C ABI library on CPU: it loads without a GPU, exports exactly the entry
points include/lunara_b200.h declares (with the signatures the ctypes binding
assumes), and its argument validation answers before touching the device."""
import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from lunara_b200.runtime import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "lunara_b200.h"
SELFTEST_HEADER = HEADER.with_name("lunara_b200_selftest.h")


def header_functions(header=HEADER):
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(lunara_\w+)\s*\(", text)))


def exported_functions():
    """Every `lunara_*` function the shared library defines (dynamic symbol table)."""
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    return sorted({ln.split()[-1] for ln in out.splitlines() if ln.split()[-1].startswith("lunara_")})


def test_library_loads_without_gpu():
    lib = _lib.load()
    assert lib.lunara_version() == 10000


def test_exports_every_declared_symbol():
    lib = _lib.load()
    declared = header_functions()
    assert len(declared) == 16
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(_lib.SIGNATURES) == declared


@pytest.mark.skipif(shutil.which("nm") is None, reason="needs nm")
def test_export_set_equals_header_declarations():
    """Both ways: nothing exported that no header declares, nothing declared that is not exported."""
    declared = sorted(set(header_functions()) | set(header_functions(SELFTEST_HEADER)))
    assert exported_functions() == declared
    assert sorted(_lib.SELFTEST_SIGNATURES) == header_functions(SELFTEST_HEADER)


def test_selftest_arity_matches_header():
    text = re.sub(r"/\*.*?\*/", "", SELFTEST_HEADER.read_text(), flags=re.S)
    for name, (argtypes, _) in _lib.SELFTEST_SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\(([^)]*)\)", text)
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(argtypes), name


def test_selftest_wait_rejects_bad_arguments_on_host():
    lib = _lib.load()
    assert lib.lunara_selftest_bounded_wait(10, 0x401, None) == 1           # budget below 1 us
    assert lib.lunara_selftest_bounded_wait(10 ** 10, 0x401, None) == 1     # budget above 1 s
    assert lib.lunara_selftest_bounded_wait(10 ** 6, 0x101, None) == 1      # a product kernel's site code


def test_signature_arity_matches_header():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, (argtypes, _) in _lib.SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\(([^)]*)\)", text)
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(argtypes), name


def test_enum_values_match_header():
    text = HEADER.read_text()
    for cname, val in [("LUNARA_F16", _lib.F16), ("LUNARA_BF16", _lib.BF16), ("LUNARA_F32", _lib.F32),
                       ("LUNARA_ACT_GELU_TANH", _lib.ACT_GELU_TANH), ("LUNARA_ACT_TANH", _lib.ACT_TANH),
                       ("LUNARA_B_NK", _lib.B_NK), ("LUNARA_ERR_DEVICE", _lib.ERR_DEVICE),
                       ("LUNARA_BIN_MUL", _lib.BIN_MUL)]:
        assert re.search(rf"\b{cname}\s*=\s*{val}\b", text), cname


def _err(lib):
    return lib.lunara_last_error_string().decode()


@pytest.mark.parametrize("call,needle", [
    (lambda L: L.lunara_gemm(1, 1, 1, None, None, 4, 4, 4, 4, 4, 4, 0, 0, 9, 0, None, None), "dtype"),
    (lambda L: L.lunara_gemm(1, 1, 1, None, None, 4, 4, 4, 4, 4, 4, 0, 0, 0, 17, None, None), "activation"),
    (lambda L: L.lunara_gemm(1, 1, 1, None, None, 4, 4, 4, 4, 4, 4, 0, 5, 0, 0, None, None), "b_layout"),
    (lambda L: L.lunara_gemm(1, 1, 1, None, None, 4, 8, 4, 2, 8, 8, 0, 0, 0, 0, None, None), "lda"),
    (lambda L: L.lunara_gemm(1, 1, 1, None, None, -1, 8, 4, 4, 8, 8, 0, 0, 0, 0, None, None), "negative"),
    (lambda L: L.lunara_layernorm(1, 1, 1, 1, 4, 0, 1e-5, 0, None), "shape"),
    (lambda L: L.lunara_gemm_layernorm(1, 1, 1, None, None, 1, 1, 4, 768, 8, 8, 8, 768, 0, 1, 0, -1.0, None, None),
     "eps"),
    (lambda L: L.lunara_gemm_layernorm(1, 1, 1, None, None, None, 1, 4, 768, 8, 8, 8, 768, 0, 1, 0, 1e-5, None,
                                       None), "NULL"),
    (lambda L: L.lunara_gemm_layernorm(1, 1, 1, None, None, 1, 1, 4, 100, 8, 8, 8, 100, 0, 1, 0, 1e-5, None, None),
     "run lunara_gemm then lunara_layernorm"),
    (lambda L: L.lunara_layernorm(1, 1, 1, 1, 4, 8, -1.0, 0, None), "eps"),
    (lambda L: L.lunara_softmax(1, 1, 4, 8, 3, None), "dtype"),
    (lambda L: L.lunara_eltwise_unary(42, 1, 1, 8, 0, None), "op"),
    (lambda L: L.lunara_eltwise_binary(3, 1, 1, 1, 8, 0, None), "op"),
    (lambda L: L.lunara_copy_strided(1, 1, 9, None, None, 2, None), "ndim"),
    (lambda L: L.lunara_copy_strided(1, 1, 1, _lib.i64_array([4]), _lib.i64_array([1]), 3, None), "elem_bytes"),
    (lambda L: L.lunara_attention(1, 1, 1, 1, 1, 1, 8, 8, 512, *(_lib.i64_array([0, 0, 0, 1]),) * 4, 0.1, 0, 0,
                                  None), "head dim"),
    (lambda L: L.lunara_slice(1, 1, 1, _lib.i64_array([10]), _lib.i64_array([8]), _lib.i64_array([1]),
                              _lib.i64_array([4]), 2, None), "outside"),
    (lambda L: L.lunara_slice(1, 1, 1, _lib.i64_array([10]), _lib.i64_array([0]), _lib.i64_array([0]),
                              _lib.i64_array([4]), 2, None), "step"),
])
def test_invalid_arguments_rejected_on_host(call, needle):
    lib = _lib.load()
    rc = call(lib)
    assert rc in (_lib.ERR_INVALID_ARG, _lib.ERR_UNSUPPORTED)
    assert needle in _err(lib)


def test_empty_work_is_ok_without_device():
    lib = _lib.load()
    assert lib.lunara_gemm(None, None, 1, None, None, 0, 8, 8, 8, 8, 8, 0, 0, 0, 0, None, None) == _lib.OK
    assert lib.lunara_layernorm(None, None, None, None, 0, 8, 1e-5, 0, None) == _lib.OK
    assert lib.lunara_gather(None, None, None, 0, 5, 16, None) == _lib.OK


def test_check_raises_with_library_message():
    lib = _lib.load()
    rc = lib.lunara_softmax(1, 1, 4, 8, 3, None)
    with pytest.raises(ValueError, match="dtype"):
        _lib.check(rc)
    with pytest.raises(_lib.LunaraError):
        _lib.check(_lib.ERR_LAUNCH)


def test_ctypes_config_struct_layout():
    assert ctypes.sizeof(_lib.GemmConfig) == 16
