"""The C ABI library loads and exports every function the header declares;
argument errors are reported (these calls touch no GPU)."""
import ctypes as C
import os
import re

from turbompc_b200 import _ffi

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "tmpc_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int32_t|uint32_t|int64_t|size_t|const char\*)\s+(tmpc_\w+)\s*\(", src, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = _ffi.load()
    names = declared_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(_ffi.exported_symbols())


def test_error_codes_without_gpu():
    lib = _ffi.load()
    assert lib.tmpc_version() >= 100
    assert b"null" in lib.tmpc_error_string(-1)
    cfg = _ffi.TmpcAdmmConfig()
    assert lib.tmpc_admm_solve_f32(None, None, None, None, None, C.byref(cfg), None, None, None, None, 0, None) == -1
    bad = _ffi.TmpcDims(1, 1, 4, 2, 2, 0)  # T < 2
    assert lib.tmpc_admm_solve_f64(C.byref(bad), None, None, None, None, C.byref(cfg), None, None, None, None, 0,
                                   None) == -2
    assert lib.tmpc_packed_operator_bytes(C.byref(_ffi.TmpcDims(1, 3, 40, 20, 20, 0)), 4) == 0  # n > 32
    d = _ffi.TmpcDims(2, 5, 16, 12, 12, 4)
    assert lib.tmpc_packed_operator_bytes(C.byref(d), 4) > 0


def test_transfer_poll_limit_hook_round_trips():
    lib = _ffi.load()
    prev = lib.tmpc_set_transfer_poll_limit(1234)
    assert prev == 1 << 26
    assert lib.tmpc_set_transfer_poll_limit(prev) == 1234


def test_iteration_timing_hook_round_trips():
    lib = _ffi.load()
    assert lib.tmpc_admm_iteration_timing(1) == 0
    assert lib.tmpc_admm_iteration_timing(0) == 1
    buf = (C.c_float * 4)()
    assert lib.tmpc_admm_iteration_timing_read(buf, 4) == 0  # nothing recorded without a solve


def test_interleaved_sizes_without_gpu():
    lib = _ffi.load()
    assert lib.tmpc_interleaved_elems(37, 10) == 64 * 10
    assert lib.tmpc_interleaved_elems(32, 10) == 32 * 10
    assert lib.tmpc_interleaved_elems(0, 10) == 0
    d = _ffi.TmpcDims(5, 4, 3, 2, 0, 0)  # T = 4, n = 3: 4 * 6 + 3 * 9
    assert lib.tmpc_riccati_il_elems_per_problem(C.byref(d)) == 4 * 6 + 3 * 9


def test_ffi_handlers_compile_to_nothing_without_xla_headers(tmp_path):
    """csrc/ffi/admm_b200_ffi.cc is guarded by __has_include on the jaxlib
    FFI header: without it (here) it must still compile, to an empty object."""
    import shutil
    import subprocess
    from turbompc_b200 import build
    gxx = shutil.which("g++")
    if gxx is None:
        import pytest
        pytest.skip("no g++")
    obj = tmp_path / "ffi.o"
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(build.nvcc())), "include")
    res = subprocess.run([gxx, "-std=c++17", "-c", build.FFI_SRC, "-I" + build.INCLUDE, "-I" + cuda_inc, "-o",
                          str(obj)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    nm = subprocess.run(["nm", str(obj)], capture_output=True, text=True).stdout
    assert "AdmmB200Cuda" not in nm
