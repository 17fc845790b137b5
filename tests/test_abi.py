"""The C-ABI library loads without a GPU and exports every declared entry point."""
import ctypes
import re

from conftest import ROOT


def declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(hk_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_headers_declare_the_boundary():
    names = declared_functions()
    for required in ("hk_create", "hk_replica", "hk_score", "hk_score_device", "hk_capabilities_get",
                     "hk_last_error", "hk_destroy", "hk_op_gemm"):
        assert required in names


def test_library_exports_every_declared_symbol(native_lib):
    missing = [n for n in sorted(declared_functions()) if not hasattr(native_lib, n)]
    assert not missing, missing


def test_python_binding_lists_model_api(native_lib):
    from huncho_b200 import _native
    for n in _native.EXPORTED:
        assert hasattr(native_lib, n)


def test_errors_without_gpu(native_lib):
    """Calls that need no device fail cleanly with argument errors."""
    h = ctypes.c_void_p()
    assert native_lib.hk_create(None, 0, 1, 512, ctypes.byref(h)) == -5
    assert native_lib.hk_create(b"/nonexistent", 0, 1, 0, ctypes.byref(h)) == -5
    assert native_lib.hk_last_error(None) == b"null handle"
    assert native_lib.hk_kernel_launches(None) == 0


def test_packed_gemm_rejects_bad_shapes_without_gpu(native_lib):
    """The packed projection entry point checks its shape before any device
    call: a width that is not a whole number of Q8_0 blocks, an input wider
    than the packed width, or a short output stride is an error."""
    f = native_lib.hk_op_gemm_packed
    f.argtypes = [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 5 + \
        [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    native_lib.hk_op_last_error.restype = ctypes.c_char_p
    for M, N, K, kp, ldx, ldo in [(4, 8, 40, 40, 40, 8),    # kp not a multiple of 32
                                  (4, 8, 70, 64, 70, 8),    # K > kp
                                  (4, 8, 32, 32, 32, 4),    # ldo < N
                                  (-1, 8, 32, 32, 32, 8)]:  # negative rows
        rc = f(M, N, K, kp, None, ldx, None, None, None, None, None, ldo, 0, None)
        assert rc < 0
        assert b"bad shape" in native_lib.hk_op_last_error()

