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
