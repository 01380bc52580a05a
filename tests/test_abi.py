"""The C ABI without a GPU: libxdna_b200.so loads, exports every function include/xdna_b200.h declares,
and its argument checks reject bad calls before touching a device (no compute is launched)."""

import ctypes
import re

from conftest import LIB, ROOT, ensure_built

HEADER = ROOT / "include" / "xdna_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(xdna_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for required in ("xdna_last_error", "xdna_quant_rows_i8", "xdna_gemm_i8", "xdna_conv3x3_i8",
                     "xdna_conv_quant_nhwc", "xdna_take_device_error"):
        assert required in names, names


def test_library_exports_every_declared_symbol():
    ensure_built()
    lib = ctypes.CDLL(str(LIB))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared in {HEADER.name} but not exported: {missing}"


def test_abi_version_and_error_text():
    ensure_built()
    lib = ctypes.CDLL(str(LIB))
    assert lib.xdna_abi_version() == 1
    lib.xdna_last_error.restype = ctypes.c_char_p
    assert isinstance(lib.xdna_last_error(), bytes)


def test_package_binding_matches_header():
    """Every function the Python binding declares exists in the header (and so in the library)."""
    import torch_xdna.kernels as k

    src = (ROOT / "torch-xdna_b200" / "torch_xdna" / "kernels.py").read_text()
    bound = set(re.findall(r'"(xdna_\w+)":', src))
    assert bound <= set(declared_functions()), bound - set(declared_functions())
    assert k.LIB_PATH == LIB
