"""C-ABI checks that need no GPU: the library loads, exports every entry point
declared in include/astro_moe.h, and rejects bad geometry on the host before
any CUDA call (as the reference validates before any kernel runs)."""
import ctypes
import os
import re

import numpy as np
import pytest

from astronomical_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_entry_points():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"\b(astro_moe_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = declared_entry_points()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding declares a signature for each of them
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_abi_version():
    assert _lib.lib().astro_moe_abi_version() == 2


def test_struct_layouts_match_the_header(tmp_path):
    """The ctypes mirrors of the ABI's structs have the C compiler's sizes and
    field offsets (a mismatch would misread every weight pointer)."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"astro_moe_affine": _lib.Affine, "astro_moe_layer_weights": _lib.LayerWeights,
               "astro_moe_options": _lib.Options, "astro_moe_block_taps": _lib.BlockTaps,
               "astro_moe_block_path": _lib.BlockPath, "astro_moe_pager_stats": _lib.PagerStats,
               "astro_moe_attribution": _lib.Attribution}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "astro_moe.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'  printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("  return 0;\n}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), "-o", str(exe), str(src)], check=True)
    got = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    c_side = {tuple(l.split()[:2]): int(l.split()[2]) for l in got if l.strip()}
    for cname, py in structs.items():
        assert c_side[(cname, "size")] == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert c_side[(cname, f)] == getattr(py, f).offset, (cname, f)


def test_host_validation_rejects_bad_geometry():
    L = _lib.lib()
    # top_k larger than the router dimension (routing.rs:133-140)
    assert L.astro_moe_route_experts(None, 1, 4, 4, 5, 1, None, None, None) == _lib.ERR_INVALID_ARGUMENT
    assert b"no larger than the router dimension" in L.astro_moe_last_error()
    # unsupported dtype
    assert L.astro_moe_route_experts(None, 9, 4, 4, 2, 1, None, None, None) == _lib.ERR_INVALID_ARGUMENT
    # affine profile (mlx_quantized_operations.rs:339-346)
    st = L.astro_moe_gather_qmm(None, 1, 64, None, None, 1, None, None, None, 1, 2, 48, 4, 0,
                                None, None)
    assert st == _lib.ERR_INVALID_ARGUMENT and b"group size" in L.astro_moe_last_error()
    st = L.astro_moe_gather_qmm(None, 1, 64, None, None, 1, None, None, None, 1, 2, 64, 7, 0,
                                None, None)
    assert st == _lib.ERR_INVALID_ARGUMENT and b"bit width" in L.astro_moe_last_error()
    # null context / unregistered layer
    assert L.astro_moe_register_layer(None, 0, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.astro_moe_block_forward(None, 0, None, 1, None) == _lib.ERR_INVALID_ARGUMENT


def test_invert_assignment_order_on_host():
    # hermetic/sparse_experts.rs:5-36 through the C ABI (a host-only entry point)
    L = _lib.lib()
    order = np.array([1, 3, 5, 4, 2, 0], np.uint32)
    inv = np.empty_like(order)
    assert L.astro_moe_invert_assignment_order(order.ctypes.data, 6, inv.ctypes.data) == 0
    assert inv.tolist() == [5, 0, 4, 1, 3, 2]
    dup = np.array([0, 0], np.uint32)
    assert L.astro_moe_invert_assignment_order(dup.ctypes.data, 2, inv.ctypes.data) == \
        _lib.ERR_DUPLICATE_SLOT
    oor = np.array([0, 2], np.uint32)
    assert L.astro_moe_invert_assignment_order(oor.ctypes.data, 2, inv.ctypes.data) == \
        _lib.ERR_OUT_OF_RANGE_SLOT


def test_numerics_check_rejects_bad_arguments_on_the_host():
    L = _lib.lib()
    fake = ctypes.c_void_p(16)  # never dereferenced: the host checks come first
    for which in (-1, 4, 99):
        assert L.astro_moe_numerics_check(which, fake, fake, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.astro_moe_numerics_check(0, None, fake, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.astro_moe_numerics_check(3, fake, None, None) == _lib.ERR_INVALID_ARGUMENT
    assert b"numerics_check" in L.astro_moe_last_error()


def test_tensor_core_probe_rejects_bad_shapes_on_the_host():
    L = _lib.lib()
    fake = ctypes.c_void_p(256)  # never dereferenced: rejected before any CUDA call
    assert L.astro_moe_tensor_core_probe(0, fake, fake, fake, fake, 1, 24, 1, 0, fake, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert L.astro_moe_tensor_core_probe(0, fake, fake, fake, fake, 1, 16, 1, 0, None, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert L.astro_moe_tensor_core_probe(1, fake, fake, fake, fake, 1, 8, 65, 1, None, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert L.astro_moe_tensor_core_probe(2, fake, fake, fake, fake, 1, 8, 1, 1, None, None) == \
        _lib.ERR_INVALID_ARGUMENT
