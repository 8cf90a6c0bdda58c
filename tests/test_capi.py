"""CPU checks of the C-ABI boundary: the library loads and exports every
symbol the public header declares; the Python bindings declare them all."""
import os
import re

import pytest

from mlx_gsplat_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gsplat_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gs_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("gs_launch_fused_adam_step", "gs_clear_buffer_cache", "gs_cull", "gs_project_forward",
              "gs_render_forward", "gs_render_backward", "gs_project_backward", "gs_fused_adam_slab"):
        assert n in names


@pytest.mark.skipif(not os.path.exists(_lib.LIB_PATH), reason="library not built")
def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for n in declared_functions():
        assert hasattr(lib, n), n


@pytest.mark.skipif(not os.path.exists(_lib.LIB_PATH), reason="library not built")
def test_bindings_cover_header():
    assert set(declared_functions()) <= set(_lib.exported_names())


@pytest.mark.skipif(not os.path.exists(_lib.LIB_PATH), reason="library not built")
def test_cpu_only_calls():
    lib = _lib.load()
    assert lib.gs_abi_version() == 3
    assert lib.gs_clear_buffer_cache() == 0
    assert lib.gs_radix_sort_scratch_bytes(1000) > 8000
    assert lib.gs_cull_scratch_bytes(5000) > 0
    # argument validation happens before any CUDA call
    st = lib.gs_fused_adam_slab(None, None, None, None, None, 10, 70, 60, 60, None, None, None, -1,
                                1e-3, 0.9, 0.999, 1e-8, 0.0, 1, 1.0, 0, None, None, None, 70, 0, None, 0, None)
    assert st == _lib.GS_ERR_INVALID
    assert b"ncols" in lib.gs_last_error()


def test_compute_calls_fail_loudly_without_cuda(monkeypatch):
    import torch
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(_lib.GsplatError):
        _lib.lib()
