"""CPU checks of the C ABI: the library loads without a GPU and exports every
function include/osm_b200.h declares; the Python declarations cover them."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "osm_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(osm_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from osm_b200 import _lib, build

    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_functions()
    assert "osm_moe_forward" in names and "osm_router_topk" not in names
    assert len(names) >= 35


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def declared_arity():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(osm_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", src, flags=re.S):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_python_signatures_match_header_arity(lib):
    from osm_b200 import _lib

    ar = declared_arity()
    for name, (_, args) in _lib._SIGS.items():
        assert len(args) == ar[name], (name, len(args), ar[name])


def test_python_binding_covers_header(lib):
    from osm_b200 import _lib

    assert sorted(_lib.declared_symbols()) == declared_functions()


def test_layout_packed_matches_oracle(lib):
    import osm_b200 as osm
    import pyoracle

    for H, I in ((2048, 512), (2048, 768), (128, 64), (256, 64)):
        L = osm.expert_layout(H, I)
        ref = pyoracle.slot_layout(H, I)
        for name in ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b", "down_w", "down_s",
                     "down_b", "stride"):
            assert getattr(L, name) == ref[name]


def test_context_create_without_gpu_fails_cleanly(lib):
    import ctypes

    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    assert lib.osm_context_create(0, 4, ctypes.byref(h)) != 0
    assert not h.value


def test_product_does_not_reference_oracle():
    """The product path never imports, links or loads the checkers."""
    pkg = os.path.join(ROOT, "orbi-streammoe_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".hpp", ".h", "Makefile")):
                text = open(os.path.join(dirpath, f), errors="ignore").read()
                assert "pyoracle" not in text and "liboracle" not in text, f
                assert "libosm_ref" not in text, f
