"""CPU tests of the C-ABI boundary: the library loads, exports every entry point
include/droidcorr.h declares, and its host-only calls behave (no GPU needed)."""
import ctypes
import os
import re
import subprocess

import pytest

from slam_hands_b200 import _lib as L

HEADER = L.HEADER


def declared_functions(header=HEADER):
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b(dc_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_boundary():
    names = declared_functions()
    for n in ["dc_create", "dc_destroy", "dc_set_frames", "dc_build_volume", "dc_pool_2x2",
              "dc_lookup", "dc_lookup_single", "dc_build_and_lookup", "dc_alt_lookup",
              "dc_last_error", "dc_status_string", "dc_default_config"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = L.load()
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(dc_\w+)$", out, flags=re.M))
    for name in declared_functions():
        assert name in exported, name
        assert hasattr(lib, name)
        assert name in L.SIGNATURES, f"{name} has no ctypes signature"


def test_library_targets_sm100a_only():
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", L.LIB_PATH],
                         capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    archs = set(re.findall(r"sm_(\d+a?)", out.stdout))
    assert archs == {"100a"}, archs


def test_host_only_calls():
    lib = L.load()
    assert lib.dc_status_string(L.DC_OK) == b"ok"
    assert b"invalid" in lib.dc_status_string(L.DC_ERR_INVALID_ARG)
    cfg = L.DcConfig()
    lib.dc_default_config(ctypes.byref(cfg), 48, 64)
    assert (cfg.h, cfg.w, cfg.channels, cfg.levels, cfg.radius) == (48, 64, 128, 4, 3)
    assert cfg.max_edges == 48 and cfg.precision == L.DC_PREC_FP16
    assert cfg.alpha == pytest.approx(1 / 16)


def test_create_rejects_bad_configs_before_touching_a_device():
    lib = L.load()
    h = ctypes.c_void_p()
    for bad in [dict(h=0), dict(channels=100), dict(levels=5), dict(radius=4),
                dict(precision=7), dict(max_edges=0), dict(h=4, levels=4)]:
        cfg = L.DcConfig()
        lib.dc_default_config(ctypes.byref(cfg), 48, 64)
        for k, v in bad.items():
            setattr(cfg, k, v)
        assert lib.dc_create(ctypes.byref(cfg), ctypes.byref(h)) == L.DC_ERR_INVALID_ARG
    assert lib.dc_create(None, ctypes.byref(h)) == L.DC_ERR_INVALID_ARG


def test_null_context_is_an_error_not_a_crash():
    lib = L.load()
    assert lib.dc_set_frames(None, None, 0, 0, 1, None) == L.DC_ERR_INVALID_ARG
    assert lib.dc_build_and_lookup(None, None, None, 1, None, None, None) == L.DC_ERR_INVALID_ARG
    assert lib.dc_alt_lookup(None, None, None, 1, None, None, None) == L.DC_ERR_INVALID_ARG
    assert lib.dc_destroy(None) == L.DC_OK
    assert lib.dc_pool_2x2(None, None, 0, 4, 4, None) == L.DC_OK  # empty: nothing to do
    assert lib.dc_pool_2x2(None, None, 1, 4, 4, None) == L.DC_ERR_INVALID_ARG
    for order in (L.DC_ORDER_SOURCE, L.DC_ORDER_WINDOW_ROW, L.DC_ORDER_AUTO, 7):
        assert lib.dc_set_tile_order(None, order) == L.DC_ERR_INVALID_ARG
    assert lib.dc_context_bytes(None) == 0


def test_product_path_does_not_reference_the_oracle():
    pkg = os.path.dirname(L.LIB_PATH)
    pat = re.compile(r"import\s+oracle|from\s+oracle|liboracle|libref|oracle/")
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                assert not pat.search(open(os.path.join(root, f)).read()), f


def test_cudadroid_shim_header_compiles(tmp_path):
    # the C++ drop-in for CudaDroid's correlation methods builds against the C ABI
    src = tmp_path / "shim.cpp"
    src.write_text('#include "droidcorr_cudadroid.hpp"\nint main() { DroidCorrShim s; return 0; }\n')
    inc = os.path.dirname(HEADER)
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", inc,
                        "-I", "/usr/local/cuda/include", str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
