"""The C-ABI library loads without a GPU and exports every function include/mkb_image.h declares; calls that need a
device fail with an error code rather than crashing. CPU only."""

import ctypes
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "include", "mkb_image.h")
LIB = os.path.join(ROOT, "mako-image_b200", "lib", "libmkb_image.so")


def _declared():
    text = open(HDR).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mkb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = _declared()
    for n in ("mkb_dit_create", "mkb_dit_begin", "mkb_dit_step", "mkb_dit_step_cfg", "mkb_proj", "mkb_attention",
              "mkb_sigmas", "mkb_er_sde_step", "mkb_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB), "build the library first (make -C mako-image_b200)"
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (mkb_[a-z0-9_]+)", out))
    missing = [n for n in _declared() if n not in exported]
    assert not missing, missing
    lib = ctypes.CDLL(LIB)
    for n in _declared():
        assert getattr(lib, n, None) is not None


def test_errors_are_codes_not_crashes():
    import sys

    sys.path.insert(0, os.path.join(ROOT, "mako-image_b200"))
    import mkimage

    # invalid arguments are rejected before any device work
    assert mkimage.lib.mkb_sigmas(None, 0, 10, None) != 0
    assert mkimage.lib.mkb_dit_create(None, None) != 0
    assert "null" in mkimage.lib.mkb_last_error().decode()
    assert mkimage.lib.mkb_er_sde_create(None, 1, 0, 0.0, None) != 0
