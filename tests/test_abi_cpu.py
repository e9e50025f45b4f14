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


def test_nccl_binding_takes_every_entry_point(tmp_path):
    """The run-time NCCL binding (the sequence-parallel exchanges' all-gather, send / receive and group calls) binds
    all nine entry points from the library MKB_NCCL_LIB names: with the stand-in the failure tests use, making a
    communicator id succeeds, and a library lacking one of them is refused with a message. No GPU involved."""
    so = tmp_path / "libfake_nccl.so"
    src = os.path.join(ROOT, "tests", "fake_nccl", "fake_nccl.c")
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(so), src], check=True)
    short = tmp_path / "libshort_nccl.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-DFAKE_NCCL_NO_P2P", "-o", str(short), src], check=True)
    code = ("import ctypes, sys; sys.path.insert(0, {pkg!r}); import mkimage; "
            "buf = ctypes.create_string_buffer(128); "
            "r = mkimage.lib.mkb_nccl_unique_id(buf, 128); print(r, mkimage.lib.mkb_last_error().decode())")
    code = code.format(pkg=os.path.join(ROOT, "mako-image_b200"))
    for lib, want in ((so, "0 "), (short, "2 ")):  # MKB_OK, MKB_ERR_CUDA
        r = subprocess.run(["python", "-c", code], env=dict(os.environ, MKB_NCCL_LIB=str(lib)), capture_output=True,
                           text=True, timeout=120)
        assert r.returncode == 0, r.stderr
        assert r.stdout.startswith(want), r.stdout
        if want == "2 ":
            assert "lacks an expected symbol" in r.stdout, r.stdout
