"""The C-ABI library loads and exports every symbol include/wfd_b200.h declares
(no compute calls: these run without a GPU)."""
from __future__ import annotations

import ctypes
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "wfd_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(wfd_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    import __graft_entry__
    __graft_entry__.build()
    from wavefront_decoding_b200 import _abi
    return _abi.load()


def test_header_declares_entry_points():
    names = declared_functions()
    assert "wfd_wave_attn" in names and "wfd_commit_window" in names and "wfd_append" in names


def test_every_declared_symbol_exported(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in wfd_b200.h but not exported"


def test_python_binding_covers_header(lib):
    from wavefront_decoding_b200 import _abi
    assert set(_abi.EXPORTED) == set(declared_functions())


def test_abi_version_and_status_strings(lib):
    assert lib.wfd_abi_version() == 6
    assert lib.wfd_status_string(0) == b"ok"
    assert b"workspace" in lib.wfd_status_string(3)


def test_item_struct_layout(lib):
    from wavefront_decoding_b200 import _abi
    assert ctypes.sizeof(_abi.wfd_item) == 20
    # the ctypes mirror of the scheduler parameters matches the compiled struct
    assert ctypes.sizeof(_abi.wfd_sched_params) == lib.wfd_sched_params_bytes()
    assert ctypes.sizeof(_abi.wfd_linear_params) == lib.wfd_linear_params_bytes()


def test_product_does_not_import_oracle():
    pkg = ROOT / "wavefront-decoding_b200"
    for p in pkg.rglob("*.py"):
        src = p.read_text()
        assert "oracle" not in re.findall(r"^\s*(?:from|import)\s+(\w+)", src, flags=re.M), p


def test_linear_rejects_bad_arguments_on_the_host(lib):
    """wfd_linear's argument checks run before any device work: bad shapes, modes and
    missing pointers come back as WFD_ERR_INVALID_ARG (no GPU needed), and an empty
    call is a no-op."""
    from wavefront_decoding_b200 import _abi

    def call(**kw):
        p = _abi.wfd_linear_params()
        p.x, p.w, p.out, p.err = 16, 32, 48, 64   # never dereferenced: the checks below fail first
        p.n_rows, p.K, p.F, p.ldx, p.ldo = 4, 256, 256, 256, 256
        p.mode = _abi.WFD_LINEAR_PLAIN
        for k, v in kw.items():
            setattr(p, k, v)
        return lib.wfd_linear(ctypes.byref(p), None)

    INVALID = 1
    assert lib.wfd_linear(None, None) == INVALID
    assert call(n_rows=-1) == INVALID
    assert call(K=100) == INVALID                 # K % 8
    assert call(F=0) == INVALID
    assert call(ldx=128) == INVALID               # ldx < K
    assert call(mode=7) == INVALID
    assert call(n_rows=0) == 0                    # nothing to do
    assert call(x=None) == INVALID
    assert call(mode=_abi.WFD_LINEAR_ROPE, Dh=64, H=0, Hkv=1) == INVALID
    assert call(mode=_abi.WFD_LINEAR_ROPE, Dh=64, H=1, Hkv=1, F=256, q=16, k=16, v=16,
                cos_tab=16, sin_tab=16, max_pos=8, pos_period=0) == INVALID   # neither pos nor a period
    assert call(mode=_abi.WFD_LINEAR_SWIGLU, F=192, ldo=96) == INVALID          # F % 128
