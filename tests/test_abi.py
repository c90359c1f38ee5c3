"""The C-ABI library loads, exports every entry point include/ngdn2.h
declares, and validates arguments the reference's way -- all host-side, no
kernel launches, so these run without a GPU."""

import ctypes
import pathlib
import re

import pytest

from nested_recurrent_memory_b200 import _lib

HEADER = pathlib.Path(__file__).resolve().parents[1] / "include" / "ngdn2.h"


def declared_functions():
    text = HEADER.read_text()
    return re.findall(r"NGDN2_API\s+[\w\s\*]+?\b(ngdn2_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_header_declares_the_entry_points():
    names = set(declared_functions())
    assert {"ngdn2_fwd", "ngdn2_update_state", "ngdn2_fwd_workspace_size"} <= names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) == set(_lib.EXPORTS)


def test_struct_layouts_match(lib):
    _lib.check_layout(lib)


def _fake_fwd(**over):
    """Arguments with non-null dummy pointers: only host validation runs."""
    a = _lib.FwdArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.T, a.H, a.K, a.V, a.L = 2, 256, 2, 64, 64, 3
    a.chunk_size = 64
    a.promotion = 0
    a.scale = 0.125
    a.n_max = 16
    for i in range(2):
        a.n_queries[i] = 16
    for i, f in enumerate((1, 2, 4)):
        a.firing[i] = f
    for name in ("q", "k", "v", "g", "b", "w", "mix", "query_banks", "key_projections",
                 "b_projections", "w_projections", "g_projections", "o", "final_state"):
        setattr(a, name, 0x1000)
    for k, v in over.items():
        if k in ("n_queries", "firing"):
            arr = getattr(a, k)
            for i, x in enumerate(v):
                arr[i] = x
        else:
            setattr(a, k, v)
    return a


def _ws(lib, a):
    n = ctypes.c_size_t(0)
    return lib.ngdn2_fwd_workspace_size(ctypes.byref(a), ctypes.byref(n)), n.value


def test_workspace_size_is_positive(lib):
    rc, n = _ws(lib, _fake_fwd())
    assert rc == 0 and n > 0


@pytest.mark.parametrize(("over", "code"), [
    (dict(chunk_size=32), _lib.ERR_CHUNK_SIZE),
    (dict(n_queries=(24, 16)), _lib.ERR_N_POW2),
    (dict(n_queries=(8, 16)), _lib.ERR_N_POW2),
    (dict(K=48, promotion=1), _lib.ERR_N_POW2),
    (dict(q=None), -9),
    (dict(abi_version=99), -13),
    (dict(firing=(1, 0, 4)), -14),
    (dict(K=200), -7),
    (dict(dtype=7), -8),
    (dict(gate=0x2000), -9),  # a start gate needs a status word to report into
])
def test_fwd_validation_codes(lib, over, code):
    rc, _ = _ws(lib, _fake_fwd(**over))
    assert rc == code
    assert lib.ngdn2_fwd(ctypes.byref(_fake_fwd(**over)), None) == code


def test_fwd_rejects_missing_workspace(lib):
    a = _fake_fwd()
    assert lib.ngdn2_fwd(ctypes.byref(a), None) == -10


def test_gate_adds_one_launch(lib):
    plain = lib.ngdn2_fwd_num_launches(ctypes.byref(_fake_fwd()))
    gated = lib.ngdn2_fwd_num_launches(ctypes.byref(_fake_fwd(gate=0x2000, status=0x3000)))
    assert plain > 0 and gated == plain + 1


def _fake_bwd(**over):
    a = _lib.BwdArgs()
    a.abi_version = _lib.ABI_VERSION
    fa = _fake_fwd(**{k: v for k, v in over.items() if k in _lib.FwdArgs.__dict__})
    fa.o = None
    fa.final_state = None   # not used by the backward
    a.fwd = fa
    for name in ("d_o", "dq", "dk", "dv", "dg", "db", "dw", "dmix"):
        setattr(a, name, 0x1000)
    for k, v in over.items():
        if k not in _lib.FwdArgs.__dict__:
            setattr(a, k, v)
    return a


def test_bwd_workspace_size_is_positive(lib):
    n = ctypes.c_size_t(0)
    assert lib.ngdn2_bwd_workspace_size(ctypes.byref(_fake_bwd()), ctypes.byref(n)) == 0
    assert n.value > 0
    assert lib.ngdn2_bwd_num_launches(ctypes.byref(_fake_bwd())) == 6


@pytest.mark.parametrize(("over", "code"), [
    (dict(chunk_size=32), _lib.ERR_CHUNK_SIZE),
    (dict(n_queries=(24, 16)), _lib.ERR_N_POW2),
    (dict(d_o=None), -9),
    (dict(dmix=None), -9),
    (dict(d_o_dtype=5), -8),
    (dict(abi_version=99), -13),
])
def test_bwd_validation_codes(lib, over, code):
    n = ctypes.c_size_t(0)
    a = _fake_bwd(**over)
    assert lib.ngdn2_bwd_workspace_size(ctypes.byref(a), ctypes.byref(n)) == code
    assert lib.ngdn2_bwd(ctypes.byref(a), None) == code


def test_bwd_rejects_missing_workspace(lib):
    assert lib.ngdn2_bwd(ctypes.byref(_fake_bwd()), None) == -10


def _fake_update(**over):
    u = _lib.UpdateArgs()
    u.abi_version = _lib.ABI_VERSION
    u.B, u.NF, u.NG, u.H, u.K, u.V, u.N = 1, 4, 4, 1, 16, 32, 16
    u.block_v = 16
    for i, s in enumerate((4 * 16 * 16, 16 * 16, 16 * 16, 16, 1)):
        u.keys_stride[i] = s
    for name in ("keys", "values", "g", "b", "w", "states", "final_state"):
        setattr(u, name, 0x1000)
    for k, v in over.items():
        if k == "k_stride":
            u.keys_stride[4] = v
        else:
            setattr(u, k, v)
    return u


@pytest.mark.parametrize(("over", "code"), [
    (dict(N=8), _lib.ERR_N_POW2),
    (dict(block_v=8), _lib.ERR_BLOCK_V),
    (dict(V=24), _lib.ERR_DIVISIBLE),
    (dict(k_stride=2), _lib.ERR_UNIT_STRIDE),
    (dict(NG=9), _lib.ERR_INCONSISTENT),
])
def test_update_validation_codes_follow_the_reference_order(lib, over, code):
    assert lib.ngdn2_update_state(ctypes.byref(_fake_update(**over)), None) == code


def test_error_strings(lib):
    assert _lib.error_string(_lib.ERR_CHUNK_SIZE) == "chunk_size must be 64"
    assert "unit-stride" in _lib.error_string(_lib.ERR_UNIT_STRIDE)


def _fake_step(**over):
    a = _lib.StepArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.H, a.K, a.V, a.L = 2, 2, 64, 64, 3
    a.chunk_size = 64
    a.scale = 0.125
    a.n_max = 16
    for i in range(2):
        a.n_queries[i] = 16
    for i, f in enumerate((1, 2, 4)):
        a.firing[i] = f
    for name in ("q", "k", "v", "g", "b", "w", "mix", "query_banks", "key_projections",
                 "b_projections", "w_projections", "g_projections", "state_in", "state_out", "o"):
        setattr(a, name, 0x1000)
    for k, v in over.items():
        if k == "n_queries":
            for i, x in enumerate(v):
                a.n_queries[i] = x
        else:
            setattr(a, k, v)
    return a


@pytest.mark.parametrize(("over", "code"), [
    (dict(n_queries=(24, 16)), _lib.ERR_N_POW2),
    (dict(state_out=None), -9),
    (dict(chunk_size=0), -7),
    (dict(abi_version=5), -13),
])
def test_step_validation_codes(lib, over, code):
    n = ctypes.c_size_t(0)
    assert lib.ngdn2_step_workspace_size(ctypes.byref(_fake_step(**over)), ctypes.byref(n)) == code
    assert lib.ngdn2_step(ctypes.byref(_fake_step(**over)), None) == code


def test_step_needs_its_workspace_for_promotions(lib):
    n = ctypes.c_size_t(0)
    assert lib.ngdn2_step_workspace_size(ctypes.byref(_fake_step()), ctypes.byref(n)) == 0
    assert n.value > 0
    assert lib.ngdn2_step(ctypes.byref(_fake_step()), None) == -10
    one = _fake_step(L=1)
    assert lib.ngdn2_step_workspace_size(ctypes.byref(one), ctypes.byref(n)) == 0 and n.value == 0
