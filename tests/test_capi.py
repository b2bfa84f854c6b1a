"""The C ABI surface, without a GPU: the library loads, exports every function
include/sae_b200.h declares, and rejects bad arguments with status codes
before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest

HEADER = Path(__file__).resolve().parents[1] / "include" / "sae_b200.h"


def _declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sae_b200_\w+)\s*\(", text)))


def test_library_exports_every_declared_function():
    from sae_b200 import _lib as L
    lib = L.load()
    names = _declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
    # and the Python binding knows every one of them
    assert set(names) == set(L.exported_symbols())


def test_workspace_queries():
    from sae_b200 import _lib as L
    small = L.workspace_bytes(256, 128, 512, 1024)
    big = L.workspace_bytes(32768, 1536, 49152, 32768 * 512)
    assert 0 < small < big
    off = L.workspace_offsets(300, 128, 512, 1024)
    total = L.workspace_bytes(300, 128, 512, 1024)
    assert len(set(off.values())) == len(off)            # distinct regions
    assert all(v % 256 == 0 and v < total for v in off.values())
    for n in (1, 63, 64, 65, 32768):
        p = L.pre_pitch(n)
        assert p >= n and p % 64 == 0 and (p & (p - 1)) != 0


def test_bad_arguments_are_rejected_without_a_device():
    from sae_b200 import _lib as L
    lib = L.load()
    assert lib.sae_b200_version() >= 1
    rc = lib.sae_b200_train_forward(None, None, 0, None, None, 0, None, None, None, None)
    assert rc == L.SAE_ERR_INVALID_ARGUMENT
    assert b"model" in lib.sae_b200_last_error()
    m = L.Model(0, 10, 1, 1, 1, 1, 1, 1, 1)
    assert lib.sae_b200_grad_norm(ctypes.byref(m), None, 1.0, None, 0, None, None) != L.SAE_OK
    out = ctypes.c_size_t(0)
    assert lib.sae_b200_workspace_bytes(-1, 4, 4, 0, ctypes.byref(out)) == L.SAE_ERR_INVALID_ARGUMENT
    with pytest.raises(L.SaeB200Error) as e:
        L.call("sae_b200_gemm", 0, 4, 4, 1.0, None, 0, 1, 1, None, 0, 1, 1, 0.0, None, 0, 1, 1,
               None, None)
    assert e.value.code == L.SAE_ERR_INVALID_ARGUMENT
    cfg = L.StepConfig(16, 1024, 0.0, 0.0, 0.0, 0.0, 1, 0, 1, 0)   # ste_bandwidth 0 is invalid
    m = L.Model(64, 128, 16, 16, 16, 16, 16, 16, 16)
    rc = lib.sae_b200_train_forward(ctypes.byref(m), 16, 1, ctypes.byref(cfg), 256, 1 << 30, 16,
                                    None, None, None)
    assert rc == L.SAE_ERR_INVALID_ARGUMENT
    assert b"ste_bandwidth" in lib.sae_b200_last_error()


def test_full_pre_store_and_pre_flag_are_checked_without_a_device():
    """sae_b200_store_full_pre validates its model, config and workspace
    before any launch; the dense backward and the aux forward refuse a
    microbatch whose forward stored pre only at the entries."""
    from sae_b200 import _lib as L
    lib = L.load()
    assert lib.sae_b200_store_full_pre(None, None, None, 0, None) == L.SAE_ERR_INVALID_ARGUMENT
    m = L.Model(64, 128, 16, 16, 16, 16, 16, 16, 16)
    bad = L.StepConfig(16, 1024, 0.0, 0.0, 0.0, 0.0, 1, 0, 1, 0)          # ste_bandwidth 0
    assert lib.sae_b200_store_full_pre(ctypes.byref(m), ctypes.byref(bad), 256, 1 << 30,
                                       None) == L.SAE_ERR_INVALID_ARGUMENT
    entries = L.StepConfig(16, 1024, 0.0, 0.0, 0.0, 0.1, 1, 0, 1, 0, 0, 1)
    assert entries.pre_entries_only == 1
    m = L.Model(1536, 49152, 256, 256, 256, 256, 256, 256, 256)
    g = L.Grads(256, 256, 256, 256, 256)
    rc = lib.sae_b200_train_backward_dense(ctypes.byref(m), ctypes.byref(g), ctypes.byref(entries),
                                           256, 1 << 40, 256, 256, 1 << 40, None)
    assert rc == L.SAE_ERR_INVALID_ARGUMENT
    assert b"pre_entries_only" in lib.sae_b200_last_error()
    # a dense scratch below sae_b200_dense_scratch_bytes is refused before any launch
    full = L.StepConfig(16, 1024, 0.0, 0.0, 0.0, 0.1, 1, 0, 1, 0, 0, 0)
    need = L.dense_scratch_bytes(16, 1536, 49152)
    assert need >= 49152 * L.pre_pitch(16) * 2
    rc = lib.sae_b200_train_backward_dense(ctypes.byref(m), ctypes.byref(g), ctypes.byref(full),
                                           256, 1 << 40, 256, 256, 1024, None)
    assert rc == L.SAE_ERR_WORKSPACE_TOO_SMALL
    assert b"dense_scratch" in lib.sae_b200_last_error()


def test_norm_from_backward_partials_is_checked_without_a_device():
    """sae_b200_grad_norm_sampled validates its arguments before any launch:
    NULL gradients, a GEMM-backward config (whose backward writes no
    per-feature partials), a too-small norm workspace and a step workspace
    smaller than the backward's layout are refused."""
    from sae_b200 import _lib as L
    lib = L.load()
    m = L.Model(64, 128, 256, 256, 256, 256, 256, 256, 256)
    g = L.Grads(256, 256, 256, 256, 256)
    ok = L.StepConfig(16, 1024, 0.0, 0.0, 0.0, 0.1, 1, 0, 1, 0, 0, 1)
    gemm = L.StepConfig(16, 1024, 0.0, 0.0, 0.0, 0.1, 1, 0, 1, 0, 1, 0)
    norm_ws = L.GRAD_NORM_WORKSPACE_BYTES
    assert lib.sae_b200_grad_norm_sampled(ctypes.byref(m), None, ctypes.byref(ok), 256, 1 << 30,
                                          1.0, 256, norm_ws, 256, None) \
        == L.SAE_ERR_INVALID_ARGUMENT
    assert lib.sae_b200_grad_norm_sampled(ctypes.byref(m), ctypes.byref(g), ctypes.byref(gemm),
                                          256, 1 << 30, 1.0, 256, norm_ws, 256, None) \
        == L.SAE_ERR_INVALID_ARGUMENT
    assert b"grad_feat_gemm" in lib.sae_b200_last_error()
    assert lib.sae_b200_grad_norm_sampled(ctypes.byref(m), ctypes.byref(g), ctypes.byref(ok),
                                          256, 1 << 30, 1.0, 256, 4, 256, None) \
        == L.SAE_ERR_WORKSPACE_TOO_SMALL
    assert lib.sae_b200_grad_norm_sampled(ctypes.byref(m), ctypes.byref(g), ctypes.byref(ok),
                                          256, 64, 1.0, 256, norm_ws, 256, None) \
        == L.SAE_ERR_WORKSPACE_TOO_SMALL
