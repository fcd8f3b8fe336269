"""The C-ABI library loads, exports every symbol include/wattn.h declares,
and rejects bad arguments before touching a GPU (no compute calls here)."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "wattn.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(wattn_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def wattn():
    import wattn as W
    return W


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for must in ("wattn_attention_fwd", "wattn_decode_fwd", "wattn_kv_create", "wattn_kv_attend",
                 "wattn_flash_attention_2", "wattn_single_token_mha_d64",
                 "wattn_multi_head_attention_with_cache", "wattn_last_error"):
        assert must in syms


def test_library_exports_every_declared_symbol(wattn):
    out = subprocess.run(["nm", "-D", "--defined-only", wattn.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (wattn_[a-z0-9_]+)$", out, flags=re.M))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    # and the Python host module binds exactly the declared set
    assert sorted(wattn.EXPORTED_SYMBOLS) == declared_symbols()


def test_status_strings(wattn):
    assert wattn.status_string(0) == "ok"
    assert "unsupported" in wattn.status_string(-2)
    assert wattn.lib.wattn_version() >= 100


def test_reference_asserts_become_errors(wattn):
    # attention.rs:79-84: n_heads == 0 and d_model % n_heads != 0 are asserts;
    # here they are WATTN_ERR_INVALID, and d_head != 64 is WATTN_ERR_UNSUPPORTED.
    # All are rejected before any CUDA call.
    q = np.zeros(128 * 4, np.float32)
    o = np.zeros_like(q)
    with pytest.raises(wattn.WattnError) as e:
        wattn.flash_attention_2(q, q, q, 4, 4, 0, 128, False, o)
    assert e.value.status == -1
    with pytest.raises(wattn.WattnError) as e:
        wattn.flash_attention_2(q, q, q, 4, 4, 3, 128, False, o)
    assert e.value.status == -1
    qq = np.zeros(160 * 4, np.float32)
    with pytest.raises(wattn.WattnError) as e:
        wattn.flash_attention_2(qq, qq, qq, 4, 4, 2, 160, False, np.zeros_like(qq))
    assert e.value.status == -2
    with pytest.raises(wattn.WattnError) as e:  # length mismatch (attention.rs:85-88)
        wattn.flash_attention_2(q, q, q, 5, 4, 2, 128, False, o)
    assert e.value.status == -1
    # no-op shapes return before touching a device
    wattn.flash_attention_2(np.zeros(0, np.float32), q, q, 0, 4, 2, 128, False,
                            np.zeros(0, np.float32))


def test_device_entry_points_validate_first(wattn):
    L = wattn.lib
    # head dim 80 -> unsupported, before any pointer is touched
    rc = L.wattn_attention_fwd(None, None, None, None, 1, 1, 1, 4, 4, 2, 80, 160, 160, 160, 0, 0, 0,
                               0.125, 0, 0, None)
    assert rc == -2
    buf = ctypes.create_string_buffer(256)
    assert L.wattn_last_error(buf, 256) == -2 and b"head dimension" in buf.value
    # negative scale, bad dtype
    assert L.wattn_attention_fwd(None, None, None, None, 1, 1, 1, 4, 4, 2, 64, 128, 128, 128, 0, 0,
                                 0, -1.0, 0, 0, None) == -1
    assert L.wattn_decode_fwd(None, None, None, None, 7, 1, 1, 1, 1, 10, 2, 64, 128, 128, 0, 128,
                              0.125, None, 0, None) == -1
    # zero-size calls are valid no-ops
    assert L.wattn_attention_fwd(None, None, None, None, 1, 1, 0, 4, 4, 2, 64, 128, 128, 128, 0, 0,
                                 0, 0.125, 0, 0, None) == 0
    assert L.wattn_decode_workspace_bytes(32, 5, 1500, 20) > 0


def test_capture_selection_is_validated_first(wattn):
    # capture_cross_attention_heads (decoder.rs:796-828) selections that the
    # fused capture cannot serve are rejected before any CUDA call.
    q = np.zeros(2 * 128, np.float32)
    k = np.zeros(10 * 128, np.float32)
    out = np.zeros(2 * 2 * 10, np.float32)
    cases = [([(0, 1), (1, 1)], -2),   # one head in two slots
             ([(2, 0)], -6),           # slot outside n_selected
             ([(0, 5)], -6)]           # head outside n_heads
    for sel, status in cases:
        with pytest.raises(wattn.WattnError) as e:
            wattn.capture_cross_attention_heads(q, k, 2, 10, 2, 128, sel, 2, 0, out)
        assert e.value.status == status, sel
    # d_model != n_heads * 64
    with pytest.raises(wattn.WattnError) as e:
        wattn.capture_cross_attention_heads(q, k, 2, 10, 4, 128, [(0, 0)], 2, 0, out)
    assert e.value.status in (-1, -2)
    assert (out == 0).all()



def test_misaligned_pointers_are_argument_errors(wattn):
    # Kernels that read or write elements one at a time need pointers aligned
    # to the element size; a caller's misaligned pointer must come back as
    # WATTN_ERR_INVALID from the host-side checks, never reach a launch.
    # The addresses below are made up and never dereferenced; on a machine
    # with a GPU this test stands aside (a check that let one through would
    # hand the address to a kernel there).
    import torch
    if torch.cuda.is_available():
        pytest.skip("made-up device addresses are only passed where no GPU can run them")
    L = wattn.lib
    buf = ctypes.create_string_buffer(256)
    base = 1 << 20  # 16-byte aligned
    F32, F16 = wattn.F32, wattn.F16

    def last():
        L.wattn_last_error(buf, 256)
        return buf.value

    # decode: f32 q, then the f32 output, one byte off
    rc = L.wattn_decode_fwd(base + 1, base, base, base, F32, F16, F32, 1, 1, 10, 2, 64, 128, 128,
                            1280, 128, 0.125, None, 0, None)
    assert rc == -1 and b"aligned" in last()
    rc = L.wattn_decode_fwd(base, base, base, base + 2, F16, F16, F32, 1, 1, 10, 2, 64, 128, 128,
                            1280, 128, 0.125, None, 0, None)
    assert rc == -1 and b"aligned" in last()
    rc = L.wattn_decode_fwd_noalloc(base, base, base, base + 1, F16, F16, F16, 1, 1, 10, 2, 64,
                                    128, 128, 1280, 128, 0.125, None)
    assert rc == -1 and b"aligned" in last()
    # linear: the output, then the bias
    rc = L.wattn_linear_fwd(base, base, None, base + 2, F16, F32, 4, 8, 64, 64, 64, 8, None)
    assert rc == -1 and b"aligned" in last()
    rc = L.wattn_linear_fwd(base, base, ctypes.cast(base + 2, wattn._fp), base, F16, F32, 4, 8, 64,
                            64, 64, 8, None)
    assert rc == -1 and b"aligned" in last()
    # cross K/V projection: the value bias
    rc = L.wattn_cross_kv_project(base, base, base, ctypes.cast(base + 1, wattn._fp), base, base,
                                  F16, F16, 4, 64, 64, 64, None)
    assert rc == -1 and b"aligned" in last()
    # encoder block with the residual: the f32 residual stream
    ws = base << 4
    rc = L.wattn_encoder_attention_residual(ctypes.cast(base + 2, wattn._fp),
                                            ctypes.cast(base, wattn._fp),
                                            ctypes.cast(base, wattn._fp), base,
                                            ctypes.cast(base, wattn._fp), base,
                                            ctypes.cast(base, wattn._fp), F16, 1, 4, 1, ws,
                                            1 << 30, None)
    assert rc == -1 and b"aligned" in last()
