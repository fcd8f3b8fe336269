"""ctypes front end of the CPU oracle (``liboracle.so``).

TEST INFRASTRUCTURE ONLY. This module is the parity checker for the CUDA
path and the timed CPU baseline of ``bench.py``; only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` leg and
reference arm may import it. The product path never does.

Each wrapper takes numpy f32 arrays in the reference's row-major layout
(``[t, n_heads * d_head]``, head ``h`` at columns ``h*d_head..``) and mirrors
the reference function named in its docstring.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_sz = ctypes.c_size_t


def build(force: bool = False) -> str:
    """Compile liboracle.so with the Makefile beside this file."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH)
        < max(os.path.getmtime(os.path.join(_HERE, f)) for f in ("wattn_oracle.c", "wattn_oracle.h"))
    ):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "liboracle.so"],
                       check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.ora_flash_attention_2.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz,
                                            ctypes.c_int, _f32p, ctypes.c_int]
        L.ora_flash_attention_2_batched.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz,
                                                    ctypes.c_int, _f32p, ctypes.c_int]
        L.ora_single_token_mha_d64.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _f32p]
        L.ora_single_token_mha_d64_scalar.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _f32p]
        L.ora_mha_with_cache.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, _f32p]
        L.ora_linear.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _f32p, ctypes.c_int]
        L.ora_layer_norm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_float, _sz, _sz, _f32p]
        _i32p = ctypes.POINTER(ctypes.c_int)
        L.ora_capture_heads.argtypes = [_f32p, _f32p, _sz, _sz, _sz, _sz, _i32p, _i32p, _sz, _sz,
                                        _sz, _f32p]
        L.ora_materialized.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, ctypes.c_int, _f32p]
        L.ora_decode_grouped.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, _f32p,
                                         ctypes.c_int]
        L.ora_softmax_inplace.argtypes = [_f32p, _sz]
        L.ora_xorshift_fill.argtypes = [ctypes.POINTER(ctypes.c_uint32), _f32p, _sz]
        for name in ("ora_flash_attention_2", "ora_flash_attention_2_batched",
                     "ora_single_token_mha_d64", "ora_single_token_mha_d64_scalar",
                     "ora_mha_with_cache", "ora_materialized", "ora_decode_grouped"):
            getattr(L, name).restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], "oracle wants C-contiguous f32"
    return a.ctypes.data_as(_f32p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _check(rc: int, what: str):
    if rc != 0:
        raise ValueError(f"{what}: invalid arguments (the reference asserts here)")


def flash_attention_2(q, k, v, t_q, t_kv, n_heads, d_model, causal, n_threads=0):
    """crates/tensor/src/ops/attention.rs:68-242 -> new [t_q, d_model] f32 array."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(t_q * d_model, np.float32)
    _check(lib().ora_flash_attention_2(_p(q), _p(k), _p(v), t_q, t_kv, n_heads, d_model,
                                       int(bool(causal)), _p(out), n_threads), "flash_attention_2")
    return out


def flash_attention_2_batched(q, k, v, batch, t_q, t_kv, n_heads, d_model, causal, n_threads=0):
    """`batch` independent attention.rs:68 calls on [batch, t, d_model] buffers."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(batch * t_q * d_model, np.float32)
    _check(lib().ora_flash_attention_2_batched(_p(q), _p(k), _p(v), batch, t_q, t_kv, n_heads,
                                               d_model, int(bool(causal)), _p(out), n_threads),
           "flash_attention_2_batched")
    return out


def single_token_mha_d64(q, k, v, t_kv, n_heads, d_model, scalar=False):
    """crates/tensor/src/ops/attention.rs:246-434 (AVX2 order, or the scalar twin)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(d_model, np.float32)
    fn = lib().ora_single_token_mha_d64_scalar if scalar else lib().ora_single_token_mha_d64
    _check(fn(_p(q), _p(k), _p(v), t_kv, n_heads, d_model, _p(out)), "single_token_mha_d64")
    return out


def layer_norm(x, gamma, beta, rows, d, eps=1e-5):
    """crates/tensor/src/ops/norm.rs:116-142."""
    x, g, b = _f32(x), _f32(gamma), _f32(beta)
    y = np.empty(rows * d, np.float32)
    _check(lib().ora_layer_norm(_p(x), _p(g), _p(b), eps, rows, d, _p(y)), "layer_norm")
    return y


def linear(x, w, bias, m, n, k, n_threads=None):
    """crates/tensor/src/ops/matmul.rs:4-110: y = x W^T (+ bias), f32."""
    x, w = _f32(x), _f32(w)
    b = _f32(bias) if bias is not None else None
    y = np.empty(m * n, np.float32)
    _check(lib().ora_linear(_p(x), _p(w), _p(b) if b is not None else None, m, n, k, _p(y),
                            n_threads or os.cpu_count() or 1), "linear")
    return y


def capture_heads(q, k, n_tokens, n_audio, n_heads, d_model, selected, n_selected, row_offset,
                  out):
    """crates/whisper/src/decoder.rs:796-828 (capture_cross_attention_heads):
    writes the selected heads' softmax rows into ``out`` (f32, modified in
    place) at [(row_offset + t) * n_selected + slot][n_audio]."""
    q, k = _f32(q), _f32(k)
    assert out.dtype == np.float32 and out.flags.c_contiguous
    slots = (ctypes.c_int * max(1, len(selected)))(*[int(a) for a, _ in selected])
    heads = (ctypes.c_int * max(1, len(selected)))(*[int(b) for _, b in selected])
    _check(lib().ora_capture_heads(_p(q), _p(k), n_tokens, n_audio, n_heads, d_model, slots,
                                   heads, len(selected), n_selected, row_offset, _p(out)),
           "capture_cross_attention_heads")
    return out


def mha_with_cache(q, k, v, n_tokens, total_tokens, t_past, n_heads, d_model):
    """crates/whisper/src/decoder.rs:835-892 (causal attention over a slot's cache)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(n_tokens * d_model, np.float32)
    _check(lib().ora_mha_with_cache(_p(q), _p(k), _p(v), n_tokens, total_tokens, t_past,
                                    n_heads, d_model, _p(out)), "multi_head_attention_with_cache")
    return out


def materialized(q, k, v, t_q, t_kv, n_heads, d_model, causal):
    """crates/tensor/tests/test_flash_attention_tiled.rs:41-89 (the tests' reference)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(t_q * d_model, np.float32)
    _check(lib().ora_materialized(_p(q), _p(k), _p(v), t_q, t_kv, n_heads, d_model,
                                  int(bool(causal)), _p(out)), "reference_materialized")
    return out


def decode_grouped(q, k, v, n_groups, group_size, t_kv, n_heads, d_model, n_threads=0):
    """One single_token_mha_d64 per query row; rows of a group share K/V
    (cross-attention of the beams of one utterance, decoder.rs:688-724)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(n_groups * group_size * d_model, np.float32)
    _check(lib().ora_decode_grouped(_p(q), _p(k), _p(v), n_groups, group_size, t_kv, n_heads,
                                    d_model, _p(out), n_threads), "decode_grouped")
    return out


def softmax_inplace(x: np.ndarray) -> np.ndarray:
    """crates/tensor/src/ops/softmax.rs:1-24."""
    x = _f32(x).copy()
    lib().ora_softmax_inplace(_p(x), x.size)
    return x


class XorShift:
    """crates/tensor/tests/test_flash_attention_tiled.rs:15-35."""

    def __init__(self, seed: int):
        self.state = ctypes.c_uint32(seed & 0xFFFFFFFF)

    def fill(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().ora_xorshift_fill(ctypes.byref(self.state), _p(out), n)
        return out


def kat_inputs(t_q: int, t_kv: int, n_heads: int, d_head: int):
    """Inputs of max_abs_error() in test_flash_attention_tiled.rs:93-98: seed
    0x1234_5678 ^ (t_q << 16) ^ t_kv, then q, k, v filled in that order."""
    d_model = n_heads * d_head
    rng = XorShift(0x12345678 ^ ((t_q << 16) & 0xFFFFFFFF) ^ t_kv)
    q = rng.fill(t_q * d_model)
    k = rng.fill(t_kv * d_model)
    v = rng.fill(t_kv * d_model)
    return q, k, v


def xorshift_f32_numpy(seed: int, n: int) -> np.ndarray:
    """Pure-numpy twin of XorShift.fill, used to check the C generator."""
    x = np.uint32(seed)
    out = np.empty(n, np.float32)
    denom = np.float32(4294967295.0)
    with np.errstate(over="ignore"):
        for i in range(n):
            x ^= np.uint32((int(x) << 13) & 0xFFFFFFFF)
            x ^= np.uint32(int(x) >> 17)
            x ^= np.uint32((int(x) << 5) & 0xFFFFFFFF)
            out[i] = (np.float32(x) / denom) * np.float32(2.0) - np.float32(1.0)
    return out
