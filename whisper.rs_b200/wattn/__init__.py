"""Python host side of the B200 attention path (ctypes over libwattn.so).

Mirrors the reference interface of whisper.rs's attention hot path:

* ``flash_attention_2`` / ``multi_head_attention`` -- crates/tensor/src/ops/attention.rs:68 / :29
* ``single_token_mha_d64``                          -- attention.rs:246
* ``multi_head_attention_with_cache``               -- crates/whisper/src/decoder.rs:835
* ``DeviceKvCache``                                 -- DecoderKvCache, decoder.rs:131-264

The four reference-signature functions take host f32 arrays (numpy) in the
reference layout ``[t, n_heads*64]`` and write ``output`` in place, as the
Rust functions do; argument errors raise ``WattnError`` where the reference
panics. ``attention_fwd`` / ``decode_fwd`` and ``DeviceKvCache`` work on CUDA
tensors (torch) on the caller's current stream.

There is no fallback: if libwattn.so is missing or fails to load, importing
this module raises.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

__all__ = [
    "F32", "F16", "BF16", "WattnError", "lib", "LIB_PATH", "status_string",
    "flash_attention_2", "multi_head_attention", "single_token_mha_d64",
    "multi_head_attention_with_cache", "attention_host", "decode_host",
    "attention_fwd", "decode_fwd", "decode_fwd_noalloc", "decode_workspace_bytes", "DeviceKvCache",
    "device_status", "selftest_bounded_wait", "EXPORTED_SYMBOLS",
]

F32, F16, BF16 = 0, 1, 2
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_NOMEM, ERR_RANGE = 0, -1, -2, -3, -4, -5, -6

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libwattn.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `python whisper.rs_b200/build.py` "
        "(there is no CPU fallback)")

lib = ctypes.CDLL(LIB_PATH)

_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
_f = ctypes.c_float
_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int)

# name -> (restype, argtypes); every symbol declared in include/wattn.h.
_SIGS = {
    "wattn_version": (_i, []),
    "wattn_status_string": (ctypes.c_char_p, [_i]),
    "wattn_last_error": (_i, [ctypes.c_char_p, _sz]),
    "wattn_device_status": (_i, [_i, _ip]),
    "wattn_attention_fwd": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i,
                                 _i64, _i64, _i64, _i64, _i64, _i64, _f, _i, _i, _vp]),
    "wattn_decode_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "wattn_decode_fwd": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i,
                              _i64, _i64, _i64, _i64, _f, _vp, _sz, _vp]),
    "wattn_decode_fwd_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i,
                                      _i64, _i64, _i64, _i64, _f, _vp]),
    "wattn_decode_fwd_capture": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i,
                                      _i64, _i64, _i64, _i64, _f, _vp, _sz, _ip, _ip, _i, _i, _i,
                                      _vp, _vp]),
    "wattn_linear_fwd": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i64, _i64, _i64, _vp]),
    "wattn_cross_kv_project": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i64, _i64,
                                    _vp]),
    "wattn_encoder_attention_workspace_bytes": (_sz, [_i, _i, _i]),
    "wattn_encoder_attention": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz,
                                     _vp]),
    "wattn_encoder_attention_residual": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i,
                                              _vp, _sz, _vp]),
    "wattn_kv_create": (_i, [ctypes.POINTER(_vp), _i, _i, _i, _i, _i, _i, _i, _i]),
    "wattn_kv_destroy": (_i, [_vp]),
    "wattn_kv_clear": (_i, [_vp]),
    "wattn_kv_clear_slot": (_i, [_vp, _i]),
    "wattn_kv_ensure_slots": (_i, [_vp, _i]),
    "wattn_kv_copy_slot": (_i, [_vp, _i, _i, _vp]),
    "wattn_kv_assign_beams": (_i, [_vp, _ip, _i, _ip]),
    "wattn_kv_slot_len": (_i, [_vp, _i, _ip]),
    "wattn_kv_slide_to_fit": (_i, [_vp, _i, _i, _i, _ip]),
    "wattn_kv_set_t_past": (_i, [_vp, _i, _i]),
    "wattn_kv_advance": (_i, [_vp, _ip, _ip, _i]),
    "wattn_kv_append": (_i, [_vp, _i, _ip, _ip, _i, _vp, _vp, _i, _i64, _vp]),
    "wattn_kv_workspace_bytes": (_sz, [_vp, _i]),
    "wattn_kv_attend": (_i, [_vp, _i, _ip, _ip, _i, _vp, _i, _i64, _vp, _i, _i64, _f, _vp, _sz,
                             _vp]),
    "wattn_kv_read_slot": (_i, [_vp, _i, _i, _i, _vp, _i, _vp]),
    "wattn_kv_stats": (_i, [_vp, _ip, _ip]),
    "wattn_flash_attention_2": (_i, [_fp, _fp, _fp, _sz, _sz, _sz, _sz, _i, _fp]),
    "wattn_multi_head_attention": (_i, [_fp, _fp, _fp, _sz, _sz, _sz, _sz, _i, _fp]),
    "wattn_single_token_mha_d64": (_i, [_fp, _fp, _fp, _sz, _sz, _sz, _fp]),
    "wattn_multi_head_attention_with_cache": (_i, [_fp, _fp, _fp, _sz, _sz, _sz, _sz, _sz, _fp]),
    "wattn_capture_cross_attention_heads": (_i, [_fp, _fp, _sz, _sz, _sz, _sz, _ip, _ip, _sz, _sz,
                                                 _sz, _fp]),
    "wattn_attention_host": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i]),
    "wattn_decode_host": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f]),
    "wattn_selftest_bounded_wait": (_i, [_i, _vp]),
}
EXPORTED_SYMBOLS = tuple(_SIGS)

for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class WattnError(RuntimeError):
    """A non-zero status from libwattn; ``.status`` holds the code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


def status_string(status: int) -> str:
    return lib.wattn_status_string(status).decode()


def _check(rc: int, what: str) -> None:
    if rc != OK:
        buf = ctypes.create_string_buffer(512)
        lib.wattn_last_error(buf, 512)
        raise WattnError(rc, f"{what}: {status_string(rc)}: {buf.value.decode(errors='replace')}")


# ---------------------------------------------------------------- host mirrors

def _f32_host(a, name: str) -> np.ndarray:
    if not isinstance(a, np.ndarray) or a.dtype != np.float32 or not a.flags["C_CONTIGUOUS"]:
        raise TypeError(f"{name} must be a C-contiguous float32 numpy array")
    return a


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(_fp)


def _expect_len(a: np.ndarray, n: int, name: str):
    # attention.rs:85-88 assert_eq!(q.len(), t_q * d_model) and friends
    if a.size != n:
        raise WattnError(ERR_INVALID, f"{name}.len() = {a.size}, expected {n}")


def flash_attention_2(q, k, v, t_q, t_kv, n_heads, d_model, causal, output) -> None:
    """attention.rs:68 ``flash_attention_2(q, k, v, t_q, t_kv, n_heads, d_model, causal, output)``.

    Host f32 slices in the reference layout; ``output`` is overwritten."""
    q, k, v, output = (_f32_host(x, n) for x, n in ((q, "q"), (k, "k"), (v, "v"), (output, "output")))
    if n_heads == 0 or d_model % n_heads:
        _check(lib.wattn_flash_attention_2(None, None, None, t_q, t_kv, n_heads, d_model,
                                           int(bool(causal)), None), "flash_attention_2")
    for a, n, nm in ((q, t_q * d_model, "q"), (k, t_kv * d_model, "k"), (v, t_kv * d_model, "v"),
                     (output, t_q * d_model, "output")):
        _expect_len(a, n, nm)
    _check(lib.wattn_flash_attention_2(_fptr(q), _fptr(k), _fptr(v), t_q, t_kv, n_heads, d_model,
                                       int(bool(causal)), _fptr(output)), "flash_attention_2")


def multi_head_attention(q, k, v, t_q, t_kv, n_heads, d_model, causal, output) -> None:
    """attention.rs:29 -- same as flash_attention_2."""
    flash_attention_2(q, k, v, t_q, t_kv, n_heads, d_model, causal, output)


def single_token_mha_d64(q, k, v, t_kv, n_heads, d_model, output) -> None:
    """attention.rs:246 ``single_token_mha_d64(q, k, v, t_kv, n_heads, d_model, output)``."""
    q, k, v, output = (_f32_host(x, n) for x, n in ((q, "q"), (k, "k"), (v, "v"), (output, "output")))
    _expect_len(q, d_model, "q")
    _expect_len(output, d_model, "output")
    if k.size < t_kv * d_model or v.size < t_kv * d_model:
        raise WattnError(ERR_INVALID, "k / v shorter than t_kv * d_model")
    _check(lib.wattn_single_token_mha_d64(_fptr(q), _fptr(k), _fptr(v), t_kv, n_heads, d_model,
                                          _fptr(output)), "single_token_mha_d64")


def multi_head_attention_with_cache(q, k, v, n_tokens, total_tokens, t_past, n_heads, d_model,
                                    output) -> None:
    """decoder.rs:835 ``multi_head_attention_with_cache``: causal attention of n_tokens
    queries at positions t_past.. over the slot's total_tokens cached rows."""
    q, k, v, output = (_f32_host(x, n) for x, n in ((q, "q"), (k, "k"), (v, "v"), (output, "output")))
    _expect_len(q, n_tokens * d_model, "q")
    _expect_len(k, total_tokens * d_model, "k")
    _expect_len(v, total_tokens * d_model, "v")
    _expect_len(output, n_tokens * d_model, "output")
    _check(lib.wattn_multi_head_attention_with_cache(_fptr(q), _fptr(k), _fptr(v), n_tokens,
                                                     total_tokens, t_past, n_heads, d_model,
                                                     _fptr(output)),
           "multi_head_attention_with_cache")


def capture_cross_attention_heads(q, k, n_tokens, n_audio, n_heads, d_model, selected,
                                  n_selected, row_offset, out) -> None:
    """decoder.rs:796 ``capture_cross_attention_heads``: for each (slot, head)
    in ``selected`` and token row t, out[row_offset + t][slot][:] = the
    softmax over the n_audio keys of q_t . k / sqrt(d_head) for that head."""
    q, k, out = (_f32_host(x, n) for x, n in ((q, "q"), (k, "k"), (out, "out")))
    _expect_len(q, n_tokens * d_model, "q")
    _expect_len(k, n_audio * d_model, "k")
    if out.size < (row_offset + n_tokens) * n_selected * n_audio:
        raise WattnError(f"out: {out.size} elements, "
                         f"{(row_offset + n_tokens) * n_selected * n_audio} needed")
    slots = [int(a) for a, _ in selected]
    heads = [int(b) for _, b in selected]
    _check(lib.wattn_capture_cross_attention_heads(_fptr(q), _fptr(k), n_tokens, n_audio, n_heads,
                                                   d_model, _iarr(slots), _iarr(heads),
                                                   len(selected), n_selected, row_offset,
                                                   _fptr(out)),
           "capture_cross_attention_heads")


def _dt_of(a) -> int:
    name = str(a.dtype).rsplit(".", 1)[-1]  # "torch.bfloat16" / numpy "float32"
    if name == "float32":
        return F32
    if name == "float16":
        return F16
    if name == "bfloat16":
        return BF16
    raise TypeError(f"unsupported dtype {a.dtype}")


def _host_ptr(a):
    """Address of a host buffer (numpy array or CPU torch tensor)."""
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if a.is_cuda:
        raise TypeError("host entry points take host (CPU) buffers")
    if not a.is_contiguous():
        raise TypeError("host buffers must be contiguous")
    return a.data_ptr()


def attention_host(q, k, v, o, batch, t_q, t_kv, n_heads, scale, causal=False) -> None:
    """Batched host-buffer encoder attention (``wattn_attention_host``): contiguous
    [batch][t][n_heads*64] buffers; pinned CPU torch tensors copy fastest."""
    _check(lib.wattn_attention_host(_host_ptr(q), _host_ptr(k), _host_ptr(v), _host_ptr(o),
                                    _dt_of(q), _dt_of(o), batch, t_q, t_kv, n_heads, scale,
                                    int(bool(causal))), "attention_host")


def decode_host(q, k, v, o, n_groups, group_size, t_kv, n_heads, scale) -> None:
    """Batched host-buffer decode (``wattn_decode_host``)."""
    _check(lib.wattn_decode_host(_host_ptr(q), _host_ptr(k), _host_ptr(v), _host_ptr(o),
                                 _dt_of(q), _dt_of(k), _dt_of(o), n_groups, group_size, t_kv,
                                 n_heads, scale), "decode_host")


# ---------------------------------------------------------------- device API

def _stream_ptr(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


def _dev(t):
    if not getattr(t, "is_cuda", False):
        raise TypeError("device entry points take CUDA tensors")
    return t.data_ptr()


def attention_fwd(q, k, v, o, *, batch, t_q, t_kv, n_heads, scale, causal=False, q_pos_offset=0,
                  q_row_stride=None, kv_row_stride=None, o_row_stride=None, q_batch_stride=None,
                  kv_batch_stride=None, o_batch_stride=None, stream=None) -> None:
    """``wattn_attention_fwd`` on CUDA tensors (strides in elements; default:
    contiguous [batch][t][n_heads*64])."""
    w = n_heads * 64
    q_rs = q_row_stride or w
    kv_rs = kv_row_stride or w
    o_rs = o_row_stride or w
    q_bs = q_batch_stride if q_batch_stride is not None else t_q * q_rs
    kv_bs = kv_batch_stride if kv_batch_stride is not None else t_kv * kv_rs
    o_bs = o_batch_stride if o_batch_stride is not None else t_q * o_rs
    _check(lib.wattn_attention_fwd(_dev(q), _dev(k), _dev(v), _dev(o), _dt_of(q), _dt_of(o), batch,
                                   t_q, t_kv, n_heads, 64, q_rs, kv_rs, o_rs, q_bs, kv_bs, o_bs,
                                   scale, int(bool(causal)), q_pos_offset, _stream_ptr(stream)),
           "attention_fwd")


def decode_workspace_bytes(n_groups, group_size, t_kv, n_heads) -> int:
    return lib.wattn_decode_workspace_bytes(n_groups, group_size, t_kv, n_heads)


def decode_fwd(q, k, v, o, *, n_groups, group_size, t_kv, n_heads, scale, q_row_stride=None,
               kv_row_stride=None, kv_group_stride=None, o_row_stride=None, workspace=None,
               stream=None) -> None:
    """``wattn_decode_fwd`` on CUDA tensors. ``workspace``: a zero-filled CUDA
    tensor of at least decode_workspace_bytes() bytes, or None."""
    w = n_heads * 64
    kv_rs = kv_row_stride or w
    kv_gs = kv_group_stride if kv_group_stride is not None else t_kv * kv_rs
    ws_ptr = _dev(workspace) if workspace is not None else None
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    _check(lib.wattn_decode_fwd(_dev(q), _dev(k), _dev(v), _dev(o), _dt_of(q), _dt_of(k), _dt_of(o),
                                n_groups, group_size, t_kv, n_heads, 64, q_row_stride or w, kv_rs,
                                kv_gs, o_row_stride or w, scale, ws_ptr, ws_bytes,
                                _stream_ptr(stream)), "decode_fwd")


def decode_fwd_capture(q, k, v, o, *, n_groups, group_size, t_kv, n_heads, scale, selected,
                       n_selected, capture, row_offset=0, q_row_stride=None, kv_row_stride=None,
                       kv_group_stride=None, o_row_stride=None, workspace=None,
                       stream=None) -> None:
    """``wattn_decode_fwd_capture``: decode_fwd plus the alignment-head
    capture; ``selected`` lists (slot, head) pairs, ``capture`` is a CUDA f32
    tensor [rows][n_selected][t_kv] (rows from row_offset)."""
    w = n_heads * 64
    kv_rs = kv_row_stride or w
    kv_gs = kv_group_stride if kv_group_stride is not None else t_kv * kv_rs
    ws_ptr = _dev(workspace) if workspace is not None else None
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    slots = [int(a) for a, _ in selected]
    heads = [int(b) for _, b in selected]
    _check(lib.wattn_decode_fwd_capture(_dev(q), _dev(k), _dev(v), _dev(o), _dt_of(q), _dt_of(k),
                                        _dt_of(o), n_groups, group_size, t_kv, n_heads, 64,
                                        q_row_stride or w, kv_rs, kv_gs, o_row_stride or w, scale,
                                        ws_ptr, ws_bytes, _iarr(slots), _iarr(heads),
                                        len(selected), n_selected, row_offset, _dev(capture),
                                        _stream_ptr(stream)), "decode_fwd_capture")


def linear_fwd(x, w, y, *, m, n, k, bias=None, x_row_stride=None, w_row_stride=None,
               y_row_stride=None, stream=None) -> None:
    """``wattn_linear_fwd``: y = x W^T (+ bias) on CUDA tensors (x, W 16-bit of
    one type, bias f32 or None)."""
    _check(lib.wattn_linear_fwd(_dev(x), _dev(w), _dev(bias) if bias is not None else None,
                                _dev(y), _dt_of(x), _dt_of(y), m, n, k, x_row_stride or k,
                                w_row_stride or k, y_row_stride or n, _stream_ptr(stream)),
           "linear_fwd")


def cross_kv_project(enc, wk, wv, bv, k_out, v_out, *, n_tokens, d_model, enc_row_stride=None,
                     kv_row_stride=None, stream=None) -> None:
    """``wattn_cross_kv_project``: one layer of precompute_cross_attn
    (decoder.rs:423-447) on the device."""
    _check(lib.wattn_cross_kv_project(_dev(enc), _dev(wk), _dev(wv), _dev(bv), _dev(k_out),
                                      _dev(v_out), _dt_of(enc), _dt_of(k_out), n_tokens, d_model,
                                      enc_row_stride or d_model, kv_row_stride or d_model,
                                      _stream_ptr(stream)), "cross_kv_project")


def encoder_attention_workspace_bytes(batch, t, n_heads) -> int:
    return lib.wattn_encoder_attention_workspace_bytes(batch, t, n_heads)


def encoder_attention(x, w_qkv, b_qkv, w_out, b_out, y, *, batch, t, n_heads, workspace,
                      stream=None) -> None:
    """``wattn_encoder_attention``: QKV projection, attention over the fused
    rows and output projection of an encoder layer (encoder.rs:276-303)."""
    _check(lib.wattn_encoder_attention(_dev(x), _dev(w_qkv), _dev(b_qkv), _dev(w_out),
                                       _dev(b_out), _dev(y), _dt_of(x), _dt_of(y), batch, t,
                                       n_heads, _dev(workspace),
                                       workspace.numel() * workspace.element_size(),
                                       _stream_ptr(stream)), "encoder_attention")


def encoder_attention_residual(x, ln_w, ln_b, w_qkv, b_qkv, w_out, b_out, *, batch, t, n_heads,
                               workspace, stream=None) -> None:
    """``wattn_encoder_attention_residual``: x (f32, updated in place) +=
    the attention sub-block of an encoder layer (encoder.rs:266-304)."""
    _check(lib.wattn_encoder_attention_residual(
        _dev(x), _dev(ln_w), _dev(ln_b), _dev(w_qkv), _dev(b_qkv), _dev(w_out), _dev(b_out),
        _dt_of(w_qkv), batch, t, n_heads, _dev(workspace),
        workspace.numel() * workspace.element_size(), _stream_ptr(stream)),
        "encoder_attention_residual")


def decode_fwd_noalloc(q, k, v, o, *, n_groups, group_size, t_kv, n_heads, scale,
                       q_row_stride=None, kv_row_stride=None, kv_group_stride=None,
                       o_row_stride=None, stream=None) -> None:
    """``wattn_decode_fwd_noalloc``: decode_fwd for callers that must not
    allocate device memory; its scratch is a fixed 8 MiB array inside the
    library, shared by every call on a device (calls that overlap on the GPU
    race)."""
    w = n_heads * 64
    kv_rs = kv_row_stride or w
    kv_gs = kv_group_stride if kv_group_stride is not None else t_kv * kv_rs
    _check(lib.wattn_decode_fwd_noalloc(_dev(q), _dev(k), _dev(v), _dev(o), _dt_of(q), _dt_of(k),
                                        _dt_of(o), n_groups, group_size, t_kv, n_heads, 64,
                                        q_row_stride or w, kv_rs, kv_gs, o_row_stride or w, scale,
                                        _stream_ptr(stream)), "decode_fwd_noalloc")


def device_status(device: int = -1) -> int:
    s = ctypes.c_int(0)
    _check(lib.wattn_device_status(device, ctypes.byref(s)), "device_status")
    return s.value


def selftest_bounded_wait(limit_us: int = 1000, stream=None) -> int:
    """Runs the bounded-wait self-test; returns its status (ERR_TIMEOUT by design)."""
    return lib.wattn_selftest_bounded_wait(limit_us, _stream_ptr(stream) if stream is not None else None)


def _iarr(xs):
    """Int list -> int* argument. A C-contiguous int32 numpy array is passed
    without copying (build it once when the same list goes to every call)."""
    if isinstance(xs, np.ndarray) and xs.dtype == np.int32 and xs.flags.c_contiguous:
        return xs.ctypes.data_as(_ip)
    return (ctypes.c_int * max(1, len(xs)))(*xs)


class DeviceKvCache:
    """Device-resident paged KV cache with the methods of DecoderKvCache
    (crates/whisper/src/decoder.rs:131-264) plus append / attend / advance
    (the per-layer steps of decode_batch_inner, decoder.rs:616-647, 765-767)."""

    def __init__(self, n_layers, n_slots, n_heads, max_ctx, *, page_rows=64, n_pages=0,
                 dtype=F16):
        h = _vp()
        _check(lib.wattn_kv_create(ctypes.byref(h), n_layers, n_slots, n_heads, 64, max_ctx,
                                   page_rows, n_pages, dtype), "kv_create")
        self._h = h
        self.n_layers, self.n_heads, self.max_ctx, self.dtype = n_layers, n_heads, max_ctx, dtype
        self.d_model = n_heads * 64

    def close(self):
        if self._h:
            lib.wattn_kv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def clear(self):
        _check(lib.wattn_kv_clear(self._h), "kv_clear")

    def clear_slot(self, slot):
        _check(lib.wattn_kv_clear_slot(self._h, slot), "kv_clear_slot")

    def ensure_slots(self, n_slots):
        _check(lib.wattn_kv_ensure_slots(self._h, n_slots), "kv_ensure_slots")

    def copy_slot(self, dst, src, stream=None):
        _check(lib.wattn_kv_copy_slot(self._h, dst, src, _stream_ptr(stream)), "kv_copy_slot")

    def assign_beams(self, parent_slots) -> list:
        """beam.rs:418-460: slots for the retained branches whose parents are
        ``parent_slots`` (ranking order), forking where a parent has several."""
        n = len(parent_slots)
        out = (ctypes.c_int * max(1, n))()
        _check(lib.wattn_kv_assign_beams(self._h, _iarr(parent_slots), n, out), "kv_assign_beams")
        return list(out[:n])

    def slot_len(self, slot) -> int:
        n = ctypes.c_int(0)
        _check(lib.wattn_kv_slot_len(self._h, slot, ctypes.byref(n)), "kv_slot_len")
        return n.value

    def slide_to_fit(self, slot, n_new, max_ctx) -> int:
        pos = ctypes.c_int(0)
        _check(lib.wattn_kv_slide_to_fit(self._h, slot, n_new, max_ctx, ctypes.byref(pos)),
               "kv_slide_to_fit")
        return pos.value

    def set_t_past(self, slot, n_past):
        _check(lib.wattn_kv_set_t_past(self._h, slot, n_past), "kv_set_t_past")

    def advance(self, slots, n_tokens):
        _check(lib.wattn_kv_advance(self._h, _iarr(slots), _iarr(n_tokens), len(slots)),
               "kv_advance")

    def append(self, layer, slots, n_tokens, k_rows, v_rows, stream=None):
        _check(lib.wattn_kv_append(self._h, layer, _iarr(slots), _iarr(n_tokens), len(slots),
                                   _dev(k_rows), _dev(v_rows), _dt_of(k_rows),
                                   k_rows.stride(0) if k_rows.dim() > 1 else self.d_model,
                                   _stream_ptr(stream)), "kv_append")

    def workspace_bytes(self, n_rows) -> int:
        return lib.wattn_kv_workspace_bytes(self._h, n_rows)

    def attend(self, layer, slots, n_tokens, q, o, scale=0.125, workspace=None, stream=None):
        ws_ptr = _dev(workspace) if workspace is not None else None
        ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
        _check(lib.wattn_kv_attend(self._h, layer, _iarr(slots), _iarr(n_tokens), len(slots),
                                   _dev(q), _dt_of(q), q.stride(0) if q.dim() > 1 else self.d_model,
                                   _dev(o), _dt_of(o), o.stride(0) if o.dim() > 1 else self.d_model,
                                   scale, ws_ptr, ws_bytes, _stream_ptr(stream)), "kv_attend")

    def read_slot(self, layer, slot, which, out, stream=None):
        _check(lib.wattn_kv_read_slot(self._h, layer, slot, which, _dev(out), _dt_of(out),
                                      _stream_ptr(stream)), "kv_read_slot")

    def stats(self):
        used, total = ctypes.c_int(0), ctypes.c_int(0)
        _check(lib.wattn_kv_stats(self._h, ctypes.byref(used), ctypes.byref(total)), "kv_stats")
        return used.value, total.value
