"""The no-allocation decode entry point (wattn_decode_fwd_noalloc).

It serves callers that may not allocate device memory at all, so they can
neither hand wattn_decode_fwd a workspace nor let it allocate one; its
scratch is a fixed array compiled into the library. This test calls it
through the C ABI twice in a row (the second call reuses the scratch left by
the first) and checks each output against wattn_decode_fwd on the same
inputs, within the 16-bit tolerance used by the other decode tests. It also
checks the clear error for a call too large for the fixed array.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

from tests.helpers import check_16bit

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


def _call_noalloc(W, q, k, v, o, n_groups, g, t_kv, h):
    d = h * 64
    return W.lib.wattn_decode_fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                          W.F16, W.F16, W.F32, n_groups, g, t_kv, h, 64, d, d,
                                          t_kv * d, d, 0.125, None)


def test_noalloc_decode_matches_workspace_decode_twice(W):
    import torch
    n_groups, g, t_kv, h = 32, 5, 1500, 20   # one config-4 layer (several splits)
    d = h * 64
    gen = torch.Generator().manual_seed(1234)
    outs = []
    for call in range(2):
        q = torch.randn(n_groups * g * d, generator=gen).half().cuda()
        k = torch.randn(n_groups * t_kv * d, generator=gen).half().cuda()
        v = torch.randn(n_groups * t_kv * d, generator=gen).half().cuda()
        ref = torch.empty(n_groups * g * d, device="cuda")
        W.decode_fwd(q, k, v, ref, n_groups=n_groups, group_size=g, t_kv=t_kv, n_heads=h,
                     scale=0.125)
        out = torch.full((n_groups * g * d,), float("nan"), device="cuda")
        rc = _call_noalloc(W, q, k, v, out, n_groups, g, t_kv, h)
        assert rc == 0, W.status_string(rc)
        torch.cuda.synchronize()
        check_16bit(out.cpu().numpy(), ref.cpu().numpy(), f"no-alloc call {call}")
        outs.append(out.cpu().numpy())
    assert not np.array_equal(outs[0], outs[1])  # two different inputs, both checked


def test_noalloc_rejects_calls_beyond_its_scratch(W):
    import torch
    # f32 K/V take the CUDA-core kernel, whose 12 splits of 128 keys here need
    # 800 rows x 20 heads x 12 partials (~51 MB), far beyond the fixed 8 MiB.
    # K/V are allocated at full size so that nothing is read out of bounds
    # even if the call were accepted.
    n_groups, g, t_kv, h = 100, 8, 1500, 20
    d = h * 64
    q = torch.zeros(n_groups * g * d, device="cuda")
    kv = torch.zeros(n_groups * t_kv * d, device="cuda")
    out = torch.zeros(n_groups * g * d, device="cuda")
    rc = W.lib.wattn_decode_fwd_noalloc(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), out.data_ptr(),
                                        W.F32, W.F32, W.F32, n_groups, g, t_kv, h, 64, d, d,
                                        t_kv * d, d, 0.125, None)
    torch.cuda.synchronize()
    assert rc == -6
    buf = ctypes.create_string_buffer(256)
    W.lib.wattn_last_error(buf, 256)
    assert b"scratch" in buf.value
