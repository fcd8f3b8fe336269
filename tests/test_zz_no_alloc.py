"""The no-allocation decode entry point (wattn_decode_fwd_noalloc).

It serves callers that may not allocate device memory at all: code running
inside a real-time audio callback, under an allocator frozen after start-up,
or in a host that only hands out pre-registered buffers. Those callers can
neither pass wattn_decode_fwd a workspace nor let it allocate one, so this
entry point keeps the split partials and merge counters in a fixed array
compiled into the library.

The tests call it through the C ABI:
  * on shapes whose keys are split (so the partials and counters in the
    fixed array are really used), twice in a row with different inputs, each
    output checked against the CPU oracle (the tolerance of the other decode
    tests: 1e-5 for f32, the 16-bit bar otherwise), with the entry point
    called before any wattn_decode_fwd of the process;
  * in a fresh process, that its calls take no device memory beyond the
    fixed array itself (loaded with the library's module on first use);
  * that arguments wattn_decode_fwd rejects are rejected here too, before
    any launch, and that a call too large for the array gets a clear error.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes
import json
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from tests.helpers import check_16bit, check_f32, randn, rounded

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SCRATCH_BYTES = 8 << 20  # the fixed array's size


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


def _call(W, q, k, v, o, dt, n_groups, g, t_kv, h, q_rs=None):
    d = h * 64
    return W.lib.wattn_decode_fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                          dt, dt, W.F32, n_groups, g, t_kv, h, 64, q_rs or d, d,
                                          t_kv * d, d, 0.125, None)


# (K/V dtype, groups, rows per group, keys, heads). The first two split the
# keys: one f16 row group of one head has a single item, so its 4000 keys are
# cut into 13 splits of 320; f32 K/V take the CUDA-core kernel, which cuts
# 1500 keys into 24 splits of 64 for 80 items (about 4.3 MB of partials).
# The last is one config-4 layer (640 items, no split).
CASES = [(1, 1, 5, 4000, 1), (0, 4, 8, 1500, 20), (1, 32, 5, 1500, 20)]


@pytest.mark.parametrize("dt,n_groups,g,t_kv,h", CASES,
                         ids=["f16-split", "f32-split", "f16-config4"])
def test_noalloc_matches_oracle_twice(W, oracle, dt, n_groups, g, t_kv, h):
    import torch
    d = h * 64
    outs = []
    for call in range(2):
        seed = 5000 + 10 * call + dt
        (kd, kf), (vd, vf) = rounded(randn(seed, n_groups * t_kv * d), dt), \
            rounded(randn(seed + 1, n_groups * t_kv * d), dt)
        qd, qf = rounded(randn(seed + 2, n_groups * g * d), dt)
        out = torch.full((n_groups * g * d,), float("nan"), device="cuda")
        rc = _call(W, qd, kd, vd, out, dt, n_groups, g, t_kv, h)
        assert rc == 0, W.status_string(rc)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        ref = oracle.decode_grouped(qf, kf, vf, n_groups, g, t_kv, h, d)
        if dt == 0:
            check_f32(got, ref, f"no-alloc call {call}")
        else:
            check_16bit(got, ref, f"no-alloc call {call}")
        outs.append(got)
    assert not np.array_equal(outs[0], outs[1])  # two different inputs, both checked
    assert W.device_status() == 0


_FRESH = textwrap.dedent("""
    import json, sys
    sys.path[:0] = [{root!r}, {pkg!r}]
    import torch
    import wattn as W
    torch.cuda.set_device(0)
    n_groups, g, t_kv, h = 4, 8, 1500, 20
    d = h * 64
    gen = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(n, generator=gen).cuda()
               for n in (n_groups * g * d, n_groups * t_kv * d, n_groups * t_kv * d))
    ref = torch.empty(n_groups * g * d, device="cuda")
    outs = [torch.full_like(ref, float("nan")) for _ in range(3)]
    # Loads the decode kernels with a workspace the caller provides, so that
    # nothing below is charged for them.
    ws = torch.zeros(W.decode_workspace_bytes(n_groups, g, t_kv, h), dtype=torch.uint8,
                     device="cuda")
    W.decode_fwd(q, k, v, ref, n_groups=n_groups, group_size=g, t_kv=t_kv, n_heads=h,
                 scale=0.125, workspace=ws)
    torch.cuda.synchronize()
    free, rcs = [torch.cuda.mem_get_info()[0]], []
    for o in outs:
        rcs.append(W.lib.wattn_decode_fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                  o.data_ptr(), 0, 0, 0, n_groups, g, t_kv, h, 64,
                                                  d, d, t_kv * d, d, 0.125, None))
        torch.cuda.synchronize()
        free.append(torch.cuda.mem_get_info()[0])
    err = max(float((o - ref).abs().max()) for o in outs)
    print(json.dumps({{"rc": rcs, "free": free, "err": err,
                      "plan": W.decode_workspace_bytes(n_groups, g, t_kv, h)}}))
""")


def test_noalloc_takes_no_device_memory_in_a_fresh_process(W):
    # A fresh interpreter: the no-allocation entry point's first call there
    # loads the library's module holding the fixed array (8 MiB, plus the
    # driver's rounding) and must take nothing else; the decode kernels'
    # own workspace for this shape (about 4.3 MB) would show if it did.
    # Later calls take nothing at all.
    script = _FRESH.format(root=ROOT, pkg=os.path.join(ROOT, "whisper.rs_b200"))
    res = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    r = json.loads(res.stdout.strip().splitlines()[-1])
    assert r["rc"] == [0, 0, 0], r
    assert r["plan"] > 4 << 20, r  # a hidden workspace would be at least this large
    free = r["free"]
    first = free[0] - free[1]
    assert first <= SCRATCH_BYTES + (3 << 20) + (1 << 19), f"first call took {first} bytes"
    assert free[1] == free[2] == free[3], f"later calls took device memory: {free}"
    assert r["err"] <= 1e-5, r


def test_noalloc_rejects_what_decode_fwd_rejects(W):
    import torch
    n_groups, g, t_kv, h = 2, 5, 300, 2
    d = h * 64
    q = torch.zeros(n_groups * g * (d + 1), dtype=torch.float16, device="cuda")
    kv = torch.zeros(n_groups * t_kv * d, dtype=torch.float16, device="cuda")
    out = torch.full((n_groups * g * d,), 7.0, device="cuda")
    # A 16-bit q with an odd row stride: its rows are read as 32-bit pairs,
    # so both entry points refuse it on the host.
    for fn in ("wattn_decode_fwd_noalloc", "wattn_decode_fwd"):
        args = [q.data_ptr(), kv.data_ptr(), kv.data_ptr(), out.data_ptr(), W.F16, W.F16, W.F32,
                n_groups, g, t_kv, h, 64, d + 1, d, t_kv * d, d, 0.125]
        if fn == "wattn_decode_fwd":
            args += [None, 0]
        assert getattr(W.lib, fn)(*args, None) == -1, fn
    # K/V rows whose stride is not a multiple of 16 bytes.
    rc = W.lib.wattn_decode_fwd_noalloc(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), out.data_ptr(),
                                        W.F16, W.F16, W.F32, n_groups, g, t_kv - 1, h, 64, d,
                                        d + 4, t_kv * d, d, 0.125, None)
    assert rc == -1
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was launched


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
