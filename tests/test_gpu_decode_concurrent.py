"""Repeated decode calls whose key range ends inside a 64-key sub-tile, while
another kernel runs on a second stream.

The streaming decode kernel walks several items per CTA through a 4-stage
K/V ring. When the last sub-tile of an item is partial and the ring wraps,
letting the TMA zero-fill the rows past the key range made items whose
stages a later item reuses come out wrong now and then (on B200: a quarter
of the calls for 32 groups x 16 rows over 70 keys, more often beside a
concurrent kernel); the kernel now copies such sub-tiles itself. This test
repeats that shape with an encoder attention call on a second stream every
third time, and requires every output to be bitwise identical to the first
and the first to match the oracle (decode_grouped, attention.rs:246-434, at
the 16-bit bar). The old kernel failed it within a few dozen calls.
"""
import numpy as np
import pytest

from tests.helpers import check_16bit, rounded

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


@pytest.mark.parametrize("t_kv", [70, 76, 204])
def test_partial_last_sub_tile_under_a_concurrent_kernel(W, oracle, t_kv):
    import torch
    n_groups, g, h, reps = 32, 16, 20, 300
    d = h * 64
    rng = np.random.default_rng(40 + t_kv)
    qd, qf = rounded(rng.standard_normal(n_groups * g * d).astype(np.float32), 1)
    kd, kf = rounded(rng.standard_normal(n_groups * t_kv * d).astype(np.float32), 1)
    vd, vf = rounded(rng.standard_normal(n_groups * t_kv * d).astype(np.float32), 1)
    ref = oracle.decode_grouped(qf, kf, vf, n_groups, g, t_kv, h, d)
    # the decode gets its own workspace; the concurrent call uses the library's
    ws = torch.zeros(W.decode_workspace_bytes(n_groups, g, t_kv, h), dtype=torch.uint8,
                     device="cuda")
    side = torch.cuda.Stream()
    bt, tt, ht = 4, 1500, 20
    aq = torch.randn(bt * tt * ht * 64, device="cuda").to(torch.bfloat16)
    ao = torch.empty_like(aq)
    torch.cuda.synchronize()
    first, differ = None, 0
    for r in range(reps):
        if r % 3 == 1:
            W.attention_fwd(aq, aq, aq, ao, batch=bt, t_q=tt, t_kv=tt, n_heads=ht, scale=0.125,
                            stream=side)
        o = torch.full((n_groups * g * d,), 3.0, device="cuda")
        W.decode_fwd(qd, kd, vd, o, n_groups=n_groups, group_size=g, t_kv=t_kv, n_heads=h,
                     scale=0.125, workspace=ws)
        if first is None:
            torch.cuda.synchronize()
            first = o.clone()
            continue
        differ += int(bool((o != first).any()))
    torch.cuda.synchronize()
    assert W.device_status() == 0
    check_16bit(first.cpu().numpy(), ref, f"t_kv={t_kv}")
    assert differ == 0, f"{differ} of {reps - 1} calls differ from the first"
