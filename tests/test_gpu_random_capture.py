"""A seeded random sweep of the decode with alignment-head capture
(wattn_decode_fwd_capture: multi_head_attention + capture_cross_attention_heads,
crates/whisper/src/decoder.rs:698-722, 796-828) against the oracle.

The fixed capture cases use three shapes and fixed selections; these draw,
from a fixed seed, 1-20 groups of 1-16 rows, 1-3000 keys (log-uniform: one
key, ragged sub-tiles and key splits all come up), 1-20 heads, each input
type, a random subset of the heads spread over random slots of a buffer with
spare slots, and a random row offset. Every captured row must match the
oracle (2e-5), be finite, non-negative and sum to 1 within 1e-4 (what the
reference's own DTW test asks, crates/whisper/tests/test_dtw_alignment.rs:
57-71); slots not selected and rows before the offset keep their contents;
the attention output must match the decode oracle as without the capture.
"""
import numpy as np
import pytest

import tests.test_gpu_capture as cap_tests
from tests.helpers import check_16bit, check_f32, rounded

pytestmark = pytest.mark.gpu

N_CASES = 30


def _draw(i):
    r = np.random.default_rng(9700 + i)
    dt = i % 3
    n_groups = int(np.exp(r.uniform(0, np.log(20))))
    g = int(r.integers(1, 17))
    t_kv = int(np.exp(r.uniform(0, np.log(3000))))
    h = int(r.integers(1, 21))
    while n_groups * g * t_kv * h > 4e6 and n_groups > 1:  # the oracle's share
        n_groups -= 1
    n_sel = int(r.integers(1, h + 1))
    heads = [int(x) for x in r.choice(h, size=n_sel, replace=False)]
    n_selected = n_sel + int(r.integers(0, 3))
    slots = [int(x) for x in r.choice(n_selected, size=n_sel, replace=False)]
    return dict(dt=dt, n_groups=n_groups, g=g, t_kv=t_kv, h=h,
                selected=list(zip(slots, heads)), n_selected=n_selected,
                row_offset=int(r.integers(0, 6)), seed=9700 + i)


CASES = [_draw(i) for i in range(N_CASES)]


def _id(c):
    return (f"{'f32 f16 bf16'.split()[c['dt']]}-{c['n_groups']}x{c['g']}-t{c['t_kv']}-h{c['h']}-"
            f"sel{len(c['selected'])}of{c['n_selected']}")


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


@pytest.mark.parametrize("c", CASES, ids=[_id(c) for c in CASES])
def test_random_capture_call(W, oracle, c):
    import torch
    dt, n_groups, g, t_kv, h = c["dt"], c["n_groups"], c["g"], c["t_kv"], c["h"]
    d = h * 64
    sel, n_selected, row_offset = c["selected"], c["n_selected"], c["row_offset"]
    rng = np.random.default_rng(c["seed"])
    kd, kf = rounded(rng.standard_normal(n_groups * t_kv * d).astype(np.float32), dt)
    vd, vf = rounded(rng.standard_normal(n_groups * t_kv * d).astype(np.float32), dt)
    qd, qf = rounded(rng.standard_normal(n_groups * g * d).astype(np.float32), dt)
    rows = row_offset + n_groups * g
    sentinel = cap_tests.SENTINEL
    cap = torch.full((rows * n_selected * t_kv,), sentinel, device="cuda")
    o = torch.empty(n_groups * g * d, device="cuda")
    W.decode_fwd_capture(qd, kd, vd, o, n_groups=n_groups, group_size=g, t_kv=t_kv, n_heads=h,
                         scale=0.125, selected=sel, n_selected=n_selected, capture=cap,
                         row_offset=row_offset)
    torch.cuda.synchronize()
    assert W.device_status() == 0
    got = cap.cpu().numpy().reshape(rows, n_selected, t_kv)
    exp = cap_tests._oracle_capture(oracle, qf, kf, n_groups, g, t_kv, h, sel, n_selected,
                                    row_offset)
    err = float(np.abs(got - exp).max())
    assert err < cap_tests.CAP_TOL, f"{_id(c)}: capture max-abs {err}"
    cap_tests._check_rows(got, sel, slice(row_offset, rows))
    untouched = [s for s in range(n_selected) if s not in {a for a, _ in sel}]
    assert (got[:, untouched] == sentinel).all()
    assert (got[:row_offset] == sentinel).all()
    ref = oracle.decode_grouped(qf, kf, vf, n_groups, g, t_kv, h, d)
    if dt == 0:
        check_f32(o.cpu().numpy(), ref, _id(c))
    else:
        check_16bit(o.cpu().numpy(), ref, _id(c))
