"""Alignment-head capture fused into the cross-attention decode
(decode_with_alignment_heads: multi_head_attention + capture_cross_attention_heads,
crates/whisper/src/decoder.rs:698-722, 796-828) against the oracle's
restatement of capture_cross_attention_heads.

Besides matching the oracle, every captured row must be what the reference's
own test asks of it (crates/whisper/tests/test_dtw_alignment.rs:57-71):
finite, non-negative and summing to 1 within 1e-4. Slots that a call does
not select keep their contents.
"""
import numpy as np
import pytest

from tests.helpers import check_16bit, check_f32, randn, rounded

pytestmark = pytest.mark.gpu

SENTINEL = -7.0
CAP_TOL = 2e-5  # probabilities: same rounded inputs on both sides, f32 dots and softmax


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


def _oracle_capture(oracle, qf, kf, n_groups, g, t_kv, h, selected, n_selected, row_offset):
    d = h * 64
    out = np.full((row_offset + n_groups * g) * n_selected * t_kv, SENTINEL, np.float32)
    for grp in range(n_groups):
        q = qf.reshape(n_groups * g, d)[grp * g:(grp + 1) * g]
        k = kf.reshape(n_groups, t_kv, d)[grp]
        oracle.capture_heads(q, k, g, t_kv, h, d, selected, n_selected, row_offset + grp * g, out)
    return out.reshape(-1, n_selected, t_kv)


def _check_rows(cap, selected, rows):
    for slot, _ in selected:
        p = cap[rows, slot]
        assert np.isfinite(p).all() and (p >= 0).all()
        assert np.abs(p.sum(-1) - 1.0).max() < 1e-4


@pytest.mark.parametrize("dt", [1, 2, 0], ids=["f16", "bf16", "f32"])
@pytest.mark.parametrize("shape", [(2, 5, 1500, 20), (1, 3, 4033, 2), (3, 13, 700, 4)],
                         ids=["large_v3", "split_keys", "two_row_chunks"])
def test_capture_matches_oracle(W, oracle, dt, shape):
    import torch
    n_groups, g, t_kv, h = shape
    d = h * 64
    selected = [(0, h - 1), (2, 0)] + ([(3, 7)] if h > 7 else [])
    n_selected, row_offset = 5, 2
    (kd, kf), (vd, vf) = rounded(randn(11 + t_kv, n_groups * t_kv * d), dt), \
        rounded(randn(12 + t_kv, n_groups * t_kv * d), dt)
    qd, qf = rounded(randn(13 + g, n_groups * g * d), dt)
    rows = row_offset + n_groups * g
    cap = torch.full((rows * n_selected * t_kv,), SENTINEL, device="cuda")
    o = torch.empty(n_groups * g * d, device="cuda")
    W.decode_fwd_capture(qd, kd, vd, o, n_groups=n_groups, group_size=g, t_kv=t_kv, n_heads=h,
                         scale=0.125, selected=selected, n_selected=n_selected, capture=cap,
                         row_offset=row_offset)
    torch.cuda.synchronize()
    got = cap.cpu().numpy().reshape(rows, n_selected, t_kv)
    exp = _oracle_capture(oracle, qf, kf, n_groups, g, t_kv, h, selected, n_selected, row_offset)
    err = np.abs(got - exp).max()
    assert err < CAP_TOL, f"capture max-abs {err}"
    _check_rows(got, selected, slice(row_offset, rows))
    # unselected slots and rows before row_offset untouched
    untouched = [s for s in range(n_selected) if s not in {a for a, _ in selected}]
    assert (got[:, untouched] == SENTINEL).all()
    assert (got[:row_offset] == SENTINEL).all()
    # the attention output is the same as without the capture
    ref = oracle.decode_grouped(qf, kf, vf, n_groups, g, t_kv, h, d)
    if dt == 0:
        check_f32(o.cpu().numpy(), ref, "decode with capture")
    else:
        check_16bit(o.cpu().numpy(), ref, "decode with capture")


def test_capture_per_layer_slots(W, oracle):
    """Two layers' calls fill disjoint slots of one capture buffer, as the
    decoder does with each layer's subset of the alignment heads."""
    import torch
    n_groups, g, t_kv, h = 1, 4, 1500, 6
    d = h * 64
    layers = [[(0, 1), (1, 4)], [(2, 0)]]
    n_selected = 3
    cap = torch.full((g * n_selected * t_kv,), SENTINEL, device="cuda")
    exp = np.full(g * n_selected * t_kv, SENTINEL, np.float32)
    for li, sel in enumerate(layers):
        kd, kf = rounded(randn(50 + li, t_kv * d), 1)
        qd, qf = rounded(randn(60 + li, g * d), 1)
        o = torch.empty(g * d, dtype=torch.float16, device="cuda")
        W.decode_fwd_capture(qd, kd, kd, o, n_groups=n_groups, group_size=g, t_kv=t_kv,
                             n_heads=h, scale=0.125, selected=sel, n_selected=n_selected,
                             capture=cap)
        oracle.capture_heads(qf, kf, g, t_kv, h, d, sel, n_selected, 0, exp)
    torch.cuda.synchronize()
    got = cap.cpu().numpy()
    assert np.abs(got - exp).max() < CAP_TOL
    assert not (got == SENTINEL).any()


def test_capture_host_mirror(W, oracle):
    """wattn_capture_cross_attention_heads on host f32 slices, the reference's
    signature (d_head 64 here, scale 1/8)."""
    n_tokens, n_audio, h = 5, 1500, 6
    d = h * 64
    q, k = randn(70, n_tokens * d), randn(71, n_audio * d)
    selected, n_selected, row_offset = [(1, 5), (0, 2)], 3, 1
    out = np.full((row_offset + n_tokens) * n_selected * n_audio, SENTINEL, np.float32)
    exp = out.copy()
    W.capture_cross_attention_heads(q, k, n_tokens, n_audio, h, d, selected, n_selected,
                                    row_offset, out)
    oracle.capture_heads(q, k, n_tokens, n_audio, h, d, selected, n_selected, row_offset, exp)
    assert np.abs(out - exp).max() < CAP_TOL
    got = out.reshape(-1, n_selected, n_audio)
    _check_rows(got, selected, slice(row_offset, row_offset + n_tokens))
    assert (got[:, 2] == SENTINEL).all() and (got[0] == SENTINEL).all()
