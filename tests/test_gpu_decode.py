"""Split-KV decode attention on the GPU against the CPU oracle
(single_token_mha_d64 restated, attention.rs:246-434; grouped as the
decoder's cross-attention, decoder.rs:688-724)."""
import numpy as np
import pytest

from tests.helpers import check_16bit, check_f32, randn, rounded

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


def _decode(W, qd, kd, vd, out_dt, n_groups, g, t_kv, h, workspace=None, **kw):
    import torch
    o = torch.empty(n_groups * g * h * 64, dtype={0: torch.float32, 1: torch.float16,
                                                  2: torch.bfloat16}[out_dt], device="cuda")
    W.decode_fwd(qd, kd, vd, o, n_groups=n_groups, group_size=g, t_kv=t_kv, n_heads=h, scale=0.125,
                 workspace=workspace, **kw)
    torch.cuda.synchronize()
    return o.float().cpu().numpy()


@pytest.mark.parametrize("kv_dt", [0, 1, 2], ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("t_kv", [1, 64, 65, 257, 1500])
@pytest.mark.parametrize("g", [1, 5, 13])
def test_decode_dense(W, oracle, kv_dt, t_kv, g):
    n_groups, h = 3, 4
    d = h * 64
    (kd, kf), (vd, vf) = rounded(randn(100 + t_kv, n_groups * t_kv * d), kv_dt), \
        rounded(randn(200 + t_kv, n_groups * t_kv * d), kv_dt)
    qd, qf = rounded(randn(300 + g, n_groups * g * d), kv_dt)
    ref = oracle.decode_grouped(qf, kf, vf, n_groups, g, t_kv, h, d)
    out = _decode(W, qd, kd, vd, 0, n_groups, g, t_kv, h)
    if kv_dt == 0:
        check_f32(out, ref, f"f32 t_kv={t_kv} g={g}")
    else:
        check_16bit(out, ref, f"dt={kv_dt} t_kv={t_kv} g={g}")


@pytest.mark.parametrize("kv_dt", [1, 2], ids=["f16", "bf16"])
@pytest.mark.parametrize("t_kv", [4000, 4033])
def test_decode_many_splits(W, oracle, kv_dt, t_kv):
    # One utterance, one head: few items, so the keys are split (16 splits of
    # 256 keys here) and merged by log-sum-exp; the second length leaves a
    # ragged last split.
    n_groups, g, h = 1, 5, 1
    d = h * 64
    (kd, kf), (vd, vf) = rounded(randn(40 + t_kv, t_kv * d), kv_dt), \
        rounded(randn(41 + t_kv, t_kv * d), kv_dt)
    qd, qf = rounded(randn(42, g * d), kv_dt)
    ref = oracle.decode_grouped(qf, kf, vf, n_groups, g, t_kv, h, d)
    out = _decode(W, qd, kd, vd, 0, n_groups, g, t_kv, h)
    check_16bit(out, ref, f"dt={kv_dt} t_kv={t_kv}")


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
@pytest.mark.parametrize("t_kv", [2, 4, 5, 18, 33])
def test_decode_bf16_short_key_ranges(W, oracle, t_kv, seed):
    # bf16 q and K/V on the streaming tensor-core kernel with few keys, where
    # one or two weights dominate each row: P rounded to bf16 alone (8
    # significant bits) gave max-abs errors up to 5.2e-3 here; the kernel
    # carries P's rounding residual as a second bf16 part.
    n_groups, g, h = 11, 14, 20
    d = h * 64
    (kd, kf), (vd, vf) = rounded(randn(500 + 7 * seed + t_kv, n_groups * t_kv * d), 2), \
        rounded(randn(600 + 7 * seed + t_kv, n_groups * t_kv * d), 2)
    qd, qf = rounded(randn(700 + seed, n_groups * g * d), 2)
    ref = oracle.decode_grouped(qf, kf, vf, n_groups, g, t_kv, h, d)
    check_16bit(_decode(W, qd, kd, vd, 0, n_groups, g, t_kv, h), ref, f"bf16 t_kv={t_kv}")
    check_16bit(_decode(W, qd, kd, vd, 2, n_groups, g, t_kv, h), ref, f"bf16 out t_kv={t_kv}", 2)


def test_decode_cross_attention_large_v3(W, oracle):
    # Config 4 at full size, one layer: 32 utterances x 5 beams, 20 heads,
    # f16 K/V of 1500 encoder states shared by the beams of an utterance.
    import torch
    n_groups, g, t_kv, h = 32, 5, 1500, 20
    d = h * 64
    (kd, kf), (vd, vf) = rounded(randn(1, n_groups * t_kv * d), 1), rounded(randn(2, n_groups * t_kv * d), 1)
    qd, qf = rounded(randn(3, n_groups * g * d), 1)
    ref = oracle.decode_grouped(qf, kf, vf, n_groups, g, t_kv, h, d)
    nbytes = W.decode_workspace_bytes(n_groups, g, t_kv, h)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    out1 = _decode(W, qd, kd, vd, 1, n_groups, g, t_kv, h, workspace=ws)
    check_16bit(out1, ref, "C4", 1)
    # the workspace is left zeroed: a second call gives the same bits
    out2 = _decode(W, qd, kd, vd, 1, n_groups, g, t_kv, h, workspace=ws)
    assert np.array_equal(out1, out2)


def test_decode_strided_rows(W, oracle):
    # Query / output rows with a stride (rows of a wider buffer) and K/V rows
    # read from a fused [t, 2*d] K|V buffer.
    import torch
    n_groups, g, t_kv, h = 2, 3, 200, 2
    d = h * 64
    kv, kvf = rounded(randn(5, n_groups * t_kv * 2 * d), 2)
    kvf = kvf.reshape(n_groups, t_kv, 2 * d)
    q, qf = rounded(randn(6, n_groups * g * 3 * d), 2)
    qf = qf.reshape(n_groups * g, 3 * d)[:, :d]
    ref = oracle.decode_grouped(np.ascontiguousarray(qf), np.ascontiguousarray(kvf[:, :, :d]),
                                np.ascontiguousarray(kvf[:, :, d:]), n_groups, g, t_kv, h, d)
    o = torch.zeros(n_groups * g * 2 * d, device="cuda")
    W.decode_fwd(q, kv, kv[d:], o, n_groups=n_groups, group_size=g, t_kv=t_kv, n_heads=h,
                 scale=0.125, q_row_stride=3 * d, kv_row_stride=2 * d,
                 kv_group_stride=t_kv * 2 * d, o_row_stride=2 * d)
    torch.cuda.synchronize()
    out = o.view(n_groups * g, 2 * d)[:, :d].cpu().numpy()
    check_16bit(out, ref, "strided")
    assert (o.view(n_groups * g, 2 * d)[:, d:] == 0).all()


def test_decode_host_entry(W, oracle):
    n_groups, g, t_kv, h = 4, 5, 333, 3
    d = h * 64
    q, k, v = randn(7, n_groups * g * d), randn(8, n_groups * t_kv * d), randn(9, n_groups * t_kv * d)
    o = np.empty_like(q)
    W.decode_host(q, k, v, o, n_groups, g, t_kv, h, 0.125)
    check_f32(o, oracle.decode_grouped(q, k, v, n_groups, g, t_kv, h, d), "decode_host")
