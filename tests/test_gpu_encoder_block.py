"""Encoder attention sub-block (crates/whisper/src/encoder.rs:276-303): the
fused QKV projection, attention over the fused rows read in place, and the
output projection, chained on the device. Each stage is checked against the
oracle's linear / flash_attention_2 on the intermediates the device stored,
and the result against an all-f32 chain by direction."""
import numpy as np
import pytest

from tests.helpers import check_16bit, half_ulp, randn, rounded

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


@pytest.mark.parametrize("dt", [2, 1], ids=["bf16", "f16"])
@pytest.mark.parametrize("shape", [(2, 300, 6), (1, 1500, 20), (3, 129, 2)],
                         ids=["base_like", "large_v3_one", "ragged"])
def test_encoder_attention_block(W, oracle, dt, shape):
    import torch
    b, t, h = shape
    d = h * 64
    rows = b * t
    s = 1.0 / np.sqrt(d)
    xd, xf = rounded(randn(1, rows * d), dt)
    wqkv_d, wqkv_f = rounded(randn(2, 3 * d * d) * s, dt)
    wo_d, wo_f = rounded(randn(3, d * d) * s, dt)
    bqkv, bo = randn(4, 3 * d) * 0.1, randn(5, d) * 0.1
    y = torch.empty(rows * d, device="cuda")
    ws = torch.empty(W.encoder_attention_workspace_bytes(b, t, h), dtype=torch.uint8, device="cuda")
    W.encoder_attention(xd, wqkv_d, torch.from_numpy(bqkv).cuda(), wo_d,
                        torch.from_numpy(bo).cuda(), y, batch=b, t=t, n_heads=h, workspace=ws)
    torch.cuda.synchronize()
    # Each stage against the oracle on the stage's own inputs as the device
    # stored them (16-bit), at that stage's bar: the projections to f32
    # accumulation order (relative 2e-5 plus the storage rounding), the
    # attention to the 16-bit attention bar.
    tdt = {1: torch.float16, 2: torch.bfloat16}[dt]
    n_qkv = rows * 3 * d
    off = ((n_qkv * 2 + 255) // 256) * 256
    qkv_dev = ws[:n_qkv * 2].view(tdt).float().cpu().numpy()
    attn_dev = ws[off:off + rows * d * 2].view(tdt).float().cpu().numpy()
    qkv_ref = oracle.linear(xf, wqkv_f, bqkv, rows, 3 * d, d)
    assert (np.abs(qkv_dev - qkv_ref) <= 2e-5 * np.abs(qkv_ref).max() + half_ulp(qkv_ref, dt)
            + 1e-6).all(), "QKV projection"
    qkv3 = qkv_dev.reshape(b, t, 3 * d)
    attn_ref = np.empty((b, t, d), np.float32)
    for u in range(b):
        q, k, v = (np.ascontiguousarray(qkv3[u, :, i * d:(i + 1) * d]) for i in range(3))
        attn_ref[u] = oracle.flash_attention_2(q, k, v, t, t, h, d, False).reshape(t, d)
    check_16bit(attn_dev, attn_ref.ravel(), f"attention in the block {shape}", dt)
    y_ref = oracle.linear(attn_dev, wo_f, bo, rows, d, d)
    got = y.cpu().numpy()
    assert (np.abs(got - y_ref) <= 2e-5 * np.abs(y_ref).max() + 1e-6).all(), "output projection"
    # end to end against an all-f32 chain: the direction of the result holds
    qkv_f = oracle.linear(xf, wqkv_f, bqkv, rows, 3 * d, d).reshape(b, t, 3 * d)
    attn_f = np.empty((b, t, d), np.float32)
    for u in range(b):
        q, k, v = (np.ascontiguousarray(qkv_f[u, :, i * d:(i + 1) * d]) for i in range(3))
        attn_f[u] = oracle.flash_attention_2(q, k, v, t, t, h, d, False).reshape(t, d)
    y_f = oracle.linear(attn_f.ravel(), wo_f, bo, rows, d, d)
    assert float(np.dot(got, y_f) / (np.linalg.norm(got) * np.linalg.norm(y_f))) > 0.9999


@pytest.mark.parametrize("dt", [2, 1], ids=["bf16", "f16"])
@pytest.mark.parametrize("shape", [(2, 300, 6), (3, 129, 2)], ids=["base_like", "ragged"])
def test_encoder_attention_residual(W, oracle, dt, shape):
    """Steps (a)-(d) of encoder.rs:266-304 in place on the f32 residual
    stream: layer norm, projections, attention and residual add; each stage
    checked on the device's own intermediates (read back from the
    workspace), as above."""
    import torch
    b, t, h = shape
    d = h * 64
    rows = b * t
    s = 1.0 / np.sqrt(d)
    x0 = randn(10, rows * d) * 2.0 + 0.5
    ln_w, ln_b = 1.0 + 0.1 * randn(11, d), 0.1 * randn(12, d)
    wqkv_d, wqkv_f = rounded(randn(13, 3 * d * d) * s, dt)
    wo_d, wo_f = rounded(randn(14, d * d) * s, dt)
    bqkv, bo = randn(15, 3 * d) * 0.1, randn(16, d) * 0.1
    x = torch.from_numpy(x0.copy()).cuda()
    ws = torch.empty(W.encoder_attention_workspace_bytes(b, t, h), dtype=torch.uint8, device="cuda")
    cuda = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    W.encoder_attention_residual(x, cuda(ln_w), cuda(ln_b), wqkv_d, cuda(bqkv), wo_d, cuda(bo),
                                 batch=b, t=t, n_heads=h, workspace=ws)
    torch.cuda.synchronize()
    tdt = {1: torch.float16, 2: torch.bfloat16}[dt]
    r256 = lambda n: ((n + 255) // 256) * 256  # noqa: E731
    o_qkv, o_attn, o_xn = 0, r256(rows * 3 * d * 2), r256(rows * 3 * d * 2) + r256(rows * d * 2)
    xn_dev = ws[o_xn:o_xn + rows * d * 2].view(tdt).float().cpu().numpy()
    qkv_dev = ws[o_qkv:o_qkv + rows * 3 * d * 2].view(tdt).float().cpu().numpy()
    attn_dev = ws[o_attn:o_attn + rows * d * 2].view(tdt).float().cpu().numpy()
    # (a) layer norm, stored 16-bit: within f32 rounding plus the storage rounding
    xn_ref = oracle.layer_norm(x0, ln_w, ln_b, rows, d)
    assert (np.abs(xn_dev - xn_ref) <= 1e-5 * np.abs(xn_ref).max() + half_ulp(xn_ref, dt)).all()
    # (b) QKV projection of the stored normalised rows
    qkv_ref = oracle.linear(xn_dev, wqkv_f, bqkv, rows, 3 * d, d)
    assert (np.abs(qkv_dev - qkv_ref) <= 2e-5 * np.abs(qkv_ref).max() + half_ulp(qkv_ref, dt)
            + 1e-6).all()
    # (c) attention over the stored QKV rows
    qkv3 = qkv_dev.reshape(b, t, 3 * d)
    attn_ref = np.empty((b, t, d), np.float32)
    for u in range(b):
        q, k, v = (np.ascontiguousarray(qkv3[u, :, i * d:(i + 1) * d]) for i in range(3))
        attn_ref[u] = oracle.flash_attention_2(q, k, v, t, t, h, d, False).reshape(t, d)
    check_16bit(attn_dev, attn_ref.ravel(), f"attention {shape}", dt)
    # (d) output projection plus the residual, f32 in place
    y_ref = x0 + oracle.linear(attn_dev, wo_f, bo, rows, d, d)
    got = x.cpu().numpy()
    assert (np.abs(got - y_ref) <= 2e-5 * np.abs(y_ref).max() + 1e-6).all()


def test_encoder_attention_rejects_a_small_workspace(W):
    import torch
    b, t, h = 1, 64, 2
    d = h * 64
    x = torch.zeros(b * t * d, dtype=torch.bfloat16, device="cuda")
    wq = torch.zeros(3 * d * d, dtype=torch.bfloat16, device="cuda")
    wo = torch.zeros(d * d, dtype=torch.bfloat16, device="cuda")
    bq, bo = torch.zeros(3 * d, device="cuda"), torch.zeros(d, device="cuda")
    y = torch.empty(b * t * d, device="cuda")
    ws = torch.empty(W.encoder_attention_workspace_bytes(b, t, h) - 256, dtype=torch.uint8,
                     device="cuda")
    with pytest.raises(W.WattnError) as e:
        W.encoder_attention(x, wq, bq, wo, bo, y, batch=b, t=t, n_heads=h, workspace=ws)
    assert e.value.status == -1
