"""A seeded random sweep of the encoder attention sub-block entry points
(wattn_encoder_attention and wattn_encoder_attention_residual,
crates/whisper/src/encoder.rs:266-304) against the oracle, stage by stage.

The fixed block tests run three shapes; these draw 1-3 utterances of 1-1500
frames with 1-8 heads from a fixed seed, in both input types, and check what
the fixed tests cannot see at those shapes: that the chained kernels keep to
the workspace wattn_encoder_attention_workspace_bytes() sizes (the bytes
after it, and after the output, hold a guard pattern that must survive) at
every row count, including single frames and ragged query and key tiles.
Each stage is checked on the intermediates the device stored, at the bars of
the fixed tests: projections to 2e-5 of their largest output plus the 16-bit
storage rounding, attention to 2e-3 / cosine 0.9999.
"""
import numpy as np
import pytest

from tests.helpers import check_16bit, half_ulp, rounded

pytestmark = pytest.mark.gpu

N_CASES = 16
GUARD = 4096  # guard bytes after the workspace and the output


def _draw(i):
    r = np.random.default_rng(9900 + i)
    b = int(r.integers(1, 4))
    t = int(np.exp(r.uniform(0, np.log(1500))))
    h = int(r.integers(1, 9))
    while b * t * h > 9000 and b > 1:  # keeps the oracle's share short
        b -= 1
    while b * t * h > 9000:
        h -= 1
    return dict(b=b, t=t, h=h, dt=int(r.integers(1, 3)), residual=bool(i % 2), seed=9900 + i)


CASES = [_draw(i) for i in range(N_CASES)]


def _id(c):
    return (f"{'f16' if c['dt'] == 1 else 'bf16'}-b{c['b']}t{c['t']}h{c['h']}"
            f"{'-residual' if c['residual'] else ''}")


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


def _attention_ref(oracle, qkv, b, t, h, d):
    qkv3 = qkv.reshape(b, t, 3 * d)
    out = np.empty((b, t, d), np.float32)
    for u in range(b):
        q, k, v = (np.ascontiguousarray(qkv3[u, :, i * d:(i + 1) * d]) for i in range(3))
        out[u] = oracle.flash_attention_2(q, k, v, t, t, h, d, False).reshape(t, d)
    return out.ravel()


@pytest.mark.parametrize("c", CASES, ids=[_id(c) for c in CASES])
def test_random_encoder_block(W, oracle, c):
    import torch
    b, t, h, dt = c["b"], c["t"], c["h"], c["dt"]
    d, rows = h * 64, b * t
    g = np.random.default_rng(c["seed"])
    s = 1.0 / np.sqrt(d)
    f32 = lambda n: g.standard_normal(n).astype(np.float32)  # noqa: E731
    wqkv_d, wqkv_f = rounded(f32(3 * d * d) * s, dt)
    wo_d, wo_f = rounded(f32(d * d) * s, dt)
    bqkv, bo = f32(3 * d) * 0.1, f32(d) * 0.1
    cuda = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    need = W.encoder_attention_workspace_bytes(b, t, h)
    ws_all = torch.full((need + GUARD,), 0xA5, dtype=torch.uint8, device="cuda")
    ws = ws_all[:need]
    tdt = {1: torch.float16, 2: torch.bfloat16}[dt]
    r256 = lambda n: ((n + 255) // 256) * 256  # noqa: E731
    o_attn = r256(rows * 3 * d * 2)
    if c["residual"]:
        x0 = f32(rows * d) * 2.0 + 0.5
        ln_w, ln_b = 1.0 + 0.1 * f32(d), 0.1 * f32(d)
        x_all = torch.full((rows * d + GUARD // 4,), 7.0, device="cuda")
        x_all[:rows * d] = cuda(x0)
        W.encoder_attention_residual(x_all[:rows * d], cuda(ln_w), cuda(ln_b), wqkv_d, cuda(bqkv),
                                     wo_d, cuda(bo), batch=b, t=t, n_heads=h, workspace=ws)
        torch.cuda.synchronize()
        o_xn = o_attn + r256(rows * d * 2)
        xn = ws[o_xn:o_xn + rows * d * 2].view(tdt).float().cpu().numpy()
        xn_ref = oracle.layer_norm(x0, ln_w, ln_b, rows, d)
        assert (np.abs(xn - xn_ref) <= 1e-5 * np.abs(xn_ref).max() + half_ulp(xn_ref, dt)).all()
        gemm_in, base, out_all = xn, x0, x_all
    else:
        xd, xf = rounded(f32(rows * d), dt)
        y_all = torch.full((rows * d + GUARD // 4,), 7.0, device="cuda")
        W.encoder_attention(xd, wqkv_d, cuda(bqkv), wo_d, cuda(bo), y_all[:rows * d], batch=b,
                            t=t, n_heads=h, workspace=ws)
        torch.cuda.synchronize()
        gemm_in, base, out_all = xf, 0.0, y_all
    assert W.device_status() == 0
    qkv = ws[:rows * 3 * d * 2].view(tdt).float().cpu().numpy()
    attn = ws[o_attn:o_attn + rows * d * 2].view(tdt).float().cpu().numpy()
    qkv_ref = oracle.linear(gemm_in, wqkv_f, bqkv, rows, 3 * d, d)
    assert (np.abs(qkv - qkv_ref) <= 2e-5 * np.abs(qkv_ref).max() + half_ulp(qkv_ref, dt)
            + 1e-6).all(), "QKV projection"
    check_16bit(attn, _attention_ref(oracle, qkv, b, t, h, d), f"{_id(c)} attention", dt)
    y_ref = base + oracle.linear(attn, wo_f, bo, rows, d, d)
    got = out_all[:rows * d].cpu().numpy()
    assert (np.abs(got - y_ref) <= 2e-5 * np.abs(y_ref).max() + 1e-6).all(), "output projection"
    assert bool((ws_all[need:] == 0xA5).all()), "bytes past the workspace written"
    assert bool((out_all[rows * d:] == 7.0).all()), "bytes past the output written"
