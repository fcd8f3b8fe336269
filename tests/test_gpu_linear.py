"""Tensor-core linear projection (Weight::linear, crates/tensor/src/ops/matmul.rs:4-110)
and the device-resident cross-attention K/V precompute built on it
(precompute_cross_attn, crates/whisper/src/decoder.rs:423-447) against the
oracle's restatement, on the same 16-bit-rounded inputs."""
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


def _check_linear(got, ref, out_dt, what):
    # f32 accumulation on both sides, in different orders: relative 2e-5 of
    # the largest output, plus half an output ulp when the output is 16-bit.
    bound = 2e-5 * float(np.abs(ref).max()) + (half_ulp(ref, out_dt) if out_dt else 0.0)
    err = np.abs(got - ref)
    assert (err <= bound + 1e-6).all(), f"{what}: max-abs {err.max()} vs bound {np.max(bound)}"


@pytest.mark.parametrize("dt", [1, 2], ids=["f16", "bf16"])
@pytest.mark.parametrize("out_dt", [0, 2], ids=["out_f32", "out_bf16"])
@pytest.mark.parametrize("mnk", [(300, 1280, 1280), (1500, 384, 384), (37, 200, 72), (129, 257, 64)],
                         ids=["large_v3", "tiny", "ragged", "edges"])
def test_linear_matches_oracle(W, oracle, dt, out_dt, mnk):
    import torch
    m, n, k = mnk
    xd, xf = rounded(randn(1 + m, m * k), dt)
    wd, wf = rounded(randn(2 + n, n * k), dt)
    bias = randn(3, n)
    y = torch.empty(m * n, dtype={0: torch.float32, 2: torch.bfloat16}[out_dt], device="cuda")
    W.linear_fwd(xd, wd, y, m=m, n=n, k=k, bias=torch.from_numpy(bias).cuda())
    torch.cuda.synchronize()
    ref = oracle.linear(xf, wf, bias, m, n, k)
    _check_linear(y.float().cpu().numpy(), ref, out_dt, f"linear {mnk}")


def test_linear_strided_rows(W, oracle):
    """x rows read from a wider buffer (the fused [T, 3d] QKV activations of
    encoder.rs:276), y written into every other column block."""
    import torch
    m, n, k = 200, 256, 128
    xd, xf = rounded(randn(7, m * 3 * k), 2)
    wd, wf = rounded(randn(8, n * k), 2)
    y = torch.zeros(m * 2 * n, device="cuda")
    W.linear_fwd(xd[k:], wd, y, m=m, n=n, k=k, x_row_stride=3 * k, y_row_stride=2 * n)
    torch.cuda.synchronize()
    ref = oracle.linear(np.ascontiguousarray(xf.reshape(m, 3 * k)[:, k:2 * k]), wf, None, m, n, k)
    got = y.view(m, 2 * n)
    _check_linear(got[:, :n].cpu().numpy().ravel(), ref, 0, "strided")
    assert (got[:, n:] == 0).all()


def test_cross_kv_project_feeds_decode(W, oracle):
    """precompute_cross_attn for one large-v3 layer on the device, then the
    beams' cross-attention over the projected K/V: the chain matches the
    oracle's projections followed by its attention."""
    import torch
    n_audio, d, g, h = 1500, 1280, 5, 20
    enc_d, enc_f = rounded(randn(20, n_audio * d), 1)
    wk_d, wk_f = rounded(randn(21, d * d) * 0.03, 1)
    wv_d, wv_f = rounded(randn(22, d * d) * 0.03, 1)
    bv = randn(23, d)
    k_out = torch.empty(n_audio * d, dtype=torch.float16, device="cuda")
    v_out = torch.empty_like(k_out)
    W.cross_kv_project(enc_d, wk_d, wv_d, torch.from_numpy(bv).cuda(), k_out, v_out,
                       n_tokens=n_audio, d_model=d)
    torch.cuda.synchronize()
    k_ref = oracle.linear(enc_f, wk_f, None, n_audio, d, d)
    v_ref = oracle.linear(enc_f, wv_f, bv, n_audio, d, d)
    _check_linear(k_out.float().cpu().numpy(), k_ref, 1, "K")
    _check_linear(v_out.float().cpu().numpy(), v_ref, 1, "V")
    # cross-attention of 5 beams over the projected (f16) K/V
    qd, qf = rounded(randn(24, g * d), 1)
    o = torch.empty(g * d, device="cuda")
    W.decode_fwd(qd, k_out, v_out, o, n_groups=1, group_size=g, t_kv=n_audio, n_heads=h,
                 scale=0.125)
    torch.cuda.synchronize()
    ref = oracle.decode_grouped(qf, k_out.float().cpu().numpy(), v_out.float().cpu().numpy(), 1, g,
                                n_audio, h, d)
    check_16bit(o.cpu().numpy(), ref, "decode over projected K/V")
