"""A seeded random sweep of the tensor-core projection (wattn_linear_fwd,
Weight::linear, crates/tensor/src/ops/matmul.rs:4-110) against the oracle.

The fixed cases use Whisper's widths; the entry point accepts any m, n and
k (x and W rows need only 16-byte aligned strides, y rows only their element
size), so this sweep draws, from a fixed seed: 1-2500 rows, 1-1500 outputs
and 1-1500 inputs (log-uniform: k below one 64-wide K tile, ragged K, M and
N tiles and single rows all come up), f16 or bf16 inputs, f32, f16 or bf16
outputs, with or without a bias, and row strides with padding: the padding
of x and W holds NaN (a read past k would show), the padding of y a sentinel
that must survive (odd y strides take the epilogue's element-wise stores).
Tolerance as in the fixed linear tests: both sides accumulate in f32 in
different orders, 2e-5 of the largest output, plus half an output ulp for a
16-bit output.
"""
import numpy as np
import pytest

from tests.helpers import half_ulp, rounded

pytestmark = pytest.mark.gpu

N_CASES = 40
SENTINEL = 9.0


def _draw(i):
    r = np.random.default_rng(9500 + i)
    m = int(np.exp(r.uniform(0, np.log(2500))))
    n = int(np.exp(r.uniform(0, np.log(1500))))
    k = int(np.exp(r.uniform(0, np.log(1500))))
    k8 = (k + 7) // 8 * 8
    return dict(m=m, n=n, k=k, dt=int(r.integers(1, 3)), out_dt=int(r.integers(0, 3)),
                bias=bool(r.random() < 0.6), x_rs=k8 + 8 * int(r.integers(0, 3)),
                w_rs=k8 + 8 * int(r.integers(0, 3)), y_rs=n + int(r.integers(0, 10)),
                seed=9500 + i)


CASES = [_draw(i) for i in range(N_CASES)]


def _id(c):
    n = "f32 f16 bf16".split()
    return f"{n[c['dt']]}-o{n[c['out_dt']]}-{c['m']}x{c['n']}x{c['k']}{'-bias' if c['bias'] else ''}"


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


@pytest.mark.parametrize("c", CASES, ids=[_id(c) for c in CASES])
def test_random_linear_call(W, oracle, c):
    import torch
    tdt = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}
    m, n, k = c["m"], c["n"], c["k"]
    g = np.random.default_rng(c["seed"])
    xd, xf = rounded(g.standard_normal(m * k).astype(np.float32), c["dt"])
    wd, wf = rounded(g.standard_normal(n * k).astype(np.float32), c["dt"])
    bias = g.standard_normal(n).astype(np.float32) if c["bias"] else None
    x = torch.full((m, c["x_rs"]), float("nan"), dtype=tdt[c["dt"]], device="cuda")
    x[:, :k] = xd.view(m, k)
    w = torch.full((n, c["w_rs"]), float("nan"), dtype=tdt[c["dt"]], device="cuda")
    w[:, :k] = wd.view(n, k)
    y = torch.full((m, c["y_rs"]), SENTINEL, dtype=tdt[c["out_dt"]], device="cuda")
    W.linear_fwd(x.view(-1), w.view(-1), y.view(-1), m=m, n=n, k=k,
                 bias=torch.from_numpy(bias).cuda() if bias is not None else None,
                 x_row_stride=c["x_rs"], w_row_stride=c["w_rs"], y_row_stride=c["y_rs"])
    torch.cuda.synchronize()
    assert W.device_status() == 0
    got = y.float().cpu().numpy()
    ref = oracle.linear(xf, wf, bias, m, n, k).reshape(m, n)
    bound = 2e-5 * float(np.abs(ref).max()) + (half_ulp(ref, c["out_dt"]) if c["out_dt"] else 0.0)
    err = np.abs(got[:, :n] - ref)
    assert np.all(np.isfinite(got[:, :n])), _id(c)
    assert (err <= bound + 1e-6).all(), f"{_id(c)}: max-abs {err.max()} vs bound {np.max(bound)}"
    assert np.all(got[:, n:] == SENTINEL), "y padding columns written"
