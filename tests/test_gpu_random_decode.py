"""A seeded random sweep of decode calls (wattn_decode_fwd) against the CPU
oracle.

The hand-picked decode cases use one type for q and K/V and a few fixed
shapes; this sweep draws, from a fixed seed, the combinations they leave
out: q, K/V and output types chosen independently (matching 16-bit q and K/V
take the streaming tensor-core kernel, everything else the CUDA-core one),
1-40 groups of 1-16 query rows (the beams of an utterance), 1-4000 keys
(log-uniform: single keys, ragged sub-tiles and key splits all come up),
1-20 heads, and padded strides: q and output rows wider than the heads,
K/V rows wider than the heads and groups separated by gap rows. The padding
and the gap rows of q, K and V hold NaN (a read outside the attended rows
and columns would show in the result); the output padding holds a sentinel
that must survive. Half of the calls pass their own zeroed workspace, half
use the library's. Tolerances are the other decode tests': max-abs 1e-5
when q, K and V are all f32 (single_token_mha_d64's f32 arithmetic,
attention.rs:246-434), otherwise 2e-3 with cosine > 0.9999 (plus half an
output ulp for a 16-bit output).
"""
import numpy as np
import pytest

from tests.helpers import check_16bit, check_f32, rounded

pytestmark = pytest.mark.gpu

N_CASES = 60
SENTINEL = 3.0


def _draw(i):
    r = np.random.default_rng(9100 + i)
    q_dt, kv_dt, out_dt = (int(x) for x in r.integers(0, 3, size=3))
    if r.random() < 0.4:  # matching 16-bit q and K/V: the streaming kernel
        kv_dt = int(r.integers(1, 3))
        q_dt = kv_dt
    n_groups = int(np.exp(r.uniform(0, np.log(40))))
    g = int(r.integers(1, 17))
    t_kv = int(np.exp(r.uniform(0, np.log(4000))))
    heads = int(r.integers(1, 21))
    while n_groups * heads * t_kv > 1.2e7 and n_groups > 1:  # keeps the oracle's share short
        n_groups -= 1
    return dict(q_dt=q_dt, kv_dt=kv_dt, out_dt=out_dt, n_groups=n_groups, g=g, t_kv=t_kv,
                heads=heads, q_pad=int(r.choice([0, 8, 64])), kv_pad=int(r.choice([0, 8, 64])),
                gap=int(r.choice([0, 3])), o_pad=int(r.choice([0, 8])),
                own_ws=bool(r.random() < 0.5), seed=9100 + i)


CASES = [_draw(i) for i in range(N_CASES)]


def _id(c):
    n = "f32 f16 bf16".split()
    return (f"q{n[c['q_dt']]}-kv{n[c['kv_dt']]}-o{n[c['out_dt']]}-"
            f"{c['n_groups']}x{c['g']}-t{c['t_kv']}-h{c['heads']}")


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


@pytest.mark.parametrize("c", CASES, ids=[_id(c) for c in CASES])
def test_random_decode_call(W, oracle, c):
    import torch
    tdt = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}
    ng, g, t_kv, h = c["n_groups"], c["g"], c["t_kv"], c["heads"]
    w = h * 64
    q_rs, kv_rs, o_rs = w + c["q_pad"], w + c["kv_pad"], w + c["o_pad"]
    kv_gs = (t_kv + c["gap"]) * kv_rs
    rng = np.random.default_rng(c["seed"])
    qd, qf = rounded(rng.standard_normal(ng * g * w).astype(np.float32), c["q_dt"])
    kd, kf = rounded(rng.standard_normal(ng * t_kv * w).astype(np.float32), c["kv_dt"])
    vd, vf = rounded(rng.standard_normal(ng * t_kv * w).astype(np.float32), c["kv_dt"])
    q = torch.full((ng * g, q_rs), float("nan"), dtype=tdt[c["q_dt"]], device="cuda")
    q[:, :w] = qd.view(ng * g, w)
    k = torch.full((ng, t_kv + c["gap"], kv_rs), float("nan"), dtype=tdt[c["kv_dt"]], device="cuda")
    v = torch.full_like(k, float("nan"))
    k[:, :t_kv, :w] = kd.view(ng, t_kv, w)
    v[:, :t_kv, :w] = vd.view(ng, t_kv, w)
    o = torch.full((ng * g, o_rs), SENTINEL, dtype=tdt[c["out_dt"]], device="cuda")
    ws = None
    if c["own_ws"]:
        ws = torch.zeros(max(1, W.decode_workspace_bytes(ng, g, t_kv, h)), dtype=torch.uint8,
                         device="cuda")
    W.decode_fwd(q.view(-1), k.view(-1), v.view(-1), o.view(-1), n_groups=ng, group_size=g,
                 t_kv=t_kv, n_heads=h, scale=0.125, q_row_stride=q_rs, kv_row_stride=kv_rs,
                 kv_group_stride=kv_gs, o_row_stride=o_rs, workspace=ws)
    torch.cuda.synchronize()
    assert W.device_status() == 0
    out = o.float().cpu().numpy()
    ref = oracle.decode_grouped(qf, kf, vf, ng, g, t_kv, h, w)
    if c["q_dt"] == 0 and c["kv_dt"] == 0 and c["out_dt"] == 0:
        check_f32(out[:, :w], ref, _id(c))
    else:
        check_16bit(out[:, :w], ref, _id(c), c["out_dt"])
    assert np.all(out[:, w:] == SENTINEL), "output padding columns written"
