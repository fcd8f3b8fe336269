"""A seeded random sweep of attention calls against the CPU oracle.

The hand-picked cases elsewhere cover the shapes whisper.rs runs and the
edges found while building the kernels; this sweep draws the combinations
those do not list, from a fixed seed so every run checks the same cases:
each input type (f32: split-f16 products on the tensor cores; f16 and bf16:
the tcgen05 kernel, bf16 with V's f16 copy), 1-4 utterances, 1-8 heads,
1-1500 queries and 1-1600 keys (log-uniform, so single rows and ragged last
tiles come up often), no mask, the causal mask of the encoder-style call
(query i sees keys j <= i, attention.rs:161-165) or the decoder prefill's
(query i at position t_kv - t_q + i, decoder.rs:864), and row strides with
padding columns. The padding of Q, K and V holds NaN, so a read outside a
head's 64 columns would show in the result; the padding of the output holds
a sentinel that must survive. Tolerances are the other tests': max-abs 1e-5
for f32 inputs, 2e-3 with cosine > 0.9999 for 16-bit inputs (plus half an
output ulp when the output itself is 16-bit).
"""
import numpy as np
import pytest

from tests.helpers import check_16bit, check_f32, rounded

pytestmark = pytest.mark.gpu

N_CASES = 90
SENTINEL = 5.0


def _draw(i):
    r = np.random.default_rng(7000 + i)
    dt = i % 3                                   # F32, F16, BF16 in turn
    out_dt = 0 if dt == 0 or r.random() < 0.5 else dt
    batch = int(r.integers(1, 5))
    heads = int(r.integers(1, 9 if dt else 5))
    t_q = int(np.exp(r.uniform(0, np.log(1500))))
    t_kv = int(np.exp(r.uniform(0, np.log(1600))))
    while batch * heads * t_q * t_kv > 2.5e7 and batch > 1:  # keeps the oracle's share short
        batch -= 1
    mode = ["none", "causal", "prefill"][int(r.integers(0, 3))]
    if mode == "prefill" and t_kv < t_q:
        t_q, t_kv = t_kv, t_q
    # padding columns per row, a multiple of 16 bytes for every type
    pad_in = int(r.choice([0, 8, 64]))
    pad_out = int(r.choice([0, 8, 64]))
    return dict(dt=dt, out_dt=out_dt, batch=batch, heads=heads, t_q=t_q, t_kv=t_kv, mode=mode,
                pad_in=pad_in, pad_out=pad_out, seed=7000 + i)


CASES = [_draw(i) for i in range(N_CASES)]


def _id(c):
    return (f"{'f32 f16 bf16'.split()[c['dt']]}-b{c['batch']}h{c['heads']}-"
            f"{c['t_q']}x{c['t_kv']}-{c['mode']}")


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


def _padded(x, rows, w, rs, dtype, device):
    """[rows][w] values in [rows][rs] rows whose padding holds NaN."""
    import torch
    t = torch.full((rows, rs), float("nan"), dtype=dtype, device=device)
    t[:, :w] = x.reshape(rows, w).to(device)
    return t.reshape(-1)


@pytest.mark.parametrize("c", CASES, ids=[_id(c) for c in CASES])
def test_random_attention_call(W, oracle, c):
    import torch
    tdt = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}
    b, h, t_q, t_kv, dt = c["batch"], c["heads"], c["t_q"], c["t_kv"], c["dt"]
    w = h * 64
    rs_in, rs_out = w + c["pad_in"], w + c["pad_out"]
    g = np.random.default_rng(c["seed"])
    q = [rounded(g.standard_normal(t_q * w).astype(np.float32), dt) for _ in range(b)]
    k = [rounded(g.standard_normal(t_kv * w).astype(np.float32), dt) for _ in range(b)]
    v = [rounded(g.standard_normal(t_kv * w).astype(np.float32), dt) for _ in range(b)]
    dq = _padded(torch.cat([x[0].cpu() for x in q]), b * t_q, w, rs_in, tdt[dt], "cuda")
    dk = _padded(torch.cat([x[0].cpu() for x in k]), b * t_kv, w, rs_in, tdt[dt], "cuda")
    dv = _padded(torch.cat([x[0].cpu() for x in v]), b * t_kv, w, rs_in, tdt[dt], "cuda")
    o = torch.full((b * t_q * rs_out,), SENTINEL, dtype=tdt[c["out_dt"]], device="cuda")
    causal = c["mode"] != "none"
    offset = t_kv - t_q if c["mode"] == "prefill" else 0
    W.attention_fwd(dq, dk, dv, o, batch=b, t_q=t_q, t_kv=t_kv, n_heads=h, scale=0.125,
                    causal=causal, q_pos_offset=offset, q_row_stride=rs_in, kv_row_stride=rs_in,
                    o_row_stride=rs_out)
    torch.cuda.synchronize()
    assert W.device_status() == 0
    out = o.float().cpu().numpy().reshape(b, t_q, rs_out)
    for u in range(b):
        qf, kf, vf = q[u][1], k[u][1], v[u][1]
        if c["mode"] == "prefill":
            ref = oracle.mha_with_cache(qf, kf, vf, t_q, t_kv, offset, h, w)
        else:
            ref = oracle.flash_attention_2(qf, kf, vf, t_q, t_kv, h, w, causal)
        what = f"{_id(c)} utterance {u}"
        if dt == 0:
            check_f32(out[u, :, :w], ref, what)
        else:
            check_16bit(out[u, :, :w], ref, what, c["out_dt"])
    assert np.all(out[:, :, w:] == SENTINEL), "output padding columns written"
