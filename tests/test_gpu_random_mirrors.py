"""A seeded random sweep of the host-buffer entry points against the oracle.

The reference-signature mirrors (wattn_flash_attention_2 / _multi_head_attention,
attention.rs:68 / :29; wattn_single_token_mha_d64, attention.rs:246;
wattn_multi_head_attention_with_cache, decoder.rs:835) are what a
whisper.rs build binds in place of its own functions: f32 host slices in the
reference layout, results at the reference's own bar (max-abs 1e-5). The
golden vectors and fixed cases check them on the reference tests' shapes;
these calls draw, from a fixed seed, 1-8 heads, 1-1500 queries and keys
(log-uniform, so the single-query dispatch to the decode kernel,
attention.rs:102-104, comes up), causal or not, and decoder-cache calls of
1-50 new tokens after 0-600 cached ones. The batched host-buffer call
(wattn_attention_host: chunks over two streams with the copies inside) is
drawn the same way in every input type.
"""
import numpy as np
import pytest

from tests.helpers import check_16bit, check_f32

pytestmark = pytest.mark.gpu

N_MIRROR = 40
N_HOST = 12


def _log_uniform(r, hi):
    return int(np.exp(r.uniform(0, np.log(hi))))


def _draw_mirror(i):
    r = np.random.default_rng(9300 + i)
    fn = ["flash_attention_2", "multi_head_attention", "single_token_mha_d64",
          "multi_head_attention_with_cache"][i % 4]
    h = int(r.integers(1, 9))
    c = dict(fn=fn, h=h, seed=9300 + i, causal=bool(r.random() < 0.5))
    if fn == "multi_head_attention_with_cache":
        c.update(n=_log_uniform(r, 50), t_past=int(r.integers(0, 601)))
    else:
        c.update(t_q=1 if fn == "single_token_mha_d64" or r.random() < 0.2 else _log_uniform(r, 1500),
                 t_kv=_log_uniform(r, 1500))
    return c


def _draw_host(i):
    r = np.random.default_rng(9400 + i)
    dt = i % 3
    return dict(dt=dt, out_dt=0 if dt == 0 or r.random() < 0.5 else dt, b=int(r.integers(1, 4)),
                h=int(r.integers(1, 9)), t_q=_log_uniform(r, 1500), t_kv=_log_uniform(r, 1500),
                causal=bool(r.random() < 0.3), pinned=bool(r.random() < 0.5), seed=9400 + i)


MIRRORS = [_draw_mirror(i) for i in range(N_MIRROR)]
HOSTS = [_draw_host(i) for i in range(N_HOST)]


def _mid(c):
    if "n" in c:
        return f"{c['fn']}-h{c['h']}-n{c['n']}-past{c['t_past']}"
    return f"{c['fn']}-h{c['h']}-{c['t_q']}x{c['t_kv']}{'-causal' if c['causal'] else ''}"


def _hid(c):
    n = "f32 f16 bf16".split()
    return (f"{n[c['dt']]}-o{n[c['out_dt']]}-b{c['b']}h{c['h']}-{c['t_q']}x{c['t_kv']}"
            f"{'-causal' if c['causal'] else ''}{'-pinned' if c['pinned'] else ''}")


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


@pytest.mark.parametrize("c", MIRRORS, ids=[_mid(c) for c in MIRRORS])
def test_random_reference_mirror(W, oracle, c):
    g = np.random.default_rng(c["seed"])
    h = c["h"]
    d = h * 64
    f32 = lambda n: g.standard_normal(n).astype(np.float32)  # noqa: E731
    if c["fn"] == "multi_head_attention_with_cache":
        n, t_past = c["n"], c["t_past"]
        total = t_past + n
        q, k, v = f32(n * d), f32(total * d), f32(total * d)
        out = np.full(n * d, np.nan, np.float32)
        W.multi_head_attention_with_cache(q, k, v, n, total, t_past, h, d, out)
        ref = oracle.mha_with_cache(q, k, v, n, total, t_past, h, d)
    elif c["fn"] == "single_token_mha_d64":
        t_kv = c["t_kv"]
        q, k, v = f32(d), f32(t_kv * d), f32(t_kv * d)
        out = np.full(d, np.nan, np.float32)
        W.single_token_mha_d64(q, k, v, t_kv, h, d, out)
        ref = oracle.single_token_mha_d64(q, k, v, t_kv, h, d)
    else:
        t_q, t_kv, causal = c["t_q"], c["t_kv"], c["causal"]
        q, k, v = f32(t_q * d), f32(t_kv * d), f32(t_kv * d)
        out = np.full(t_q * d, np.nan, np.float32)
        getattr(W, c["fn"])(q, k, v, t_q, t_kv, h, d, causal, out)
        ref = oracle.flash_attention_2(q, k, v, t_q, t_kv, h, d, causal)
    check_f32(out, ref, _mid(c))


@pytest.mark.parametrize("c", HOSTS, ids=[_hid(c) for c in HOSTS])
def test_random_attention_host(W, oracle, c):
    import torch
    tdt = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}
    b, h, t_q, t_kv = c["b"], c["h"], c["t_q"], c["t_kv"]
    d = h * 64
    g = np.random.default_rng(c["seed"])
    mk = lambda n: torch.from_numpy(g.standard_normal(n).astype(np.float32)).to(tdt[c["dt"]])  # noqa: E731
    q, k, v = mk(b * t_q * d), mk(b * t_kv * d), mk(b * t_kv * d)
    o = torch.full((b * t_q * d,), float("nan"), dtype=tdt[c["out_dt"]])
    if c["pinned"]:
        q, k, v, o = (x.pin_memory() for x in (q, k, v, o))
    W.attention_host(q, k, v, o, b, t_q, t_kv, h, 0.125, causal=c["causal"])
    ref = oracle.flash_attention_2_batched(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                           b, t_q, t_kv, h, d, c["causal"])
    got = o.float().numpy()
    if c["dt"] == 0:
        check_f32(got, ref, _hid(c))
    else:
        check_16bit(got, ref, _hid(c), c["out_dt"])
