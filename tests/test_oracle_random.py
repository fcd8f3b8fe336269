"""The CPU oracle against float64 NumPy on seeded random shapes.

Every GPU parity test trusts the oracle; the golden vectors pin it on the
reference tests' own shapes, and this sweep checks it, as a second and
independent restatement, on the shapes the random GPU sweeps draw: the
flash_attention_2 tiling with ragged tiles and both masks
(attention.rs:68-242), multi_head_attention_with_cache at random offsets
(decoder.rs:835-892), the grouped single-token decode (attention.rs:246-434,
grouped as decoder.rs:688-724) and the projection (ops/matmul.rs:4-110),
each against a direct float64 computation. The bar is the reference's own
1e-5; the decode oracle's p < 1e-7 skip (attention.rs:366, 425) stays far
inside it at these sizes.
"""
import numpy as np
import pytest

N_CASES = 12


def _f64_attention(q, k, v, t_q, t_kv, n_heads, d_model, offset=None):
    """Softmax attention in float64; offset None: no mask, else query i sees
    keys j <= i + offset."""
    dh = d_model // n_heads
    Q = q.reshape(t_q, n_heads, dh).astype(np.float64)
    K = k.reshape(t_kv, n_heads, dh).astype(np.float64)
    V = v.reshape(t_kv, n_heads, dh).astype(np.float64)
    s = np.einsum("ihd,jhd->hij", Q, K) / np.sqrt(dh)
    if offset is not None:
        mask = np.arange(t_kv)[None, :] > (np.arange(t_q)[:, None] + offset)
        s = np.where(mask[None], -np.inf, s)
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("hij,jhd->ihd", p, V).reshape(t_q * d_model)


def _rng_arrays(seed, *sizes):
    g = np.random.default_rng(seed)
    return [g.standard_normal(n).astype(np.float32) for n in sizes]


@pytest.mark.parametrize("i", range(N_CASES))
def test_flash_attention_2_against_float64(oracle, i):
    r = np.random.default_rng(300 + i)
    t_q, t_kv = int(r.integers(1, 300)), int(r.integers(1, 400))
    h = int(r.integers(1, 5))
    d = h * 64
    causal = bool(i % 2)
    q, k, v = _rng_arrays(400 + i, t_q * d, t_kv * d, t_kv * d)
    out = oracle.flash_attention_2(q, k, v, t_q, t_kv, h, d, causal)
    ref = _f64_attention(q, k, v, t_q, t_kv, h, d, 0 if causal else None)
    assert np.abs(out - ref).max() <= 1e-5, (t_q, t_kv, h, causal)


@pytest.mark.parametrize("i", range(N_CASES))
def test_mha_with_cache_against_float64(oracle, i):
    r = np.random.default_rng(500 + i)
    n, t_past = int(r.integers(1, 40)), int(r.integers(0, 200))
    h = int(r.integers(1, 5))
    d = h * 64
    total = t_past + n
    q, k, v = _rng_arrays(600 + i, n * d, total * d, total * d)
    out = oracle.mha_with_cache(q, k, v, n, total, t_past, h, d)
    ref = _f64_attention(q, k, v, n, total, h, d, t_past)
    assert np.abs(out - ref).max() <= 1e-5, (n, t_past, h)


@pytest.mark.parametrize("i", range(N_CASES))
def test_decode_grouped_against_float64(oracle, i):
    r = np.random.default_rng(700 + i)
    ng, g, t_kv = int(r.integers(1, 5)), int(r.integers(1, 9)), int(r.integers(1, 500))
    h = int(r.integers(1, 5))
    d = h * 64
    q, k, v = _rng_arrays(800 + i, ng * g * d, ng * t_kv * d, ng * t_kv * d)
    out = oracle.decode_grouped(q, k, v, ng, g, t_kv, h, d).reshape(ng, g * d)
    for grp in range(ng):
        ref = np.concatenate([
            _f64_attention(q[(grp * g + row) * d:(grp * g + row + 1) * d],
                           k[grp * t_kv * d:(grp + 1) * t_kv * d],
                           v[grp * t_kv * d:(grp + 1) * t_kv * d], 1, t_kv, h, d)
            for row in range(g)])
        assert np.abs(out[grp] - ref).max() <= 1e-5, (ng, g, t_kv, h)


@pytest.mark.parametrize("i", range(N_CASES))
def test_linear_against_float64(oracle, i):
    r = np.random.default_rng(900 + i)
    m, n, k = int(r.integers(1, 200)), int(r.integers(1, 200)), int(r.integers(1, 300))
    x, w, b = _rng_arrays(1000 + i, m * k, n * k, n)
    bias = b if i % 2 else None
    out = oracle.linear(x, w, bias, m, n, k)
    ref = x.reshape(m, k).astype(np.float64) @ w.reshape(n, k).astype(np.float64).T
    if bias is not None:
        ref += bias.astype(np.float64)
    # f32 dot products of length k: relative to the magnitude of the terms
    tol = 1e-6 * np.sqrt(k) * 4 + 1e-6
    assert np.abs(out.reshape(m, n) - ref).max() <= tol, (m, n, k)
