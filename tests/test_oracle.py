"""CPU oracle pinned against the reference's own known-answer tests.

The golden vectors (tests/golden/kat_attention.npz, made by gen_golden.py)
hold the outputs of the reference tests' checker on the reference tests' own
inputs; the oracle's restatement of flash_attention_2 must match them within
the reference's tolerance (1e-5, test_flash_attention_tiled.rs:123-130).
"""
import hashlib
import os

import numpy as np
import pytest

from tests.helpers import TOL_F32_MAXABS, randn

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kat_attention.npz")


def _cases():
    z = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in z.files})
    return z, names


def _inputs(O, name, meta):
    t_q, t_kv, n_heads, d_head, causal, seed = (int(x) for x in meta)
    if seed == -2:  # test_flash_attention.rs:10-23 pattern inputs
        d_model = 64
        q = np.array([((i % 17) - 8.0) * 0.1 for i in range(t_q * d_model)], np.float32)
        k = np.array([((i % 19) - 9.0) * 0.1 for i in range(t_kv * d_model)], np.float32)
        v = np.array([((i % 23) - 11.0) * 0.1 for i in range(t_kv * d_model)], np.float32)
        return q, k, v
    if seed == -1:
        return O.kat_inputs(t_q, t_kv, n_heads, d_head)
    rng = O.XorShift(seed)
    d_model = n_heads * d_head
    return rng.fill(t_q * d_model), rng.fill(t_kv * d_model), rng.fill(t_kv * d_model)


def test_xorshift_matches_reference_generator(oracle):
    # The C generator and a direct numpy transcription of
    # test_flash_attention_tiled.rs:22-30 agree bit for bit.
    for seed in (0x12345678, 0xFEEDFACE, 1):
        assert np.array_equal(oracle.XorShift(seed).fill(300), oracle.xorshift_f32_numpy(seed, 300))


def test_golden_inputs_reproduce(oracle):
    z, names = _cases()
    for name in names:
        if f"{name}/sha256" not in z.files:
            continue
        q, k, v = _inputs(oracle, name, z[f"{name}/meta"])
        digest = hashlib.sha256(q.tobytes() + k.tobytes() + v.tobytes()).digest()
        assert digest == z[f"{name}/sha256"].tobytes(), name


def test_oracle_flash_attention_2_matches_golden(oracle):
    z, names = _cases()
    for name in names:
        meta = z[f"{name}/meta"]
        t_q, t_kv, n_heads, d_head, causal, _ = (int(x) for x in meta)
        q, k, v = _inputs(oracle, name, meta)
        out = oracle.flash_attention_2(q, k, v, t_q, t_kv, n_heads, n_heads * d_head, causal)
        tol = 1e-4 if name.startswith("pattern") else TOL_F32_MAXABS
        err = np.abs(out - z[f"{name}/out"]).max()
        assert err <= tol, (name, err)


def test_causal_single_query_returns_first_value(oracle):
    # test_flash_attention_tiled.rs:186-205
    rng = oracle.XorShift(0xFEEDFACE)
    q, k, v = rng.fill(64), rng.fill(17 * 64), rng.fill(17 * 64)
    out = oracle.flash_attention_2(q, k, v, 1, 17, 1, 64, True)
    assert np.abs(out - v[:64]).max() <= 1e-6


def test_single_token_twins_agree(oracle):
    # AVX2-order and scalar restatements of attention.rs:293-434 both meet 1e-5.
    q, k, v = oracle.kat_inputs(1, 257, 4, 64)
    ref = oracle.materialized(q, k, v, 1, 257, 4, 256, False)
    a = oracle.single_token_mha_d64(q, k, v, 257, 4, 256)
    b = oracle.single_token_mha_d64(q, k, v, 257, 4, 256, scalar=True)
    assert np.abs(a - ref).max() <= TOL_F32_MAXABS
    assert np.abs(b - ref).max() <= TOL_F32_MAXABS


@pytest.mark.parametrize("t_past,n_tokens", [(0, 1), (5, 1), (10, 3), (0, 7), (40, 9)])
def test_mha_with_cache_is_offset_causal(oracle, t_past, n_tokens):
    # decoder.rs:835-892: query i sees keys 0..=t_past+i. Equal to the
    # materialized causal attention of the full prefix, restricted to the last
    # n_tokens rows.
    n_heads, d_model = 2, 128
    total = t_past + n_tokens
    kq = randn(1, total * d_model)
    k, v = randn(2, total * d_model), randn(3, total * d_model)
    full = oracle.materialized(kq, k, v, total, total, n_heads, d_model, True)
    q = kq[t_past * d_model:]
    out = oracle.mha_with_cache(q, k, v, n_tokens, total, t_past, n_heads, d_model)
    # random N(0,1) rows are far from the 1e-7 skip threshold at this length
    assert np.abs(out - full[t_past * d_model:]).max() <= 1e-5


def test_decode_grouped_matches_per_row(oracle):
    n_groups, g, t_kv, n_heads = 3, 5, 300, 2
    d = n_heads * 64
    q = randn(4, n_groups * g * d)
    k, v = randn(5, n_groups * t_kv * d), randn(6, n_groups * t_kv * d)
    out = oracle.decode_grouped(q, k, v, n_groups, g, t_kv, n_heads, d)
    for r in range(n_groups * g):
        gi = r // g
        ref = oracle.materialized(q[r * d:(r + 1) * d], k[gi * t_kv * d:(gi + 1) * t_kv * d],
                                  v[gi * t_kv * d:(gi + 1) * t_kv * d], 1, t_kv, n_heads, d, False)
        assert np.abs(out[r * d:(r + 1) * d] - ref).max() <= 1e-5


def test_oracle_matches_float64_random(oracle):
    from tests.golden.gen_golden import f64_attention
    for (t_q, t_kv, causal) in ((300, 517, False), (300, 517, True), (1500, 1500, False)):
        n_heads, d = 2, 128
        q, k, v = randn(7, t_q * d), randn(8, t_kv * d), randn(9, t_kv * d)
        out = oracle.flash_attention_2(q, k, v, t_q, t_kv, n_heads, d, causal)
        assert np.abs(out - f64_attention(q, k, v, t_q, t_kv, n_heads, d, causal)).max() <= 2e-6


def test_oracle_edge_cases(oracle):
    q = randn(1, 4 * 128)
    # t_kv == 0 -> zeros (attention.rs:93-96)
    out = oracle.flash_attention_2(q, np.zeros(0, np.float32), np.zeros(0, np.float32), 4, 0, 2, 128,
                                   False)
    assert np.all(out == 0)
    # argument errors the reference asserts on (attention.rs:79-84)
    with pytest.raises(ValueError):
        oracle.flash_attention_2(q, q, q, 4, 4, 0, 128, False)
    with pytest.raises(ValueError):
        oracle.flash_attention_2(q, q, q, 4, 4, 3, 128, False)


def test_softmax_inplace(oracle):
    x = randn(10, 33)
    y = oracle.softmax_inplace(x)
    e = np.exp(x.astype(np.float64) - x.max())
    assert np.abs(y - e / e.sum()).max() < 1e-7


def test_capture_heads_is_the_softmax_of_the_scaled_dots(oracle):
    """capture_cross_attention_heads (decoder.rs:796-828): each captured row is
    softmax_j(q . k_j / sqrt(d_head)) of the selected head, laid out
    [row][slot][n_audio]; unselected slots are left alone. Checked against a
    float64 evaluation of that formula."""
    rng = np.random.default_rng(5)
    n_tokens, n_audio, n_heads, d_head = 3, 257, 4, 64
    d = n_heads * d_head
    q = rng.standard_normal(n_tokens * d).astype(np.float32)
    k = rng.standard_normal(n_audio * d).astype(np.float32)
    selected, n_selected, row_offset = [(2, 3), (0, 1)], 3, 1
    out = np.full((row_offset + n_tokens) * n_selected * n_audio, -1.0, np.float32)
    oracle.capture_heads(q, k, n_tokens, n_audio, n_heads, d, selected, n_selected, row_offset, out)
    out = out.reshape(-1, n_selected, n_audio)
    q64 = q.reshape(n_tokens, n_heads, d_head).astype(np.float64)
    k64 = k.reshape(n_audio, n_heads, d_head).astype(np.float64)
    for slot, head in selected:
        s = q64[:, head] @ k64[:, head].T / np.sqrt(d_head)
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        assert np.abs(out[row_offset:, slot] - p).max() < 1e-6
    assert (out[:, 1] == -1.0).all() and (out[0] == -1.0).all()

