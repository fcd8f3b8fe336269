"""Generates the committed golden vectors of tests/golden/.

The reference (Rust) cannot be built in this environment, so the vectors pin
the reference's own known-answer tests instead:

* inputs are produced exactly as crates/tensor/tests/test_flash_attention_tiled.rs
  produces them (xorshift32 -> U[-1,1), seeds from :95, :192, :214, :252) and as
  crates/tensor/tests/test_flash_attention.rs:10-23 produces its pattern inputs;
* expected outputs come from the reference tests' own checker,
  `reference_materialized` (test_flash_attention_tiled.rs:41-89) and
  `reference_mha` (test_flash_attention.rs:99-143), restated in oracle/, and
  are cross-checked here against float64 torch attention.

Run from the repository root: python tests/golden/gen_golden.py
"""
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

OUT = os.path.join(ROOT, "tests", "golden", "kat_attention.npz")

# (name, t_q, t_kv, n_heads, d_head, causal, seed or None = KAT seed rule)
CASES = [
    ("d64_noncausal", 100, 137, 3, 64, False, None),      # test_flash_attention_tiled.rs:133-137
    ("d64_causal", 100, 137, 3, 64, True, None),          # :139-142
    ("d80_noncausal", 37, 91, 2, 80, False, None),        # :144-147
    ("d80_causal", 37, 91, 2, 80, True, None),            # :149-152
    ("tile_p1_noncausal", 129, 129, 2, 64, False, None),  # :155-163
    ("tile_p1_causal", 129, 129, 2, 64, True, None),
    ("tile_2p_noncausal", 259, 261, 4, 64, False, None),
    ("tile_2p_causal", 259, 261, 4, 64, True, None),
    ("fewer_keys_causal_a", 90, 33, 3, 64, True, None),   # :166-172
    ("fewer_keys_causal_b", 168, 37, 3, 64, True, None),
    ("decode_d64", 1, 257, 4, 64, False, None),           # :174-178
    ("decode_d80", 1, 193, 2, 80, False, None),           # :180-184
    ("causal_single_query", 1, 17, 1, 64, True, 0xFEEDFACE),   # :186-205
    ("mha_48x70", 48, 70, 5, 64, False, 0x0BADC0DE),      # :207-241
    ("stale_output_causal", 40, 100, 2, 64, True, 0xDEADBEEF),  # :243-263
]


def inputs(t_q, t_kv, n_heads, d_head, seed):
    if seed is None:
        return O.kat_inputs(t_q, t_kv, n_heads, d_head)
    rng = O.XorShift(seed)
    d_model = n_heads * d_head
    return rng.fill(t_q * d_model), rng.fill(t_kv * d_model), rng.fill(t_kv * d_model)


def pattern_inputs():
    """test_flash_attention.rs:6-23 (t_q 64, t_kv 128, 4 heads, d_model 64)."""
    t_q, t_kv, d_model = 64, 128, 64
    q = np.array([((i % 17) - 8.0) * 0.1 for i in range(t_q * d_model)], np.float32)
    k = np.array([((i % 19) - 9.0) * 0.1 for i in range(t_kv * d_model)], np.float32)
    v = np.array([((i % 23) - 11.0) * 0.1 for i in range(t_kv * d_model)], np.float32)
    return q, k, v


def f64_attention(q, k, v, t_q, t_kv, n_heads, d_model, causal):
    dh = d_model // n_heads
    Q = q.astype(np.float64).reshape(t_q, n_heads, dh).transpose(1, 0, 2)
    K = k.astype(np.float64).reshape(t_kv, n_heads, dh).transpose(1, 0, 2)
    V = v.astype(np.float64).reshape(t_kv, n_heads, dh).transpose(1, 0, 2)
    S = Q @ K.transpose(0, 2, 1) / np.sqrt(dh)
    if causal:
        S = np.where(np.arange(t_kv)[None, None, :] > np.arange(t_q)[None, :, None], -np.inf, S)
    S = S - S.max(-1, keepdims=True)
    P = np.exp(S)
    P /= P.sum(-1, keepdims=True)
    return (P @ V).transpose(1, 0, 2).reshape(-1)


def main():
    O.build()
    blobs = {}
    for name, t_q, t_kv, n_heads, d_head, causal, seed in CASES:
        q, k, v = inputs(t_q, t_kv, n_heads, d_head, seed)
        d_model = n_heads * d_head
        out = O.materialized(q, k, v, t_q, t_kv, n_heads, d_model, causal)
        err = np.abs(out - f64_attention(q, k, v, t_q, t_kv, n_heads, d_model, causal)).max()
        assert err < 1e-6, (name, err)
        digest = hashlib.sha256(q.tobytes() + k.tobytes() + v.tobytes()).hexdigest()
        blobs[f"{name}/meta"] = np.array([t_q, t_kv, n_heads, d_head, int(causal),
                                          -1 if seed is None else seed], np.int64)
        blobs[f"{name}/sha256"] = np.frombuffer(bytes.fromhex(digest), np.uint8)
        blobs[f"{name}/out"] = out
    q, k, v = pattern_inputs()
    for causal in (False, True):
        out = O.materialized(q, k, v, 64, 128, 4, 64, causal)
        blobs[f"pattern_{'causal' if causal else 'noncausal'}/out"] = out
        blobs[f"pattern_{'causal' if causal else 'noncausal'}/meta"] = np.array(
            [64, 128, 4, 16, int(causal), -2], np.int64)
    np.savez_compressed(OUT, **blobs)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(CASES) + 2} cases)")


if __name__ == "__main__":
    main()
