"""Seeded random histories of the device paged KV cache against the host
DecoderKvCache model and the causal attention oracle (decoder.rs:131-264,
616-647, 835-892).

The scripted history in test_gpu_kv_cache.py follows one beam search; these
draw, from fixed seeds, sequences of the operations whisper.rs's decoder
issues in other orders: batched steps over random subsets of slots with one
token or a prefill of up to 40 (made to fit by slide_to_fit first, as the
decoder does, decoder.rs:248-263), forks (copy_slot, shared pages and copy
on write), rewinds (the C API's n_past, crates/ffi/src/lib.rs:2352), slot
clears and slides, for every cache type (f32 on the CUDA-core kernel, f16
and bf16 on the streaming tensor-core kernel), with random head counts,
context limits and page sizes. After every operation the device rows must
equal the model's (bit-exact) and every attention output must match the
oracle (max-abs 1e-5 for f32, 2e-3 with cosine > 0.9999 for 16-bit).
"""
import numpy as np
import pytest

from tests.test_gpu_kv_cache import Harness

pytestmark = pytest.mark.gpu

N_HISTORIES = 15
N_OPS = 40


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


def _make_room(h, slot, n, max_ctx):
    if h.ref.t_past[slot] + n > max_ctx:
        assert h.dev.slide_to_fit(slot, n, max_ctx) == h.ref.slide_to_fit(slot, n, max_ctx)


@pytest.mark.parametrize("seed", range(N_HISTORIES))
def test_random_cache_history(W, oracle, seed):
    r = np.random.default_rng(8200 + seed)
    dtype = seed % 3
    n_slots = int(r.integers(2, 7))
    heads = int(r.integers(1, 7))
    max_ctx = int(r.choice([64, 130, 257, 448]))
    page_rows = int(r.choice([64, 128]))
    h = Harness(W, oracle, dtype, n_layers=2, n_slots=n_slots, n_heads=heads, max_ctx=max_ctx,
                page_rows=page_rows)
    h.seed = 50_000 + 1000 * seed
    for _ in range(N_OPS):
        x = r.random()
        if x < 0.6:
            k = int(r.integers(1, n_slots + 1))
            slots = [int(s) for s in sorted(r.choice(n_slots, size=k, replace=False))]
            toks = [1 if r.random() < 0.7 else int(r.integers(2, min(40, max_ctx) + 1))
                    for _ in slots]
            for s, n in zip(slots, toks):
                _make_room(h, s, n, max_ctx)
            h.step(slots, toks)  # checks outputs and rows
            continue
        if x < 0.72:
            src, dst = (int(v) for v in r.choice(n_slots, size=2, replace=False))
            h.dev.copy_slot(dst, src)
            h.ref.copy_slot(dst, src)
        elif x < 0.82:
            s = int(r.integers(0, n_slots))
            n_past = int(r.integers(0, h.ref.t_past[s] + 1))
            h.dev.set_t_past(s, n_past)
            h.ref.set_t_past(s, n_past)
        elif x < 0.9:
            s = int(r.integers(0, n_slots))
            h.dev.clear_slot(s)
            h.ref.clear_slot(s)
        else:
            s = int(r.integers(0, n_slots))
            _make_room(h, s, int(r.integers(1, max_ctx + 1)), max_ctx)
        h.check_rows()
    h.dev.clear()
    h.ref.clear()
    h.check_rows()
    assert h.dev.stats()[0] == 0
