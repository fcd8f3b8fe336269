"""Device paged KV cache against the host DecoderKvCache model and the
causal attention oracle (decoder.rs:131-264, 616-647, 835-892).

A scripted beam-search history runs on both: prompt prefill across a page
boundary, single-token steps, forks (copy_slot, shared pages and copy on
write), a slide (slide_to_fit), a rewind (the C API's n_past) and slot
clears. After every step the device rows must equal the model's rows
(bit-exact for an f32 cache) and every attention output must match the
oracle's multi_head_attention_with_cache on those rows.
"""
import numpy as np
import pytest

from oracle.kv_cache_oracle import DecoderKvCacheOracle
from tests.helpers import check_16bit, check_f32, randn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


class Harness:
    def __init__(self, W, oracle, dtype, n_layers=2, n_slots=4, n_heads=3, max_ctx=200, page_rows=64):
        import torch
        self.torch = torch
        self.W, self.O, self.dtype = W, oracle, dtype
        self.L, self.H, self.max_ctx = n_layers, n_heads, max_ctx
        self.d = n_heads * 64
        self.dev = W.DeviceKvCache(n_layers, n_slots, n_heads, max_ctx, page_rows=page_rows,
                                   dtype=dtype)
        self.ref = DecoderKvCacheOracle(n_layers, n_slots, self.d)
        self.seed = 1000

    def _rows(self, n):
        self.seed += 1
        x = randn(self.seed, n * self.d).reshape(n, self.d)
        if self.dtype != 0:  # the cache stores 16-bit rows; the model keeps the rounded values
            t = self.torch.from_numpy(x).to({1: self.torch.float16, 2: self.torch.bfloat16}[self.dtype])
            x = t.float().numpy()
        return x

    def step(self, slots, n_tokens):
        """One decode_batch_inner pass: per layer append + attend, then advance."""
        torch = self.torch
        total = sum(n_tokens)
        for layer in range(self.L):
            k, v, q = self._rows(total), self._rows(total), self._rows(total)
            self.dev.append(layer, slots, n_tokens, torch.from_numpy(k).cuda(),
                            torch.from_numpy(v).cuda())
            o = torch.zeros(total, self.d, device="cuda")
            self.dev.attend(layer, slots, n_tokens, torch.from_numpy(q).cuda(), o)
            torch.cuda.synchronize()
            out = o.cpu().numpy()
            r0 = 0
            for s, n in zip(slots, n_tokens):
                self.ref.append(layer, s, k[r0:r0 + n], v[r0:r0 + n])
                t_past = self.ref.t_past[s]
                K, V = self.ref.k_self[layer][s], self.ref.v_self[layer][s]
                exp = self.O.mha_with_cache(q[r0:r0 + n].ravel(), K.ravel(), V.ravel(), n,
                                            t_past + n, t_past, self.H, self.d)
                if self.dtype == 0:
                    check_f32(out[r0:r0 + n], exp, f"slot {s} layer {layer}")
                else:
                    check_16bit(out[r0:r0 + n], exp, f"slot {s} layer {layer}")
                r0 += n
        self.dev.advance(slots, n_tokens)
        for s, n in zip(slots, n_tokens):
            self.ref.advance(s, n)
        self.check_rows()

    def check_rows(self):
        torch = self.torch
        for s in range(len(self.ref.t_past)):
            assert self.dev.slot_len(s) == self.ref.t_past[s]
            n = self.ref.t_past[s]
            if n == 0:
                continue
            for layer in range(self.L):
                for which, arr in ((0, self.ref.k_self), (1, self.ref.v_self)):
                    buf = torch.empty(n, self.d, device="cuda")
                    self.dev.read_slot(layer, s, which, buf)
                    torch.cuda.synchronize()
                    assert np.array_equal(buf.cpu().numpy(), arr[layer][s][:n]), (s, layer, which)


@pytest.mark.parametrize("dtype", [0, 1], ids=["f32", "f16"])
def test_beam_history(W, oracle, dtype):
    h = Harness(W, oracle, dtype)
    h.step([0], [70])                 # prompt prefill across the first page boundary
    for _ in range(3):
        h.step([0], [1])              # greedy steps
    for dst in (1, 2):                # beam fork (beam.rs:455 -> copy_slot)
        h.dev.copy_slot(dst, 0)
        h.ref.copy_slot(dst, 0)
    h.check_rows()
    used_after_fork, _ = h.dev.stats()
    h.step([0, 1, 2], [1, 1, 1])      # all three write into the shared partial page
    used, _ = h.dev.stats()
    assert used == used_after_fork + 2  # two copy-on-write pages, the last writer keeps the original
    for _ in range(60):               # grow past the second page boundary
        h.step([2, 0], [1, 1])
    # slide: drop the oldest rows of slot 2 so 5 more fit in a 100-token context
    pos_dev = h.dev.slide_to_fit(2, 5, 100)
    pos_ref = h.ref.slide_to_fit(2, 5, 100)
    assert pos_dev == pos_ref == 95
    h.check_rows()
    h.step([2], [5])
    # rewind slot 0 to 50 tokens (the C API's n_past, crates/ffi/src/lib.rs:2352)
    h.dev.set_t_past(0, 50)
    h.ref.set_t_past(0, 50)
    h.step([0, 1], [3, 2])
    h.dev.clear_slot(1)
    h.ref.clear_slot(1)
    h.check_rows()
    h.dev.copy_slot(3, 2)
    h.ref.copy_slot(3, 2)
    h.step([3], [1])
    h.dev.clear()
    h.ref.clear()
    h.check_rows()
    assert h.dev.stats()[0] == 0


@pytest.mark.parametrize("dtype", [1, 2], ids=["f16", "bf16"])
def test_ragged_batch_many_rows(W, oracle, dtype):
    """Many slots of ragged lengths at 20 heads: one attend call spans several
    kernel launches (more rows than one launch's table holds), entries are
    reordered by length inside each launch and every CTA of the persistent
    grid serves several (row, head) items."""
    rng = np.random.default_rng(7)
    h = Harness(W, oracle, dtype, n_layers=1, n_slots=40, n_heads=20, max_ctx=448, page_rows=64)
    slots = list(range(40))
    h.step(slots, [int(x) for x in rng.integers(1, 300, size=40)])  # ragged prefill
    h.step(slots, [1] * 40)                                           # one decode step
    h.step(slots[::3], [int(x) for x in rng.integers(1, 12, size=len(slots[::3]))])


@pytest.mark.parametrize("src, dst, pad", [(1, 1, 3), (0, 2, 0), (2, 2, 8)],
                         ids=["f16_unaligned_rows", "f32_to_bf16", "bf16_padded_rows"])
def test_append_row_layouts(W, src, dst, pad):
    """Rows appended from strided sources (row stride = width + pad, so some
    are not 16-byte aligned and take the element-wise path) and with a type
    conversion land bit-exact in the pages."""
    import torch
    tdt = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}
    H, n = 4, 37
    d = H * 64
    c = W.DeviceKvCache(1, 2, H, 128, page_rows=64, dtype=dst)
    g = torch.Generator(device="cuda").manual_seed(3)
    base_k = torch.randn(n, d + pad, generator=g, device="cuda").to(tdt[src])
    base_v = torch.randn(n, d + pad, generator=g, device="cuda").to(tdt[src])
    k, v = base_k[:, :d], base_v[:, :d]       # row stride d + pad
    c.append(0, [1], [n], k, v)
    c.advance([1], [n])
    for which, ref in ((0, k), (1, v)):
        out = torch.empty(n, d, dtype=tdt[dst], device="cuda")
        c.read_slot(0, 1, which, out)
        torch.cuda.synchronize()
        assert torch.equal(out, ref.to(tdt[dst])), which
    c.close()


def test_assign_beams(W, oracle):
    """BeamSearch::step's slot hand-out (beam.rs:418-460) on the device cache
    against the host model: same slots, same rows, and appends after a
    multi-way fork land copy-on-write in the right slots."""
    h = Harness(W, oracle, 1, n_layers=2, n_slots=8, n_heads=3, max_ctx=300)
    h.step([0], [70])
    for dst in (2, 4):
        h.dev.copy_slot(dst, 0)
        h.ref.copy_slot(dst, 0)
    h.step([0, 2, 4], [5, 9, 1])         # three diverged beams
    parents = [2, 0, 2, 2, 4]
    got = h.dev.assign_beams(parents)
    assert got == h.ref.assign_beams(parents) == [2, 0, 1, 3, 4]
    h.check_rows()
    h.step(got, [1] * len(got))          # every retained beam appends a token
    h.step([1, 3], [2, 1])
    # more branches than slots: rejected, nothing changes
    used = h.dev.stats()[0]
    lens = [h.dev.slot_len(s) for s in range(8)]
    with pytest.raises(W.WattnError) as e:
        h.dev.assign_beams([0] * 9)
    assert e.value.status == -6
    assert h.dev.stats()[0] == used and [h.dev.slot_len(s) for s in range(8)] == lens
    h.check_rows()


def test_cache_errors(W):
    c = W.DeviceKvCache(1, 2, 2, 128)
    with pytest.raises(W.WattnError) as e:
        c.copy_slot(5, 0)
    assert e.value.status == -6
    with pytest.raises(W.WattnError):
        c.advance([0], [1])           # nothing appended yet
    with pytest.raises(W.WattnError):
        c.set_t_past(0, 3)
    with pytest.raises(W.WattnError) as e:
        W.DeviceKvCache(1, 1, 2, 128, page_rows=48)
    assert e.value.status == -1
    c.close()
