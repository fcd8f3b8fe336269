"""Host model of DecoderKvCache (oracle/kv_cache_oracle.py) against the
reference's own inline tests (crates/whisper/src/decoder.rs:894-925) and the
semantics of decode_batch_inner (decoder.rs:616-647, 765-767)."""
import numpy as np
import pytest

from oracle.kv_cache_oracle import DecoderKvCacheOracle


def test_slide_to_fit_drops_oldest_rows():  # decoder.rs:899-914
    c = DecoderKvCacheOracle(1, 1, 2)
    rows = np.array([[1, 1], [2, 2], [3, 3], [4, 4]], np.float32)
    c.append(0, 0, rows, rows)
    c.advance(0, 4)
    assert c.slide_to_fit(0, 2, 4) == 2
    assert c.t_past[0] == 2
    assert np.array_equal(c.k_self[0][0], rows[2:])
    assert np.array_equal(c.v_self[0][0], rows[2:])


def test_slide_to_fit_is_a_noop_when_room_exists():  # decoder.rs:916-924
    c = DecoderKvCacheOracle(1, 1, 2)
    rows = np.array([[1, 1], [2, 2], [3, 3]], np.float32)
    c.append(0, 0, rows, rows)
    c.advance(0, 3)
    assert c.slide_to_fit(0, 1, 8) == 3
    assert c.t_past[0] == 3
    assert c.k_self[0][0].shape[0] == 3


def test_copy_slot_rewind_and_clear():
    c = DecoderKvCacheOracle(2, 2, 4)
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    for layer in range(2):
        c.append(layer, 0, a + layer, -a)
    c.advance(0, 3)
    c.copy_slot(1, 0)  # decoder.rs:220-234
    assert c.slot_len(1) == 3
    assert np.array_equal(c.k_self[1][1], a + 1)
    c.set_t_past(0, 1)  # the C API rewind; the next append truncates
    c.append(0, 0, a[:1] * 10, a[:1])
    assert c.k_self[0][0].shape[0] == 2
    assert np.array_equal(c.k_self[0][0][1], a[0] * 10)
    c.clear_slot(1)
    assert c.slot_len(1) == 0 and c.k_self[0][1].shape[0] == 0
    c.ensure_slots(5)
    assert len(c.t_past) == 5
    with pytest.raises(IndexError):
        c.copy_slot(7, 0)
    c.clear()
    assert c.t_past == [0] * 5


def test_assign_beams_follows_the_reference_slot_hand_out():
    """beam.rs:418-460 worked by hand: parents [2, 0, 2, 2, 4] over 8 slots.
    Reserved {0, 2, 4}; branches 0, 1 and 4 keep their parents' slots, the two
    extra children of slot 2 take the free slots 1 and 3 and fork it."""
    import numpy as np
    from oracle.kv_cache_oracle import DecoderKvCacheOracle
    c = DecoderKvCacheOracle(1, 8, 4)
    for s, n in ((0, 3), (2, 5), (4, 1)):
        c.append(0, s, np.full((n, 4), s, np.float32), np.full((n, 4), -s, np.float32))
        c.advance(s, n)
    assert c.assign_beams([2, 0, 2, 2, 4]) == [2, 0, 1, 3, 4]
    for s in (1, 3):
        assert c.t_past[s] == 5 and (c.k_self[0][s] == 2).all() and (c.v_self[0][s] == -2).all()
    assert c.t_past[5:] == [0, 0, 0]
    with pytest.raises(RuntimeError):
        c.assign_beams([0] * 9)  # nine branches on eight slots

