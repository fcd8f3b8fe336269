"""Host-side restatement of whisper.rs's ``DecoderKvCache`` semantics.

TEST INFRASTRUCTURE ONLY: the checker for the device paged cache. It restates
crates/whisper/src/decoder.rs:131-264 (arena of flat per-(layer, slot) row
buffers) plus the per-layer truncate/append of decode_batch_inner
(decoder.rs:616-647) and the slot advance (decoder.rs:765-767), on numpy f32
rows of width ``d_model``.
"""
from __future__ import annotations

import numpy as np


class DecoderKvCacheOracle:
    """decoder.rs:131-264."""

    def __init__(self, n_layers: int, n_slots: int, d_model: int):  # :147-156
        self.n_layers = n_layers
        self.d_model = d_model
        self.k_self = [[np.zeros((0, d_model), np.float32) for _ in range(n_slots)]
                       for _ in range(n_layers)]
        self.v_self = [[np.zeros((0, d_model), np.float32) for _ in range(n_slots)]
                       for _ in range(n_layers)]
        self.t_past = [0] * n_slots

    def clear(self):  # :161-173
        for layer in range(self.n_layers):
            for s in range(len(self.t_past)):
                self.k_self[layer][s] = self.k_self[layer][s][:0]
                self.v_self[layer][s] = self.v_self[layer][s][:0]
        self.t_past = [0] * len(self.t_past)

    def clear_slot(self, slot: int):  # :176-186
        if not slot < len(self.t_past):
            raise IndexError(f"slot {slot} out of range")
        for layer in range(self.n_layers):
            self.k_self[layer][slot] = self.k_self[layer][slot][:0]
            self.v_self[layer][slot] = self.v_self[layer][slot][:0]
        self.t_past[slot] = 0

    def ensure_slots(self, n_slots: int):  # :203-214
        while len(self.t_past) < n_slots:
            for layer in range(self.n_layers):
                self.k_self[layer].append(np.zeros((0, self.d_model), np.float32))
                self.v_self[layer].append(np.zeros((0, self.d_model), np.float32))
            self.t_past.append(0)

    def assign_beams(self, parent_slots):
        """crates/whisper/src/beam.rs:418-460 (the slot hand-out at the end of
        BeamSearch::step), applied to this cache: returns each branch's slot."""
        n_slots = len(self.t_past)
        reserved = [False] * n_slots
        for p in parent_slots:
            if not p < n_slots:
                raise IndexError(f"slot {p} out of range")
            reserved[p] = True
        claimed = [False] * n_slots
        out = []
        free_cursor = 0
        for parent in parent_slots:
            if not claimed[parent]:
                claimed[parent] = True
                out.append(parent)
                continue
            new_slot = free_cursor
            while new_slot < n_slots and (reserved[new_slot] or claimed[new_slot]):
                new_slot += 1
            if new_slot >= n_slots:
                raise RuntimeError("beam slot arena exhausted")
            claimed[new_slot] = True
            self.copy_slot(new_slot, parent)
            out.append(new_slot)
            free_cursor = new_slot
        return out

    def copy_slot(self, dst: int, src: int):  # :220-234
        if not dst < len(self.t_past):
            raise IndexError(f"slot {dst} out of range")
        if not src < len(self.t_past):
            raise IndexError(f"slot {src} out of range")
        if dst == src:
            return
        n = self.t_past[src]
        for layer in range(self.n_layers):
            self.k_self[layer][dst] = self.k_self[layer][src][:n].copy()
            self.v_self[layer][dst] = self.v_self[layer][src][:n].copy()
        self.t_past[dst] = n

    def slot_len(self, slot: int) -> int:  # :237-239
        return self.t_past[slot]

    def slide_to_fit(self, slot: int, n_new: int, max_ctx: int) -> int:  # :248-263
        t_past = self.t_past[slot]
        if t_past + n_new > max_ctx:
            drop = min(t_past + n_new - max_ctx, t_past)
            for layer in range(self.n_layers):
                self.k_self[layer][slot] = self.k_self[layer][slot][drop:]
                self.v_self[layer][slot] = self.v_self[layer][slot][drop:]
            t_past -= drop
            self.t_past[slot] = t_past
        return t_past

    def set_t_past(self, slot: int, n_past: int):
        """The C API rewind: whisper_decode_with_state sets t_past[0] = n_past
        (crates/ffi/src/lib.rs:2352); the next append truncates to it."""
        self.t_past[slot] = n_past

    def append(self, layer: int, slot: int, k_rows: np.ndarray, v_rows: np.ndarray):
        """decoder.rs:631-635: truncate the slot to t_past rows, then extend."""
        t_past = self.t_past[slot]
        self.k_self[layer][slot] = np.concatenate(
            [self.k_self[layer][slot][:t_past], np.asarray(k_rows, np.float32)])
        self.v_self[layer][slot] = np.concatenate(
            [self.v_self[layer][slot][:t_past], np.asarray(v_rows, np.float32)])

    def advance(self, slot: int, n: int):  # decoder.rs:765-767
        self.t_past[slot] += n
