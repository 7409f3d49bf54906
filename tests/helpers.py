"""Oracle-side mirror of the device state used by the parity tests.

``OracleState`` keeps a per-layer KV cache and replays Task 18 / 19 / 20 with
the CPU oracle on the same weights the device context holds, so that every
device output can be compared bit for bit.
"""
from __future__ import annotations

import numpy as np


class OracleState:
    def __init__(self, O, oshape, model_layers, norms, payload=1):
        self.O = O
        self.s = oshape
        self.layers = model_layers          # list of dense blobs (np.int16, C-contiguous)
        self.norms = np.ascontiguousarray(norms, np.int16)
        self.payload = payload
        hd = oshape.hidden // oshape.heads
        self.rope = O.rope_table(hd, oshape.max_seq)
        self.kc = [np.zeros((oshape.kv_heads, oshape.max_seq, hd), np.int16) for _ in model_layers]
        self.vc = [np.zeros_like(k) for k in self.kc]

    def task18(self, layer, hidden, position):
        return self.O.task18(self.s, self.layers[layer], self.norms[2 * layer], self.rope,
                             self.kc[layer], self.vc[layer], hidden, position, self.payload)

    def task19(self, layer, hidden):
        return self.O.task19(self.s, self.layers[layer], self.norms[2 * layer + 1], hidden)

    def task20(self, hidden):
        return self.O.rmsnorm(hidden, self.norms[2 * self.s.layers])

    def stack(self, hidden, position, layer_begin=0, layer_count=None, final_norm=True):
        layer_count = len(self.layers) - layer_begin if layer_count is None else layer_count
        h = np.ascontiguousarray(hidden, np.int16)
        for l in range(layer_begin, layer_begin + layer_count):
            h = self.task19(l, self.task18(l, h, position))
        return self.task20(h) if final_norm else h


def oracle_shape(O, xshape):
    return O.Shape(*xshape.tuple())


def random_kv(rng, kv_heads, count, hd, scale=600):
    k = np.clip(rng.normal(0, scale, (kv_heads, count, hd)), -32768, 32767).astype(np.int16)
    v = np.clip(rng.normal(0, scale, (kv_heads, count, hd)), -32768, 32767).astype(np.int16)
    return k, v


def diff_report(a, b):
    a = np.asarray(a, np.int32)
    b = np.asarray(b, np.int32)
    bad = np.argwhere(a != b)
    if len(bad) == 0:
        return "identical"
    idx = tuple(bad[0])
    return f"{len(bad)} mismatches, first at {idx}: device={a[idx]} oracle={b[idx]}, max|d|={np.abs(a - b).max()}"
