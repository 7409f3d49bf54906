"""Generate a reference-format packed checkpoint (tests/golden/packed_small/).

Writes the files model_data_t::load reads (host/host_qwen_8x64.cpp:789-840):
token_embedding.fix16.bin, norm_weights.fix16.bin, lm_head.fix16.bin and the
16 weight shards layer_weights_shardNN.fix16.bin (shard_path :736-747), with
every projection weight placed where projection_weight_raw (:899-935) looks
for it: per layer the projections Q, K, V, O, Gate, Up, Down are consecutive
runs of 16x16 tiles (output-tile-major, then input tile; model_config.hpp
:98-125), global tile t goes to shard group t & 1 at 512-bit word t >> 1, and
tile lane (out % 16) * 16 + in % 16 is value lane % 32 of shard
group * 8 + lane / 32.  Lanes outside the projection are zero.

The model is a small seeded one whose FFN width (120) is not a multiple of
16, so the padding of partial tiles is exercised.  This restatement is written
from the reference's indexing rules, independently of the library's loader,
which the tests check against it.  Usage: python make_packed_fixture.py
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "packed_small")
# (vocab, hidden, inter, layers, heads, kv_heads, max_seq): the "small" profile with inter 120
SHAPE = dict(vocab=64, hidden=64, inter=120, layers=2, heads=4, kv_heads=2, max_seq=32)
SEED = 20261202


def dense_model():
    """Seeded dense tensors: embedding, norms, LM head and per layer the seven
    projections [out][in] (int16, including the extremes -32768 and 32767)."""
    s = SHAPE
    H, I, L = s["hidden"], s["inter"], s["layers"]
    KV = s["kv_heads"] * H // s["heads"]
    rng = np.random.default_rng(SEED)

    def w(o, i):
        a = rng.normal(0, 900, (o, i)).round().clip(-32768, 32767).astype(np.int16)
        a.flat[0], a.flat[-1] = -32768, 32767
        return a
    emb = rng.integers(-1200, 1200, (s["vocab"], H)).astype(np.int16)
    norms = rng.integers(200, 300, (2 * L + 1, H)).astype(np.int16)
    head = rng.integers(-900, 900, (s["vocab"], H)).astype(np.int16)
    layers = [[w(H, H), w(KV, H), w(KV, H), w(H, H), w(I, H), w(I, H), w(H, I)] for _ in range(L)]
    return emb, norms, head, layers


def pack_shards(layers):
    """The 16 shard arrays [words][32] of the packed layout."""
    def tiles(o, i):
        return -(-o // 16) * -(-i // 16)
    per_layer = sum(tiles(*m.shape) for m in layers[0])
    total = per_layer * len(layers)
    words = -(-total // 2)
    shards = np.zeros((16, words, 32), np.int16)
    for l, mats in enumerate(layers):
        base = l * per_layer
        for m in mats:
            o_dim, i_dim = m.shape
            it = -(-i_dim // 16)
            out, inp = np.meshgrid(np.arange(o_dim), np.arange(i_dim), indexing="ij")
            tile = base + (out // 16) * it + inp // 16
            lane = (out % 16) * 16 + inp % 16
            shard = (tile & 1) * 8 + lane // 32
            shards[shard, tile >> 1, lane % 32] = m
            base += tiles(o_dim, i_dim)
    return shards


def main():
    emb, norms, head, layers = dense_model()
    os.makedirs(OUT, exist_ok=True)
    emb.astype("<i2").tofile(os.path.join(OUT, "token_embedding.fix16.bin"))
    norms.astype("<i2").tofile(os.path.join(OUT, "norm_weights.fix16.bin"))
    head.astype("<i2").tofile(os.path.join(OUT, "lm_head.fix16.bin"))
    for k, sh in enumerate(pack_shards(layers)):
        sh.astype("<i2").tofile(os.path.join(OUT, f"layer_weights_shard{k:02d}.fix16.bin"))


if __name__ == "__main__":
    main()
