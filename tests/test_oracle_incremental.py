"""The oracle's incremental-KV Task 18/19 equals the reference's full-prefix
recompute (golden_prefill_decoder_layer_sequence host:4854-4978), so it can
serve as both the checker and the timed CPU baseline."""
import numpy as np
import pytest

from helpers import OracleState


@pytest.mark.parametrize("profile,blocks", [("small", [8, 3, 1, 1, 5]), ("qwen-layer", [3, 5, 1])])
def test_incremental_equals_full_prefix(oracle, profile, blocks):
    s = oracle.shape(profile)
    keep = min(s.layers, 2)
    emb, norms, dense = oracle.ref_random_model(s, 5, keep, with_embedding=False)
    s = oracle.shape(profile, layers=keep)
    norms = np.concatenate([norms[:2 * keep], norms[-1:]])
    st = OracleState(oracle, s, [dense[l] for l in range(keep)], norms)
    rope = oracle.rope_table(s.head_dim, s.max_seq)
    rng = np.random.default_rng(4)
    seq = rng.integers(-300, 300, (sum(blocks), s.hidden)).astype(np.int16)
    pos = 0
    for rows in blocks:
        out = st.stack(seq[pos:pos + rows], pos)
        h = seq[:pos + rows]
        for l in range(keep):
            _, h = oracle.prefill_sequence_layer(s, dense[l], norms[2 * l], norms[2 * l + 1], rope, h, 1)
        assert np.array_equal(out, oracle.rmsnorm(h, norms[2 * keep])[pos:pos + rows])
        pos += rows
