"""Pin the CPU oracle against the reference's own known-answer values.

K1 (scripts/test_q214_payload_golden.sh:30-63): golden-only regression of the
Q2.14 raw-payload vs direct attention semantics on the qwen-layer profile.
K2/K3 (results/qwen3b-e2e-*/host*.log): full qwen2.5-3b random model, tokens
0..7, 1 and 2 layers, two generated tokens.

What is pinned exactly: the random-model generator (mt19937 + libstdc++-9
uniform_int), RMSNorm, projections, RoPE, the Q2.14 softmax exp table, the
tile-sequential online softmax with both PV semantics, O projection and
residual (all of K1's post-attention fingerprint), the LM head and the
generated tokens of K2/K3.  What is not: the SiLU exp table
(hls::exp(ap_fixed<16,8>), Xilinx library source not available) -- the
truncated exact exponential differs from it by one Q8.8 LSB in a few entries,
which shows up as small post-FFN differences; the stated tolerance is checked.
"""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _cmp(a, b, tol):
    err = np.abs(a.astype(np.int32) - b.astype(np.int32))
    bad = np.argwhere(err > tol)
    return int(err.max()), len(bad), [[int(r), int(c), int(a[r, c]), int(b[r, c])] for r, c in bad[:4]]


@pytest.fixture(scope="module")
def k1(oracle):
    s = oracle.shape("qwen-layer")
    emb, norms, dense = oracle.ref_random_model(s, 20260718, 1, with_embedding=False)
    rope = oracle.rope_table(s.head_dim, s.max_seq)
    want = json.load(open(os.path.join(GOLDEN, "k1_q214_payload.json")))
    return s, norms, dense, rope, want


@pytest.mark.parametrize("rows", [2, 8])
def test_k1_q214_payload_golden(oracle, k1, rows):
    s, norms, dense, rope, want = k1
    w = want[f"p{rows}"]
    hidden = oracle.mt_uniform(20260718 ^ 0x626C6F63, -48, 48, (rows, s.hidden))
    pa_p, out_p = oracle.prefill_sequence_layer(s, dense[0], norms[0], norms[1], rope, hidden, 1)
    pa_d, out_d = oracle.prefill_sequence_layer(s, dense[0], norms[0], norms[1], rope, hidden, 0)
    fin_p, fin_d = oracle.rmsnorm(out_p, norms[2]), oracle.rmsnorm(out_d, norms[2])
    # exact: the whole attention sublayer under both PV semantics
    mx, n, first = _cmp(pa_p, pa_d, 0)
    assert (mx, n) == (w["post_attention"]["max_raw_error"], w["post_attention"]["mismatches"])
    if n:
        assert first == w["post_attention"]["first"]
    # FFN: SiLU exp table within one Q8.8 LSB of hls::exp<16,8>
    mx, n, first = _cmp(out_p, out_d, 0)
    if rows == 2:
        assert (mx, n) == (0, 0)
        key = "probes_row1"
    else:
        assert abs(mx - w["post_ffn"]["max_raw_error"]) <= 2
        assert abs(n - w["post_ffn"]["mismatches"]) <= 0.01 * w["post_ffn"]["mismatches"]
        for got, ref in zip(first, w["post_ffn"]["first"]):
            assert got[:2] == ref[:2] and abs(got[2] - ref[2]) <= 1 and abs(got[3] - ref[3]) <= 1
        key = "probes_row3"
    r = 1 if rows == 2 else 3
    for c, rp, rd in zip(w[key]["cols"], w[key]["raw_payload"], w[key]["direct"]):
        # final RMSNorm multiplies by 25.87 * norm weight (~29): one post-FFN LSB
        assert abs(int(fin_p[r, c]) - rp) <= 64 and abs(int(fin_d[r, c]) - rd) <= 64


@pytest.mark.slow
def test_k2_k3_generated_tokens(oracle):
    """Full qwen2.5-3b reference random model (3.1 G draws); two layers kept."""
    want = json.load(open(os.path.join(GOLDEN, "e2e_tokens.json")))
    s = oracle.shape("qwen2.5-3b")
    emb, norms, dense = oracle.ref_random_model(s, want["seed"], 2)
    s16 = oracle.shape("qwen2.5-3b", max_seq=16)
    rope = oracle.rope_table(s.head_dim, 16)

    def final_rows(tokens, L):
        h = emb[tokens].copy()
        for l in range(L):
            _, h = oracle.prefill_sequence_layer(s16, dense[l], norms[2 * l], norms[2 * l + 1], rope, h, 1)
        return oracle.rmsnorm(h, norms[2 * s.layers])

    for L in (1, 2):
        w = want[f"layers_{L}"]
        prompt = list(want["prompt_tokens"])
        t1 = oracle.lm_head_argmax(final_rows(prompt, L)[-1], emb)
        t2 = oracle.lm_head_argmax(final_rows(prompt + [t1], L)[-1], emb)
        assert [t1, t2] == w["generated"]
