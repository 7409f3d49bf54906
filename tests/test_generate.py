"""Greedy generation on the device (llmx_generate) vs the reference's generate mode.

llmx_generate restates the coarse-task branch of main's generate mode
(host/host_qwen_8x64.cpp:9016-9132): prompt blocks through
run_composed_decoder_stack, the last one final-normed, then the LM-head argmax
of the last row (model_data_t::lm_head_argmax :937-977) fed back through
run_token (:7665-7700).  The embedding gather and the argmax run on the GPU.
Integer arithmetic throughout, so tokens and hidden rows must match exactly.
"""
import json
import os

import numpy as np
import pytest

from helpers import OracleState, diff_report, oracle_shape

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _host_generate(llmx, acc, m, prompt, max_new, block_rows):
    """The same loop on the host entry points (run_prompt_block / run_token and
    the host LM-head argmax)."""
    ex = llmx.Executor(acc, m)
    acc.reset_kv()
    out = None
    for b0 in range(0, len(prompt), block_rows):
        blk = prompt[b0:b0 + block_rows]
        last = b0 + len(blk) == len(prompt)
        out = ex.run_prompt_block(blk, b0, materialize=last)
    tokens, h = [], out[-1]
    for step in range(max_new):
        nxt = m.lm_head_argmax(h)
        tokens.append(nxt)
        if step + 1 < max_new:
            h = ex.run_token(nxt, len(prompt) + step)[0]
    return tokens, out


@pytest.mark.parametrize("block_rows", [8, 3, 1])
def test_small_generate_matches_host_loop_and_oracle(llmx, oracle, block_rows):
    s = llmx.shape("small")
    m = llmx.Model(s).init_reference_random(11)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    acc.upload_vocab(m)
    prompt = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5]
    max_new = s.max_seq - len(prompt) + 1  # the last decode forward sits at max_seq - 1
    acc.reset_kv()
    got, rows = acc.generate(prompt, max_new, block_rows=block_rows, last_block=True)
    want, want_rows = _host_generate(llmx, acc, m, prompt, max_new, block_rows)
    assert got == want
    assert np.array_equal(rows, want_rows), diff_report(rows, want_rows)
    # the oracle's full-prefix stack for the last block, and its argmax
    ref = OracleState(oracle, oracle_shape(oracle, s), [m.layer(l) for l in range(s.layers)], m.norms())
    table = m.embed(np.arange(s.vocab))
    for b0 in range(0, len(prompt), block_rows):
        blk = prompt[b0:b0 + block_rows]
        o = ref.stack(m.embed(blk), b0, final_norm=b0 + len(blk) == len(prompt))
    assert np.array_equal(rows, o), diff_report(rows, o)
    assert got[0] == oracle.lm_head_argmax(o[-1], table)
    acc.close()


def test_generate_gaussian_untied_and_layer_count(llmx, oracle):
    """Synthetic Gaussian model with an untied LM head; only the first two of
    three layers run (layer_count).  The device loop must equal the host loop
    and the oracle's incremental stack + argmax over the regenerated head."""
    s = llmx.shape("qwen2.5-3b", layers=3, max_seq=64, vocab=4096)
    m = llmx.Model(s).init_gaussian(20260718, 0.02, lm_head=True)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    acc.upload_vocab(m)
    prompt = list(range(100, 120))
    acc.reset_kv()
    got = acc.generate(prompt, 6, block_rows=8, layer_count=2)
    # host loop over the same two layers
    acc.reset_kv()
    h = None
    for b0 in range(0, len(prompt), 8):
        blk = prompt[b0:b0 + 8]
        h = acc.stack(m.embed(blk), layer_count=2, position=b0, include_final_norm=b0 + len(blk) == len(prompt))
    want = []
    for step in range(6):
        want.append(m.lm_head_argmax(h[-1]))
        if step < 5:
            h = acc.stack(m.embed([want[-1]]), layer_count=2, position=len(prompt) + step)
    assert got == want
    # oracle leg: its own prompt blocks + decodes over layers 0-1, argmax over the
    # LM head regenerated from its seed (stream 0x20, N(0, 0.02) in Q4.12)
    ref = OracleState(oracle, oracle_shape(oracle, s), [m.layer(0), m.layer(1)], m.norms())
    head = oracle.gaussian_lm_head(oracle_shape(oracle, s), 20260718, 0.02)
    for b0 in range(0, len(prompt), 8):
        blk = prompt[b0:b0 + 8]
        o = ref.stack(m.embed(blk), b0, layer_count=2, final_norm=b0 + len(blk) == len(prompt))
    ref_tokens = []
    for step in range(6):
        ref_tokens.append(oracle.lm_head_argmax(o[-1], head))
        if step < 5:
            o = ref.stack(m.embed([ref_tokens[-1]]), len(prompt) + step, layer_count=2)
    assert got == ref_tokens
    assert m.lm_head_argmax(o[-1]) == oracle.lm_head_argmax(o[-1], head)
    acc.close()


def test_generate_argument_and_state_errors(llmx):
    s = llmx.shape("small")
    m = llmx.Model(s).init_reference_random(3)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    with pytest.raises(llmx.LlmxError) as e:
        acc.generate([1, 2], 1)
    assert e.value.code == llmx.ERR_STATE  # vocabulary not uploaded
    acc.upload_vocab(m)
    with pytest.raises(llmx.LlmxError) as e:
        acc.generate([1, s.vocab], 1)
    assert e.value.code == llmx.ERR_ARG  # prompt token outside the vocabulary
    with pytest.raises(llmx.LlmxError) as e:
        acc.generate([1, 2], s.max_seq)
    assert e.value.code == llmx.ERR_ARG  # last decode position past max_seq
    with pytest.raises(llmx.LlmxError) as e:
        acc.generate([1, 2], 1, layer_count=s.layers + 1)
    assert e.value.code == llmx.ERR_ARG
    assert acc.generate([1, 2], 2) == acc.generate([1, 2], 2)  # context still usable
    acc.close()


def test_reference_e2e_tokens(llmx, oracle):
    """The reference's end-to-end runs (results/qwen3b-e2e-20260820/host.evidence.log,
    results/qwen3b-e2e-l2-20260821/host.raw.log): qwen2.5-3b reference random
    model, seed 20260718, tied embeddings, prompt 0..7 in one block, one and two
    layers -> the generated tokens, exactly.  The final-normed prompt rows match
    the oracle bit for bit; the FNV checksums the reference printed for them are
    not compared, because the SiLU exponential table of Vitis HLS is restated
    only to within one LSB."""
    want = json.load(open(os.path.join(GOLDEN, "e2e_tokens.json")))
    s = llmx.shape("qwen2.5-3b", max_seq=16)
    m = llmx.Model(s).init_reference_random(want["seed"], 2)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)  # layers 0 and 1 and every norm row
    acc.upload_vocab(m)
    prompt = want["prompt_tokens"]
    for L in (1, 2):
        w = want[f"layers_{L}"]
        acc.reset_kv()
        toks, rows = acc.generate(prompt, len(w["generated"]), block_rows=8, layer_count=L, last_block=True)
        assert toks == w["generated"], f"layers {L}"
        ref = OracleState(oracle, oracle_shape(oracle, s), [m.layer(0), m.layer(1)], m.norms())
        o = ref.stack(m.embed(prompt), 0, layer_count=L)
        assert np.array_equal(rows, o), diff_report(rows, o)
    acc.close()
