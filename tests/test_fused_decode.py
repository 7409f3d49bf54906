"""Fused one-row decode (one cooperative kernel per stack) vs the per-task kernels.

Both paths implement run_composed_decoder_stack (host/host_qwen_8x64.cpp:1258-1493)
with the same integer arithmetic, so outputs and KV caches must be identical
bit for bit; each path is also checked against the CPU oracle elsewhere.
LLMX_FUSED_DECODE=1 at context creation selects the fused kernel for one-row
stacks (the per-task kernels are the default).
"""
import numpy as np
import pytest

from helpers import OracleState, diff_report, oracle_shape, random_kv

pytestmark = pytest.mark.gpu


def _pair(llmx, monkeypatch, s, m):
    monkeypatch.setenv("LLMX_FUSED_DECODE", "1")
    fused = llmx.Accelerator(s)
    fused.upload_model(m)
    monkeypatch.setenv("LLMX_FUSED_DECODE", "0")
    plain = llmx.Accelerator(s)
    plain.upload_model(m)
    monkeypatch.delenv("LLMX_FUSED_DECODE")
    return fused, plain


def _same(a, b, what):
    assert np.array_equal(a, b), f"{what}: {diff_report(a, b)}"


def test_fused_matches_per_task_long_context(llmx, monkeypatch):
    """Qwen2.5-3B layer, Gaussian weights, random KV prefix; decode rows at tile
    edges up to context 2048, with and without the final norm."""
    s = llmx.shape("qwen-layer-long")
    m = llmx.Model(s).init_gaussian(20260718, 0.02)
    fused, plain = _pair(llmx, monkeypatch, s, m)
    rng = np.random.default_rng(5)
    k, v = random_kv(rng, s.kv_heads, s.max_seq, s.head_dim)
    for acc in (fused, plain):
        acc.write_kv(0, 0, k, v)
    for pos in (0, 1, 63, 64, 65, 511, 1000, 2047):
        d = m.embed([int(rng.integers(0, s.vocab))])
        for final in (True, False):
            a = fused.stack(d, position=pos, include_final_norm=final)
            assert fused.kernel_launches == 2, "fused path not taken"
            b = plain.stack(d, position=pos, include_final_norm=final)
            assert plain.kernel_launches > 2
            _same(a, b, f"pos {pos} final_norm {final}")
        ka, va = fused.read_kv(0, pos, 1)
        kb, vb = plain.read_kv(0, pos, 1)
        _same(ka, kb, f"K row {pos}")
        _same(va, vb, f"V row {pos}")
    fused.close()
    plain.close()


def test_fused_small_generate_vs_oracle(llmx, oracle, monkeypatch):
    """Two-layer small shape (generic loop path, head_dim 16): a prompt block,
    then decode rows through the fused kernel, each against the oracle."""
    s = llmx.shape("small")
    m = llmx.Model(s).init_reference_random(11)
    fused, plain = _pair(llmx, monkeypatch, s, m)
    ref = OracleState(oracle, oracle_shape(oracle, s), [m.layer(l) for l in range(s.layers)], m.norms())
    rng = np.random.default_rng(9)
    h = rng.integers(-700, 700, (8, s.hidden)).astype(np.int16)
    want = ref.stack(h, 0)
    _same(fused.stack(h, position=0), want, "block")
    _same(plain.stack(h, position=0), want, "block (per task)")
    for pos in range(8, s.max_seq):
        d = rng.integers(-900, 900, (1, s.hidden)).astype(np.int16)
        want = ref.stack(d, pos)
        _same(fused.stack(d, position=pos), want, f"fused decode {pos}")
        _same(plain.stack(d, position=pos), want, f"per-task decode {pos}")
    fused.close()
    plain.close()


def test_fused_multi_layer_stack_ranges(llmx, monkeypatch):
    """Layer sub-ranges (layer_begin / layer_count) of a 3-layer stack."""
    s = llmx.shape("qwen2.5-3b", layers=3, max_seq=256, vocab=512)
    m = llmx.Model(s).init_gaussian(7, 0.02)
    fused, plain = _pair(llmx, monkeypatch, s, m)
    rng = np.random.default_rng(2)
    prompt = m.embed(rng.integers(0, s.vocab, 8))
    _same(fused.stack(prompt, position=0), plain.stack(prompt, position=0), "prompt")
    for pos, (lb, lc) in zip(range(8, 14), [(0, 3), (1, 2), (0, 1), (2, 1), (0, 3), (1, 1)]):
        d = m.embed([int(rng.integers(0, s.vocab))])
        a = fused.stack(d, layer_begin=lb, layer_count=lc, position=pos, include_final_norm=False)
        b = plain.stack(d, layer_begin=lb, layer_count=lc, position=pos, include_final_norm=False)
        _same(a, b, f"layers [{lb}, {lb + lc}) at {pos}")
    fused.close()
    plain.close()
