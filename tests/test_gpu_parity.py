"""Device parity: every coarse task through the C ABI vs the CPU oracle, bit-exact.

Mirrors the reference's numerical gates (host/host_qwen_8x64.cpp verify-* modes,
compare_tensors host:3761-3811 with tolerance 0) on the resident Task 18/19/20
path.  Integer / fixed-point work, so the bar is exact equality.
"""
import numpy as np
import pytest

from helpers import OracleState, diff_report, oracle_shape, random_kv

pytestmark = pytest.mark.gpu


def _assert_same(dev, ref, what):
    assert np.array_equal(dev, ref), f"{what}: {diff_report(dev, ref)}"


@pytest.fixture(scope="module")
def small(llmx, oracle):
    s = llmx.shape("small")
    m = llmx.Model(s).init_reference_random(7)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    layers = [m.layer(l) for l in range(s.layers)]
    yield s, m, acc, layers
    acc.close()


def test_small_tasks_step_by_step(llmx, oracle, small):
    """Task 18 / 19 / 20 one at a time (execute_bound_resident_task) over a prompt
    of 11 rows in blocks of 8 and 3, then 5 decode rows; hidden state and KV
    cache compared after every task."""
    s, m, acc, layers = small
    acc.reset_kv()
    ref = OracleState(oracle, oracle_shape(oracle, s), layers, m.norms())
    rng = np.random.default_rng(1)
    blocks = [(0, 8), (8, 3)] + [(11 + i, 1) for i in range(5)]
    for pos, rows in blocks:
        h = rng.integers(-600, 600, (rows, s.hidden)).astype(np.int16)
        acc.write_hidden(1, h)
        hr = h
        for l in range(s.layers):
            acc.bind(0, 1)
            rc, st = acc.task(llmx.OP_ATTENTION, l, pos, rows)
            hr = ref.task18(l, hr, pos)
            _assert_same(acc.read_hidden(0, rows), hr, f"task18 layer {l} pos {pos}")
            k, v = acc.read_kv(l, 0, pos + rows)
            _assert_same(k, ref.kc[l][:, :pos + rows], f"K cache layer {l}")
            _assert_same(v, ref.vc[l][:, :pos + rows], f"V cache layer {l}")
            code, exp = llmx.validate_task(s, llmx.OP_ATTENTION, l, pos, rows)
            assert st.as_dict() == exp.as_dict()
            acc.bind(1, 0)
            acc.task(llmx.OP_FFN, l, pos, rows)
            hr = ref.task19(l, hr)
            _assert_same(acc.read_hidden(1, rows), hr, f"task19 layer {l} pos {pos}")
        acc.bind(0, 1)
        acc.task(llmx.OP_FINAL_NORM, 0, pos, rows)
        _assert_same(acc.read_hidden(0, rows), ref.task20(hr), f"task20 pos {pos}")


def test_small_stack_graph_matches_full_prefix_golden(llmx, oracle, small):
    """run_composed_decoder_stack as one CUDA graph, prompt blocks + decodes, vs
    the golden full-prefix recompute (golden_e2e_sequence_final_hidden)."""
    s, m, acc, layers = small
    acc.reset_kv()
    os_ = oracle_shape(oracle, s)
    rope = oracle.rope_table(s.head_dim, s.max_seq)
    norms = m.norms()
    rng = np.random.default_rng(2)
    seq = rng.integers(-500, 500, (19, s.hidden)).astype(np.int16)
    pos = 0
    for rows in (8, 8, 1, 1, 1):
        out = acc.stack(seq[pos:pos + rows], position=pos)
        h = seq[:pos + rows]
        for l in range(s.layers):
            _, h = oracle.prefill_sequence_layer(os_, layers[l], norms[2 * l], norms[2 * l + 1], rope, h, 1)
        golden = oracle.rmsnorm(h, norms[2 * s.layers])
        _assert_same(out, golden[pos:pos + rows], f"stack rows {pos}..{pos + rows}")
        pos += rows


def test_small_executor_generate(llmx, oracle, small):
    """qwen_executor_t: embedding, prompt block, decode, host LM-head argmax."""
    s, m, acc, layers = small
    acc.reset_kv()
    ref = OracleState(oracle, oracle_shape(oracle, s), layers, m.norms())
    ex = llmx.Executor(acc, m)
    tokens = [3, 1, 4, 1, 5, 9, 2]
    out = ex.run_prompt_block(tokens, 0)
    emb = m.embed(tokens)
    _assert_same(out, ref.stack(emb, 0), "prompt block")
    nxt = m.lm_head_argmax(out[-1])
    assert nxt == oracle.lm_head_argmax(out[-1], m.embed(np.arange(s.vocab)))
    for step in range(3):
        pos = len(tokens) + step
        o = ex.run_token(nxt, pos)
        _assert_same(o, ref.stack(m.embed([nxt]), pos), f"decode {step}")
        nxt = m.lm_head_argmax(o[0])


@pytest.mark.parametrize("rows", [1, 2, 3, 5, 8])
def test_qwen_layer_reference_model(llmx, oracle, rows):
    """Full Qwen2.5-3B layer shape (hidden 2048, FFN 11008, 16/2 heads) with the
    reference random model: Task 18/19/20 for a block, then one decode row."""
    s = llmx.shape("qwen-layer")
    m = llmx.Model(s).init_reference_random(20260718)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    ref = OracleState(oracle, oracle_shape(oracle, s), [m.layer(0)], m.norms())
    hidden = oracle.mt_uniform(20260718 ^ 0x626C6F63, -48, 48, (rows, s.hidden))
    out = acc.stack(hidden, position=0)
    _assert_same(out, ref.stack(hidden, 0), f"qwen layer block rows={rows}")
    dec = oracle.mt_uniform(99, -128, 128, (1, s.hidden))
    out = acc.stack(dec, position=rows)
    _assert_same(out, ref.stack(dec, rows), "qwen layer decode")
    acc.close()


def test_long_context_gaussian(llmx, oracle):
    """Gaussian N(0,0.02) weights / N(0,1) rows (the benchmark workload), KV cache
    preloaded to 1000 positions: an 8-row block straddling a 64-tile boundary
    and decode rows at tile edges (1023, 1024, 1025 context)."""
    s = llmx.shape("qwen-layer-long")
    m = llmx.Model(s).init_gaussian(20260718, 0.02)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    ref = OracleState(oracle, oracle_shape(oracle, s), [m.layer(0)], m.norms())
    rng = np.random.default_rng(3)
    k, v = random_kv(rng, s.kv_heads, 1015, s.head_dim)
    acc.write_kv(0, 0, k, v)
    ref.kc[0][:, :1015] = k
    ref.vc[0][:, :1015] = v
    h = m.embed(rng.integers(0, s.vocab, 8))
    out = acc.stack(h, position=1015)
    _assert_same(out, ref.stack(h, 1015), "block at 1015")
    for pos in (1023, 1024):  # context 1024 (16 full tiles), then 1025 (a 1-position tile)
        d = m.embed([int(rng.integers(0, s.vocab))])
        out = acc.stack(d, position=pos)
        _assert_same(out, ref.stack(d, pos), f"decode at {pos}")
    kd, vd = acc.read_kv(0, 0, 1025)
    _assert_same(kd, ref.kc[0][:, :1025], "K cache")
    _assert_same(vd, ref.vc[0][:, :1025], "V cache")
    acc.close()


@pytest.mark.parametrize("heads,kv_heads,hidden", [(4, 1, 512), (2, 1, 256)])
def test_long_context_few_heads(llmx, oracle, monkeypatch, heads, kv_heads, hidden):
    """A layer with as few query heads as a tensor-parallel rank holds (4 / 2):
    one-row decodes at contexts above 16 tiles run 16-CTA attention clusters
    (3 tiles per CTA); the same rows with 8-CTA clusters (LLMX_ATTN_WIDE=0) and
    the oracle must agree."""
    s = llmx.shape("qwen-layer-long", hidden=hidden, heads=heads, kv_heads=kv_heads, inter=hidden * 2 + 256)
    m = llmx.Model(s).init_gaussian(20260718 + heads, 0.02)
    wide = llmx.Accelerator(s)
    monkeypatch.setenv("LLMX_ATTN_WIDE", "0")
    narrow = llmx.Accelerator(s)
    monkeypatch.delenv("LLMX_ATTN_WIDE")
    ref = OracleState(oracle, oracle_shape(oracle, s), [m.layer(0)], m.norms())
    rng = np.random.default_rng(heads)
    P = 1900
    k, v = random_kv(rng, s.kv_heads, P, s.head_dim)
    ref.kc[0][:, :P] = k
    ref.vc[0][:, :P] = v
    for acc in (wide, narrow):
        acc.upload_model(m)
        acc.write_kv(0, 0, k, v)
    h = m.embed(rng.integers(0, s.vocab, 8))
    want = ref.stack(h, P)
    for acc, what in ((wide, "wide"), (narrow, "narrow")):
        _assert_same(acc.stack(h, position=P), want, f"block at {P} ({what})")
    for pos in (1919, 1983, 1984, 2047):
        d = m.embed([int(rng.integers(0, s.vocab))])
        want = ref.stack(d, pos)
        for acc, what in ((wide, "wide"), (narrow, "narrow")):
            _assert_same(acc.stack(d, position=pos), want, f"decode at {pos} ({what})")
    wide.close()
    narrow.close()


def test_status_and_errors_on_device(llmx, small):
    """Controller status codes (include/control_cache_8x64.hpp:279-286) from
    the device entry point: bad rows / operator / layer / position."""
    s, m, acc, layers = small
    assert acc.task(llmx.OP_ATTENTION, 0, 0, 9, raise_on_error=False)[0] == llmx.BAD_TOKEN_COUNT
    assert acc.task(llmx.OP_ATTENTION, 0, 0, 0, raise_on_error=False)[0] == llmx.BAD_TOKEN_COUNT
    assert acc.task(7, 0, 0, 1, raise_on_error=False)[0] == llmx.BAD_OPERATOR
    assert acc.task(llmx.OP_FFN, s.layers, 0, 1, raise_on_error=False)[0] == llmx.BAD_LAYER
    assert acc.task(llmx.OP_ATTENTION, 0, s.max_seq - 2, 3, raise_on_error=False)[0] == llmx.BAD_POSITION
    rc, st = acc.task(llmx.OP_NOP, 0, 0, 1, raise_on_error=False)
    assert rc == 0 and st.op == 0 and st.last_task == 1


def test_bounded_wait_expires_with_error_status(llmx, oracle, small):
    """Failure detection without a fault: the receiving side of the peer
    all-reduce waits on an exchange region that nothing writes; the bounded
    wait expires, the kernel records its error status and returns, the call
    reports LLMX_ERR_TIMEOUT, and the same context then runs a stack that
    matches the oracle."""
    s, m, acc, layers = small
    assert acc.selftest_ar_timeout(2000) == llmx.ERR_TIMEOUT
    assert "bounded wait expired" in llmx.last_error()
    assert acc.selftest_ar_timeout(0) == llmx.ERR_ARG
    acc.reset_kv()
    ref = OracleState(oracle, oracle_shape(oracle, s), layers, m.norms())
    h = np.random.default_rng(9).integers(-600, 600, (3, s.hidden)).astype(np.int16)
    _assert_same(acc.stack(h, position=0), ref.stack(h, 0), "stack after the expired wait")


def test_prefill_sweep_device_built_cache(llmx, oracle):
    """BASELINE config 2 on one Qwen2.5-3B-shaped layer (Gaussian weights, N(0,1)
    embedding rows): a 1024-token prompt as 128 consecutive P8 blocks, the KV
    cache built by the device itself (nothing preloaded).  Prompts of 8, 64,
    256 and 1024 tokens are its prefixes.  Every block's final-normed rows are
    compared with the oracle's incremental state, and the whole K/V cache at
    each prompt length (the reference's P/D sweep,
    results/q214-pd-20260811/performance.tsv:2-9)."""
    s = llmx.shape("qwen2.5-3b", layers=1, max_seq=1024, vocab=4096)
    m = llmx.Model(s).init_gaussian(20260718, 0.02)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    oracle.set_threads(8)
    ref = OracleState(oracle, oracle_shape(oracle, s), [m.layer(0)], m.norms())
    toks = np.random.default_rng(1024).integers(0, s.vocab, 1024)
    try:
        for b in range(128):
            h = m.embed(toks[8 * b:8 * b + 8])
            _assert_same(acc.stack(h, position=8 * b), ref.stack(h, 8 * b), f"P8 block {b}")
            n = 8 * (b + 1)
            if n in (8, 64, 256, 1024):
                k, v = acc.read_kv(0, 0, n)
                _assert_same(k, ref.kc[0][:, :n], f"K cache after {n} prompt tokens")
                _assert_same(v, ref.vc[0][:, :n], f"V cache after {n} prompt tokens")
    finally:
        oracle.set_threads(1)
        acc.close()


@pytest.mark.parametrize("env", [{"LLMX_MMA_PROJ": "15"}, {"LLMX_MMA": "0"}], ids=["all_tensor_core", "all_dp2a"])
@pytest.mark.parametrize("rows", [3, 8])
def test_projection_kernels_both_paths(llmx, oracle, monkeypatch, env, rows):
    """Blocks of 3..8 rows run Gate/Up and Down on the tensor cores by default
    (byte-split int8 tcgen05.mma) and QKV / O on the dp2a kernel; every
    projection has both kernels.  Force each choice for all four projections
    (LLMX_MMA_PROJ=15: all on the tensor cores; LLMX_MMA=0: all dp2a) and match
    the oracle on a Gaussian layer, a block at a tile edge and a decode row."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    s = llmx.shape("qwen-layer-long")
    m = llmx.Model(s).init_gaussian(20260718 + rows, 0.02)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    ref = OracleState(oracle, oracle_shape(oracle, s), [m.layer(0)], m.norms())
    rng = np.random.default_rng(rows)
    k, v = random_kv(rng, s.kv_heads, 61, s.head_dim)
    acc.write_kv(0, 0, k, v)
    ref.kc[0][:, :61] = k
    ref.vc[0][:, :61] = v
    h = m.embed(rng.integers(0, s.vocab, rows))
    _assert_same(acc.stack(h, position=61), ref.stack(h, 61), f"{rows}-row block")
    d = m.embed([int(rng.integers(0, s.vocab))])
    _assert_same(acc.stack(d, position=61 + rows), ref.stack(d, 61 + rows), "decode")
    acc.close()


@pytest.mark.parametrize("rows", [1, 8])
def test_attention_saturating_operands(llmx, oracle, rows):
    """K and V caches over the whole int16 range (many |k|, |v| >= 8.0, i.e. raw
    >= 2048, where the Q4.12 conversion saturates) and hidden rows at the int16
    extremes (saturated queries, some exactly -32768): the per-product rounding
    and the saturating banks of both attention kernels must agree with the
    oracle, for one row and an 8-row block."""
    s = llmx.shape("qwen-layer-long")
    m = llmx.Model(s).init_reference_random(5)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    ref = OracleState(oracle, oracle_shape(oracle, s), [m.layer(0)], m.norms())
    rng = np.random.default_rng(77)
    P = 200
    k = rng.integers(-32768, 32768, (s.kv_heads, P, s.head_dim)).astype(np.int16)
    v = rng.integers(-32768, 32768, (s.kv_heads, P, s.head_dim)).astype(np.int16)
    k[:, ::3] = np.clip(k[:, ::3] // 16, -2047, 2047)  # a third of the positions unsaturated
    v[:, :64] = np.clip(v[:, :64] // 16, -2047, 2047)  # the first tile of V unsaturated
    acc.write_kv(0, 0, k, v)
    ref.kc[0][:, :P] = k
    ref.vc[0][:, :P] = v
    h = rng.choice(np.array([-32768, 32767, -30000, 31000], np.int16), (rows, s.hidden))
    _assert_same(acc.stack(h, position=P), ref.stack(h, P), f"{rows} saturating rows")
    d = rng.integers(-2000, 2000, (1, s.hidden)).astype(np.int16)
    _assert_same(acc.stack(d, position=P + rows), ref.stack(d, P + rows), "decode after")
    acc.close()


@pytest.mark.parametrize("env", [{}, {"LLMX_ATTN_FUSE_O": "0"}, {"LLMX_ATTN_TRIGGER_TILES": "0"}],
                         ids=["o_fused", "o_kernel", "early_trigger"])
def test_decode_attention_paths(llmx, oracle, monkeypatch, env):
    """One-row decode runs the O projection inside the attention kernel (its
    int64 sums finished by the Gate/Up prologue and cleared by Down); with
    LLMX_ATTN_FUSE_O=0 the separate O kernel runs, and LLMX_ATTN_TRIGGER_TILES
    moves the point where attention lets the next kernel launch.  Every variant
    must match the oracle through a 3-layer stack of decode rows on both sides
    of the 16-tile trigger threshold, and single Task 18 / 19 calls after it."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    s = llmx.shape("qwen-layer-long", layers=3)
    m = llmx.Model(s).init_gaussian(20260719, 0.02)
    acc = llmx.Accelerator(s)
    try:
        acc.upload_model(m)
        assert acc.decode_fuses_o == (env.get("LLMX_ATTN_FUSE_O") != "0")
        layers = [m.layer(l) for l in range(s.layers)]
        ref = OracleState(oracle, oracle_shape(oracle, s), layers, m.norms())
        rng = np.random.default_rng(11)
        P = 1020
        for l in range(s.layers):
            k, v = random_kv(rng, s.kv_heads, P, s.head_dim)
            acc.write_kv(l, 0, k, v)
            ref.kc[l][:, :P] = k
            ref.vc[l][:, :P] = v
        for pos in range(P, P + 6):  # contexts 1021..1026: 16 tiles, then 17
            d = m.embed([int(rng.integers(0, s.vocab))])
            _assert_same(acc.stack(d, position=pos), ref.stack(d, pos), f"decode at {pos}")
        h = m.embed([int(rng.integers(0, s.vocab))])  # the coarse tasks one by one
        acc.write_hidden(1, h)
        acc.bind(0, 1)
        acc.task(llmx.OP_ATTENTION, 0, P + 6, 1)
        want = ref.task18(0, h, P + 6)
        _assert_same(acc.read_hidden(0, 1), want, "task 18")
        acc.bind(1, 0)
        acc.task(llmx.OP_FFN, 0, P + 6, 1)
        _assert_same(acc.read_hidden(1, 1), ref.task19(0, want), "task 19")
    finally:
        acc.close()
