"""Per-operator API: the controller's legacy operator modes next to the coarse tasks.

* ops 1-10 (feature operators) through ``llmx_run_feature``, the counterpart of
  ``run_feature`` host/host_qwen_8x64.cpp:1088-1130, checked the way
  ``run_random_verification`` host:3813-3940 checks them (golden_projection,
  golden_residual, golden_rmsnorm, golden_silu_mul) but bit-exact;
* op 16, the compatibility full-layer task (run_decoder_layer host:1136-1176),
  through ``llmx_task``: Task 18 followed by Task 19;
* op 17, the prefill block attention (run_prefill_attention_block
  host:1647-1690), against the oracle's tiled Q2.14 attention per token.

Status records follow the controller testbench (tests/control_cache_8x64_tb.cpp).
"""
import numpy as np
import pytest

from helpers import OracleState, diff_report, oracle_shape


def _same(dev, ref, what):
    assert np.array_equal(dev, ref), f"{what}: {diff_report(dev, ref)}"


def cdiv(a, b):
    return -(-a // b)


# ---------------------------------------------------------------- host-only --

def test_feature_dims_follow_the_host_table(llmx):
    """feature_input_dim / feature_output_dim / needs_rhs host:2015-2061."""
    s = llmx.shape("qwen2.5-3b")
    H, I, KV = s.hidden, s.inter, s.kv_channels
    want = {1: (H, H, False), 2: (H, KV, False), 3: (H, KV, False), 4: (H, H, False), 5: (H, I, False),
            6: (H, I, False), 7: (I, H, False), 8: (H, H, True), 9: (I, I, True), 10: (H, H, True)}
    for op, dims in want.items():
        assert llmx.feature_dims(s, op) == dims, op
    for op in (0, 11, 15, 16, 17, 18, 20):
        with pytest.raises(llmx.LlmxError):
            llmx.feature_dims(s, op)


def test_resident_image_accepts_only_the_layer_tasks(llmx):
    """The production image rejects every per-operator mode (control_cache_8x64.cpp:6484-6494)."""
    s = llmx.shape("qwen2.5-3b")
    for op in range(21):
        code, st = llmx.validate_task(s, op, 0, 0, 1)
        ok = op in (0, 16, 18, 19, 20)
        assert code == (llmx.OK if ok else llmx.BAD_OPERATOR), op
        assert st.op == op and st.last_task == 1
    code, _ = llmx.validate_task(s, 21, 0, 0, 1)
    assert code == llmx.BAD_OPERATOR


def test_full_image_validation_order(llmx):
    """Rows first (:5891-5897), then the operator, then the layer; feature operators
    have no position check; tile diagnostics 11-15 are not served."""
    s = llmx.shape("qwen2.5-3b")
    code, st = llmx.validate_operator(s, 5, 99, 0, 9)
    assert code == llmx.BAD_TOKEN_COUNT and st.op == llmx.OP_NOP
    for op in range(11, 16):
        assert llmx.validate_operator(s, op, 0, 0, 1)[0] == llmx.BAD_OPERATOR
    assert llmx.validate_operator(s, llmx.OP_FFN_GATE, s.layers, 0, 1)[0] == llmx.BAD_LAYER
    assert llmx.validate_operator(s, llmx.OP_FFN_GATE, 0, 10 ** 6, 1)[0] == llmx.OK
    assert llmx.validate_operator(s, llmx.OP_ATTN_PREFILL_BLOCK, 0, 0, 0)[0] == llmx.BAD_TOKEN_COUNT
    assert llmx.validate_operator(s, llmx.OP_ATTN_PREFILL_BLOCK, 0, s.max_seq - 3, 4)[0] == llmx.BAD_POSITION
    assert llmx.validate_operator(s, llmx.OP_ATTN_PREFILL_BLOCK, 0, s.max_seq - 4, 4)[0] == llmx.OK


def test_feature_status_counters(llmx):
    """Projection waves (:7273-7405; repeated-gate case tb:700-770) and the two-core
    vector split (:7411-7497; SiLU-Mul case tb:2485-2575)."""
    s = llmx.shape("qwen2.5-3b")
    for op in range(1, 8):
        out_dim = llmx.feature_dims(s, op)[1]
        code, st = llmx.validate_operator(s, op, 3, 0, 5)
        w = cdiv(out_dim, 128)
        assert code == 0 and (st.output_waves, st.mm_tasks, st.vector_tasks, st.completed_packets) == (
            w, 2 * w, 0, 2 * w * 32), op
    for op in (8, 9, 10):
        out_dim = llmx.feature_dims(s, op)[1]
        for rows in (1, 4, 5, 8):
            code, st = llmx.validate_operator(s, op, 0, 0, rows)
            cores = (rows > 0) + (rows > 4)
            assert (st.mm_tasks, st.vector_tasks, st.completed_packets) == (0, cores, rows * cdiv(out_dim, 16))


def test_decoder_layer_status_counters(llmx):
    """run_resident_decoder_layer_route_case tb:2680-2880: one token at position 0."""
    s = llmx.shape("qwen2.5-3b")
    H, I, KV, hd = s.hidden, s.inter, s.kv_channels, s.head_dim
    waves = (cdiv(H, 128) + 2 * cdiv(KV, 128) + (1 + cdiv(hd, 64)) + cdiv(H, 128) + 2 * cdiv(I, 128)
             + cdiv(H, 128))
    packets = waves * 2 * 32 + 4 * cdiv(H, 16) + cdiv(I, 16)
    code, st = llmx.validate_task(s, llmx.OP_DECODER_LAYER, 0, 0, 1)
    assert code == 0
    assert (st.output_waves, st.mm_tasks, st.vector_tasks, st.completed_packets) == (waves, 2 * waves, 5, packets)
    # a longer block is the sum of its two sublayers
    for pos, rows in ((0, 8), (100, 5), (2040, 8)):
        _, a = llmx.validate_task(s, llmx.OP_ATTENTION, 1, pos, rows)
        _, f = llmx.validate_task(s, llmx.OP_FFN, 1, pos, rows)
        _, d = llmx.validate_task(s, llmx.OP_DECODER_LAYER, 1, pos, rows)
        for k in ("output_waves", "mm_tasks", "vector_tasks", "completed_packets"):
            assert getattr(d, k) == getattr(a, k) + getattr(f, k), (pos, rows, k)


def test_prefill_block_status_counters(llmx):
    """Prefill block status (tb:2065-2085, check_prefill_block_attention_status host:5587-5604)."""
    s = llmx.shape("qwen2.5-3b")
    G, pv = s.heads // s.kv_heads, cdiv(s.head_dim, 64)
    for pos, rows in ((0, 1), (0, 8), (60, 8), (1000, 3)):
        code, st = llmx.validate_operator(s, llmx.OP_ATTN_PREFILL_BLOCK, 0, pos, rows)
        tasks = 2 * cdiv(pos + rows, 64) * G * (1 + pv)
        assert code == 0 and (st.output_waves, st.mm_tasks, st.completed_packets) == (pv, tasks, tasks * 32)


# --------------------------------------------------------------------- GPU --

def _views(oracle, s, blob):
    q, k, v, o, g, u, d = oracle.layer_views(oracle_shape(oracle, s), blob)
    return {1: q, 2: k, 3: v, 4: o, 5: g, 6: u, 7: d}


@pytest.fixture(scope="module", params=["small", "qwen-layer"])
def feature_ctx(request, llmx, oracle):
    s = llmx.shape(request.param)
    m = llmx.Model(s)
    if request.param == "small":
        m.init_reference_random(11)
    else:
        m.init_gaussian(20260718, 0.02)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    yield s, m, acc
    acc.close()


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [1, 5, 8])
def test_feature_operators_match_oracle(llmx, oracle, feature_ctx, rows):
    """Every feature operator on random rows (make_random_tensor ranges of
    run_random_verification) and on saturating rows, vs the oracle, exactly."""
    s, m, acc = feature_ctx
    rng = np.random.default_rng(rows)
    views = _views(oracle, s, m.layer(s.layers - 1))
    norms = m.norms()
    for scale in (600, 32767):
        x_h = rng.integers(-scale, scale + 1, (rows, s.hidden)).astype(np.int16)
        x_i = rng.integers(-scale, scale + 1, (rows, s.inter)).astype(np.int16)
        for op in range(1, 8):
            x = x_i if op == llmx.OP_FFN_DOWN else x_h
            out, st = acc.run_feature(op, x, layer=s.layers - 1)
            _same(out, oracle.projection(x, views[op]), f"op {op} scale {scale}")
            assert st.as_dict() == llmx.validate_operator(s, op, s.layers - 1, 0, rows)[1].as_dict()
        w = norms[2 * (s.layers - 1)]
        out, st = acc.run_feature(llmx.OP_RMSNORM, x_h, w[None, :])
        _same(out, oracle.rmsnorm(x_h, w), f"rmsnorm scale {scale}")
        up = rng.integers(-scale, scale + 1, (rows, s.inter)).astype(np.int16)
        out, st = acc.run_feature(llmx.OP_SILU_MUL, x_i, up)
        _same(out, oracle.silu_mul(x_i, up), f"silu_mul scale {scale}")
        rhs = rng.integers(-scale, scale + 1, (rows, s.hidden)).astype(np.int16)
        out, st = acc.run_feature(llmx.OP_RESIDUAL_ADD, x_h, rhs)
        _same(out, oracle.residual(x_h, rhs), f"residual scale {scale}")
        assert st.as_dict() == llmx.validate_operator(s, llmx.OP_RESIDUAL_ADD, 0, 0, rows)[1].as_dict()


@pytest.mark.gpu
def test_feature_operator_errors(llmx, feature_ctx):
    """run_feature's shape checks (runtime_error) come before any launch; controller
    codes come back as codes."""
    s, m, acc = feature_ctx
    x = np.zeros((2, s.hidden), np.int16)
    for bad in (lambda: acc.run_feature(llmx.OP_Q_PROJECTION, np.zeros((2, s.hidden + 8), np.int16)),
                lambda: acc.run_feature(llmx.OP_Q_PROJECTION, np.zeros((9, s.hidden), np.int16)),
                lambda: acc.run_feature(llmx.OP_RMSNORM, x),
                lambda: acc.run_feature(llmx.OP_RMSNORM, x, np.zeros((2, s.hidden), np.int16)),
                lambda: acc.run_feature(llmx.OP_RESIDUAL_ADD, x, np.zeros((1, s.hidden), np.int16)),
                lambda: acc.run_feature(llmx.OP_ATTENTION, x)):
        with pytest.raises(llmx.LlmxError) as e:
            bad()
        assert e.value.code == llmx.ERR_ARG
    with pytest.raises(llmx.LlmxError) as e:
        acc.run_feature(llmx.OP_FFN_GATE, x, layer=s.layers)
    assert e.value.code == llmx.BAD_LAYER
    out, _ = acc.run_feature(llmx.OP_RESIDUAL_ADD, x, x)  # the context stays usable
    assert not out.any()


@pytest.mark.gpu
def test_decoder_layer_task_matches_sublayers(llmx, oracle):
    """Op 16 = Task 18 then Task 19 on the bound pairs; the input pair is unchanged and
    the KV cache is appended as by Task 18."""
    s = llmx.shape("small")
    m = llmx.Model(s).init_reference_random(5)
    acc = llmx.Accelerator(s)
    try:
        acc.upload_model(m)
        layers = [m.layer(l) for l in range(s.layers)]
        ref = OracleState(oracle, oracle_shape(oracle, s), layers, m.norms())
        rng = np.random.default_rng(16)
        pos = 0
        for rows in (8, 3, 1, 1):
            h = rng.integers(-700, 700, (rows, s.hidden)).astype(np.int16)
            for l in range(s.layers):
                acc.write_hidden(1, h)
                acc.bind(0, 1)
                rc, st = acc.task(llmx.OP_DECODER_LAYER, l, pos, rows)
                want = ref.task19(l, ref.task18(l, h, pos))
                _same(acc.read_hidden(0, rows), want, f"decoder layer {l} pos {pos}")
                _same(acc.read_hidden(1, rows), h, "input pair unchanged")
                k, v = acc.read_kv(l, 0, pos + rows)
                _same(k, ref.kc[l][:, :pos + rows], f"K cache layer {l}")
                _same(v, ref.vc[l][:, :pos + rows], f"V cache layer {l}")
                assert st.as_dict() == llmx.validate_task(s, llmx.OP_DECODER_LAYER, l, pos, rows)[1].as_dict()
                h = want
            pos += rows
    finally:
        acc.close()


@pytest.mark.gpu
@pytest.mark.parametrize("pos,rows", [(0, 1), (0, 8), (60, 8), (127, 1), (1000, 5), (2040, 8)])
def test_prefill_block_attention_matches_oracle(llmx, oracle, pos, rows):
    """Op 17 over a preloaded cache (initialize_kv_cache_heads host:7104-7117 then
    run_prefill_attention_block), every token's G heads vs the oracle's tiled Q2.14
    attention over positions 0..position+t."""
    s = llmx.shape("qwen-layer-long")
    acc = llmx.Accelerator(s)
    try:
        rng = np.random.default_rng(pos * 10 + rows)
        G, hd, KVh = s.heads // s.kv_heads, s.head_dim, s.kv_heads
        ctx = pos + rows
        k = rng.integers(-900, 900, (KVh, ctx, hd)).astype(np.int16)
        v = rng.integers(-900, 900, (KVh, ctx, hd)).astype(np.int16)
        k[:, ::7] = 32767  # saturating K and V entries as well
        v[:, ::5] = -32768
        acc.write_kv(0, 0, k, v)
        q = rng.integers(-1500, 1500, (KVh, rows, G, hd)).astype(np.int16)
        out, st = acc.run_prefill_attention_block(q, pos)
        for p in range(KVh):
            for t in range(rows):
                want = oracle.attention_group(q[p, t], k[p, :pos + t + 1], v[p, :pos + t + 1])
                _same(out[p, t], want, f"kv head {p} token {t} (position {pos + t})")
        assert st.as_dict() == llmx.validate_operator(s, llmx.OP_ATTN_PREFILL_BLOCK, 0, pos, rows)[1].as_dict()
    finally:
        acc.close()
