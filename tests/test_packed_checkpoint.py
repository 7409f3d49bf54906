"""Packed-checkpoint loader (model_data_t::load host/host_qwen_8x64.cpp:789-840,
tile/shard order of projection_weight_raw :899-935) against a reference-format
fixture written by tests/golden/make_packed_fixture.py, which restates the
reference's indexing independently of the library's loader."""
import os
import sys

import numpy as np
import pytest

from helpers import OracleState, diff_report, oracle_shape

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "packed_small")
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_packed_fixture as fx  # noqa: E402


def _load(llmx):
    s = llmx.shape("small", inter=fx.SHAPE["inter"])
    m = llmx.Model(s)
    m.load_packed(FIXTURE, tie_embeddings=False)
    return s, m


def test_fixture_files_are_the_generator_output():
    """The committed files are exactly what the generator writes."""
    emb, norms, head, layers = fx.dense_model()
    shards = fx.pack_shards(layers)
    for k in range(16):
        got = np.fromfile(os.path.join(FIXTURE, f"layer_weights_shard{k:02d}.fix16.bin"), "<i2")
        assert np.array_equal(got, shards[k].ravel()), f"shard {k}"
    assert np.array_equal(np.fromfile(os.path.join(FIXTURE, "norm_weights.fix16.bin"), "<i2"), norms.ravel())


def test_loader_reads_reference_layout(llmx):
    s, m = _load(llmx)
    emb, norms, head, layers = fx.dense_model()
    for l in range(s.layers):
        want = np.concatenate([w.ravel() for w in layers[l]])
        assert np.array_equal(m.layer(l), want), f"layer {l}"
    assert np.array_equal(m.norms(), norms)
    assert np.array_equal(m.embed(np.arange(s.vocab)), emb)
    for r in (emb[3], emb[40] // 3):
        scores = head.astype(np.int64) @ r.astype(np.int64)
        assert m.lm_head_argmax(r) == int(np.argmax(scores))  # untied head, first maximum


def test_loader_rejects_truncated_shard(llmx, tmp_path):
    import shutil
    for f in os.listdir(FIXTURE):
        shutil.copy(os.path.join(FIXTURE, f), tmp_path / f)
    p = tmp_path / "layer_weights_shard07.fix16.bin"
    p.write_bytes(p.read_bytes()[:-64])
    s = llmx.shape("small", inter=fx.SHAPE["inter"])
    with pytest.raises(llmx.LlmxError) as e:
        llmx.Model(s).load_packed(str(tmp_path))
    assert e.value.code == llmx.ERR_IO


@pytest.mark.gpu
def test_packed_checkpoint_on_device_matches_oracle(llmx, oracle):
    """The loaded checkpoint through the device stack (prompt block + decodes),
    bit-exact against the oracle on the generator's dense weights."""
    s, m = _load(llmx)
    emb, norms, head, layers = fx.dense_model()
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    ref = OracleState(oracle, oracle_shape(oracle, s), [np.concatenate([w.ravel() for w in L]) for L in layers], norms)
    toks = [5, 9, 2, 33, 61, 7]
    out = acc.stack(emb[toks], position=0)
    want = ref.stack(emb[toks], 0)
    assert np.array_equal(out, want), diff_report(out, want)
    for i in range(3):
        out = acc.stack(emb[[toks[i]]], position=6 + i)
        want = ref.stack(emb[[toks[i]]], 6 + i)
        assert np.array_equal(out, want), diff_report(out, want)
    acc.close()
