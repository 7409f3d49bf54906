"""C ABI and host-side logic, no GPU needed.

The library must load, export every symbol include/llmx.h declares, and its
host logic (shapes, controller validation and status records, constant tables,
model generators, embedding, LM head) must agree with the oracle.
"""
import ctypes as C
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_header_symbols(llmx):
    header = open(os.path.join(ROOT, "include", "llmx.h")).read()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    names = sorted(set(re.findall(r"\b(llmx_\w+)\s*\(", header)))
    assert len(names) > 30
    lib = C.CDLL(llmx.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_timeline_only_in_the_measurement_build(tmp_path):
    """The launch timeline (csrc/timeline.cuh) exists only when compiled with
    -DLLMX_TIMELINE: the product library exports none of its symbols, and the
    instrumented form of the header and of an argument struct compiles."""
    lib = C.CDLL(os.path.join(ROOT, "llm-accel_b200", "libllmx.so"))
    assert not hasattr(lib, "llmx_timeline_read") and not hasattr(lib, "llmx_tl_table_gemv")
    nvcc = "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    src = tmp_path / "tl_probe.cu"
    src.write_text('#include "kernels.cuh"\n'
                   "__global__ void k_probe(const llmx::NormArgs a) { LLMX_TL_GUARD(a.tl_slot); }\n"
                   "int llmx::tl_take(const char *) { return 0; }\n"
                   "void probe_take(llmx::NormArgs &a) { LLMX_TL_TAKE(a, \"probe\"); }\n"
                   "LLMX_TL_READER(probe)\n")
    csrc = os.path.join(ROOT, "llm-accel_b200", "csrc")
    import subprocess
    r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-DLLMX_TIMELINE",
                        "-I", csrc, "-I", os.path.join(ROOT, "include"), "-c", str(src), "-o",
                        str(tmp_path / "tl_probe.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]


def test_profiles(llmx, oracle):
    for name, vals in oracle.PROFILES.items():
        assert llmx.profile(name).tuple() == vals
    with pytest.raises(llmx.LlmxError):
        llmx.profile("nope")


def test_shape_validation(llmx):
    assert llmx.lib().llmx_shape_validate(C.byref(llmx.shape("qwen2.5-3b"))) == 0
    bad = llmx.shape("small", heads=3)  # 64 % 3 != 0
    assert llmx.lib().llmx_shape_validate(C.byref(bad)) == llmx.ERR_ARG
    bad = llmx.shape("small", hidden=64 * 3, heads=1, kv_heads=1)  # head_dim 192 > 128
    assert llmx.lib().llmx_shape_validate(C.byref(bad)) == llmx.ERR_UNSUPPORTED


def test_controller_validation_order(llmx):
    """kernel/control_cache_8x64.cpp:5891-5972: row count before operator,
    NOP always OK, layer, then per-task row/position rules."""
    s = llmx.shape("qwen2.5-3b")
    code, st = llmx.validate_task(s, 99, 0, 0, 9)
    assert code == llmx.BAD_TOKEN_COUNT and st.op == 0
    assert llmx.validate_task(s, 99, 0, 0, 1)[0] == llmx.BAD_OPERATOR
    assert llmx.validate_task(s, 16, 0, 0, 1)[0] == llmx.OK  # compatibility full-layer task (:6031-6036)
    assert llmx.validate_task(s, 17, 0, 0, 1)[0] == llmx.BAD_OPERATOR  # per-operator modes: not this image
    assert llmx.validate_task(s, 16, 0, 2041, 8)[0] == llmx.BAD_POSITION
    assert llmx.validate_task(s, 0, 999, 9999, 1)[0] == llmx.OK
    assert llmx.validate_task(s, 18, 36, 0, 1)[0] == llmx.BAD_LAYER
    assert llmx.validate_task(s, 20, 36, 0, 1)[0] == llmx.BAD_LAYER
    assert llmx.validate_task(s, 19, 0, 0, 0)[0] == llmx.BAD_TOKEN_COUNT
    assert llmx.validate_task(s, 18, 0, 2048, 1)[0] == llmx.BAD_POSITION
    assert llmx.validate_task(s, 18, 0, 2041, 8)[0] == llmx.BAD_POSITION
    assert llmx.validate_task(s, 18, 0, 2040, 8)[0] == llmx.OK
    assert llmx.validate_task(s, 20, 0, 5000, 8)[0] == llmx.OK  # final norm ignores position


def test_status_counters(llmx):
    """Counter formulas of tests/closed_loop_8x64_cosim_tb.cpp:523-626 (CC8
    outputs/wave 128, attention tile 64, 16-lane packets)."""
    s = llmx.shape("qwen2.5-3b")
    code, st = llmx.validate_task(s, 18, 0, 8, 1)
    waves = 16 + 2 * 2 + 1 * 3 + 16  # Q, K+V, ceil(9/64)*(1+2), O
    assert st.output_waves == waves and st.mm_tasks == 2 * waves
    assert st.vector_tasks == 2 and st.completed_packets == waves * 64 + 2 * 128
    code, st = llmx.validate_task(s, 19, 3, 100, 8)
    waves = 2 * 86 + 16
    assert (st.output_waves, st.vector_tasks) == (waves, 6)
    assert st.completed_packets == waves * 64 + 8 * (2 * 128 + 688)
    code, st = llmx.validate_task(s, 20, 0, 0, 5)
    assert (st.output_waves, st.mm_tasks, st.vector_tasks, st.completed_packets) == (0, 0, 2, 5 * 128)
    assert st.last_task == 1 and st.op == 20 and st.token_count == 5


def test_tables_match_oracle(llmx, oracle):
    e, p = llmx.exp_tables()
    oe, op = oracle.exp_tables(oracle.EXP_TRUNC)
    assert np.array_equal(e, oe) and np.array_equal(p, op)
    assert p[2048] == 16384 and e[2048] == 256
    for hd, ms in ((16, 32), (128, 2304)):
        assert np.array_equal(llmx.rope_table(hd, ms), oracle.rope_table(hd, ms))


def test_gauss_sampler_matches_oracle(llmx, oracle):
    for sigma, stream, idx0 in ((81.92, 0x1000, 0), (256.0, 0x10, 123456789), (3.5, 7, 5)):
        a = llmx.gauss_fill(20260718, stream, sigma, 200000, idx0)
        b = oracle.gauss_fill(20260718, stream, sigma, 200000, idx0)
        assert np.array_equal(a, b)
    # sanity of the distribution: N(0, 0.02) in Q4.12 has raw sigma 81.92
    a = llmx.gauss_fill(1, 2, 81.92, 400000).astype(np.float64)
    assert abs(a.mean()) < 0.5 and abs(a.std() - 81.92) < 0.5


@pytest.mark.parametrize("profile", ["small", "qwen-layer"])
def test_reference_random_model_matches_oracle(llmx, oracle, profile):
    s = llmx.shape(profile)
    m = llmx.Model(s).init_reference_random(20260718)
    emb, norms, dense = oracle.ref_random_model(oracle.shape(profile), 20260718, s.layers)
    assert np.array_equal(m.norms(), norms)
    assert np.array_equal(m.embed(np.arange(s.vocab)), emb)
    for l in range(s.layers):
        assert np.array_equal(m.layer(l), dense[l])


def test_gaussian_model_layout(llmx, oracle):
    s = llmx.shape("small")
    m = llmx.Model(s).init_gaussian(5, 0.02)
    blob = m.layer(1)
    views = oracle.layer_views(oracle.shape("small"), blob)
    # Down projection of layer 1 is stream 0x1000 + 1*16 + 6, dense [out][in]
    d = oracle.gauss_fill(5, 0x1000 + 16 + 6, 0.02 * 4096, s.hidden * s.inter)
    assert np.array_equal(views[6].reshape(-1), d)
    assert np.all(m.norms() == 256)
    e = m.embed([3, 60])
    assert np.array_equal(e[1], oracle.gauss_fill(5, 0x10, 256.0, s.hidden, 60 * s.hidden))


def test_lm_head_argmax_matches_oracle(llmx, oracle):
    s = llmx.shape("small")
    m = llmx.Model(s).init_reference_random(3)
    table = m.embed(np.arange(s.vocab))
    rng = np.random.default_rng(0)
    for _ in range(5):
        h = rng.integers(-32768, 32767, s.hidden).astype(np.int16)
        assert m.lm_head_argmax(h) == oracle.lm_head_argmax(h, table)
    # ties: the first maximum wins (strict '>' host:961-967)
    h = np.zeros(s.hidden, np.int16)
    assert m.lm_head_argmax(h) == 0


def test_packed_checkpoint_roundtrip(llmx, oracle, tmp_path):
    """model_data_t::load host:789-840 on files written in the reference's packed
    16x16-tile / 16-shard layout (projection_weight_raw host:899-935)."""
    s = llmx.shape("small")
    src = llmx.Model(s).init_reference_random(11)
    H, I, KV = s.hidden, s.inter, s.kv_channels
    tiles = (H // 16) ** 2 * 2 + (KV // 16) * (H // 16) * 2 + (I // 16) * (H // 16) * 3
    words = (tiles * s.layers + 1) // 2
    (tmp_path / "token_embedding.fix16.bin").write_bytes(src.embed(np.arange(s.vocab)).tobytes())
    (tmp_path / "norm_weights.fix16.bin").write_bytes(np.ascontiguousarray(src.norms()).tobytes())
    shards = np.zeros((16, words, 32), np.int16)
    base = np.cumsum([0, (H // 16) ** 2, (KV // 16) * (H // 16), (KV // 16) * (H // 16), (H // 16) ** 2,
                      (I // 16) * (H // 16), (I // 16) * (H // 16), (H // 16) * (I // 16)])
    dims = [(H, H), (KV, H), (KV, H), (H, H), (I, H), (I, H), (H, I)]
    for l in range(s.layers):
        views = oracle.layer_views(oracle.shape("small"), src.layer(l))
        for op, (od, idim) in enumerate(dims):
            in_tiles = idim // 16
            for o in range(od):
                for i in range(idim):
                    gt = l * tiles + base[op] + (o // 16) * in_tiles + i // 16
                    lane_in_tile = (o % 16) * 16 + i % 16
                    shard = (gt & 1) * 8 + lane_in_tile // 32
                    shards[shard, gt >> 1, lane_in_tile % 32] = views[op][o, i]
    for k in range(16):
        (tmp_path / f"layer_weights_shard{k:02d}.fix16.bin").write_bytes(shards[k].tobytes())
    m = llmx.Model(s).load_packed(str(tmp_path), tie_embeddings=True)
    for l in range(s.layers):
        assert np.array_equal(m.layer(l), src.layer(l))
    assert np.array_equal(m.norms(), src.norms())
    (tmp_path / "norm_weights.fix16.bin").write_bytes(b"\0" * 10)
    with pytest.raises(llmx.LlmxError) as e:
        llmx.Model(s).load_packed(str(tmp_path), tie_embeddings=True)
    assert e.value.code == llmx.ERR_IO


def test_create_without_gpu_fails_loudly(llmx):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(llmx.LlmxError) as e:
        llmx.Accelerator(llmx.shape("small"))
    assert e.value.code in (llmx.ERR_CUDA, llmx.ERR_NOMEM)
