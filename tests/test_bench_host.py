"""Host-side logic of bench.py, no GPU needed.

* the algorithmic bytes behind every roofline fraction: one decode forward of
  the Qwen2.5-3B shape streams W(N) = 152,043,520 / N + 2,097,152 weight bytes
  per layer (Q, O, Gate, Up, Down sharded over N ranks; K, V replicated), reads
  1,024 B of K/V per cached position, writes 1,024 B of K/V and reads two norm
  rows; bench.py adds the RoPE row and the hidden rows in and out;
* the clock record: median SM clock under load and the throttle reasons that
  reject a run;
* the BASELINE config 0-2 legs, run against stand-ins for the device objects
  (the CUDA context, the executor and CUDA events), so that the code that
  follows the headline on the GPU box is exercised here; a failing leg must be
  reported in the returned object, never raised.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


@pytest.fixture(scope="module")
def bench(llmx):
    import bench as B
    return B


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("ctx", [513, 640, 2049])
def test_decode_bytes_follow_the_weight_stream(llmx, bench, world, ctx):
    s = llmx.shape("qwen2.5-3b", max_seq=2304)
    weights = 152_043_520 // world + 2_097_152
    kv = 1024 * ctx + 1024
    norms, rope, rows = 2 * 2 * s.hidden, 2 * s.head_dim, 4 * 2 * s.hidden
    want = s.layers * (weights + kv + norms + rope + rows) + 2 * s.hidden * 2
    assert bench.bytes_per_decode(s, world, ctx) == want
    if world == 1:  # SURVEY's per-token figure at c = 640: 5,549,064,192 B of weights
        assert s.layers * weights == 5_549_064_192


def test_clock_record(bench, tmp_path):
    c = bench.ClockSampler(0)
    c.proc = type("P", (), {"terminate": lambda self: None, "wait": lambda self: 0})()
    c.path = str(tmp_path / "clocks.csv")
    lines = ["0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active",
             "0, 1950, 1965, 810.0, 0x4, Not Active, Not Active, Not Active, Active",
             "0, 1965, 1965, 820.0, 0x0, Not Active, Not Active, Not Active, Not Active",
             "0, 345, 1965, 90.0, 0x0, Not Active, Not Active, Not Active, Not Active",  # idle sample
             "garbage line"]
    with open(c.path, "w") as f:
        f.write("\n".join(lines) + "\n")
    c.f = open(os.devnull, "w")
    rec = c.stop()
    assert rec["sm_mhz"] == 1965.0 and rec["sm_max_mhz"] == 1965.0
    assert rec["reasons"] == ["sw_power_cap"] and rec["samples"] == 4


class _FakeAccelerator:
    def __init__(self, s, **kw):
        self.shape, self.h, self.stream, self.fail = s, 1, 0, False

    def upload_model(self, m):
        pass

    def stack(self, hidden, layer_begin=0, layer_count=None, position=0, include_final_norm=True,
              materialize=True):
        assert position + len(hidden) <= self.shape.max_seq
        return np.zeros((len(hidden), self.shape.hidden), np.int16)

    def stack_async(self, rows, layer_begin, layer_count, position, include_final_norm=True):
        assert position + rows <= self.shape.max_seq and layer_begin + layer_count <= self.shape.layers

    def write_hidden(self, pair, rows):
        assert rows.shape == (8, self.shape.hidden)

    def upload_vocab(self, m):
        pass

    def reset_kv(self):
        pass

    def generate(self, prompt, max_new, **kw):
        return [0] * max_new

    def synchronize(self):
        pass

    def close(self):
        self.h = 0


class _FakeExecutor:
    def __init__(self, acc, m):
        self.acc = acc

    def run_prompt_block(self, tokens, position, materialize=True):
        return np.zeros((len(tokens), self.acc.shape.hidden), np.int16)

    def run_token(self, token, position):
        return np.zeros((1, self.acc.shape.hidden), np.int16)


class _FakeEvent:
    def __init__(self, **kw):
        pass

    def record(self, stream=None):
        pass

    def synchronize(self):
        pass

    def elapsed_time(self, other):
        return 2.0


def test_config_legs_on_stand_ins(llmx, bench, monkeypatch):
    torch = pytest.importorskip("torch")
    monkeypatch.setattr(llmx, "Accelerator", _FakeAccelerator)
    monkeypatch.setattr(llmx, "Executor", _FakeExecutor)
    monkeypatch.setattr(torch.cuda, "Event", _FakeEvent)
    monkeypatch.setattr(torch.cuda, "ExternalStream", lambda ptr: None)
    out = bench.config_legs()
    assert set(out) == {"config0", "config1", "config2"}
    for k, v in out.items():
        assert "error" not in v, (k, v)
    assert out["config0"]["cpu_oracle_ms"]["cores"] == 1
    assert set(out["config2"]["prefill_tok_s"]) == {"8", "64", "256", "1024"}
    assert out["config2"]["prefill_tok_s"]["1024"] == pytest.approx(1024 / 2e-3)


def test_config_legs_report_failures(llmx, bench, monkeypatch):
    def broken(*a, **kw):
        raise llmx.LlmxError(llmx.ERR_CUDA, "no device")
    monkeypatch.setattr(llmx, "Accelerator", broken)
    out = bench.config_legs()
    assert all("error" in out[k] for k in ("config0", "config1", "config2"))
