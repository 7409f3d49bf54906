#!/usr/bin/env python3
"""Decode / prefill tokens per second of the Qwen2.5-3B-shaped fixed-point
decoder stack (LLM-ACCEL's resident Task 18/19/20 path) on B200.

One step = one single-row decode forward through all 36 layers plus the final
RMSNorm (run_token, host/host_qwen_8x64.cpp:7665).  The workload is BASELINE
config 3 on one GPU (512-token prompt as 64 P8 blocks, then decodes at
positions 512..639) and config 4 under tensor parallelism (2048-token prompt,
decodes from 2048).  Prefill tok/s of the prompt is reported beside it.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl llmx|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...

Rank 0 prints one JSON line.  At N=1 it also carries `configs`: BASELINE
configs 0-2 (one or two layers, the prefill-length sweep) as small bounded runs
after the headline.  `--impl reference` times the reference's
fixed-point oracle (its CPU restatement in oracle/, all host threads) on the
same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llm-accel_b200"))

SEED = 20260718
W_SIGMA = 0.02
METRIC = "decode tok/s, Qwen2.5-3B-shaped 36-layer fixed-point stack (prefill tok/s, % HBM roofline alongside)"
CONFIGS = {
    3: {"prompt": 512, "decodes": 128,
        "name": "config3: 36-layer Qwen2.5-3B shape, 512-token prompt (64 P8 blocks) + 128 decode forwards, 1 GPU"},
    4: {"prompt": 2048, "decodes": 256,
        "name": "config4: 36-layer Qwen2.5-3B shape, 2048-token prompt (256 P8 blocks) + 256 decode forwards, "
                "tensor parallel"},
}


def bench_config(cfg_id, world, P, K):
    """The `config` object of both arms (same keys)."""
    return {"workload": CONFIGS[cfg_id]["name"], "layers": 36, "hidden": 2048, "ffn": 11008, "heads": 16,
            "kv_heads": 2, "prompt_tokens": P, "decode_positions": [P, P + K - 1], "rows_per_decode": 1,
            "sequence_batch": 1, "parallelism": f"tp{world}",
            "l2": "no flush: every step streams 5.5 GB/N of weights (>> 126 MB L2)"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic(name):
    """dram bytes per launch from a committed ncu summary (profiles/<name>), or None."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms in the background."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.path = f"/tmp/llmx_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu)], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        # nvidia-smi takes a while to start: the timed region begins only once it
        # is sampling (bounded wait), so that the record covers the region
        deadline = time.time() + 5.0
        while self.proc is not None and time.time() < deadline and self.proc.poll() is None:
            self.f.flush()
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.02)
        self.t0 = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        sms, maxs, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, mx = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            sms.append(sm)
            maxs.append(mx)
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in sms if s > 0.5 * max(sms)]
        return {"sm_mhz": float(np.median(loaded)), "sm_max_mhz": max(maxs), "reasons": sorted(reasons),
                "samples": len(sms)}


def embed_rows(tokens, hidden):
    import llmx
    return np.stack([llmx.gauss_fill(SEED, 0x10, 256.0, hidden, int(t) * hidden) for t in tokens])


def bytes_per_decode(shape, world, ctx):
    """Algorithmic HBM bytes of one decode forward per GPU at context `ctx`
    (weights once, KV rows read + appended, norm rows, RoPE row, hidden rows)."""
    H, I, hd, KV = shape.hidden, shape.inter, shape.head_dim, shape.kv_channels
    w = 2 * (2 * H * H // world + 2 * KV * H + 3 * I * H // world)
    per_layer = w + 2 * 2 * KV * ctx + 2 * 2 * KV + 2 * 2 * H + 2 * hd + 4 * 2 * H
    return shape.layers * per_layer + 2 * H * 2


def run_llmx(args, cfg_id, world, rank, local, K, W):
    import torch
    import llmx

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    cfg = CONFIGS[cfg_id]
    P = cfg["prompt"]
    ndec = max(K, W, cfg["decodes"])
    shape = llmx.shape("qwen2.5-3b", max_seq=P + ndec)
    H, L = shape.hidden, shape.layers
    tp_id = None
    if world > 1:
        obj = [llmx.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        tp_id = obj[0]
    acc = llmx.Accelerator(shape, device=local, tp_rank=rank, tp_size=world, tp_id=tp_id)

    t_setup = time.time()
    model = None
    if world == 1:
        model = llmx.Model(shape).init_gaussian(SEED, W_SIGMA, lm_head=False)
        acc.upload_model(model)
    else:  # generate layer by layer (each rank slices its own shard on upload)
        sizes = [H * H, shape.kv_channels * H, shape.kv_channels * H, H * H, shape.inter * H,
                 shape.inter * H, H * shape.inter]
        buf = np.empty(sum(sizes), np.int16)
        for l in range(L):
            off = 0
            for op, n in enumerate(sizes):
                buf[off:off + n] = llmx.gauss_fill(SEED, 0x1000 + 16 * l + op, W_SIGMA * 4096.0, n)
                off += n
            acc.upload_layer(l, buf)
        acc.upload_norms(np.full((2 * L + 1, H), 256, np.int16))
    setup_s = time.time() - t_setup

    rng = np.random.default_rng(SEED)
    prompt = rng.integers(0, shape.vocab, P)
    dec = rng.integers(0, shape.vocab, ndec)
    rows = embed_rows(np.concatenate([prompt, dec]), H).astype(np.int16)
    dev_rows = torch.from_numpy(rows).cuda()
    stream = torch.cuda.ExternalStream(acc.stream)

    class _Dev:
        def __init__(self, ptr, shp):
            self.__cuda_array_interface__ = {"shape": shp, "typestr": "<i2", "data": (ptr, False),
                                             "version": 3, "strides": None}

    hid1 = torch.as_tensor(_Dev(acc.hidden_ptr(1), (8, H)), device="cuda")
    launches = [0]

    def prefill():
        nb = P // 8
        for b in range(nb):
            with torch.cuda.stream(stream):
                hid1[:8].copy_(dev_rows[8 * b:8 * b + 8], non_blocking=True)
            acc.stack_async(8, 0, L, 8 * b, include_final_norm=(b == nb - 1))
            launches[0] += acc.kernel_launches

    def decode(i):
        with torch.cuda.stream(stream):
            hid1[:1].copy_(dev_rows[P + i:P + i + 1], non_blocking=True)
        acc.stack_async(1, 0, L, P + i, include_final_norm=True)
        launches[0] += acc.kernel_launches

    def device_time(fn):
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        e1.synchronize()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if dist:
            t = torch.tensor([ms], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms

    clocks = ClockSampler(local)
    prefill()                                   # warm-up pass: graph capture for 8 rows
    acc.synchronize()
    clocks.start()
    prefill_ms = device_time(prefill)           # timed prefill of the whole prompt
    for i in range(W):                          # warm-up decodes at positions P..P+W-1
        decode(i)
    acc.synchronize()
    launches[0] = 0
    decode_ms = device_time(lambda: [decode(i) for i in range(K)])
    gpu_launches = launches[0]
    clock = clocks.stop()

    # end to end through the public API: the step's embedding row copied from the
    # host table (rows, drawn before timing -- a resident table as in
    # model_data_t::embedding host:871-884) into pinned memory, H2D, the stack,
    # final norm, D2H of the output row, every step
    in_p = torch.empty((1, H), dtype=torch.int16).pin_memory()
    out_p = torch.empty((1, H), dtype=torch.int16).pin_memory()
    in_np = in_p.numpy()
    e2e_outputs = []

    def e2e():
        for i in range(K):
            in_np[0] = rows[P + i]
            acc.stack_raw(in_p.data_ptr(), 1, 0, L, P + i, True, out_p.data_ptr())
            if len(e2e_outputs) < 8:
                e2e_outputs.append(out_p.numpy().copy())
    t0 = time.time()
    e2e_ms = device_time(e2e)
    e2e_wall_ms = (time.time() - t0) * 1e3

    # dominant kernel (Gate/Up + SiLU, ~59% of the decode bytes): mean device time per launch
    Il = shape.inter // world
    # every kernel of a decode layer at context P + 1 on this rank (no all-reduce in these launches)
    kernel_us = {n: acc.time_kernel(i, 0, P, 1, 2 * L) * 1e3
                 for i, n in enumerate(["qkv", "attention", "o_proj", "gate_up", "down", "final_norm"])}
    if acc.decode_fuses_o:  # the decode layer's attention launch also does the O projection
        kernel_us["attention_with_o"] = kernel_us.pop("attention")
        kernel_us.pop("o_proj")
    gu_ms = acc.time_kernel(llmx.KERNEL_GATE_UP, 0, P, 1, 3 * L)
    down_ms = acc.time_kernel(llmx.KERNEL_DOWN, 0, P, 1, 3 * L)
    gu_bytes = 2 * Il * H * 2 + H * 2 + H * 2 + Il * 2
    peak, peak_kind = peaks()
    gu_gbs = gu_bytes / (gu_ms * 1e-3) / 1e9
    step_bytes = [bytes_per_decode(shape, world, P + i + 1) for i in range(K)]
    dec_gbs = sum(step_bytes) / (decode_ms * 1e-3) / 1e9

    gen = None
    if world == 1:
        gen = generate_leg(acc, model, shape, prompt, device_time, stream)

    cpu = None
    if not args.no_cpu_baseline:
        # parity of this run: the device's post-prefill KV of layers 0-1 against
        # the oracle's own prefill of those layers; decode rows against the oracle
        # (N=1: a timed sample; N>1: one forward on rank 0, and every rank's row)
        kv_ok = prefill_kv_check(acc, shape, rows[:P], P, rank) if rank == 0 else None
        if world == 1:
            cpu = cpu_baseline(acc, model, shape, rows[P:], P, e2e_outputs)
        else:
            cpu = tp_parity(acc, shape, rank, world, dist, rows[P:], P, e2e_outputs[0])
        if rank == 0:
            cpu["prefill_kv_layers_0_1_match"] = kv_ok
            cpu["matches_gpu"] = bool(cpu["matches_gpu"] and kv_ok)

    result = {
        "metric": METRIC,
        "value": K / (decode_ms * 1e-3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": decode_ms / K,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int16",
        "data": "synthetic: seeded N(0,0.02)->Q4.12 weights, N(0,1)->Q8.8 embedding rows, norm weights 1.0 "
                "(random-init, no checkpoint)",
        "config": bench_config(cfg_id, world, P, K),
        "prefill": {"value": P / (prefill_ms * 1e-3), "unit": "tok/s", "ms_per_p8_block": prefill_ms / (P // 8),
                    "hbm_frac": (P // 8) * bytes_per_decode(shape, world, P // 2) / (prefill_ms * 1e-3) / 1e9
                    / peak},
        "decode_roofline": {"bound": "hbm", "achieved": dec_gbs, "peak": peak, "unit": "GB/s",
                            "frac": dec_gbs / peak, "bytes_per_step": int(np.mean(step_bytes)),
                            "peak_source": peak_kind},
        "roofline": {"bound": "hbm", "kernel": "k_gemv<1,EPI_SILU,8,1> (RMSNorm + Gate/Up + SiLU x Up, decode)",
                     "achieved": gu_gbs, "peak": peak, "unit": "GB/s", "frac": gu_gbs / peak,
                     # ncu dram bytes only from a capture of this same launch shape (one GPU, full FFN)
                     "traffic": ncu_traffic("gate_up_decode_ncu.txt") if world == 1 else None,
                     "bytes_per_launch": gu_bytes,
                     "ms_per_launch": gu_ms, "down_ms_per_launch": down_ms, "peak_source": peak_kind},
        "e2e": {"value": K / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": H * 2,
                "d2h_bytes_per_step": H * 2, "wall_ms_per_step": e2e_wall_ms / K,
                "api": "llmx_stack (run_token boundary: host embedding-table row -> H2D -> 36x Task18/19 -> Task20 -> D2H)"},
        "kernel_us": kernel_us,
        "gpu_launches": gpu_launches,
        "clocks": clock,
        "setup_s": setup_s,
    }
    if gen is not None:
        result["generate"] = gen
    if cpu is not None:
        result["cpu_baseline"] = cpu
    if world == 1 and not args.no_configs:  # BASELINE configs 0-2 beside the headline, on a free device
        acc.close()
        result["configs"] = config_legs()
    if rank == 0:
        emit(json.dumps(result))
    acc.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def generate_leg(acc, model, shape, prompt, device_time, stream, new_tokens=64):
    """Greedy generation on the device (llmx_generate): the prompt in P8 blocks,
    then new_tokens tokens, each an LM-head argmax over the tied 151,936-row
    table fed back as a decode row.  Per-token cost = (T(1 + n) - T(1)) / n, so
    the prompt's cost cancels.  The host argmax of the same row is timed once
    beside it (the reference's sampler runs on the host)."""
    import torch
    import llmx

    t0 = time.time()
    acc.upload_vocab(model)
    upload_s = time.time() - t0
    prompt = [int(t) for t in prompt]
    acc.generate(prompt, 2)                     # warm-up: graphs, argmax kernels
    toks = [None, None]

    def run(n, slot):
        toks[slot] = acc.generate(prompt, n)
    t1 = device_time(lambda: run(1, 0))
    tn = device_time(lambda: run(1 + new_tokens, 1))
    assert toks[1][0] == toks[0][0]
    # the argmax alone on one final-normed row already on the device
    h_row = acc.hidden_ptr(0)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    table = llmx.lib().llmx_model_embedding(model.h)
    w = torch.from_numpy(np.ctypeslib.as_array(table, shape=(shape.vocab, shape.hidden)).copy()).cuda()
    for _ in range(3):
        llmx.lm_head_argmax_device(h_row, 1, shape.hidden, w.data_ptr(), shape.vocab, tok.data_ptr(), acc.stream)
    reps = 20
    am_ms = device_time(lambda: [llmx.lm_head_argmax_device(h_row, 1, shape.hidden, w.data_ptr(), shape.vocab,
                                                            tok.data_ptr(), acc.stream) for _ in range(reps)]) / reps
    row = acc.read_hidden(0, 1)[0]
    t0 = time.time()
    host_tok = model.lm_head_argmax(row)
    host_ms = (time.time() - t0) * 1e3
    assert host_tok == int(tok.item()), "device argmax differs from the host argmax"
    del w
    return {"value": new_tokens / ((tn - t1) * 1e-3), "unit": "tok/s", "new_tokens": new_tokens,
            "prompt_tokens": len(prompt), "ms_prompt_plus_first_token": t1,
            "ms_per_token": (tn - t1) / new_tokens,
            "lm_head_argmax_ms": am_ms, "lm_head_gbs": shape.vocab * shape.hidden * 2 / (am_ms * 1e-3) / 1e9,
            "host_lm_head_argmax_ms": host_ms, "host_threads": os.cpu_count(), "vocab_upload_s": upload_s,
            "api": "llmx_generate (device embedding gather + stack + LM-head argmax, one host wait)"}


def config_legs():
    """BASELINE configs 0-2 on one GPU, each a small bounded run beside the
    headline (config 3), with the same synthetic model family (seeded N(0,0.02)
    Q4.12 weights, N(0,1) Q8.8 embedding rows, norm weights 1.0):
      config 0: one layer, a P8 block at position 0 then one decode row at 8,
                through llmx_stack (host rows in, final-normed rows out), checked
                against the oracle, which is also timed (1 thread);
      config 1: two layers, P8/G2: the prompt block and one decode through the
                executor (run_prompt_block / run_token) with the untied
                151,936-row LM head argmax on the host, and the same two tokens
                from llmx_generate (argmax on the device);
      config 2: one layer, a 1024-token prompt as 128 consecutive P8 blocks with
                the KV cache built by the device: prefill tok/s after 8, 64,
                256 and 1024 tokens (CUDA events on the context stream).
    A failure is reported in the returned object, never raised."""
    import torch
    import llmx

    out = {}
    reps = 50
    O = _oracle()
    from helpers import OracleState, oracle_shape

    def e2e_ms(fn):
        fn()  # warm-up: graph capture
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) * 1e3 / reps

    # ---- config 0
    try:
        s = llmx.shape("qwen2.5-3b", layers=1, max_seq=64)
        m = llmx.Model(s).init_gaussian(SEED, W_SIGMA)
        acc = llmx.Accelerator(s)
        try:
            acc.upload_model(m)
            rows = embed_rows(range(9), s.hidden).astype(np.int16)
            got_p, got_d = acc.stack(rows[:8], position=0), acc.stack(rows[8:9], position=8)
            O.set_threads(1)
            ref = OracleState(O, oracle_shape(O, s), [m.layer(0)], m.norms())
            t0 = time.perf_counter()
            want_p = ref.stack(rows[:8], 0)
            t1 = time.perf_counter()
            want_d = ref.stack(rows[8:9], 8)
            t2 = time.perf_counter()
            p8_ms = e2e_ms(lambda: acc.stack(rows[:8], position=0))
            dec_ms = e2e_ms(lambda: acc.stack(rows[8:9], position=8))
            out["config0"] = {
                "workload": "1 Qwen2.5-3B-shaped layer: P8 block at position 0, then one decode row at position 8",
                "p8_block_ms": p8_ms, "decode_ms": dec_ms, "prefill_tok_s": 8 / (p8_ms * 1e-3),
                "decode_tok_s": 1 / (dec_ms * 1e-3),
                "matches_oracle": bool(np.array_equal(got_p, want_p) and np.array_equal(got_d, want_d)),
                "cpu_oracle_ms": {"p8_block": (t1 - t0) * 1e3, "decode": (t2 - t1) * 1e3, "cores": 1},
                "timing": f"llmx_stack end to end (host rows, H2D, graph, D2H), mean of {reps} calls"}
        finally:
            acc.close()
    except Exception as e:  # reported, not raised: the headline line must print
        out["config0"] = {"error": f"{type(e).__name__}: {e}"}

    # ---- config 1
    try:
        s = llmx.shape("qwen2.5-3b", layers=2, max_seq=64)
        m = llmx.Model(s).init_gaussian(SEED, W_SIGMA, lm_head=True)
        acc = llmx.Accelerator(s)
        try:
            acc.upload_model(m)
            ex = llmx.Executor(acc, m)
            prompt = list(range(8))

            def host_path():
                t0 = time.perf_counter()
                r = ex.run_prompt_block(prompt, 0)
                t1 = time.perf_counter()
                a = m.lm_head_argmax(r[-1])
                t2 = time.perf_counter()
                d = ex.run_token(a, 8)
                t3 = time.perf_counter()
                b = m.lm_head_argmax(d[0])
                t4 = time.perf_counter()
                return [a, b], (t1 - t0 + t3 - t2) * 1e3, (t2 - t1 + t4 - t3) * 1e3

            host_path()  # warm-up
            toks, fwd_ms, head_ms = host_path()
            acc.upload_vocab(m)
            acc.reset_kv()
            dev = acc.generate(prompt, 2)
            t0 = time.perf_counter()
            dev = acc.generate(prompt, 2)
            gen_ms = (time.perf_counter() - t0) * 1e3
            out["config1"] = {
                "workload": "2 Qwen2.5-3B-shaped layers, P8/G2: prompt tokens 0..7 in one block, one decode; "
                            "untied N(0,0.02) 151,936 x 2048 LM head",
                "generated": toks, "device_generated": dev, "device_matches_host": toks == dev,
                "host_path_ms": fwd_ms + head_ms, "forward_ms": fwd_ms, "host_lm_head_ms": head_ms,
                "host_threads": os.cpu_count(), "device_generate_ms": gen_ms,
                "timing": "wall clock of one warm call (executor + host argmax; llmx_generate)"}
        finally:
            acc.close()
    except Exception as e:
        out["config1"] = {"error": f"{type(e).__name__}: {e}"}

    # ---- config 2
    try:
        s = llmx.shape("qwen2.5-3b", layers=1, max_seq=1024)
        m = llmx.Model(s).init_gaussian(SEED, W_SIGMA)
        acc = llmx.Accelerator(s)
        try:
            acc.upload_model(m)
            stream = torch.cuda.ExternalStream(acc.stream)
            marks = (8, 64, 256, 1024)

            def sweep(events):
                for b in range(128):
                    acc.stack_async(8, 0, 1, 8 * b, include_final_norm=False)
                    if 8 * (b + 1) in events:
                        events[8 * (b + 1)].record(stream)

            acc.write_hidden(1, embed_rows(range(8), s.hidden).astype(np.int16))
            sweep({})  # warm-up: graph capture
            acc.synchronize()
            acc.reset_kv()
            e0 = torch.cuda.Event(enable_timing=True)
            ev = {n: torch.cuda.Event(enable_timing=True) for n in marks}
            e0.record(stream)
            sweep(ev)
            ev[marks[-1]].synchronize()
            acc.synchronize()
            out["config2"] = {
                "workload": "1 Qwen2.5-3B-shaped layer, prompts of 8/64/256/1024 tokens as consecutive P8 blocks, "
                            "causal KV cache built by the device",
                "prefill_tok_s": {str(n): n / (e0.elapsed_time(ev[n]) * 1e-3) for n in marks},
                "ms": {str(n): e0.elapsed_time(ev[n]) for n in marks},
                "timing": "CUDA events on the context stream around consecutive llmx_stack_async blocks"}
        finally:
            acc.close()
    except Exception as e:
        out["config2"] = {"error": f"{type(e).__name__}: {e}"}
    return out


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle as O
    O.set_exp_mode(O.EXP_TRUNC)
    return O


def _dense_layers(O, shape, layers):
    s = O.shape("qwen2.5-3b", max_seq=shape.max_seq)
    return s, [O.gaussian_layer(s, SEED, l, W_SIGMA) for l in layers]


def prefill_kv_check(acc, shape, prompt_rows, P, rank):
    """The oracle's own prefill of layers 0 and 1 (P/8 P8 blocks, all host
    threads) against the device's K/V cache of those layers after the prompt."""
    O = _oracle()
    from helpers import OracleState
    O.set_threads(len(os.sched_getaffinity(0)))
    s, dense = _dense_layers(O, shape, [0, 1])
    norms = np.full((2 * shape.layers + 1, s.hidden), 256, np.int16)
    s2 = O.shape("qwen2.5-3b", max_seq=shape.max_seq, layers=2)
    ref = OracleState(O, s2, dense, norms[:5])
    ok = True
    for b in range(P // 8):
        ref.stack(prompt_rows[8 * b:8 * b + 8], 8 * b, final_norm=False)
    for l in range(2):
        k, v = acc.read_kv(l, 0, P)
        ok &= bool(np.array_equal(k, ref.kc[l][:, :P]) and np.array_equal(v, ref.vc[l][:, :P]))
    O.set_threads(1)
    return ok


def tp_parity(acc, shape, rank, world, dist, dec_rows, P, first_out):
    """Tensor parallel: every rank's first end-to-end decode row must be the same,
    and rank 0 recomputes it with the oracle (1 thread, all 36 layers, from the
    device KV of positions < P, which every rank holds in full)."""
    import torch
    mine = torch.from_numpy(np.ascontiguousarray(first_out, np.int32)).cuda()  # NCCL has no int16
    allo = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allo, mine)
    same = all(torch.equal(allo[0], t) for t in allo)
    res = None
    if rank == 0:
        O = _oracle()
        from helpers import OracleState
        s, dense = _dense_layers(O, shape, range(shape.layers))
        norms = np.full((2 * shape.layers + 1, s.hidden), 256, np.int16)
        ref = OracleState(O, s, dense, norms)
        for l in range(shape.layers):
            k, v = acc.read_kv(l, 0, P)
            ref.kc[l][:, :P] = k
            ref.vc[l][:, :P] = v
        t0 = time.time()
        out = ref.stack(dec_rows[0:1], P)
        dt = time.time() - t0
        res = {"value": 1.0 / dt, "unit": "tok/s", "cores": 1, "kind": "port",
               "sample": f"1 decode forward (36 layers + final norm) at position {P} from the device KV state, "
                         f"integer oracle restatement, 1 thread",
               "matches_gpu": bool(same and np.array_equal(out, first_out)), "ranks_identical": bool(same)}
    dist.barrier()
    return res


def cpu_baseline(acc, model, shape, dec_rows, P, gpu_outputs):
    """The oracle restatement (1 thread) on a bounded sample of the same workload:
    decode forwards at positions P.. from the device's KV cache state; checks
    the oracle's outputs against the device outputs of the same steps."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle as O
    from helpers import OracleState, oracle_shape

    O.set_exp_mode(O.EXP_TRUNC)
    O.set_threads(1)
    L = shape.layers
    ref = OracleState(O, oracle_shape(O, shape), [model.layer(l) for l in range(L)], model.norms())
    for l in range(L):
        k, v = acc.read_kv(l, 0, P)
        ref.kc[l][:, :P] = k
        ref.vc[l][:, :P] = v
    n, t0, same = 0, time.time(), True
    while n < min(8, len(gpu_outputs)) and (time.time() - t0) < 20.0:
        out = ref.stack(dec_rows[n:n + 1], P + n)
        same &= bool(np.array_equal(out, gpu_outputs[n]))
        n += 1
    dt = time.time() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": 1, "kind": "port",
            "sample": f"{n} decode forwards (36 layers + final norm) at positions {P}..{P + n - 1} from the "
                      f"device KV state, integer oracle restatement, 1 thread",
            "matches_gpu": same}


def run_reference(args, cfg_id, world, K, W):
    """The reference's fixed-point golden model (CPU restatement, all host
    threads) on the same workload: decode forwards at positions P.. over a
    seeded KV cache."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle as O
    from helpers import OracleState

    cores = len(os.sched_getaffinity(0))
    O.set_exp_mode(O.EXP_TRUNC)
    O.set_threads(cores)
    cfg = CONFIGS[cfg_id]
    P = cfg["prompt"]
    ndec = max(K, W, cfg["decodes"])
    s = O.shape("qwen2.5-3b", max_seq=P + ndec)
    L = s.layers
    layers = [O.gaussian_layer(s, SEED, l, W_SIGMA) for l in range(L)]
    norms = np.full((2 * L + 1, s.hidden), 256, np.int16)
    ref = OracleState(O, s, layers, norms)
    rng = np.random.default_rng(SEED + 1)
    for l in range(L):  # seeded KV state for positions < P (decode cost does not depend on values)
        ref.kc[l][:, :P] = np.clip(rng.normal(0, 600, (s.kv_heads, P, s.head_dim)), -32768, 32767)
        ref.vc[l][:, :P] = np.clip(rng.normal(0, 600, (s.kv_heads, P, s.head_dim)), -32768, 32767)
    dec = np.random.default_rng(SEED).integers(0, s.vocab, P + ndec)[P:]
    rows = O.gaussian_embedding_rows(s, SEED, dec[:max(K, W)])
    t0 = time.time()
    for i in range(W):
        ref.stack(rows[i:i + 1], P + i)
    per_step = (time.time() - t0) / W
    if K * per_step > 150.0:  # bounded CPU sample: keep the whole run within a few minutes
        K = max(3, int(150.0 / per_step))
    t0 = time.time()
    for i in range(K):
        ref.stack(rows[i:i + 1], P + i)
    dt = time.time() - t0
    v = K / dt
    emit(json.dumps({
        "metric": METRIC, "value": v, "unit": "tok/s", "impl": "reference", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": dt * 1e3 / K, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int16", "data": "synthetic (same seeds as the llmx arm)",
        "config": bench_config(cfg_id, world, P, K),
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": f"{K} decode forwards (36 layers + final norm) at positions {P}..{P + K - 1}, "
                                   f"oracle restatement of the reference golden model, {cores} threads"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


_RESULT_FD = None


def emit(line):
    """The one result line, on the process's original standard output."""
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, (line + "\n").encode())


def main():
    global _RESULT_FD
    # Libraries loaded here (NCCL, CUDA) may print to standard output; send file
    # descriptor 1 to standard error so that the JSON result is the only line there.
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["llmx", "reference"], default="llmx")
    ap.add_argument("--config", type=int, choices=[3, 4], default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the BASELINE config 0-2 legs (N=1)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg_id = args.config or (3 if world == 1 else 4)
    K = args.steps if args.steps is not None else CONFIGS[cfg_id]["decodes"]
    W = max(3, args.warmup)
    if args.impl == "reference":
        if rank != 0:
            return 0
        return run_reference(args, cfg_id, world, K, W)
    return run_llmx(args, cfg_id, world, rank, local, K, W)


if __name__ == "__main__":
    sys.exit(main() or 0)
