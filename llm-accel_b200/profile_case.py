"""Small, self-contained profiling case for the path's kernels.

Builds a Qwen2.5-3B-shaped stack with a few layers (synthetic N(0,0.02)
weights), preloads a seeded KV cache to `--position`, then
  --table : prints the mean device time of every kernel (llmx_time_kernel,
            CUDA events on the context stream) for 1-row decode and 8-row blocks;
  --eager : runs `--steps` eager Task 18/19/20 sequences (no CUDA graph) so that a
            profiler sees plain launches (ncu -k regex:... -c ...);
  --argmax: runs `--steps` device LM-head argmaxes over a 151,936 x 2048 table
            (k_lm_scan + k_lm_pick) and prints their mean device time;
  --generate: greedy generation on the device (llmx_generate: k_embed_rows,
            the stack, k_lm_scan + k_lm_pick) over `--layers` layers, 8 prompt
            tokens and `--steps` new tokens.
  --timeline: after `--steps` warm-up stack calls (graph capture), one more
            `--rows`-row stack call whose launches stamp %globaltimer (the
            measurement build: `python llm-accel_b200/build.py --timeline` and
            LLMX_TIMELINE=1); prints every launch's start, duration and the idle
            gap before it, in graph order, plus per-kernel totals.  Under
            torchrun (WORLD_SIZE > 1) every rank runs its tensor-parallel shard
            (CUDA device = LOCAL_RANK) and prints its own line.
Usage: python llm-accel_b200/profile_case.py --layers 4 --position 512 --table
       LLMX_TIMELINE=1 python llm-accel_b200/profile_case.py --layers 36 --position 512 --max-seq 640 --timeline
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import llmx  # noqa: E402

NAMES = ["qkv", "attention", "o_proj", "gate_up", "down", "final_norm"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--position", type=int, default=512)
    ap.add_argument("--max-seq", type=int, default=2304)
    ap.add_argument("--table", action="store_true")
    ap.add_argument("--eager", action="store_true")
    ap.add_argument("--stack", action="store_true", help="decode steps through llmx_stack (one CUDA graph each)")
    ap.add_argument("--rows", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--iters", type=int, default=40)
    ap.add_argument("--argmax", action="store_true")
    ap.add_argument("--generate", action="store_true")
    ap.add_argument("--timeline", action="store_true")
    ap.add_argument("--kv-scale", type=float, default=600.0, help="std of the preloaded KV cache (raw Q8.8)")
    ap.add_argument("--hidden", type=int, default=0, help="override the shape (e.g. a tensor-parallel rank's heads)")
    ap.add_argument("--heads", type=int, default=0)
    ap.add_argument("--kv-heads", type=int, default=0)
    ap.add_argument("--inter", type=int, default=0)
    args = ap.parse_args()
    if args.argmax:
        return argmax_case(args.steps)
    if args.generate:
        return generate_case(args.layers, args.steps)
    over = {k: v for k, v in (("hidden", args.hidden), ("heads", args.heads), ("kv_heads", args.kv_heads),
                              ("inter", args.inter)) if v}
    s = llmx.shape("qwen2.5-3b", layers=args.layers, max_seq=args.max_seq, **over)
    m = llmx.Model(s).init_gaussian(20260718, 0.02)
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    tp = {}
    if world > 1:  # tensor parallel: the NCCL id travels over a gloo group (torchrun's env rendezvous)
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method="env://")
        obj = [llmx.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        tp = dict(device=int(os.environ.get("LOCAL_RANK", "0")), tp_rank=rank, tp_size=world, tp_id=obj[0])
    acc = llmx.Accelerator(s, **tp)
    acc.upload_model(m)
    rng = np.random.default_rng(0)
    P = args.position
    for l in range(s.layers):
        k = np.clip(rng.normal(0, args.kv_scale, (s.kv_heads, P, s.head_dim)), -32768, 32767).astype(np.int16)
        v = np.clip(rng.normal(0, args.kv_scale, (s.kv_heads, P, s.head_dim)), -32768, 32767).astype(np.int16)
        acc.write_kv(l, 0, k, v)
    acc.write_hidden(1, m.embed(rng.integers(0, s.vocab, 8)))
    if args.table:
        out = {}
        for rows in (1, 8):
            out[f"rows{rows}"] = {n: acc.time_kernel(i, 0, P, rows, args.iters) * 1e3 for i, n in enumerate(NAMES)}
        print(json.dumps({"position": P, "layers": s.layers, "us_per_launch": out}, indent=1))
    if args.stack:
        hs = m.embed(rng.integers(0, s.vocab, 8 * args.steps))
        for step in range(args.steps):
            pos = P + step * args.rows
            acc.stack(hs[step * args.rows:(step + 1) * args.rows], position=pos)
        print("stack steps done")
    if args.eager:
        for step in range(args.steps):
            pos = P + step * args.rows
            for l in range(s.layers):
                acc.bind(0, 1)
                acc.task(llmx.OP_ATTENTION, l, pos, args.rows)
                acc.bind(1, 0)
                acc.task(llmx.OP_FFN, l, pos, args.rows)
            acc.bind(0, 1)
            acc.task(llmx.OP_FINAL_NORM, 0, pos, args.rows)
        print("eager steps done")
    if args.timeline:
        timeline_case(acc, m, s, P, args, rank, world, rng)
    acc.close()


def timeline_case(acc, m, s, P, args, rank, world, rng):
    if not llmx.TIMELINE:
        raise SystemExit("--timeline needs the measurement build: build.py --timeline, then LLMX_TIMELINE=1")
    R = args.rows
    hs = m.embed(rng.integers(0, s.vocab, R * (args.steps + 1)))
    for step in range(args.steps):  # graph capture and warm-up
        acc.stack(hs[step * R:(step + 1) * R], position=P + step * R)
    pos = P + args.steps * R
    acc.timeline_reset()
    acc.stack(hs[args.steps * R:], position=pos)
    runs = acc.timeline_read()
    t0 = runs[0][2]
    launches, per_name, busy_end = [], {}, t0
    for slot, name, st, en in runs:
        launches.append({"name": name, "start_us": round((st - t0) / 1e3, 2), "dur_us": round((en - st) / 1e3, 2),
                         "idle_before_us": round(max(0, st - busy_end) / 1e3, 2)})
        busy_end = max(busy_end, en)
        d = per_name.setdefault(name, {"launches": 0, "sum_dur_us": 0.0})
        d["launches"] += 1
        d["sum_dur_us"] = round(d["sum_dur_us"] + (en - st) / 1e3, 2)
    print(json.dumps({"rank": rank, "world": world, "layers": s.layers, "rows": R, "position": pos,
                      "step_us": round((busy_end - t0) / 1e3, 2),
                      "idle_us": round(sum(x["idle_before_us"] for x in launches), 2),
                      "per_kernel": per_name, "launches": launches}))


def generate_case(layers, steps):
    s = llmx.shape("qwen2.5-3b", layers=layers, max_seq=64)
    m = llmx.Model(s).init_gaussian(20260718, 0.02)
    acc = llmx.Accelerator(s)
    acc.upload_model(m)
    acc.upload_vocab(m)
    toks = acc.generate(list(range(100, 108)), steps)
    print(json.dumps({"generated": toks}))
    acc.close()


def argmax_case(steps):
    import torch
    s = llmx.shape("qwen2.5-3b", layers=1)
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(1)
    w = torch.randint(-700, 700, (s.vocab, s.hidden), dtype=torch.int16, device=dev, generator=g)
    h = torch.randint(-2000, 2000, (1, s.hidden), dtype=torch.int16, device=dev, generator=g)
    tok = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def run():
        llmx.lm_head_argmax_device(h.data_ptr(), 1, s.hidden, w.data_ptr(), s.vocab, tok.data_ptr(),
                                   stream.cuda_stream)
    run()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        run()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    print(json.dumps({"lm_head_argmax_us": ms * 1e3, "gbs": s.vocab * s.hidden * 2 / (ms * 1e-3) / 1e9,
                      "token": int(tok.item())}))


if __name__ == "__main__":
    main()
