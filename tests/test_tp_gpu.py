"""Tensor-parallel stack on 2, 4 and 8 GPUs (int64 all-reduce after O and Down).

Two reductions are checked: the default peer all-reduce (O / Down epilogues
store their exact sums into every rank's IPC-mapped exchange region over
NVLink; the next projection's prologue -- Gate/Up after O, the next layer's
QKV after Down -- waits for them, adds, rounds and adds the residual) and NCCL
(LLMX_TP_NCCL=1).  Each rank holds its shard of the heads / FFN columns
(llmx_create with tp_size N) and runs the same llmx_stack calls; after every
call every rank must hold the one-GPU oracle's rows bit for bit (the reduction
of exact int64 partial sums is order-free, rounding happens after it).

Cases: a prompt block, decode rows and a 5-row block at short context; then one
decode row at contexts above 16 tiles (KV cache preloaded), where ranks of 4 and
2 heads run 16-CTA attention clusters.  Oracle references are computed before
any collective, so no rank can stop between collectives.  A failure case checks
that a rank whose peer skipped a step gets LLMX_ERR_TIMEOUT from the bounded
wait, not a hang.  Each case is skipped when fewer GPUs than its ranks are
visible.
"""
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port):
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "llm-accel_b200"))
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
    sys.path.insert(0, HERE)
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300))
    return dist


def _worker(rank, world, port, result_dir, nccl):
    os.environ["LLMX_TP_NCCL"] = str(nccl)
    dist = _setup(rank, world, port)
    import llmx
    import oracle as O
    from helpers import OracleState, oracle_shape, random_kv

    O.build()
    O.set_exp_mode(O.EXP_TRUNC)
    O.set_threads(4)
    s = llmx.shape("qwen2.5-3b", layers=2, max_seq=1280, vocab=256)
    m = llmx.Model(s).init_gaussian(20260718, 0.02)
    ref = OracleState(O, oracle_shape(O, s), [m.layer(l) for l in range(s.layers)], m.norms())
    rng = np.random.default_rng(23)
    steps = [(0, m.embed(rng.integers(0, s.vocab, 8)))]
    steps += [(8 + i, m.embed([int(rng.integers(0, s.vocab))])) for i in range(3)]
    steps += [(11, m.embed(rng.integers(0, s.vocab, 5)))]
    want = [ref.stack(h, pos) for pos, h in steps]  # every reference before any collective
    # long context: KV of positions [0, P) preloaded, decodes above 16 tiles
    P = 1090
    kv = [random_kv(np.random.default_rng(100 + l), s.kv_heads, P, s.head_dim) for l in range(s.layers)]
    for l in range(s.layers):
        ref.kc[l][:, :P] = kv[l][0]
        ref.vc[l][:, :P] = kv[l][1]
    long_steps = [(P + i, m.embed([int(rng.integers(0, s.vocab))])) for i in range(2)]
    want += [ref.stack(h, pos) for pos, h in long_steps]

    obj = [llmx.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    acc = llmx.Accelerator(s, device=rank, tp_rank=rank, tp_size=world, tp_id=obj[0])
    kind = acc.allreduce_kind
    acc.upload_model(m)
    got = [acc.stack(h, position=pos) for pos, h in steps]
    for l in range(s.layers):
        acc.write_kv(l, 0, kv[l][0], kv[l][1])
    got += [acc.stack(h, position=pos) for pos, h in long_steps]
    acc.close()
    dist.barrier()
    dist.destroy_process_group()
    bad = [i for i, (g, w) in enumerate(zip(got, want)) if not np.array_equal(g, w)]
    want_kind = llmx.AR_NCCL if nccl else llmx.AR_PEER
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
        if kind != want_kind:
            f.write(f"all-reduce kind {kind}, expected {want_kind}")
        else:
            f.write("ok" if not bad else f"mismatch at steps {bad}")


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("nccl", [0, 1], ids=["peer_allreduce", "nccl_allreduce"])
def test_tensor_parallel_gpus_match_oracle(tmp_path, nccl, world):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), nccl), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}.txt").read_text() == "ok", f"rank {r}"


def _skip_worker(rank, world, port, result_dir):
    """Rank 1 leaves out one stack call (between steps, nothing in flight);
    rank 0's call must end with LLMX_ERR_TIMEOUT from the bounded wait on the
    missing peer sums (short limit: LLMX_AR_POLL_LIMIT), and its device must
    still run work afterwards."""
    os.environ["LLMX_AR_POLL_LIMIT"] = "200000"
    os.environ["LLMX_TP_NCCL"] = "0"
    dist = _setup(rank, world, port)
    import llmx

    s = llmx.shape("qwen2.5-3b", layers=2, max_seq=64, vocab=256)
    m = llmx.Model(s).init_gaussian(20260718, 0.02)
    obj = [llmx.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    acc = llmx.Accelerator(s, device=rank, tp_rank=rank, tp_size=world, tp_id=obj[0])
    acc.upload_model(m)
    h = m.embed([1, 2, 3])
    dist.barrier()                            # both ranks start the first step together
    msg = "ok"
    if acc.allreduce_kind != llmx.AR_PEER:
        msg = f"all-reduce kind {acc.allreduce_kind}"
    first = acc.stack(h, position=0)          # both ranks
    if rank == 0 and msg == "ok":
        try:
            acc.stack(h, position=3)          # rank 1 does not take part
            msg = "no error although a peer skipped the step"
        except llmx.LlmxError as e:
            if e.code != llmx.ERR_TIMEOUT:
                msg = f"error code {e.code}, expected {llmx.ERR_TIMEOUT}"
        # the context and the device keep working
        back = acc.read_hidden(0, 3)
        if back.shape != (3, s.hidden):
            msg = "hidden rows unreadable after the timeout"
        one = llmx.Accelerator(llmx.shape("small"), device=rank)
        one.close()
    dist.barrier()                            # rank 1 keeps its region mapped until rank 0 is done
    acc.close()
    dist.barrier()
    dist.destroy_process_group()
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
        f.write(msg if first.shape == (3, s.hidden) else "first step failed")


def test_peer_skipping_a_step_times_out(tmp_path):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_skip_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert (tmp_path / f"rank{r}.txt").read_text() == "ok", f"rank {r}"
