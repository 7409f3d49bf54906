"""Tensor-parallel stack on two and four GPUs (int64 all-reduce after O and Down).

Two reductions are checked: the default peer all-reduce (O / Down epilogues
store their exact sums into every rank's IPC-mapped exchange region over
NVLink, a one-block kernel adds them) and NCCL (LLMX_TP_NCCL=1).  Each rank
holds its shard of the heads / FFN columns (llmx_create with tp_size 2 or 4) and
runs the same llmx_stack calls; after every call both ranks must
hold the one-GPU oracle's rows bit for bit (the reduction of exact int64
partial sums is order-free, rounding happens after it).  Oracle references are
computed before any collective, so no rank can stop between collectives.
Each case is skipped when fewer GPUs than its ranks are visible.
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


def _worker(rank, world, port, result_dir, nccl):
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "llm-accel_b200"))
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
    sys.path.insert(0, HERE)
    import datetime

    import torch
    import torch.distributed as dist

    import llmx
    import oracle as O
    from helpers import OracleState, oracle_shape

    os.environ["LLMX_TP_NCCL"] = str(nccl)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    O.build()
    O.set_exp_mode(O.EXP_TRUNC)
    s = llmx.shape("qwen2.5-3b", layers=2, max_seq=128, vocab=256)
    m = llmx.Model(s).init_gaussian(20260718, 0.02)
    ref = OracleState(O, oracle_shape(O, s), [m.layer(l) for l in range(s.layers)], m.norms())
    rng = np.random.default_rng(23)
    steps = [(0, m.embed(rng.integers(0, s.vocab, 8)))]
    steps += [(8 + i, m.embed([int(rng.integers(0, s.vocab))])) for i in range(3)]
    steps += [(11, m.embed(rng.integers(0, s.vocab, 5)))]
    want = [ref.stack(h, pos) for pos, h in steps]  # every reference before any collective

    obj = [llmx.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    acc = llmx.Accelerator(s, device=rank, tp_rank=rank, tp_size=world, tp_id=obj[0])
    acc.upload_model(m)
    got = [acc.stack(h, position=pos) for pos, h in steps]
    acc.close()
    dist.barrier()
    dist.destroy_process_group()
    bad = [i for i, (g, w) in enumerate(zip(got, want)) if not np.array_equal(g, w)]
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
        f.write("ok" if not bad else f"mismatch at steps {bad}")


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("nccl", [0, 1], ids=["peer_allreduce", "nccl_allreduce"])
def test_tensor_parallel_gpus_match_oracle(tmp_path, nccl, world):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), nccl), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}.txt").read_text() == "ok", f"rank {r}"
