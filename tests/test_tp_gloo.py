"""Tensor-parallel decomposition on two CPU ranks (gloo), against the one-rank oracle.

The device runtime shards a layer like this (runtime.cu: shard geometry,
EPI_PARTIAL epilogue, allreduce_resid): rank r of N holds query heads
[r*H/N, (r+1)*H/N) and the matching O input columns, FFN columns
[r*I/N, (r+1)*I/N) of Gate/Up and the matching Down input columns; K/V, the KV
cache, the norms and the hidden stream are replicated.  O and Down produce exact
int64 partial sums, an all-reduce adds them, and every rank applies the same
rnd4 / rnd8 / saturation and residual.  Rounding before the reduction would
break parity with one rank; integer addition makes the reduction order free.

Here two gloo processes run exactly that schedule with the CPU oracle's
primitives and a real int64 all-reduce, and must reproduce orc_task18 /
orc_task19 (the golden Task 18 / 19, host/host_qwen_8x64.cpp:4854-4978) bit
for bit on a prompt block and two decode rows over two layers.
"""
import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rope(vec, heads, hd, row):
    """rotate_fix16_pair_with_quantized_rope host:4765-4788 on (i, i + hd/2) pairs."""
    v = vec.astype(np.int64).reshape(heads, hd)
    half = hd // 2
    c, s = row[:half].astype(np.int64), row[half:].astype(np.int64)
    x0, x1 = v[:, :half], v[:, half:]
    r0 = np.clip((x0 * c - x1 * s + 128) >> 8, -32768, 32767)
    r1 = np.clip((x1 * c + x0 * s + 128) >> 8, -32768, 32767)
    return np.concatenate([r0, r1], axis=1).reshape(-1).astype(np.int16)


def _tp_task18(O, s, W, norm, rope, kc, vc, hidden, pos, rank, world, all_reduce):
    H, hd = s.hidden, s.hidden // s.heads
    G, hq = s.heads // s.kv_heads, s.heads // world
    h0 = rank * hq
    Wq, Wk, Wv, Wo = W[0], W[1], W[2], W[3]
    xn = O.rmsnorm(hidden, norm)
    q = O.projection(xn, np.ascontiguousarray(Wq[h0 * hd:(h0 + hq) * hd]))
    k, v = O.projection(xn, Wk), O.projection(xn, Wv)
    att = np.zeros((hidden.shape[0], hq * hd), np.int16)
    for t in range(hidden.shape[0]):
        p = pos + t
        qt = _rope(q[t], hq, hd, rope[p])
        kt = _rope(k[t], s.kv_heads, hd, rope[p])
        for g in range(s.kv_heads):
            kc[g, p] = kt[g * hd:(g + 1) * hd]
            vc[g, p] = v[t, g * hd:(g + 1) * hd]
        for lh in range(hq):
            g = (h0 + lh) // G
            att[t, lh * hd:(lh + 1) * hd] = O.attention_group(qt[lh * hd:(lh + 1) * hd][None, :],
                                                              kc[g, :p + 1], vc[g, :p + 1])[0]
    part = O.projection_partial(att, np.ascontiguousarray(Wo[:, h0 * hd:(h0 + hq) * hd]), 0, hq * hd)
    return O.residual(hidden, O.round_partial(all_reduce(part)))


def _tp_task19(O, s, W, norm, hidden, rank, world, all_reduce):
    Il = s.inter // world
    c0 = rank * Il
    Wg, Wu, Wd = W[4], W[5], W[6]
    xn = O.rmsnorm(hidden, norm)
    g = O.projection(xn, np.ascontiguousarray(Wg[c0:c0 + Il]))
    u = O.projection(xn, np.ascontiguousarray(Wu[c0:c0 + Il]))
    act = O.silu_mul(g, u)
    part = O.projection_partial(act, np.ascontiguousarray(Wd[:, c0:c0 + Il]), 0, Il)
    return O.residual(hidden, O.round_partial(all_reduce(part)))


def _word_all_reduce(dist, torch, p, number):
    """The device's peer all-reduce as a host model: each rank's exact partial
    sums travel as 64-bit words {sum << 16 | tag} (the sum must fit 48 bits),
    every rank receives every rank's words, checks the tag of all-reduce
    `number` ((number mod 65535) + 1) and adds the sign-extended sums."""
    p = np.ascontiguousarray(p, dtype=np.int64)
    assert np.abs(p).max(initial=0) < (1 << 47), "partial sum does not fit the 48-bit word"
    tag = number % 65535 + 1
    words = (p.astype(np.uint64) << np.uint64(16)) | np.uint64(tag)
    t = torch.from_numpy(words.view(np.int64).copy())
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    total = np.zeros_like(p)
    for o in out:
        w = o.numpy().view(np.uint64)
        assert np.all((w & np.uint64(0xFFFF)) == np.uint64(tag)), "stale or foreign word"
        total += w.view(np.int64) >> 16
    return total


def _worker(rank, world, port, profile, words=False):
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
    import torch
    import torch.distributed as dist
    import oracle as O

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        O.build()
        O.set_exp_mode(O.EXP_TRUNC)

        count = [0]

        def all_reduce(p):
            if words:
                count[0] += 1
                return _word_all_reduce(dist, torch, p, count[0] - 1)
            t = torch.from_numpy(np.ascontiguousarray(p, dtype=np.int64))
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            return t.numpy()

        s = O.shape(profile)
        _, norms, dense = O.ref_random_model(s, 20260718, s.layers, with_embedding=False)
        rope = O.rope_table(s.hidden // s.heads, s.max_seq)
        hd = s.hidden // s.heads
        kc_tp = [np.zeros((s.kv_heads, s.max_seq, hd), np.int16) for _ in range(s.layers)]
        vc_tp = [np.zeros_like(kc_tp[0]) for _ in range(s.layers)]
        kc_1 = [np.zeros_like(kc_tp[0]) for _ in range(s.layers)]
        vc_1 = [np.zeros_like(kc_tp[0]) for _ in range(s.layers)]
        rng = np.random.default_rng(17)  # same stream on every rank
        blocks = [(0, rng.integers(-900, 900, (5, s.hidden)).astype(np.int16))]
        blocks += [(5 + i, rng.integers(-900, 900, (1, s.hidden)).astype(np.int16)) for i in range(2)]
        for pos, h in blocks:
            a = b = h
            for l in range(s.layers):
                W = O.layer_views(s, dense[l])
                a = _tp_task18(O, s, W, norms[2 * l], rope, kc_tp[l], vc_tp[l], a, pos, rank, world, all_reduce)
                b = O.task18(s, dense[l], norms[2 * l], rope, kc_1[l], vc_1[l], b, pos)
                assert np.array_equal(a, b), f"rank {rank}: Task 18 layer {l} at {pos}"
                a = _tp_task19(O, s, W, norms[2 * l + 1], a, rank, world, all_reduce)
                b = O.task19(s, dense[l], norms[2 * l + 1], b)
                assert np.array_equal(a, b), f"rank {rank}: Task 19 layer {l} at {pos}"
            assert np.array_equal(kc_tp[0][:, :pos + h.shape[0]], kc_1[0][:, :pos + h.shape[0]])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("words", [False, True], ids=["sum", "tagged_words"])
@pytest.mark.parametrize("profile", ["medium", "small"])
def test_tensor_parallel_two_gloo_ranks(profile, words):
    mp = pytest.importorskip("torch.multiprocessing")
    mp.spawn(_worker, args=(2, _free_port(), profile, words), nprocs=2, join=True)


def _leave_worker(rank, world, port, result_dir):
    """Rank 1 leaves between steps (after the first all-reduce, nothing in
    flight); rank 0's next all-reduce must end with an error within the
    process group's short timeout instead of waiting for good."""
    import datetime
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    t = torch.ones(4, dtype=torch.int64)
    dist.all_reduce(t)
    msg = "ok" if int(t[0]) == world else "first step wrong"
    if rank == 1:
        dist.destroy_process_group()  # leaves the group between steps
    else:
        import time
        t0 = time.time()
        try:
            dist.all_reduce(t)
            msg = "the survivor's collective returned although its peer left"
        except Exception:  # noqa: BLE001 -- any error is the detection we want
            if time.time() - t0 > 60:
                msg = "detected, but only after the timeout bound"
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
        f.write(msg)


def test_rank_leaving_between_steps_is_detected(tmp_path):
    mp = pytest.importorskip("torch.multiprocessing")
    mp.spawn(_leave_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert (tmp_path / f"rank{r}.txt").read_text() == "ok", f"rank {r}"
