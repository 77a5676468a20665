"""Multi-rank logic of the vocab-parallel verify on CPU ranks (gloo).

Each rank reduces its contiguous vocabulary block to packed int64
(max logit, index) keys, the ranks all-reduce(MAX) the keys -- the same
collective the GPU path issues over NCCL -- and every rank decodes the
chain.  The result must equal single-device verification on the full
lm_head, including exact ties that straddle a shard boundary.  A rank that
dies before the collective must surface as an error on the others within the
process-group timeout, not as a hang.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import mtp_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "verify.npz")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, case, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=8))
        g = np.load(GOLDEN)
        h, w, d = g["h3"], g["w3"].copy(), g["d3"]
        if case == "tie_across_shards":
            lo1, _ = O.vocab_shard_bounds(w.shape[0], world)[1]
            w[lo1 + 3] = w[2]  # equal logits in rank 0 and rank 1 blocks: index 2 must win
        if case == "weak":
            # each rank holds only its own sequences; the candidates of every
            # rank are all-gathered (asynchronously, as the weak-scaling bench
            # does) before the vocabulary-sharded argmax
            bs = h.shape[0] // world
            h_loc = torch.from_numpy(np.ascontiguousarray(h[rank * bs:(rank + 1) * bs]))
            d_loc = torch.from_numpy(np.ascontiguousarray(d[rank * bs:(rank + 1) * bs]).astype(np.int32))
            h_all = torch.empty((bs * world,) + h_loc.shape[1:], dtype=h_loc.dtype)
            d_all = torch.empty((bs * world,) + d_loc.shape[1:], dtype=d_loc.dtype)
            works = [dist.all_gather_into_tensor(h_all, h_loc, async_op=True),
                     dist.all_gather_into_tensor(d_all, d_loc, async_op=True)]
            for wk in works:
                wk.wait()
            h, d = h_all.numpy(), d_all.numpy()
        B, S, K = h.shape
        lo, hi = O.vocab_shard_bounds(w.shape[0], world)[rank]
        keys = O.shard_argmax_keys(h.reshape(B * S, K), w[lo:hi], None, lo)
        if case == "dead_rank" and rank == 1:
            os._exit(3)  # leaves between steps, before its collective
        t = torch.from_numpy(keys.astype(np.int64))
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        top = O.key_index(t.numpy()).reshape(B, S)
        res = O.chain_accept(top, d)
        q.put((rank, "ok", [r.tolist() for r in res], w.tobytes() if rank == 0 else None))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, "error", repr(e), None))


def _run(world, case, expect_ranks):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(expect_ranks):
        r, status, payload, extra = q.get(timeout=120)
        out[r] = (status, payload, extra)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("world", [2, 4, 8])
def test_keys_allreduce_matches_full(world):
    g = np.load(GOLDEN)
    full = O.fused_multi_verify(g["h3"], g["w3"], None, g["d3"])
    out = _run(world, "plain", world)
    for r in range(world):
        status, payload, _ = out[r]
        assert status == "ok", payload
        for a, b in zip(payload, full):
            np.testing.assert_array_equal(np.asarray(a), b)


def test_tie_across_shard_boundary():
    out = _run(2, "tie_across_shards", 2)
    g = np.load(GOLDEN)
    w = np.frombuffer(out[0][2], dtype=np.float32).reshape(g["w3"].shape)
    full = O.fused_multi_verify(g["h3"], w, None, g["d3"])
    for r in range(2):
        status, payload, _ = out[r]
        assert status == "ok", payload
        for a, b in zip(payload, full):
            np.testing.assert_array_equal(np.asarray(a), b)


def test_dead_rank_surfaces_as_error():
    out = _run(2, "dead_rank", 1)
    status, payload, _ = out[0]
    assert status == "error", "the surviving rank should see the collective fail"


@pytest.mark.parametrize("world", [2, 3])
def test_weak_scaling_exchange(world):
    """The weak-scaling bench's data flow: every rank owns 6 / world of the
    sequences, all-gathers the candidates, folds its vocabulary block into
    keys and all-reduces them; every rank must then hold single-device
    verification of all sequences."""
    g = np.load(GOLDEN)
    full = O.fused_multi_verify(g["h3"], g["w3"], None, g["d3"])
    out = _run(world, "weak", world)
    for r in range(world):
        status, payload, _ = out[r]
        assert status == "ok", payload
        for a, b in zip(payload, full):
            np.testing.assert_array_equal(np.asarray(a), b)
