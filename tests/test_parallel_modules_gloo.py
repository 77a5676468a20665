"""The drop-in parallel layers of mtp_parallel on CPU ranks (gloo, world 2):
ParallelPrimitives' collectives and scatter (mtp_parallel.py:12-66),
RowParallelLinear (84-118) and ColumnParallelLinear (121-156) must give
what one process computes on the whole weight with the same arithmetic --
gathered / summed logits for the row split, the torch.chunk slice of x and
partial products for the column split -- and vocab_shard_range must name
torch.chunk's blocks.  CPU only."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as tmp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    for p in (REPO, os.path.join(REPO, "mtp-engine_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        import mtp_parallel as mp
        mp._reset_parallel_primitives()
        prim = mp.get_parallel_primitives()
        out = {"world": prim.world_size, "rank": prim.rank, "tp": prim.tp_size}
        torch.manual_seed(0)  # identical inputs on every rank
        x = torch.randn(3, 4, 16)
        W = torch.randn(12, 16)
        b = torch.randn(12)
        # primitives
        out["scatter"] = torch.equal(prim.scatter(x, dim=-1), torch.chunk(x, world, dim=-1)[rank])
        y = torch.full((2, 3), float(rank + 1))
        out["all_reduce"] = torch.equal(prim.all_reduce(y.clone()), torch.full((2, 3), float(sum(range(1, world + 1)))))
        g = prim.all_gather(torch.full((2, 1), float(rank)), dim=-1)
        out["all_gather"] = torch.equal(g, torch.arange(world, dtype=torch.float32).expand(2, world))
        # row split (vocabulary): this rank holds torch.chunk block `rank` of W, b
        row = mp.RowParallelLinear(16, 12, bias=True, gather_output=True)
        lo, hi = mp.vocab_shard_range(12, world, rank)
        out["shard_range"] = (lo, hi) == (rank * (12 // world), (rank + 1) * (12 // world))
        with torch.no_grad():
            row.weight.copy_(W[lo:hi])
            row.bias.copy_(b[lo:hi])
        full = torch.nn.functional.linear(x, W, b)
        out["row_gather"] = torch.allclose(row(x), full, rtol=1e-6, atol=1e-6)
        row.gather_output = False  # the reference's default: the ranks' blocks summed
        blocks = torch.nn.functional.linear(x, W, b).reshape(3, 4, world, 12 // world).sum(2)
        out["row_sum"] = torch.allclose(row(x), blocks, rtol=1e-5, atol=1e-5)
        # column split (input features): this rank holds columns [rank*K/tp, (rank+1)*K/tp)
        col = mp.ColumnParallelLinear(16, 12, bias=True, gather_output=True)
        k0, k1 = rank * (16 // world), (rank + 1) * (16 // world)
        with torch.no_grad():
            col.weight.copy_(W[:, k0:k1])
            col.bias.copy_(b)
        parts = [torch.nn.functional.linear(x[..., r * 8:(r + 1) * 8], W[:, r * 8:(r + 1) * 8], b)
                 for r in range(world)]
        out["col_gather"] = torch.allclose(col(x), torch.cat(parts, dim=-1), rtol=1e-6, atol=1e-6)
        col.gather_output = False
        out["col_local"] = torch.allclose(col(x), parts[rank], rtol=1e-6, atol=1e-6)
        out["col_shapes"] = (col.in_features_per_rank, tuple(col.weight.shape)) == (16 // world, (12, 16 // world))
        q.put((rank, out))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))


def test_parallel_layers_world2():
    world = 2
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, out in res.items():
        assert isinstance(out, dict), out
        assert out.pop("world") == world and out.pop("rank") == rank and out.pop("tp") == world
        bad = [k for k, v in out.items() if v is not True]
        assert not bad, f"rank {rank}: {bad}"


def test_single_process_defaults():
    import mtp_parallel as mp
    mp._reset_parallel_primitives()
    prim = mp.get_parallel_primitives()
    assert (prim.world_size, prim.rank, prim.tp_size, prim.initialized) == (1, 0, 1, False)
    x = torch.randn(2, 5)
    assert prim.scatter(x, dim=-1) is x and prim.all_gather(x, dim=-1) is x and prim.all_reduce(x) is x
    col = mp.ColumnParallelLinear(5, 3, bias=False)
    assert col.bias is None and torch.allclose(col(x), x @ col.weight.T)
    for V, world in ((128256, 8), (10007, 2), (10, 4), (3, 4)):
        chunks = torch.chunk(torch.arange(V), world)
        for r in range(world):
            lo, hi = mp.vocab_shard_range(V, world, r)
            ref = chunks[r] if r < len(chunks) else torch.arange(0)
            assert hi - lo == ref.numel() and (ref.numel() == 0 or (lo, hi - 1) == (int(ref[0]), int(ref[-1])))


def test_out_of_scope_names():
    import mtp_parallel as mp
    if os.environ.get("MTP_REFERENCE_PATH"):
        pytest.skip("reference path set: out-of-scope names resolve there")
    with pytest.raises(AttributeError, match="not part of the B200 hot path"):
        mp.SegmentedGraphRunner
