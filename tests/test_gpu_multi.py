"""Vocab-parallel verify on 2+ GPUs (NCCL ranks): every key exchange --
the NCCL all-reduce through torch.distributed, the peer-memory kernel, the
all-reduce fused into the shard GEMM, and the one-call C-ABI entry over its
own NCCL communicator -- must return exactly what
single-device fused_multi_verify returns on the full lm_head, on every rank,
for several calls in a row.  Runs whenever two GPUs are visible
(MTP_TEST_MULTI_GPU=0 turns it off)."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ENABLED = os.environ.get("MTP_TEST_MULTI_GPU", "1") != "0"


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p_ in (repo, os.path.join(repo, "mtp-engine_b200")):
        if p_ not in sys.path:
            sys.path.insert(0, p_)
    import torch.distributed as dist
    import mtp_fused_verify as mv
    import mtp_parallel as mp
    try:
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        prim = mp.ParallelPrimitives()
        # a second, C-ABI NCCL communicator: rank 0's id sent over the process group
        uid = [mp.NcclCommunicator.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = mp.NcclCommunicator(uid[0], rank, world, dev)
        results = []
        for call in range(3):
            g = torch.Generator(device=dev).manual_seed(100 + call)  # same inputs on every rank
            B, S, K, V = 8, 6, 512, 10007
            hid = torch.randn(B, S, K, generator=g, device=dev).to(torch.bfloat16)
            w = (0.05 * torch.randn(V, K, generator=g, device=dev)).to(torch.bfloat16)
            draft = torch.randint(0, V, (B, S - 1), generator=g, device=dev, dtype=torch.int32)
            ref = mv.fused_multi_verify(hid, w, draft)
            shard, off = mp.shard_lm_head(w, world, rank)
            for exchange in ("nccl", "p2p", "fused", "abi"):
                if exchange == "abi":
                    got = mp.vocab_parallel_multi_verify_nccl(hid, shard, draft, off, comm)
                else:
                    got = mp.vocab_parallel_multi_verify(hid, shard, draft, None, off, prim, exchange=exchange)
                torch.cuda.synchronize(dev)
                same = all(torch.equal(a, b) for a, b in zip(got, ref))
                results.append((call, exchange, same))
        comm.status()
        comm.close()
        import _mtp_native as N
        status = N.device_status(dev)
        dist.barrier(device_ids=[rank])
        mp._EXCHANGES.clear()
        dist.destroy_process_group()
        q.put((rank, results, status))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e), -1))


@pytest.mark.skipif(not ENABLED or not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs (and MTP_TEST_MULTI_GPU not 0)")
def test_vocab_parallel_exchanges_match_single_device():
    import torch.multiprocessing as tmp
    world = 2
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, results, status in out:
        assert isinstance(results, list), results
        assert status == 0
        for call, exchange, same in results:
            assert same, f"rank {rank} call {call} exchange {exchange} differs from single-device verify"
