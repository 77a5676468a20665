"""mtp_vocab_parallel_multi_verify over a C-ABI NCCL communicator on one
GPU: a single-rank communicator (the all-reduce runs, over one rank) and no
communicator must both return bit for bit what fused_multi_verify returns
on the same lm_head (mtp_fused_verify.py:237-290), and the keys must be back
at rest for the next call.  The 2-GPU case is in tests/test_gpu_multi.py.
GPU only; runs in a child process (tests/test_gpu_isolated.py)."""

import numpy as np
import pytest
import torch

from oracle import mtp_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.isolated]


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _mtp_native as N
    import mtp_fused_verify as mv
    import mtp_parallel as mp
    torch.cuda.set_device(0)
    return N, mv, mp


def inputs(seed, B, S, K, V, bias=False):
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(seed)
    hid = torch.randn(B, S, K, generator=g, device=d).to(torch.bfloat16)
    w = (0.05 * torch.randn(V, K, generator=g, device=d)).to(torch.bfloat16)
    b = (0.1 * torch.randn(V, generator=g, device=d)) if bias else None
    draft = torch.randint(0, V, (B, S - 1), generator=g, device=d, dtype=torch.int32)
    return hid, w, b, draft


@pytest.mark.parametrize("B,S,K,V,bias", [(8, 6, 512, 10007, False), (3, 1, 256, 777, True),
                                          (64, 6, 4096, 20000, False)])
def test_single_rank_communicator(mods, B, S, K, V, bias):
    N, mv, mp = mods
    hid, w, b, draft = inputs(B + V, B, S, K, V, bias)
    ref = mv.fused_multi_verify(hid, w, draft, b)
    with mp.NcclCommunicator(mp.NcclCommunicator.unique_id(), 0, 1) as comm:
        for _ in range(3):  # the keys rest again after each call
            got = mp.vocab_parallel_multi_verify_nccl(hid, w, draft, 0, comm, b)
            torch.cuda.synchronize()
            for a, r in zip(got, ref):
                assert torch.equal(a, r)
        comm.status()
    got = mp.vocab_parallel_multi_verify_nccl(hid, w, draft, 0, None, b)
    for a, r in zip(got, ref):
        assert torch.equal(a, r)
    assert N.device_status(torch.device("cuda", 0)) == 0


def test_against_oracle(mods):
    N, mv, mp = mods
    B, S, K, V = 4, 5, 256, 4096
    hid, w, _, draft = inputs(7, B, S, K, V)
    f32 = lambda t: t.float().cpu().numpy()
    top = O.logits_f32(f32(hid).reshape(-1, K), f32(w), None).argmax(-1).reshape(B, S)
    draft[:, :2] = torch.from_numpy(top[:, 1:3].astype(np.int32)).cuda()  # accept at least 2
    ra, rn, rc = O.chain_accept(top, draft.cpu().numpy())
    with mp.NcclCommunicator(mp.NcclCommunicator.unique_id(), 0, 1) as comm:
        a, n, c = mp.vocab_parallel_multi_verify_nccl(hid, w, draft, 0, comm)
    np.testing.assert_array_equal(a.cpu().numpy(), ra)
    np.testing.assert_array_equal(n.cpu().numpy(), rn)
    np.testing.assert_array_equal(c.cpu().numpy(), rc)
    assert (n.cpu().numpy() >= 2).all()


def test_wrong_device_rejected(mods):
    N, _, mp = mods
    if torch.cuda.device_count() < 2:
        pytest.skip("needs a second GPU")
    hid, w, _, draft = inputs(3, 2, 3, 64, 100)
    with mp.NcclCommunicator(mp.NcclCommunicator.unique_id(), 0, 1) as comm:  # on cuda:0
        with torch.cuda.device(1):
            h1, w1, d1 = hid.to("cuda:1"), w.to("cuda:1"), draft.to("cuda:1")
            with pytest.raises(RuntimeError, match="MTP_ERR_ARG"):
                mp.vocab_parallel_multi_verify_nccl(h1, w1, d1, 0, comm)
