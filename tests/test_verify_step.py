"""Host step after fused_multi_verify (mtp_engine.py:1244-1258, 1326-1337):
the oracle's two restatements (generate_fused, generate_optimized) agree,
and the device kernel (mtp_verify_step) equals them on every case.  The
CPU part runs without a GPU; the device part is marked gpu."""

import numpy as np
import pytest
import torch

from oracle import mtp_oracle as O


def cases():
    rng = np.random.default_rng(7)
    out = []
    for B, D in [(1, 4), (64, 5), (1000, 7), (3, 1), (5, 0)]:
        for mode in ("random", "all", "none"):
            draft = rng.integers(0, 50000, size=(B, D)).astype(np.int32)
            if mode == "all":
                acc_n = np.full(B, D, np.int32)
            elif mode == "none":
                acc_n = rng.integers(0, D + 1, size=B).astype(np.int32)
                acc_n[rng.integers(0, B)] = 0
            else:
                acc_n = rng.integers(0, D + 1, size=B).astype(np.int32)
            corr = rng.integers(0, 50000, size=B).astype(np.int32)
            out.append((draft, acc_n, corr))
    return out


def test_oracle_variants_agree():
    for draft, acc_n, corr in cases():
        a, na = O.verify_step(draft, acc_n, corr, "optimized")
        b, nb = O.verify_step(draft, acc_n, corr, "fused")
        assert na == nb and np.array_equal(a, b)


@pytest.mark.gpu
@pytest.mark.isolated
def test_device_step_matches_oracle():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mtp_fused_verify as mv
    d = torch.device("cuda", 0)
    for draft, acc_n, corr in cases():
        st, info = mv.verify_step(torch.tensor(draft, device=d), torch.tensor(acc_n, device=d),
                                  torch.tensor(corr, device=d))
        ref, n = O.verify_step(draft, acc_n, corr)
        n_dev, width = (int(x) for x in info.cpu())
        assert n_dev == n and width == ref.shape[1]
        assert np.array_equal(st[:, :width].cpu().numpy(), ref)
        assert (st[:, width:] == -1).all()  # the columns after the step's tokens hold "no token"
