"""Host-side recovery after a bounded device wait ran out (MTP_ERR_TIMEOUT):
_mtp_native.device_status() drops the device's cached workspaces so later
calls start from workspaces at rest, and mtp_parallel marks that device's
peer exchanges stale until reset_exchanges() runs (on every rank).  No GPU:
the status path is driven directly with fake cache entries."""

import pytest
import torch

import _mtp_native as N
import mtp_parallel as mp


def test_timeout_drops_device_workspaces():
    keep = (1, 111, "verify")
    drop = [(0, 111, "verify"), (0, 222, "rmsnorm_linear"), (0, 111, "vp_keys")]
    with N._ws_lock:
        for k in drop + [keep]:
            N._ws[k] = torch.empty(8, dtype=torch.uint8)
    try:
        N._reset_after_timeout(torch.device("cuda", 0))
        with N._ws_lock:
            assert not any(k in N._ws for k in drop)
            assert keep in N._ws  # another device's workspaces stay
    finally:
        with N._ws_lock:
            for k in drop + [keep]:
                N._ws.pop(k, None)


def test_timeout_marks_exchanges_stale_until_reset():
    class Fake:
        rows = 4

    mine, other = Fake(), Fake()
    mp._EXCHANGES[("p2p", 0, 7, 2)] = mine
    mp._EXCHANGES[("fused", 1, 7, 2)] = other
    try:
        N._reset_after_timeout(torch.device("cuda", 0))
        assert getattr(mine, "stale", False) and not getattr(other, "stale", False)
        with pytest.raises(N.MTPError, match="reset_exchanges"):
            mp._check_fresh(mine)
        mp._check_fresh(other)
        mp.reset_exchanges()
        assert not mp._EXCHANGES
    finally:
        mp._EXCHANGES.clear()
