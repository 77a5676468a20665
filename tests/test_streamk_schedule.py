"""The stream-K GEMM schedule, checked on the host: the library walks the
kernel's own work iterator (an __host__ __device__ function) for every CTA
and verifies that each (tile, K block) is computed exactly once and that the
slot every split part writes is the slot the summing part reads.  Also pins
which benchmark shapes the cost model sends to stream-K.  No GPU needed."""

import ctypes

import pytest

import _mtp_native as N

SMS = 148  # B200


def plan(M, Nn, K, dt=N.DT_BF16, sms=SMS, grid=0):
    info = (ctypes.c_int64 * 9)()
    N.check(N.lib().mtp_gemm_streamk_plan(M, Nn, K, dt, sms, grid, info), "mtp_gemm_streamk_plan")
    keys = ("use", "bn", "grid", "dp_rounds", "dp_tiles", "q", "tiles", "num_kb", "bytes")
    return dict(zip(keys, list(info)))


def check(M, Nn, K, dt=N.DT_BF16, sms=SMS, grid=0):
    st = N.lib().mtp_gemm_streamk_check(M, Nn, K, dt, sms, grid)
    assert st == 0, N.lib().mtp_last_error().decode()


# benchmark workloads (one GPU, and one rank of 8) plus shapes that cut tiles
# into many parts, leave CTAs without work, or have a single K block
SHAPES = [
    (384, 128256, 4096, N.DT_BF16),   # config 5 verify, 1 GPU
    (384, 16032, 4096, N.DT_BF16),    # config 5 verify, 1 of 8 ranks
    (512, 14336, 4096, N.DT_BF16),    # config 2 RMSNorm-linear, 1 GPU
    (512, 1792, 4096, N.DT_BF16),     # config 2, 1 of 8 ranks
    (1024, 14336, 4096, N.DT_E4M3),   # config 3 FP8
    (64, 128256, 4096, N.DT_BF16),
    (1, 300, 64, N.DT_BF16),
    (129, 257, 4096, N.DT_F16),
    (300, 1000, 1024, N.DT_E4M3),
]


@pytest.mark.parametrize("M,Nn,K,dt", SHAPES)
@pytest.mark.parametrize("grid", [0, 1, 3, 7, 16, 148])
def test_schedule_covers_every_block_once(M, Nn, K, dt, grid):
    p = plan(M, Nn, K, dt, grid=grid)
    if grid == 0 and not p["use"]:
        pytest.skip("cost model keeps the data-parallel schedule")
    check(M, Nn, K, dt, grid=grid)


def test_cost_model_choices():
    # verify, 1 GPU: 1503 tiles = 10.16 rounds -> 9 whole rounds + stream-K
    p = plan(384, 128256, 4096)
    assert p["use"] == 1 and p["bn"] == 256 and p["dp_rounds"] == 9 and p["tiles"] == 1503
    assert p["q"] == -(-(1503 - 9 * 148) * 64 // 148)
    # RMSNorm-linear, 1 GPU: 224 tiles = 1.51 rounds, all stream-K
    p = plan(512, 14336, 4096)
    assert p["use"] == 1 and p["dp_rounds"] == 0 and p["q"] == 97
    # verify, 1 of 8 ranks: 189 tiles
    assert plan(384, 16032, 4096)["use"] == 1
    # RMSNorm-linear, 1 of 8 ranks: 28 tiles of 256 would be cut ~5 ways;
    # the data-parallel schedule with narrower tiles is cheaper
    assert plan(512, 1792, 4096)["use"] == 0
    # whole rounds: nothing to balance
    assert plan(128 * 148, 256, 4096)["use"] == 0


def test_workspace_sizes():
    p = plan(384, 128256, 4096)
    assert p["bytes"] == 2 * 148 * 128 * 256 * 4 + N.STREAMK_TAIL
    assert N.STREAMK_TAIL == 16640


def test_schedule_switch_roundtrip():
    L = N.lib()
    assert L.mtp_gemm_schedule() in (0, 1)
    before = L.mtp_gemm_schedule()
    try:
        N.set_gemm_schedule(1)
        assert L.mtp_gemm_schedule() == 1
        N.set_gemm_schedule(0)
        assert L.mtp_gemm_schedule() == 0
        assert L.mtp_set_gemm_schedule(2) == 8  # MTP_ERR_ARG
    finally:
        N.set_gemm_schedule(before)


def test_schedule_random_shapes():
    """Property check over random shapes, dtypes and grids (seeded)."""
    import random
    rnd = random.Random(11)
    for _ in range(300):
        M = rnd.choice([1, 7, 64, 128, 129, 383, 384, 1000, 4096])
        Nn = rnd.choice([1, 64, 65, 128, 129, 256, 257, 1000, 16032, 128256])
        K = rnd.choice([16, 64, 128, 1000, 4096, 8192])
        dt = rnd.choice([N.DT_BF16, N.DT_F16, N.DT_E4M3])
        grid = rnd.choice([0, 1, 2, 5, 13, 64, 148, 300])
        sms = rnd.choice([8, 132, 148])
        p = plan(M, Nn, K, dt, sms=sms, grid=grid)
        if grid == 0 and not p["use"]:
            continue
        if p["grid"] <= 0:
            continue
        check(M, Nn, K, dt, sms=sms, grid=grid)


@pytest.mark.parametrize("M,Nn,K,dt", SHAPES)
def test_whole_tile_plan_covers_every_block_once(M, Nn, K, dt):
    """The whole-tile plan (grid < 0) the fused vocab-parallel verify runs
    when stream-K does not pay: a ragged last round must be skipped, not
    run past the last tile."""
    check(M, Nn, K, dt, grid=-1)


def tile_plan(M, Nn, sms=SMS):
    bn = ctypes.c_int(0)
    N.check(N.lib().mtp_gemm_tile_plan(M, Nn, sms, ctypes.byref(bn)), "mtp_gemm_tile_plan")
    return bn.value


def test_tile_plan_choices():
    """The tile width chosen per problem (fewest rounds x (128 + BN) operand
    rows per K block): config 5 verify 256, config 2 224."""
    assert tile_plan(384, 128256) == 256
    assert tile_plan(512, 14336) == 224
    assert tile_plan(64, 100) == 64   # N <= 128: the narrowest tile


def tile_check(M, Nn, grid):
    tiles = ctypes.c_int64(0)
    st = N.lib().mtp_gemm_tile_check(M, Nn, grid, ctypes.byref(tiles))
    assert st == 0, N.lib().mtp_last_error().decode()
    return tiles.value


@pytest.mark.parametrize("M,Nn", [(384, 128256), (384, 16032), (512, 14336), (300, 1000), (129, 64),
                                  (1000, 70000), (256, 256), (640, 9000)])
@pytest.mark.parametrize("grid", [1, 2, 3, 7, 74, 148, 149])
def test_tile_order_covers_every_tile_once(M, Nn, grid):
    tile_check(M, Nn, grid)


def test_tile_order_balances_rounds():
    """1503 tiles of 128 x 256 (config 5) on 148 CTAs: 11 rounds, no CTA
    takes more than that."""
    assert tile_check(384, 128256, SMS) == -(-(3 * -(-128256 // 256)) // SMS)
