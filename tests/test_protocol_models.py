"""Synchronisation protocols of the kernels, checked on the CPU with
randomised interleaving models (tests/protocol_models.py): the
vocab-parallel peer-memory key exchange, the exchange fused into the shard
GEMM, and the GEMM's accumulator handshake.  Each model must be clean for
the protocol the kernel uses and must catch a known-bad variant (one parity
for the exchange; the double-buffer phase formula on a single accumulator),
which shows the model can see the bug it guards against."""

import pytest

import protocol_models as PM


def _count(fn, seeds):
    bad = 0
    for seed in seeds:
        try:
            fn(seed)
        except PM.Violation:
            bad += 1
    return bad


def test_exchange_protocol():
    run = lambda par: (lambda seed: PM.run_exchange(seed, 2 + seed % 7, 6, parities=par))
    assert _count(run(2), range(300)) == 0
    assert _count(run(1), range(300)) > 0


def test_fused_exchange_protocol():
    run = lambda par: (lambda seed: PM.run_fused_exchange(seed, 2 + seed % 7, 6, parities=par))
    assert _count(run(2), range(300)) == 0
    assert _count(run(1), range(300)) > 0


@pytest.mark.parametrize("acc_bufs", [1, 2])
def test_gemm_accumulator_handshake(acc_bufs):
    """gemm_tc_kernel's double-buffered accumulators (and, as a second case
    of the same handshake, a single accumulator with its own phase rule):
    every MMA reads the stage it expects and the epilogue reads each tile's
    complete accumulator."""
    for seed in range(150):
        PM.run_gemm(seed, n_tiles=7, num_kb=5, stages=3, acc_bufs=acc_bufs)
        PM.run_gemm(seed + 1000, n_tiles=4, num_kb=1, stages=2, acc_bufs=acc_bufs)


def test_gemm_model_flags_wrong_single_buffer_phases():
    """Control: the double-buffer phase formula on a single accumulator must
    be caught (a wait passing early, a stale read, or a deadlock)."""
    flagged = 0
    for seed in range(50):
        try:
            PM.run_gemm(seed, n_tiles=7, num_kb=5, stages=3, acc_bufs=1, phase_rule="double")
        except PM.Violation:
            flagged += 1
    assert flagged == 50
