"""The synchronisation protocols of two kernels that have not yet run on a
GPU, checked on the CPU with randomised interleaving models
(tests/protocol_models.py): the 64-key tree attention's mbarrier protocol
the vocab-parallel peer-memory key exchange, and the exchange fused into
the shard GEMM.  Each model must be clean
for the protocol the kernel uses and must catch a known-bad variant (the
previous final wait of the attention kernel; one parity for the exchange),
which shows the model can see the bug it guards against."""

import protocol_models as PM


def _count(fn, seeds):
    bad = 0
    for seed in seeds:
        try:
            fn(seed)
        except PM.Violation:
            bad += 1
    return bad


def _attn(final_wait):
    return lambda seed: PM.run_attn2(seed, 1 + seed % 11, 1 + (seed // 11) % 2,
                                     p_rescale=(0.0, 0.3, 1.0)[seed % 3], final_wait=final_wait)


def test_attention_tc2_protocol():
    assert _count(_attn("o_done"), range(400)) == 0
    assert _count(_attn("pv_parity"), range(400)) > 0


def test_exchange_protocol():
    run = lambda par: (lambda seed: PM.run_exchange(seed, 2 + seed % 7, 6, parities=par))
    assert _count(run(2), range(300)) == 0
    assert _count(run(1), range(300)) > 0


def test_fused_exchange_protocol():
    run = lambda par: (lambda seed: PM.run_fused_exchange(seed, 2 + seed % 7, 6, parities=par))
    assert _count(run(2), range(300)) == 0
    assert _count(run(1), range(300)) > 0
