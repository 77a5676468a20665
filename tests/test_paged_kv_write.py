"""Batched paged KV write (mtp_paged_kv_write) against the reference's own
PagedKVCache.write_inplace (mtp_engine.py:582-586), whose results on the CPU
are the golden vectors in tests/golden/paged_kv_write.npz.  The oracle part
runs without a GPU; the device part is marked gpu.  The bar is bit-exact:
this is a copy (bf16 pools: the same round-to-nearest-even conversion)."""

import numpy as np
import pytest
import torch

from oracle import mtp_oracle as O


def test_oracle_matches_reference(golden):
    g = golden("paged_kv_write.npz")
    s = int(g["f32_start"][0])
    kp, vp = O.paged_kv_write(g["f32_k_before"], g["f32_v_before"], g["f32_page_table"], s,
                              g["f32_k_new"], g["f32_v_new"])
    assert np.array_equal(kp, g["f32_k_after"]) and np.array_equal(vp, g["f32_v_after"])
    s = int(g["bf16_start"][0])
    kb = O.bf16_bits_to_f32(g["bf16_k_before"])
    vb = O.bf16_bits_to_f32(g["bf16_v_before"])
    kp, vp = O.paged_kv_write(kb, vb, g["bf16_page_table"], s, O.round_to_bf16(g["bf16_k_new"]),
                              O.round_to_bf16(g["bf16_v_new"]))
    assert np.array_equal(O.f32_to_bf16_bits(kp), g["bf16_k_after"])
    assert np.array_equal(O.f32_to_bf16_bits(vp), g["bf16_v_after"])


@pytest.fixture(scope="module")
def mk():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mtp_kernels
    return mtp_kernels


@pytest.mark.gpu
@pytest.mark.isolated
def test_device_matches_reference(mk, golden):
    g = golden("paged_kv_write.npz")
    d = torch.device("cuda", 0)
    for name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        if dt == torch.float32:
            kp = torch.tensor(g[f"{name}_k_before"], device=d)
            vp = torch.tensor(g[f"{name}_v_before"], device=d)
        else:
            kp = torch.tensor(g[f"{name}_k_before"].view(np.int16), device=d).view(torch.bfloat16)
            vp = torch.tensor(g[f"{name}_v_before"].view(np.int16), device=d).view(torch.bfloat16)
        mk.paged_kv_write(kp, vp, torch.tensor(g[f"{name}_page_table"], device=d), int(g[f"{name}_start"][0]),
                          torch.tensor(g[f"{name}_k_new"], device=d), torch.tensor(g[f"{name}_v_new"], device=d))
        torch.cuda.synchronize()
        if dt == torch.float32:
            assert np.array_equal(kp.cpu().numpy(), g[f"{name}_k_after"])
            assert np.array_equal(vp.cpu().numpy(), g[f"{name}_v_after"])
        else:
            assert np.array_equal(kp.view(torch.int16).cpu().numpy().view(np.uint16), g[f"{name}_k_after"])
            assert np.array_equal(vp.view(torch.int16).cpu().numpy().view(np.uint16), g[f"{name}_v_after"])


@pytest.mark.gpu
@pytest.mark.isolated
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_device_tree_commit(mk, dt):
    """Commit a path of tree nodes (node_idx) with per-sequence lengths
    (count = accepted_n + 1) at the config-4 layout (page_size 16, D 128)."""
    import _mtp_native as N
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(5)
    P, B, H, ps, D, T = 64, 4, 8, 16, 128, 64
    kp = torch.randn(P, B, H, ps, D, generator=g, device=d).to(dt)
    vp = torch.randn(P, B, H, ps, D, generator=g, device=d).to(dt)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(1))
    L = (P // B) * ps
    table = torch.stack([perm[b * (P // B):(b + 1) * (P // B)].repeat_interleave(ps) for b in range(B)])
    table = table.to(torch.int32).to(d)
    tk = torch.randn(B, H, T, D, generator=g, device=d)  # fp32 source: converted on write
    tv = torch.randn(B, H, T, D, generator=g, device=d)
    n = 6
    node_idx = torch.randint(0, T, (B, n), generator=g, device=d, dtype=torch.int32)
    count = torch.tensor([6, 1, 0, 4], dtype=torch.int32, device=d)
    start = L - 40
    ref_k, ref_v = O.paged_kv_write(kp.float().cpu().numpy(), vp.float().cpu().numpy(), table.cpu().numpy(),
                                    start, tk.to(dt).float().cpu().numpy(), tv.to(dt).float().cpu().numpy(),
                                    node_idx.cpu().numpy(), count.cpu().numpy())
    mk.paged_kv_write(kp, vp, table, start, tk, tv, node_idx=node_idx, count=count)
    torch.cuda.synchronize()
    assert np.array_equal(kp.float().cpu().numpy(), ref_k)
    assert np.array_equal(vp.float().cpu().numpy(), ref_v)
    assert N.device_status(d) == 0


@pytest.mark.gpu
@pytest.mark.isolated
def test_device_bad_page_recorded(mk):
    import _mtp_native as N
    d = torch.device("cuda", 0)
    kp = torch.zeros(2, 1, 1, 4, 8, device=d)
    vp = torch.zeros_like(kp)
    table = torch.tensor([[0, 0, 0, 0, 5, 5, 5, 5]], dtype=torch.int32, device=d)  # page 5 is outside the pool
    src = torch.ones(1, 1, 8, 8, device=d)
    N.device_status(d)  # clear
    mk.paged_kv_write(kp, vp, table, 0, src, src)
    assert N.device_status(d) == 7  # MTP_ERR_DEVICE
    assert float(kp[0].sum()) == 4 * 8 and float(kp[1].sum()) == 0  # valid rows written, bad ones skipped
