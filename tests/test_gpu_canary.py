"""Out-of-bounds write checks without a sanitizer (compute-sanitizer is not
available on the GPU pool): every output and workspace is placed in the
middle of a buffer whose bytes are a canary pattern; after the call the
bytes on both sides must be untouched.  Ragged shapes (M, N, K, T not
multiples of any tile) exercise the edge paths.  Values are checked by the
parity tests.  GPU only; runs in a child process (tests/test_gpu_isolated.py)."""

import ctypes

import pytest
import torch

from oracle import mtp_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.isolated]

CANARY = 0x5A
PAD = 8192  # bytes on each side (a multiple of 256, so alignment is kept)


@pytest.fixture(scope="module")
def N():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _mtp_native
    _mtp_native.lib()
    return _mtp_native


class Guarded:
    """nbytes of device memory with PAD canary bytes before and after."""

    def __init__(self, nbytes, dtype=torch.uint8, init=None):
        self.nbytes = int(nbytes)
        self.raw = torch.full((self.nbytes + 2 * PAD,), CANARY, dtype=torch.uint8, device="cuda")
        self.ptr = ctypes.c_void_p(self.raw.data_ptr() + PAD)
        if init is not None:
            self.raw[PAD:PAD + self.nbytes].copy_(init.contiguous().view(torch.uint8).reshape(-1))

    def intact(self):
        torch.cuda.synchronize()
        return bool((self.raw[:PAD] == CANARY).all()) and bool((self.raw[PAD + self.nbytes:] == CANARY).all())


def rnd(shape, dt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, generator=g, device="cuda").to(dt)


@pytest.mark.parametrize("M,Nn,K,dt", [(130, 300, 264, torch.bfloat16), (7, 65, 72, torch.float32),
                                       (257, 1000, 4096, torch.bfloat16)])
def test_rmsnorm_linear(N, M, Nn, K, dt):
    x, w = rnd((M, K), dt, 1), (0.05 * rnd((Nn, K), torch.float32, 2)).to(dt)
    gam = 1.0 + 0.1 * rnd((K,), torch.float32, 3)
    es = x.element_size()
    y = Guarded(M * Nn * es)
    need = N.lib().mtp_rmsnorm_linear_workspace(M, K, 1)
    ws = Guarded(need)
    N.check(N.lib().mtp_rmsnorm_linear(N.ptr(x), N.dtype_code(x), N.ptr(w), N.dtype_code(w), None, 0, N.ptr(gam),
                                       N.DT_F32, y.ptr, N.dtype_code(x), M, Nn, K, 1e-5, 1.0, ws.ptr, need,
                                       N.stream_handle(x.device)), "rmsnorm_linear")
    assert y.intact() and ws.intact()


@pytest.mark.parametrize("B,S,K,V", [(5, 6, 264, 1000), (64, 6, 4096, 20000), (3, 1, 64, 77)])
def test_multi_verify(N, B, S, K, V):
    hid, w = rnd((B, S, K), torch.bfloat16, 4), (0.05 * rnd((V, K), torch.float32, 5)).to(torch.bfloat16)
    draft = torch.randint(0, V, (B, S - 1), device="cuda", dtype=torch.int32)
    acc, n, c = Guarded(B * (S - 1)), Guarded(B * 4), Guarded(B * 4)
    need = N.lib().mtp_verify_workspace(B * S)
    ws = Guarded(need)
    st = N.stream_handle(hid.device)
    N.check(N.lib().mtp_verify_workspace_init(ws.ptr, need, st), "init")
    for _ in range(2):
        N.check(N.lib().mtp_fused_multi_verify(N.ptr(hid), N.DT_BF16, N.ptr(w), N.DT_BF16, None, 0, N.ptr(draft),
                                               acc.ptr, n.ptr, c.ptr, B, S, K, V, ws.ptr, need, st), "verify")
    assert acc.intact() and n.intact() and c.intact() and ws.intact()


def test_tree_attention_paged(N):
    B, Hq, Hkv, D, ps, ctx = 3, 12, 3, 128, 16, 300
    _, tm = O.draft_tree(5, 3, "tree")
    T = tm.shape[0]
    P = B * (-(-ctx // ps)) + 1
    kp, vp = rnd((P, B, Hkv, ps, D), torch.bfloat16, 6), rnd((P, B, Hkv, ps, D), torch.bfloat16, 7)
    per = -(-ctx // ps)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(1))
    table = torch.stack([perm[b * per:(b + 1) * per].repeat_interleave(ps) for b in range(B)]).to(torch.int32).cuda()
    q = rnd((B, T, Hq, D), torch.bfloat16, 8)
    tk, tv = rnd((B, Hkv, T, D), torch.bfloat16, 9), rnd((B, Hkv, T, D), torch.bfloat16, 10)
    tmd = torch.tensor(tm, device="cuda")
    out = Guarded(q.numel() * 2)
    need = N.lib().mtp_tree_attention_paged_workspace(B, T, Hq, Hkv, D, ctx)
    ws = Guarded(max(need, 256))
    N.check(N.lib().mtp_tree_attention_paged(N.ptr(q), N.ptr(kp), N.ptr(vp), N.ptr(table), table.shape[1], ctx,
                                             N.ptr(tk), N.ptr(tv), N.ptr(tmd), out.ptr, N.DT_BF16, B, T, Hq, Hkv,
                                             D, P, ps, 1.0 / D ** 0.5, ws.ptr, max(need, 256),
                                             N.stream_handle(q.device)), "attention")
    assert out.intact() and ws.intact()


def test_tree_attn_rmsnorm_linear(N):
    B, H, D, L, Nn = 5, 2, 200, 37, 333
    q, k, v = rnd((B, H, D), torch.bfloat16, 11), rnd((B, H, L, D), torch.bfloat16, 12), rnd((B, H, L, D),
                                                                                          torch.bfloat16, 13)
    mask = (torch.rand(L, device="cuda") > 0.3).float()
    w = (0.05 * rnd((Nn, D), torch.float32, 14)).to(torch.bfloat16)
    out = Guarded(B * H * Nn * 2)
    need = N.lib().mtp_tree_attn_rmsnorm_linear_workspace(B, H, D, N.DT_BF16, N.DT_BF16)
    ws = Guarded(need)
    N.check(N.lib().mtp_tree_attn_rmsnorm_linear(N.ptr(q), N.ptr(k), N.ptr(v), N.DT_BF16, N.ptr(mask), None,
                                                 N.ptr(w), N.DT_BF16, None, 0, None, out.ptr, B, H, L, D, Nn,
                                                 D ** -0.5, 1e-6, ws.ptr, need, N.stream_handle(q.device)), "mono")
    assert out.intact() and ws.intact()


def test_verify_step_and_int4(N):
    B, D = 37, 5
    draft = torch.randint(0, 1000, (B, D), device="cuda", dtype=torch.int32)
    acc_n = torch.randint(0, D + 1, (B,), device="cuda", dtype=torch.int32)
    corr = torch.randint(0, 1000, (B,), device="cuda", dtype=torch.int32)
    tokens, info = Guarded(B * (D + 1) * 4), Guarded(8)
    N.check(N.lib().mtp_verify_step(N.ptr(draft), N.ptr(acc_n), N.ptr(corr), B, D, tokens.ptr, D + 1, info.ptr,
                                    N.stream_handle(draft.device)), "step")
    assert tokens.intact() and info.intact()
    import mtp_kernels as mk
    for M, Nn, K in ((1, 333, 1024), (5, 100, 64), (70, 129, 100)):
        pk, sc = mk.quantize_int4(rnd((Nn, K), torch.float32, 15), group=32)
        x = rnd((M, K), torch.bfloat16, 16)
        y = Guarded(M * Nn * 2)
        N.check(N.lib().mtp_int4_matmul(N.ptr(x), N.DT_BF16, N.ptr(pk), N.ptr(sc), 32, y.ptr, N.DT_BF16, M, Nn, K,
                                        N.stream_handle(x.device)), "int4")
        assert y.intact()


def test_streamk_gemm(N):
    M, Nn, K = 130, 700, 512
    a, b = rnd((M, K), torch.bfloat16, 17), rnd((Nn, K), torch.bfloat16, 18)
    info = (ctypes.c_int64 * 9)()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    N.check(N.lib().mtp_gemm_streamk_plan(M, Nn, K, N.DT_BF16, sms, 7, info), "plan")
    ws = Guarded(int(info[8]))
    N.check(N.lib().mtp_keys_fill(ws.ptr, int(info[8]) // 8, N.stream_handle(a.device)), "fill")
    c = Guarded(M * Nn * 4)
    N.check(N.lib().mtp_gemm_test_streamk(N.ptr(a), N.ptr(b), N.DT_BF16, c.ptr, M, Nn, K, 7, ws.ptr, int(info[8]),
                                          N.stream_handle(a.device)), "streamk")
    assert c.intact() and ws.intact()
