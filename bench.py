#!/usr/bin/env python
"""Tree-verification forward step benchmark (one JSON line on rank 0).

A step is one pass of the hot path over the benchmark workloads:
  1. fused RMSNorm -> linear, bf16, M=512 K=4096 N=14336 (config 2, gamma on)
  2. paged tree attention, bf16, B=16 Hq=32 Hkv=8 D=128 page 16, ctx 4096,
     64-node tree (config 4)
  3. fused_multi_verify, bf16, B=64 S=6 K=4096 V=128256 (config 5)
and verifies B*S = 384 candidate tokens.  On N GPUs (torchrun, one rank per
GPU) every rank runs stages 1 and 2 whole on its own batch and stage 3
verifies every rank's sequences against its vocabulary block of the
lm_head (candidates all-gathered, packed (logit, index) keys all-reduced
with MAX over NCCL) -- weak scaling, the north star's layout, where only
the lm_head is sharded.  With --scaling strong the 1-GPU job is split
tensor-parallel instead: stage 1 by output columns, stage 2 by KV heads,
stage 3 by vocabulary.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--scaling strong|weak] [--exchange nccl|p2p|fused|abi]
                    [--gemm-schedule dp|streamk]
    python bench.py --sweep [--sweep-only SECTIONS] [--compare]   # one line per config
    python bench.py --profile-case verify|rms|attention --steps K # the ncu capture workloads

--impl reference times the reference's eager algorithm as restated by the CPU
oracle (the reference is Python and cannot be shipped to the GPU box) on the
host cores, on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "mtp-engine_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "verified tokens/sec (fused norm-linear+tree-attn+verify); % TC/HBM roofline"
UNIT = "verified tokens/s"

# benchmark configs
C2 = dict(M=512, K=4096, N=14336, eps=1e-5)
C4 = dict(B=16, Hq=32, Hkv=8, D=128, ps=16, ctx=4096, P=4096, depth=16, branches=4)
C5 = dict(B=64, S=6, K=4096, V=128256)
TOKENS_PER_STEP = C5["B"] * C5["S"]

# algorithmic work per launch (full, unsharded job)
C2_FLOP = 2.0 * C2["M"] * C2["N"] * C2["K"]
C2_BYTES = 2.0 * (C2["M"] * C2["K"] + C2["N"] * C2["K"] + C2["M"] * C2["N"])
C4_T = 64
C4_BYTES = (2 * C4["B"] * C4["Hkv"] * C4["ctx"] * C4["D"] * 2          # context K and V
            + 2 * C4["B"] * C4["Hkv"] * C4_T * C4["D"] * 2              # tree K and V
            + 2 * C4["B"] * C4_T * C4["Hq"] * C4["D"] * 2)              # Q in, O out
C4_FLOP = 4.0 * C4["B"] * C4["Hq"] * C4_T * (C4["ctx"] + C4_T) * C4["D"]
C5_FLOP = 2.0 * C5["B"] * C5["S"] * C5["K"] * C5["V"]
C5_BYTES = 2.0 * (C5["V"] * C5["K"] + C5["B"] * C5["S"] * C5["K"])

WORKLOAD = ("tree-verification forward: rmsnorm_linear bf16 M=512 K=4096 N=14336 (cfg2) + "
            "paged tree attention bf16 B=16 Hq=32 Hkv=8 D=128 page16 ctx4096 T=64 (cfg4) + "
            "fused_multi_verify bf16 B=64 S=6 K=4096 V=128256 (cfg5)")


def arm_config(world, weak, args):
    """The `config` object of both arms' JSON lines for the same flags."""
    return {"workload": WORKLOAD, "tokens_per_step": TOKENS_PER_STEP * (world if weak else 1),
            "global_batch": C5["B"] * (world if weak else 1), "seq_len": C5["S"],
            "parallelism": "tp1" if world == 1 else
            (f"dp{world} (configs 2, 4 per GPU) + verify of {world}x{C5['B']} sequences, vocab-sharded"
             if weak else f"tp{world} (cols / kv-heads / vocab)"),
            "l2": "inputs larger than L2 (about 2.3 GB touched per step)"}


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return dict(hbm=float(p["hbm_gbs"]), bf16=float(p["bf16_tflops"]),
                    bf16_sus=float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), src="measured")
    except Exception:
        return dict(hbm=6650.0, bf16=1590.0, bf16_sus=1400.0, src="fallback")


def profile_traffic(name):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name>.md."""
    path = os.path.join(REPO, "profiles", name + ".md")
    try:
        with open(path) as f:
            m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


# --------------------------------------------------------------------------- #
# clocks during the timed region
# --------------------------------------------------------------------------- #
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_ids):
        self.proc = None
        self.gpu_ids = gpu_ids

    @staticmethod
    def job_gpus(world):
        """nvidia-smi ids of the GPUs this job runs on: local ranks 0..world-1,
        mapped through CUDA_VISIBLE_DEVICES when it is set (idle GPUs of the
        box must not enter the median)."""
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        return [vis[i] if i < len(vis) else str(i) for i in range(world)] if vis else list(range(world))

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "20"]
        if self.gpu_ids:
            cmd += ["-i", ",".join(str(i) for i in self.gpu_ids)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- #
# the verify's checker: fp32 argmax over the full vocabulary, independent of
# this library's kernels (cuBLAS fp32 with TF32 off, outside the timed region)
# --------------------------------------------------------------------------- #
MARGIN_TOL = 1e-3  # rows whose fp32 top-2 logit margin is at most this are not judged


def reference_top(hidden, lm_shard, offset, world):
    """Global argmax (lowest index on ties) of every candidate row against
    the lm_head, whose rows [offset, offset + len) this rank holds, and each
    row's top-2 margin.  Per rank: fp32 logits of its shard, its best and
    second-best value and best index; the ranks' triples are all-gathered and
    combined, as the reference's eager verify would see the whole vocabulary
    (mtp_fused_verify.py:180-183).  Returns (top [R] int64, margin [R] f32)."""
    import torch
    import torch.distributed as dist

    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        rows = hidden.reshape(-1, hidden.shape[-1]).float()
        best_v = torch.empty(rows.shape[0], device=hidden.device)
        best_i = torch.empty(rows.shape[0], dtype=torch.int64, device=hidden.device)
        second = torch.empty(rows.shape[0], device=hidden.device)
        w32 = lm_shard.float()
        for r0 in range(0, rows.shape[0], 1024):  # bounded logits memory
            lg = rows[r0:r0 + 1024] @ w32.T
            v, i = lg.max(dim=1)  # first maximal index on ties
            best_v[r0:r0 + 1024], best_i[r0:r0 + 1024] = v, i + offset
            lg.scatter_(1, i[:, None], float("-inf"))
            second[r0:r0 + 1024] = lg.max(dim=1).values
        del w32
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    trip = torch.stack([best_v.double(), best_i.double(), second.double()], 1)  # indices < 2^53: exact
    if world > 1:
        allt = [torch.empty_like(trip) for _ in range(world)]
        dist.all_gather(allt, trip)
        allt = torch.stack(allt)  # [world, R, 3]
    else:
        allt = trip[None]
    bv, bi, sv = allt[..., 0], allt[..., 1], allt[..., 2]
    gmax = bv.max(dim=0).values
    # lowest global index among the ranks holding the maximum
    cand = torch.where(bv == gmax[None], bi, torch.full_like(bi, float("inf")))
    top = cand.min(dim=0).values.long()
    # runner-up: every rank's second best, and the other ranks' bests
    is_win = (bv == gmax[None]) & (bi == top[None].double())
    others = torch.where(is_win, torch.full_like(bv, float("-inf")), bv)
    runner = torch.maximum(sv.max(dim=0).values, others.max(dim=0).values)
    return top, (gmax - runner).float()


def verify_parity(acc, n, c, prefix, top, margin):
    """Compare one verify's outputs with the drafts' construction: sequence b
    must accept exactly its drawn prefix, with `corrected` = the argmax at
    position 0.  A sequence is judged when every row that decides it
    (positions 0 .. prefix+1) has a top-2 margin above MARGIN_TOL."""
    import numpy as np
    B, D = acc.shape
    judged = mism = 0
    for b in range(B):
        a = int(prefix[b])
        if not (margin[b, :min(a + 1, D) + 1] > MARGIN_TOL).all():
            continue
        judged += 1
        want = np.zeros(D, np.int8)
        want[:a] = 1
        if int(n[b]) != a or int(c[b]) != int(top[b, 0]) or not np.array_equal(acc[b].astype(np.int8), want):
            mism += 1
    return judged, mism


# --------------------------------------------------------------------------- #
# our arm
# --------------------------------------------------------------------------- #
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import _mtp_native as N
    import mtp_fused_verify as mv
    import mtp_kernels as mk
    import mtp_parallel as mp
    from mtp_draft_tree import SpeculativeDraftTree

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    N.set_gemm_schedule(1 if args.gemm_schedule == "streamk" else 0)  # before any workspace exists
    if world > 1:
        import datetime
        opts = None
        if args.nccl_max_ctas > 0:
            # NCCL's kernels run beside this rank's own (the candidates'
            # all-gather beside stages 1-2): cap their CTAs so they fit in the
            # SMs those stages leave free instead of delaying their CTAs
            # (uncapped, the all-gather cost the stage beside it ~30 us)
            opts = dist.ProcessGroupNCCL.Options()
            opts.config.max_ctas = args.nccl_max_ctas
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev, pg_options=opts)
    prim = mp.get_parallel_primitives()
    assert C2["N"] % world == 0 and C4["Hkv"] % world == 0
    # strong: the 1-GPU job split tensor-parallel (columns / KV heads / vocabulary).
    # weak: configs 2 and 4 run whole on every GPU over that rank's own batch; the
    # verify checks every rank's candidates against a vocabulary-sharded lm_head
    # (the candidates all-gathered, the argmax keys all-reduced).
    weak = world > 1 and args.scaling == "weak"
    split = 1 if weak else world
    comm = None  # --exchange abi: the library's own NCCL communicator (C ABI)
    if world > 1 and args.exchange == "abi":
        uid = [mp.NcclCommunicator.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = mp.NcclCommunicator(uid[0], rank, world, dev)

    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    # ---- stage 1 inputs (columns split)
    Nr = C2["N"] // split
    x = torch.randn(C2["M"], C2["K"], generator=g, device=dev).to(torch.bfloat16)
    gamma = 1.0 + 0.1 * torch.randn(C2["K"], generator=g, device=dev)
    W = (0.02 * torch.randn(Nr, C2["K"], generator=g, device=dev)).to(torch.bfloat16)
    # ---- stage 2 inputs (KV heads split)
    Hkv = C4["Hkv"] // split
    Hq = Hkv * (C4["Hq"] // C4["Hkv"])
    B4, D, ps, ctx, P = C4["B"], C4["D"], C4["ps"], C4["ctx"], C4["P"]
    kp = torch.randn(P, B4, Hkv, ps, D, generator=g, device=dev).to(torch.bfloat16)
    vp = torch.randn(P, B4, Hkv, ps, D, generator=g, device=dev).to(torch.bfloat16)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(3))
    per_seq = ctx // ps
    table = torch.stack([perm[b * per_seq:(b + 1) * per_seq].repeat_interleave(ps) for b in range(B4)])
    table = table.to(torch.int32).to(dev)
    tmask_t = SpeculativeDraftTree(C4["depth"], C4["branches"], "tree").tree_mask
    tmask_np = tmask_t.numpy()
    T = tmask_np.shape[0]
    tmask = tmask_t.to(dev)
    q = torch.randn(B4, T, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    tk = torch.randn(B4, Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
    tv = torch.randn(B4, Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
    # ---- stage 3 inputs (vocabulary split)
    B5, S5, K5, V5 = C5["B"], C5["S"], C5["K"], C5["V"]
    lo, hi = mp.vocab_shard_range(V5, world, rank)
    BG = B5 * (world if weak else 1)  # sequences verified per step, all ranks
    gh = torch.Generator(device=dev).manual_seed(4)  # identical on every rank; weak: rank r owns block r
    hidden_g = torch.randn(BG, S5, K5, generator=gh, device=dev).to(torch.bfloat16)
    lm = (0.02 * torch.randn(hi - lo, K5, generator=g, device=dev)).to(torch.bfloat16)
    # drafts with per-sequence accept prefixes U{0..5}: needs the true argmax,
    # taken from the independent fp32 checker (also used for the parity check)
    top_t, margin_t = reference_top(hidden_g, lm, lo, world)
    top, margin = top_t.cpu().numpy().reshape(BG, S5), margin_t.cpu().numpy().reshape(BG, S5)
    rng = np.random.default_rng(4)
    draft_np = rng.integers(0, V5, size=(BG, S5 - 1))
    prefix = np.zeros(BG, np.int64)
    for b in range(BG):
        a = int(rng.integers(0, S5))
        prefix[b] = a
        draft_np[b, :a] = top[b, 1:a + 1]
        if a < S5 - 1:
            while draft_np[b, a] == top[b, a + 1]:
                draft_np[b, a] = rng.integers(0, V5)
    own = slice(rank * B5, (rank + 1) * B5) if weak else slice(0, B5)
    hidden = hidden_g[own].contiguous()
    draft = torch.tensor(draft_np[own], dtype=torch.int32, device=dev)
    del hidden_g
    # weak: every rank's candidates gathered here before the verify
    hid_all = torch.empty((BG, S5, K5), dtype=torch.bfloat16, device=dev) if weak else None
    dr_all = torch.empty((BG, S5 - 1), dtype=torch.int32, device=dev) if weak else None
    pending = []  # weak: an all-gather issued early in the step, awaited by the verify

    def gather(hh, dd):
        """Start the all-gather of this rank's candidates (async; it overlaps
        whatever the stream runs next)."""
        pending.append((dist.all_gather_into_tensor(hid_all, hh, async_op=True),
                        dist.all_gather_into_tensor(dr_all, dd, async_op=True)))

    def stage1(xx):
        return mk.fused_rmsnorm_linear(xx, W, None, C2["eps"], norm_weight=gamma)

    def stage2(qq, kk, vv):
        return mk.fused_tree_attention_paged(qq, kp, vp, table, kk, vv, tmask)

    def stage3(hh, dd):
        if world == 1:
            return mv.fused_multi_verify(hh, lm, dd)
        if weak:
            if not pending:
                gather(hh, dd)
            for w_ in pending.pop():
                w_.wait()  # the stream waits for the gather, the host does not
            hh, dd = hid_all, dr_all
        if comm is not None:
            return mp.vocab_parallel_multi_verify_nccl(hh, lm, dd, lo, comm)
        return mp.vocab_parallel_multi_verify(hh, lm, dd, None, lo, prim, exchange=args.exchange)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    # ---- warm-up (eager) on the stream the step runs on
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            stage1(x)
            stage2(q, tk, tv)
            stage3(hidden, draft)
    stream.synchronize()
    barrier()

    # ---- each stage captured once as a CUDA graph (kernel launches and, on
    # N > 1, the NCCL all-reduce of the verify keys); replays cost one launch
    # Graph replays are used on one GPU.  With N > 1 the stages launch
    # eagerly unless --graph is given: a graph holding an NCCL call must be
    # released before destroy_process_group (see the teardown below), and on
    # 2-8 GPUs the replays saved only a few percent.
    # With the peer-memory exchange the verify holds no NCCL call, so its graph
    # needs no special teardown: replay graphs on N > 1 too.
    use_graphs = (world == 1 or args.graph or args.exchange in ("p2p", "fused")) and not args.no_graph and not weak
    launches0 = N.lib().mtp_launch_count()
    graphs = []  # the only owner of the graph objects
    if use_graphs:
        for fn in (lambda: stage1(x), lambda: stage2(q, tk, tv), lambda: stage3(hidden, draft)):
            graphs.append(torch.cuda.CUDAGraph())
            with torch.cuda.graph(graphs[-1], stream=stream):
                outs = fn()
            graphs[-1].outputs = outs
        stream.synchronize()
        barrier()
        launches_per_step = N.lib().mtp_launch_count() - launches0
        run = [lambda i=i: graphs[i].replay() for i in range(3)]
    else:
        run = [lambda: stage1(x), lambda: stage2(q, tk, tv), lambda: stage3(hidden, draft)]

    # ---- timed region (device time, CUDA events on the launching stream)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(ClockSampler.job_gpus(world) if world > 1 else
                           ClockSampler.job_gpus(local + 1)[local:]) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.2)
    launches0 = N.lib().mtp_launch_count()
    barrier()
    with torch.cuda.stream(stream):
        t_start.record(stream)
        for i in range(args.steps):
            e = ev[i]
            e[0].record(stream)
            if weak:
                # overlaps stages 1 and 2: NCCL's kernel (capped at
                # --nccl-max-ctas CTAs) runs in the SMs the pair GEMM leaves
                # free (128 tiles take 64 pairs, 128 of the 148 SMs)
                gather(hidden, draft)
            run[0]()
            e[1].record(stream)
            run[1]()
            e[2].record(stream)
            run[2]()
            e[3].record(stream)
        t_end.record(stream)
    barrier()
    launches = N.lib().mtp_launch_count() - launches0
    if graphs:
        launches = launches_per_step * args.steps  # graph replays launch the captured kernels
    clocks = sampler.stop() if sampler else None
    total_ms = t_start.elapsed_time(t_end)
    stage_ms = [sum(e[j].elapsed_time(e[j + 1]) for e in ev) / args.steps for j in range(3)]
    t = torch.tensor([total_ms] + stage_ms, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, s1, s2, s3 = t.tolist()
    ms_per_step = total_ms / args.steps
    tokens_per_step = TOKENS_PER_STEP * (world if weak else 1)
    value = tokens_per_step * args.steps / (total_ms / 1e3)

    # ---- end to end through the public API, host buffers in and out
    pin = lambda tt: tt.cpu().pin_memory()
    h_x, h_q, h_tk, h_tv, h_hid, h_dr = (pin(a) for a in (x, q, tk, tv, hidden, draft))
    d_x, d_q, d_tk, d_tv, d_hid, d_dr = x, q, tk, tv, hidden, draft  # the captured graphs read these
    o_acc = torch.empty((B5, S5 - 1), dtype=torch.int8).pin_memory()
    o_n = torch.empty((B5,), dtype=torch.int32).pin_memory()
    o_c = torch.empty((B5,), dtype=torch.int32).pin_memory()
    h2d = sum(a.numel() * a.element_size() for a in (h_x, h_q, h_tk, h_tv, h_hid, h_dr))
    d2h = sum(a.numel() * a.element_size() for a in (o_acc, o_n, o_c))

    # Host->device copies run in the order the stages run, each stage waiting
    # only for its own inputs.  The stages are independent, so the verify --
    # the longest stage with the smallest upload (3 MB) -- runs first and the
    # other stages' 16.6 MB upload overlaps it; its result goes back on a
    # third stream while the other two stages run.  The uploads alternate
    # between two copy streams, so two copy engines share the host link (one
    # engine alone left the link part idle on some hosts).  Every step
    # uploads all inputs and the host waits for the result before the next.
    copy_streams = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    d2h_stream = torch.cuda.Stream(dev)
    order = (2, 0, 1)
    groups = {2: ((h_hid, d_hid), (h_dr, d_dr)), 0: ((h_x, d_x),), 1: ((h_q, d_q), (h_tk, d_tk), (h_tv, d_tv))}
    step_start = torch.cuda.Event()
    ready = {j: [torch.cuda.Event() for _ in groups[j]] for j in order}
    verified = torch.cuda.Event()

    def upload():
        """Every input of the step, alternating between the copy streams;
        ready[j] holds the events that stage j waits for."""
        k = 0
        for j in order:
            for (h, d_), ev in zip(groups[j], ready[j]):
                cs_ = copy_streams[k % 2]
                with torch.cuda.stream(cs_):
                    d_.copy_(h, non_blocking=True)
                    ev.record(cs_)
                k += 1

    def e2e_step():
        step_start.record(stream)
        for cs_ in copy_streams:
            cs_.wait_event(step_start)
        upload()
        with torch.cuda.stream(stream):
            for j in order:
                for ev in ready[j]:
                    stream.wait_event(ev)
                out = run[j]()
                if j == 2:
                    a, n_, c = graphs[2].outputs if graphs else out
                    if weak:  # this rank reads back its own sequences
                        a, n_, c = a[own], n_[own], c[own]
                    verified.record(stream)
                    d2h_stream.wait_event(verified)
                    with torch.cuda.stream(d2h_stream):
                        o_acc.copy_(a, non_blocking=True)
                        o_n.copy_(n_, non_blocking=True)
                        o_c.copy_(c, non_blocking=True)
        stream.synchronize()
        d2h_stream.synchronize()

    def time_e2e(step_fn):
        """Warm-up, then args.steps steps between two events; tokens/s, max over ranks."""
        for _ in range(max(1, args.warmup)):
            step_fn()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step_fn()
        e1.record(stream)
        stream.synchronize()
        barrier()
        te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return tokens_per_step * args.steps / (te.item() / 1e3)

    e2e_eager_value = time_e2e(e2e_step)
    e2e_value = e2e_eager_value
    eager_out = (o_acc.clone(), o_n.clone(), o_c.clone())

    # 1 GPU (default; --e2e-eager turns it off): the same step -- uploads on
    # the copy streams, the three stages, the read-back -- captured once as
    # one graph; a step is then one replay and the host's wait for its
    # result.  The replays copy from the same pinned host buffers, so new
    # inputs written there are picked up by the next step.  Its read-back
    # must equal the eager step's bit for bit.
    e2e_graph = None
    e2e_one_graph = False
    graph_matches_eager = None
    if not args.e2e_eager and world == 1:
        stage_fns = {0: lambda: stage1(d_x), 1: lambda: stage2(d_q, d_tk, d_tv), 2: lambda: stage3(d_hid, d_dr)}
        e2e_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(e2e_graph, stream=stream):
            for cs_ in copy_streams:
                cs_.wait_stream(stream)
            upload()
            for j in order:
                for ev in ready[j]:
                    stream.wait_event(ev)
                out = stage_fns[j]()
                if j == 2:
                    a, n_, c = out
                    verified.record(stream)
                    d2h_stream.wait_event(verified)
                    with torch.cuda.stream(d2h_stream):
                        o_acc.copy_(a, non_blocking=True)
                        o_n.copy_(n_, non_blocking=True)
                        o_c.copy_(c, non_blocking=True)
            for cs_ in copy_streams:
                stream.wait_stream(cs_)
            stream.wait_stream(d2h_stream)
        stream.synchronize()
        for o in (o_acc, o_n, o_c):
            o.fill_(-7)  # a replay that does not write its read-back shows up below

        def e2e_graph_step():
            with torch.cuda.stream(stream):
                e2e_graph.replay()
            stream.synchronize()

        e2e_value = time_e2e(e2e_graph_step)
        e2e_one_graph = True
        graph_matches_eager = all(bool(torch.equal(g, e)) for g, e in zip((o_acc, o_n, o_c), eager_out))

    # ---- parity of the verify outputs that the last end-to-end step read back
    # to the host, against the fp32 checker (every rank checks its sequences)
    judged, mism = verify_parity(o_acc.numpy(), o_n.numpy(), o_c.numpy(), prefix[own], top[own], margin[own])
    pc = torch.tensor([judged, mism, B5], dtype=torch.int64, device=dev)
    if world > 1:
        dist.all_reduce(pc, op=dist.ReduceOp.SUM)
    judged, mism, seqs = pc.tolist()
    parity = {"ok": bool(mism == 0 and judged >= 0.9 * seqs and graph_matches_eager is not False),
              "sequences": seqs, "judged": judged,
              "mismatches": mism, "margin_tol": MARGIN_TOL,
              "checker": "drawn accept prefixes and argmax from a torch fp32 matmul (TF32 off) of each "
                         "vocabulary shard, combined over ranks; outputs read back by the end-to-end step"}

    # ---- N > 1: the shard GEMM alone (same inputs), so the verify stage splits
    # into GEMM time and exchange + decode time
    verify_gemm_ms = None
    if world > 1 and comm is None and args.exchange != "fused":
        hh, _ = (hid_all, dr_all) if weak else (hidden, draft)
        rows_v, Vr = hh.shape[0] * S5, hi - lo
        kbuf = torch.full((rows_v,), -(2 ** 63), dtype=torch.int64, device=dev)
        sk_bytes = N.streamk_bytes(rows_v, Vr, K5, N.DT_BF16)
        region = torch.empty(max(sk_bytes, 256), dtype=torch.uint8, device=dev)
        N.check(N.lib().mtp_keys_fill(N.ptr(region), region.numel() // 8, N.stream_handle(dev)), "region at rest")

        def shard_gemm():
            N.check(N.lib().mtp_verify_shard_keys_ws(N.ptr(hh), N.DT_BF16, N.ptr(lm), N.DT_BF16, None, 0,
                                                     N.ptr(kbuf), rows_v, K5, Vr, lo, N.ptr(region), sk_bytes,
                                                     N.stream_handle(dev)), "shard gemm")
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                shard_gemm()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            g0.record(stream)
            for _ in range(args.steps):
                shard_gemm()
            g1.record(stream)
        barrier()
        tg = torch.tensor([g0.elapsed_time(g1) / args.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(tg, op=dist.ReduceOp.MAX)
        verify_gemm_ms = tg.item()
        del kbuf, region

    status = N.device_status(dev)
    # graphs that hold NCCL calls must be gone before destroy_process_group:
    # drop every reference (the list and the replay closures), then collect
    run = None
    e2e_graph = None
    graphs.clear()
    mp._EXCHANGES.clear()  # symmetric-memory buffers go before the process group too
    import gc
    gc.collect()
    torch.cuda.synchronize(dev)
    if comm is not None:  # after the graphs that may hold its all-reduce
        comm.close()
        comm = None
    if rank != 0:
        if world > 1:
            dist.barrier(device_ids=[local])
            dist.destroy_process_group()
        return

    peaks = load_peaks()
    # per-GPU rooflines: strong -- each rank does 1/world of every stage's work;
    # weak -- every rank does a whole config 2 and 4, and 1/world of a verify
    # over world x 64 sequences (the FLOPs of one config-5 verify)
    w = float(split)
    kernels = {
        "rmsnorm_linear": {"ms": s1, "bound": "tensor", "achieved": C2_FLOP / w / (s1 / 1e3) / 1e12,
                           "unit": "TFLOP/s", "flop_per_gpu": C2_FLOP / w, "bytes_per_gpu": C2_BYTES / w},
        "tree_attention_paged": {"ms": s2, "bound": "hbm", "achieved": C4_BYTES / w / (s2 / 1e3) / 1e9,
                                 "unit": "GB/s", "bytes_per_gpu": C4_BYTES / w, "flop_per_gpu": C4_FLOP / w},
        "fused_multi_verify": {"ms": s3, "bound": "tensor", "achieved": C5_FLOP / w / (s3 / 1e3) / 1e12,
                               "unit": "TFLOP/s", "flop_per_gpu": C5_FLOP / w, "bytes_per_gpu": C5_BYTES / w,
                               "note": "includes the NCCL key all-reduce when n_gpus > 1" +
                                       (", and the wait for the candidates' all-gather" if weak else "")},
    }
    # fractions of the measured burst peak: each stage runs for well under a
    # millisecond at a time inside a short timed region; the sustained figure
    # (a seconds-long GEMM loop at the power cap) is reported beside it
    for k in kernels.values():
        if k["bound"] == "hbm":
            k["frac"] = k["achieved"] / peaks["hbm"]
        else:
            k["frac"] = k["achieved"] / peaks["bf16"]
            k["frac_of_sustained"] = k["achieved"] / peaks["bf16_sus"]
    if verify_gemm_ms is not None:
        kv = kernels["fused_multi_verify"]
        kv["gemm_ms"] = verify_gemm_ms
        kv["exchange_ms"] = max(s3 - verify_gemm_ms, 0.0)
        kv["gemm_achieved"] = C5_FLOP / w / (verify_gemm_ms / 1e3) / 1e12  # TFLOP/s per GPU
        kv["gemm_note"] = ("shard GEMM alone (same inputs, timed separately); exchange_ms = stage time - gemm_ms: "
                           "the key all-reduce" + (", the wait for the all-gather" if weak else "") +
                           " and the acceptance scan")
    dom_name = max(kernels, key=lambda n: kernels[n]["ms"])
    dom = kernels[dom_name]
    prof_name = {"fused_multi_verify": "verify_gemm_c5", "rmsnorm_linear": "rmsnorm_linear_c2",
                 "tree_attention_paged": "tree_attention_c4"}[dom_name]
    roofline = {
        "kernel": dom_name, "bound": dom["bound"], "achieved": dom["achieved"],
        "peak": peaks["hbm"] if dom["bound"] == "hbm" else peaks["bf16"],
        "unit": dom["unit"], "frac": dom["frac"],
        "peak_source": f"{peaks['src']} ({'hbm_gbs' if dom['bound'] == 'hbm' else 'bf16_tflops, burst'})",
        "traffic": profile_traffic(prof_name) if world == 1 else None,
        "per": "GPU",
    }
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        host_threads()
        cpu = cpu_baseline_sample(x, gamma, W, kp, vp, table, q, tk, tv, tmask_np, hidden, lm, draft,
                                  budget_s=args.cpu_budget)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) activations / KV, random-init weights of the benchmark shapes",
        "config": dict(arm_config(world, weak, args), gemm_schedule=args.gemm_schedule,
                       exchange=args.exchange if world > 1 else "none"),
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "order": "verify, RMSNorm-linear, attention; uploads on two copy streams overlap earlier "
                         "stages; host waits for each step's result",
                "one_graph_per_step": e2e_one_graph, "eager_value": e2e_eager_value,
                "graph_matches_eager": graph_matches_eager},
        "gpu_launches": launches,
        "parity": parity,
        "clocks": clocks,
        "kernels": kernels,
        "device_status": status,
    }
    print(json.dumps(line), flush=True)
    if not parity["ok"]:
        print(f"bench: verify outputs differ from the fp32 checker: {parity}", file=sys.stderr, flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


# --------------------------------------------------------------------------- #
# CPU baseline: the oracle (restated reference eager path) on host cores
# --------------------------------------------------------------------------- #
SAMPLE_DESC = ("1/16 of each stage: 32 of 512 rmsnorm_linear rows, 1 of 16 attention sequences "
               "(all 64 nodes, 32 heads), 4 of 64 verify sequences (full vocabulary)")
SAMPLE_FRACTION_INV = 16


def host_threads():
    """Give the host BLAS every core this process may run on (torchrun sets
    OMP_NUM_THREADS=1 for its workers); returns the thread count.  Must run
    before numpy is first imported for the environment to reach OpenBLAS;
    threadpoolctl covers an already loaded BLAS."""
    try:
        n = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        n = os.cpu_count() or 1
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = str(n)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n)
    except Exception:
        pass
    return _blas_threads()


def _blas_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else os.cpu_count()
    except Exception:
        return os.cpu_count()


def cpu_sample_inputs_from_numpy(seed=0):
    """Host-generated inputs with the sample's shapes (reference arm: no GPU)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s, dtype=np.float32)
    ctx, ps = C4["ctx"], C4["ps"]
    _, tmask = __import__("oracle.mtp_oracle", fromlist=["x"]).draft_tree(C4["depth"], C4["branches"], "tree")
    pages = ctx // ps
    return dict(
        x=f(32, C2["K"]), gamma=1 + 0.1 * f(C2["K"]), W=0.02 * f(C2["N"], C2["K"]),
        kp=f(pages, 1, C4["Hkv"], ps, C4["D"]), vp=f(pages, 1, C4["Hkv"], ps, C4["D"]),
        table=np.repeat(np.arange(pages, dtype=np.int32), ps)[None, :],
        q=f(1, 64, C4["Hq"], C4["D"]), tk=f(1, C4["Hkv"], 64, C4["D"]), tv=f(1, C4["Hkv"], 64, C4["D"]),
        tmask=tmask, hidden=f(4, C5["S"], C5["K"]), lm=0.02 * f(C5["V"], C5["K"]),
        draft=rng.integers(0, C5["V"], size=(4, C5["S"] - 1)))


def cpu_sample_step(inp):
    from oracle import mtp_oracle as O
    O.rmsnorm_linear(inp["x"], inp["W"] * inp["gamma"][None, :], None, C2["eps"], 1.0)
    O.tree_attention_paged_fast(inp["q"], inp["kp"], inp["vp"], inp["table"], C4["ctx"], C4["ps"],
                                inp["tk"], inp["tv"], inp["tmask"], 1.0 / math.sqrt(C4["D"]))
    O.fused_multi_verify(inp["hidden"], inp["lm"], None, inp["draft"])


def cpu_baseline_sample(x, gamma, W, kp, vp, table, q, tk, tv, tmask_np, hidden, lm, draft, budget_s=20.0):
    import numpy as np
    import torch
    f32 = lambda t: t.detach().float().cpu().numpy()
    pages = table[0].view(-1, C4["ps"])[:, 0].long()
    inp = dict(x=f32(x[:32]), gamma=f32(gamma), W=f32(W),
               kp=f32(kp[pages][:, 0:1]), vp=f32(vp[pages][:, 0:1]),
               table=np.repeat(np.arange(pages.numel(), dtype=np.int32), C4["ps"])[None, :],
               q=f32(q[0:1]), tk=f32(tk[0:1]), tv=f32(tv[0:1]), tmask=tmask_np,
               hidden=f32(hidden[:4]), lm=f32(lm), draft=draft[:4].cpu().numpy())
    cpu_sample_step(inp)  # warm-up
    times = []
    t0 = time.perf_counter()
    while len(times) < 3 or (time.perf_counter() - t0 < budget_s and len(times) < 20):
        t1 = time.perf_counter()
        cpu_sample_step(inp)
        times.append(time.perf_counter() - t1)
        if time.perf_counter() - t0 > budget_s:
            break
    per_sample = statistics.median(times)
    tokens = TOKENS_PER_STEP / SAMPLE_FRACTION_INV
    return {"value": tokens / per_sample, "unit": UNIT, "cores": _blas_threads(), "kind": "port",
            "sample": SAMPLE_DESC + f" ({tokens:g} verified tokens); value = those tokens / the median time of "
                                    f"{len(times)} sample steps", "host_cpu_count": os.cpu_count()}


def run_reference(args):
    """The reference arm: the reference's eager algorithm for the path, as the
    CPU oracle restates it (the reference is Python and does not travel to the
    GPU box), on every host core of rank 0 (the other ranks exit).  Each step
    is a bounded 1/16 sample of the workload; `value` and `ms_per_step` are
    what the timed sample steps measured."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    cores = host_threads()
    inp = cpu_sample_inputs_from_numpy()
    for _ in range(args.warmup):
        cpu_sample_step(inp)
    times = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        t1 = time.perf_counter()
        cpu_sample_step(inp)
        times.append(time.perf_counter() - t1)
    wall = time.perf_counter() - t0
    per_step = sum(times) / len(times)
    tokens = TOKENS_PER_STEP / SAMPLE_FRACTION_INV
    value = tokens / per_step
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "weak" if (world > 1 and args.scaling == "weak") else "strong", "vs_baseline": None,
        "dtype": "f32", "impl": "reference",
        "data": "synthetic: seeded N(0,1) inputs of the benchmark shapes (host)",
        "config": arm_config(world, world > 1 and args.scaling == "weak", args),
        "timed_region_s": wall,
        "sample_fraction": 1.0 / SAMPLE_FRACTION_INV,
        "tokens_per_sample_step": tokens,
        "full_step_ms_estimate": per_step * SAMPLE_FRACTION_INV * 1e3,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": SAMPLE_DESC + f" per step ({tokens:g} verified tokens); value = those tokens / "
                                                 "the measured time of a sample step",
                         "host_cpu_count": os.cpu_count(), "execution": "host cpu, rank 0",
                         "note": "the reference is pure Python/torch; its eager path is timed as restated "
                                 "by the oracle (numpy fp32, BLAS threads = cores)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_sweep(args):
    """--sweep: every benchmark config timed on its own (one JSON line each,
    marked "sweep"), 1 GPU.  L2 is flushed (256 MB write) between timed
    calls; each call is bracketed by CUDA events on its stream; the median is
    reported with its roofline fraction and a CPU-oracle baseline on a bounded
    sample of the same config."""
    import numpy as np
    import torch

    import _mtp_native as N
    import mtp_fused_verify as mv
    import mtp_kernels as mk
    from mtp_draft_tree import SpeculativeDraftTree
    from oracle import mtp_oracle as O  # the CPU-baseline column of each line only

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N.set_gemm_schedule(1 if args.gemm_schedule == "streamk" else 0)
    peaks = load_peaks()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    f32 = lambda t: t.detach().float().cpu().numpy()

    def time_call(fn, iters):
        for _ in range(args.warmup):
            fn()
        ts = []
        for _ in range(iters):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) / 1e3)
        return statistics.median(ts)

    def cpu_time(fn, budget=8.0):
        if args.no_cpu_baseline:
            return float("nan")
        fn()
        ts, t0 = [], time.perf_counter()
        while not ts or (time.perf_counter() - t0 < budget and len(ts) < 5):
            t1 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t1)
        return statistics.median(ts)

    def emit(name, units, unit, t, bound, achieved, peak, peak_src, cpu_units, cpu_t, extra=None):
        line = {"sweep": True, "config": name, "metric": f"{unit} ({name})", "value": units / t, "unit": unit,
                "gemm_schedule": args.gemm_schedule,
                "ms": t * 1e3, "dtype": extra.pop("dtype") if extra and "dtype" in extra else "bf16",
                "roofline": {"bound": bound, "achieved": achieved, "peak": peak,
                             "unit": "TFLOP/s" if bound == "tensor" else "GB/s", "frac": achieved / peak,
                             "peak_source": peak_src},
                "cpu_baseline": {"value": cpu_units / cpu_t, "unit": unit, "cores": _blas_threads(),
                                 "kind": "port", "sample": f"{cpu_units} units"}}
        if extra:
            line.update(extra)
        print(json.dumps(line), flush=True)

    iters = max(5, min(args.steps, 50))
    # --compare: each GEMM config under both schedules, config 4 under both
    # attention kernels (one line per variant)
    # GEMM variants: (label, schedule)
    gemm_variants = ((("dp", 0), ("streamk", 1)) if args.compare else
                     ((args.gemm_schedule, 1 if args.gemm_schedule == "streamk" else 0),))

    def timed_gemm(fn):
        out = []
        for label, sched in gemm_variants:
            N.set_gemm_schedule(sched)
            out.append((label, time_call(fn, iters)))
        N.set_gemm_schedule(1 if args.gemm_schedule == "streamk" else 0)
        return out

    def sec_config1():
        # ---- config 1: the CPU-runnable chain (fp32, seed 0): RMSNorm-linear of the
        # 5 candidate positions, then fused_multi_verify with the first two drafts
        # set to the target's own argmax -> accepted_n = 2 (launch-bound; bytes =
        # both weights once)
        g1 = torch.Generator(device=dev).manual_seed(0)
        x1 = torch.randn(1, 5, 256, generator=g1, device=dev)
        gam1 = 1.0 + 0.1 * torch.randn(256, generator=g1, device=dev)
        W1 = 0.02 * torch.randn(256, 256, generator=g1, device=dev)
        LM1 = 0.02 * torch.randn(4096, 256, generator=g1, device=dev)
        y1 = mk.fused_rmsnorm_linear(x1[0], W1, None, 1e-6, norm_weight=gam1)
        top1 = (y1 @ LM1.T).argmax(-1)
        d1 = torch.randint(0, 4096, (1, 4), generator=g1, device=dev, dtype=torch.int32)
        d1[0, :2] = top1[1:3].to(torch.int32)
        if int(top1[3]) == int(d1[0, 2]):
            d1[0, 2] = (d1[0, 2] + 1) % 4096
        chain1 = lambda: mv.fused_multi_verify(mk.fused_rmsnorm_linear(x1[0], W1, None, 1e-6, norm_weight=gam1)[None],
                                               LM1, d1)
        n1 = int(chain1()[1][0])
        t1 = time_call(chain1, iters)
        xs1, ws1, gs1, lms1, ds1 = f32(x1[0]), f32(W1), f32(gam1), f32(LM1), d1.cpu().numpy()
        ct = cpu_time(lambda: O.fused_multi_verify(O.rmsnorm_linear(xs1, ws1 * gs1[None, :], None, 1e-6, 1.0)[None],
                                                   lms1, None, ds1))
        emit("config1_chain", 5, "verified candidates/s", t1, "hbm", 4.0 * (256 * 256 + 4096 * 256) / t1 / 1e9,
             peaks["hbm"], "measured hbm_gbs", 5, ct, {"dtype": "f32", "accepted_n": n1,
                                                       "note": "launch-bound: two launches for 4.5 MB"})
        del x1, W1, LM1

    def sec_config2():
        # ---- config 2 sweep: RMSNorm-linear bf16, gamma on
        for M in (64, 512, 2048, 8192):
            K, Nn = C2["K"], C2["N"]
            g = torch.Generator(device=dev).manual_seed(1)
            x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
            gam = 1.0 + 0.1 * torch.randn(K, generator=g, device=dev)
            W = (0.02 * torch.randn(Nn, K, generator=g, device=dev)).to(torch.bfloat16)
            times = timed_gemm(lambda: mk.fused_rmsnorm_linear(x, W, None, C2["eps"], norm_weight=gam))
            flop, byts = 2.0 * M * Nn * K, 2.0 * (M * K + Nn * K + M * Nn)
            tensor = flop / byts > 281  # ridge of the measured peaks
            rows = min(M, 16)
            xs, ws, gs = f32(x[:rows]), f32(W), f32(gam)
            ct = cpu_time(lambda: O.rmsnorm_linear(xs, ws * gs[None, :], None, C2["eps"], 1.0))
            for v, t in times:
                emit(f"config2_M{M}", M, "rows/s", t, "tensor" if tensor else "hbm",
                     flop / t / 1e12 if tensor else byts / t / 1e9, peaks["bf16"] if tensor else peaks["hbm"],
                     "measured bf16_tflops (burst)" if tensor else "measured hbm_gbs", rows, ct,
                     {"gemm_schedule": v})
            del x, W

    def sec_config3():
        # ---- config 3: FP8 E4M3, per-token activations, packed per-channel weight scales
        M, K, Nn = 1024, 8192, 28672
        g = torch.Generator(device=dev).manual_seed(2)
        x = torch.randn(M, K, generator=g, device=dev)
        x = x * (448.0 / x.abs().amax(dim=1, keepdim=True))
        xq, sx = mk.quantize_fp8_rows(x)
        wq, sw = mk.quantize_fp8_rows(0.02 * torch.randn(Nn, K, generator=g, device=dev))
        flat, offs = mk.pack_scales([sw])
        swv = mk.unpack_scale_tensor(flat, offs, 0, (Nn,))
        times = timed_gemm(lambda: mk.fused_rmsnorm_linear_fp8(xq, wq, swv, x_scale=sx, out_dtype=torch.bfloat16))
        flop = 2.0 * M * Nn * K
        rows = 4
        xd = O.e4m3_bits_to_f32(xq[:rows].view(torch.uint8).cpu().numpy()) * f32(sx)[:rows, None]
        wd = O.e4m3_bits_to_f32(wq.view(torch.uint8).cpu().numpy())
        sws = f32(sw)
        ct = cpu_time(lambda: O.rmsnorm_linear_fp8(xd, wd, sws, None, 1e-6))
        # the FP8 peak, measured here: cuBLASLt's E4M3 GEMM at 8192^3 (no FP8
        # figure is in the pool's measured peaks)
        a8 = torch.randn(8192, 8192, generator=g, device=dev).to(torch.float8_e4m3fn)
        b8 = torch.randn(8192, 8192, generator=g, device=dev).to(torch.float8_e4m3fn)
        one_a, one_b = torch.ones((8192, 1), device=dev), torch.ones((1, 8192), device=dev)
        t8 = time_call(lambda: torch._scaled_mm(a8, b8.T, scale_a=one_a, scale_b=one_b, out_dtype=torch.bfloat16),
                       iters)
        fp8_peak = 2.0 * 8192 ** 3 / t8 / 1e12
        del a8, b8
        for v, t in times:
            emit("config3_fp8", M, "rows/s", t, "tensor", flop / t / 1e12, fp8_peak,
                 "cuBLASLt E4M3 GEMM 8192^3 measured in this run (torch._scaled_mm)", rows, ct,
                 {"dtype": "e4m3", "gemm_schedule": v,
                  "frac_of_2x_bf16_burst": flop / t / 1e12 / (2 * peaks["bf16"])})
        del x, xq, wq

    def sec_config4():
        # ---- config 4: paged tree attention
        B, Hq, Hkv, D, ps, ctx, P = C4["B"], C4["Hq"], C4["Hkv"], C4["D"], C4["ps"], C4["ctx"], C4["P"]
        tm = SpeculativeDraftTree(C4["depth"], C4["branches"], "tree").tree_mask.numpy()
        T = tm.shape[0]
        g = torch.Generator(device=dev).manual_seed(3)
        kp = torch.randn(P, B, Hkv, ps, D, generator=g, device=dev).to(torch.bfloat16)
        vp = torch.randn(P, B, Hkv, ps, D, generator=g, device=dev).to(torch.bfloat16)
        perm = torch.randperm(P, generator=torch.Generator().manual_seed(3))
        per = ctx // ps
        table = torch.stack([perm[b * per:(b + 1) * per].repeat_interleave(ps) for b in range(B)]).to(torch.int32)
        tdev = table.to(dev)
        q = torch.randn(B, T, Hq, D, generator=g, device=dev).to(torch.bfloat16)
        tk = torch.randn(B, Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
        tv = torch.randn(B, Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
        tmd = torch.tensor(tm, device=dev)
        t4 = time_call(lambda: mk.fused_tree_attention_paged(q, kp, vp, tdev, tk, tv, tmd), iters)
        pages0 = table[0].view(-1, ps)[:, 0].long()
        kps, vps = f32(kp[pages0.to(dev)][:, 0:1]), f32(vp[pages0.to(dev)][:, 0:1])
        tab0 = np.repeat(np.arange(pages0.numel(), dtype=np.int32), ps)[None, :]
        q0, tk0, tv0 = f32(q[0:1]), f32(tk[0:1]), f32(tv[0:1])
        ct = cpu_time(lambda: O.tree_attention_paged_fast(q0, kps, vps, tab0, ctx, ps, tk0, tv0, tm, 1 / math.sqrt(D)))
        emit("config4_tree_attention", B * T, "tree-node queries/s", t4, "hbm", C4_BYTES / t4 / 1e9, peaks["hbm"],
             "measured hbm_gbs", T, ct, {"tflops": C4_FLOP / t4 / 1e12})
        del kp, vp

    def sec_config5():
        # ---- config 5: fused_multi_verify, tp = 1
        Bv, S, K, V = C5["B"], C5["S"], C5["K"], C5["V"]
        g = torch.Generator(device=dev).manual_seed(4)
        hid = torch.randn(Bv, S, K, generator=g, device=dev).to(torch.bfloat16)
        lm = (0.02 * torch.randn(V, K, generator=g, device=dev)).to(torch.bfloat16)
        dr = torch.randint(0, V, (Bv, S - 1), device=dev, dtype=torch.int32)
        times = timed_gemm(lambda: mv.fused_multi_verify(hid, lm, dr))
        hs, lms, ds = f32(hid[:2]), f32(lm), dr[:2].cpu().numpy()
        ct = cpu_time(lambda: O.fused_multi_verify(hs, lms, None, ds))
        for v, t in times:
            emit("config5_verify", Bv * S, "verified candidates/s", t, "tensor", C5_FLOP / t / 1e12, peaks["bf16"],
                 "measured bf16_tflops (burst)", 2 * S, ct, {"gemm_schedule": v})
        del lm

    def sec_ref_bench_fusion_verify():
        # ---- the reference's own verify benchmark geometry (bench_optimizations.py:58-113):
        # B=32, S=5, K=256, V=8192 with bias, fp32 (the CUDA-core exact-fp32 GEMM) and bf16
        for dt in (torch.float32, torch.bfloat16):
            g = torch.Generator(device=dev).manual_seed(0)
            hr = torch.randn(32, 5, 256, generator=g, device=dev).to(dt)
            wr = torch.randn(8192, 256, generator=g, device=dev).to(dt)
            br = torch.randn(8192, generator=g, device=dev)
            dr_ = torch.randint(0, 8192, (32, 4), generator=g, device=dev, dtype=torch.int32)
            t = time_call(lambda: mv.fused_multi_verify(hr, wr, dr_, br), iters)
            hs_, ws2, bs_, ds_ = f32(hr[:4]), f32(wr), f32(br), dr_[:4].cpu().numpy()
            ct = cpu_time(lambda: O.fused_multi_verify(hs_, ws2, bs_, ds_))
            flop = 2.0 * 32 * 5 * 256 * 8192
            emit(f"ref_bench_fusion_verify_{'fp32' if dt == torch.float32 else 'bf16'}", 32 * 5,
                 "verified candidates/s", t, "tensor", flop / t / 1e12, peaks["bf16"],
                 "measured bf16_tflops (burst)", 4 * 5, ct,
                 {"dtype": "f32" if dt == torch.float32 else "bf16",
                  "note": "launch-bound size (0.34 GFLOP); the reference times it at bench_optimizations.py:58-113"})
            del hr, wr

    def sec_operators():
        # ---- operators around the path (not benchmark configs): one line each
        # tree attention -> RMSNorm -> linear: the reference's own bench geometry
        # (bench_memory.py:96, fp32) and a draft-head shape (bf16, D = hidden)
        for (Bm, Hm, Dm, Lm, Nm, dt) in ((64, 4, 64, 32, 256, torch.float32),
                                        (64, 1, 4096, 64, 32000, torch.bfloat16)):
            g = torch.Generator(device=dev).manual_seed(5)
            qm = torch.randn(Bm, Hm, Dm, generator=g, device=dev).to(dt)
            km = torch.randn(Bm, Hm, Lm, Dm, generator=g, device=dev).to(dt)
            vm = torch.randn(Bm, Hm, Lm, Dm, generator=g, device=dev).to(dt)
            mm = (torch.rand(Lm, generator=g, device=dev) > 0.3).float()
            rw = 1.0 + 0.1 * torch.randn(Dm, generator=g, device=dev)
            pw = (0.05 * torch.randn(Nm, Dm, generator=g, device=dev)).to(dt)
            t = time_call(lambda: mk.fused_tree_attn_rmsnorm_linear(qm, km, vm, mm, pw, rms_w=rw), iters)
            eb = qm.element_size()
            byts = (2 * Bm * Hm * Lm * Dm + 2 * Bm * Hm * Dm + Nm * Dm) * eb + Bm * Hm * Nm * eb
            flop = 2.0 * Bm * Hm * Nm * Dm
            qs, ks, vs, ws_, ms_, rws = f32(qm[:2]), f32(km[:2]), f32(vm[:2]), f32(pw), f32(mm), f32(rw)
            ct = cpu_time(lambda: O.tree_attn_rmsnorm_linear(qs, ks, vs, ms_, rws, ws_, None, None,
                                                             1 / math.sqrt(Dm), 1e-6))
            emit(f"tree_attn_rmsnorm_linear_B{Bm}_H{Hm}_D{Dm}_L{Lm}_N{Nm}", Bm * Hm, "rows/s", t, "hbm",
                 byts / t / 1e9, peaks["hbm"], "measured hbm_gbs", 2 * Hm, ct,
                 {"dtype": "f32" if dt == torch.float32 else "bf16", "tflops": flop / t / 1e12})
        # the reference's single-query operators (CUDA-core decode kernel): paged
        # attention over a config-4-sized context, tree attention over 512 keys
        Bd, Hd, Ld, Dd, psd = 16, 32, 4096, 128, 16
        g = torch.Generator(device=dev).manual_seed(8)
        Pd = Bd * Ld // psd // Bd + 1
        kpd = torch.randn(Pd, Bd, Hd, psd, Dd, generator=g, device=dev).to(torch.bfloat16)
        vpd = torch.randn(Pd, Bd, Hd, psd, Dd, generator=g, device=dev).to(torch.bfloat16)
        tab = torch.stack([torch.randperm(Pd - 1, generator=torch.Generator().manual_seed(b))[: Ld // psd]
                           .repeat_interleave(psd) for b in range(Bd)]).to(torch.int32)
        qd = torch.randn(Bd, Hd, Dd, generator=g, device=dev).to(torch.bfloat16)
        tabd = tab.to(dev)
        decode_variants = (1, 2) if args.compare else (N.decode_kernel(),)

        def timed_decode(fn):
            out = []
            for v in decode_variants:
                N.set_decode_kernel(v)
                out.append((v, time_call(fn, iters)))
            return out

        times = timed_decode(lambda: mk.fused_paged_attention(qd, kpd, vpd, tabd, psd))
        byts = 2 * Bd * Hd * Ld * Dd * 2 + 2 * Bd * Hd * Dd * 2
        kps_, vps_ = f32(kpd[:, 0:1]), f32(vpd[:, 0:1])
        q1, tab1 = f32(qd[0:1]), tab[0:1].numpy()
        ct = cpu_time(lambda: O.paged_attention(q1, kps_, vps_, tab1, psd, 1 / math.sqrt(Dd)))
        for v, t in times:
            emit("paged_attention_B16_H32_L4096_D128", Bd * Hd, "query rows/s", t, "hbm", byts / t / 1e9,
                 peaks["hbm"], "measured hbm_gbs", Hd, ct, {"decode_kernel": v})
        del kpd, vpd
        Lt = 512
        kt = torch.randn(Bd, Hd, Lt, Dd, generator=g, device=dev).to(torch.bfloat16)
        vt = torch.randn(Bd, Hd, Lt, Dd, generator=g, device=dev).to(torch.bfloat16)
        mt = (torch.rand(Lt, generator=g, device=dev) > 0.2).float()
        times = timed_decode(lambda: mk.fused_tree_attention(qd, kt, vt, mt))
        byts = 2 * Bd * Hd * Lt * Dd * 2 + 2 * Bd * Hd * Dd * 2
        kt1, vt1, mt1 = f32(kt[0:1]), f32(vt[0:1]), f32(mt)
        ct = cpu_time(lambda: O.tree_attention(q1, kt1, vt1, mt1, 1 / math.sqrt(Dd)))
        for v, t in times:
            emit("tree_attention_B16_H32_L512_D128", Bd * Hd, "query rows/s", t, "hbm", byts / t / 1e9,
                 peaks["hbm"], "measured hbm_gbs", Hd, ct, {"decode_kernel": v})
        del kt, vt
        # INT4 weights, decode-sized M (streamed GEMV)
        Mi, Ni, Ki, gi = 1, 14336, 4096, 128
        g = torch.Generator(device=dev).manual_seed(6)
        pk, sc = mk.quantize_int4(torch.randn(Ni, Ki, generator=g, device=dev), group=gi)
        xi = torch.randn(Mi, Ki, generator=g, device=dev).to(torch.bfloat16)
        t = time_call(lambda: mk.fused_int4_matmul(xi, pk, sc, Ki, gi), iters)
        byts = Ni * Ki / 2 + sc.numel() * 4 + Mi * Ki * 2 + Mi * Ni * 2
        pks, scs, xis = pk.cpu().numpy(), sc.cpu().numpy(), f32(xi)
        ct = cpu_time(lambda: O.int4_matmul(xis, pks, scs, Ki, gi))
        emit("int4_matmul_M1_N14336_K4096_g128", Mi, "rows/s", t, "hbm", byts / t / 1e9, peaks["hbm"],
             "measured hbm_gbs", Mi, ct, {"dtype": "int4 x bf16"})
        # FP8 KV-cache decode attention
        Ba, Ha, La, Da = 16, 32, 4096, 128
        g = torch.Generator(device=dev).manual_seed(7)
        qa = torch.randn(Ba, Ha, Da, generator=g, device=dev).to(torch.bfloat16)
        ka = torch.randn(Ba, Ha, La, Da, generator=g, device=dev).to(torch.float8_e4m3fn)
        va = torch.randn(Ba, Ha, La, Da, generator=g, device=dev).to(torch.float8_e4m3fn)
        ksa = torch.rand(Ha, generator=g, device=dev) + 0.5
        vsa = torch.rand(Ha, generator=g, device=dev) + 0.5
        t = time_call(lambda: mk.fused_causal_attention_fp8(qa, ka, va, ksa, vsa), iters)
        byts = 2 * Ba * Ha * La * Da + 2 * 2 * Ba * Ha * Da
        q0, k0 = f32(qa[:1]), O.e4m3_bits_to_f32(ka[:1].view(torch.uint8).cpu().numpy())
        v0 = O.e4m3_bits_to_f32(va[:1].view(torch.uint8).cpu().numpy())
        ks0, vs0 = f32(ksa), f32(vsa)
        ct = cpu_time(lambda: O.causal_attention_scaled(q0, k0, v0, ks0, vs0, 1 / math.sqrt(Da)))
        emit("causal_attention_fp8_B16_H32_L4096_D128", Ba * Ha, "query rows/s", t, "hbm", byts / t / 1e9,
             peaks["hbm"], "measured hbm_gbs", Ha, ct, {"dtype": "e4m3 kv, bf16 q"})

    sections = (("config1", sec_config1), ("config2", sec_config2), ("config3", sec_config3),
                ("config4", sec_config4), ("config5", sec_config5),
                ("ref_bench_fusion_verify", sec_ref_bench_fusion_verify), ("operators", sec_operators))
    only = [p for p in (args.sweep_only or "").split(",") if p]
    for name, section in sections:
        if not only or any(name.startswith(p) for p in only):
            section()
    assert N.device_status(dev) == 0


def run_profile_case(args):
    """--profile-case: one operator at its benchmark config, called --steps
    times with CUDA-event timing printed per call -- the small, fixed
    workload the ncu captures in profiles/ are taken on."""
    import torch

    import _mtp_native as N
    import mtp_fused_verify as mv
    import mtp_kernels as mk
    from mtp_draft_tree import SpeculativeDraftTree

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N.set_gemm_schedule(1 if args.gemm_schedule == "streamk" else 0)
    case = args.profile_case
    if case == "attention":
        B, Hq, Hkv, D, ps, ctx, P = C4["B"], C4["Hq"], C4["Hkv"], C4["D"], C4["ps"], C4["ctx"], C4["P"]
        tm = SpeculativeDraftTree(C4["depth"], C4["branches"], "tree").tree_mask.numpy()
        T = tm.shape[0]
        g = torch.Generator(device=dev).manual_seed(3)
        kp = torch.randn(P, B, Hkv, ps, D, generator=g, device=dev).to(torch.bfloat16)
        vp = torch.randn(P, B, Hkv, ps, D, generator=g, device=dev).to(torch.bfloat16)
        perm = torch.randperm(P, generator=torch.Generator().manual_seed(3))
        per = ctx // ps
        table = torch.stack([perm[b * per:(b + 1) * per].repeat_interleave(ps) for b in range(B)])
        table = table.to(torch.int32).to(dev)
        q = torch.randn(B, T, Hq, D, generator=g, device=dev).to(torch.bfloat16)
        tk = torch.randn(B, Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
        tv = torch.randn(B, Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
        tmask = torch.tensor(tm, device=dev)
        fn = lambda: mk.fused_tree_attention_paged(q, kp, vp, table, tk, tv, tmask)
    else:
        g = torch.Generator(device=dev).manual_seed(4)
        if case == "verify":
            B, S, K, V = C5["B"], C5["S"], C5["K"], C5["V"]
            hid = torch.randn(B, S, K, generator=g, device=dev).to(torch.bfloat16)
            w = (0.02 * torch.randn(V, K, generator=g, device=dev)).to(torch.bfloat16)
            d = torch.randint(0, V, (B, S - 1), device=dev, dtype=torch.int32)
            fn = lambda: mv.fused_multi_verify(hid, w, d)
        elif case in ("verify_rank8_weak", "verify_rank8_strong"):
            # one rank's shard GEMM of an 8-way vocab-parallel verify: every
            # rank's candidates (weak: 8 x 384 rows) against V/8 lm_head rows
            import _mtp_native as Nn
            S, K, V = C5["S"], C5["K"], C5["V"]
            rows = C5["B"] * S * (8 if case.endswith("weak") else 1)
            Vr = V // 8
            hid = torch.randn(rows, K, generator=g, device=dev).to(torch.bfloat16)
            w = (0.02 * torch.randn(Vr, K, generator=g, device=dev)).to(torch.bfloat16)
            keys = torch.full((rows,), -(2 ** 63), dtype=torch.int64, device=dev)
            fn = lambda: Nn.check(Nn.lib().mtp_verify_shard_keys(Nn.ptr(hid), Nn.DT_BF16, Nn.ptr(w), Nn.DT_BF16,
                                                                 None, 0, Nn.ptr(keys), rows, K, Vr, 0,
                                                                 Nn.stream_handle(dev)), "shard keys")
        elif case == "fp8":
            M, K, Nn_ = 1024, 8192, 28672
            x = torch.randn(M, K, generator=g, device=dev)
            x = x * (448.0 / x.abs().amax(dim=1, keepdim=True))
            xq, sx = mk.quantize_fp8_rows(x)
            wq, sw = mk.quantize_fp8_rows(0.02 * torch.randn(Nn_, K, generator=g, device=dev))
            del x
            fn = lambda: mk.fused_rmsnorm_linear_fp8(xq, wq, sw, x_scale=sx, out_dtype=torch.bfloat16)
        else:  # rms
            M, K, Nn = C2["M"], C2["K"], C2["N"]
            x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
            gam = 1 + 0.1 * torch.randn(K, generator=g, device=dev)
            w = (0.02 * torch.randn(Nn, K, generator=g, device=dev)).to(torch.bfloat16)
            fn = lambda: mk.fused_rmsnorm_linear(x, w, None, 1e-5, norm_weight=gam)
    for i in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        print(f"{case} call {i}: {e0.elapsed_time(e1) * 1000:.1f} us", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch every call eagerly")
    ap.add_argument("--graph", action="store_true", help="also replay captured graphs when n_gpus > 1")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--sweep", action="store_true", help="time every benchmark config on its own (1 GPU)")
    ap.add_argument("--nccl-max-ctas", type=int, default=8,
                    help="N > 1: cap on the CTAs of NCCL's kernels (0: NCCL's own choice)")
    ap.add_argument("--exchange", choices=["nccl", "p2p", "fused", "abi"], default="nccl",
                    help="vocab-parallel key exchange on N > 1: NCCL all-reduce, the peer-memory kernel, "
                         "the all-reduce fused into the shard GEMM, or the one-call C-ABI verify over the "
                         "library's own NCCL communicator")
    ap.add_argument("--e2e-eager", action="store_true",
                    help="1 GPU: report the eager end-to-end step only (by default the step is also captured "
                         "as one CUDA graph -- uploads, stages, read-back -- and the graph's rate is e2e.value)")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="weak",
                    help="N > 1: weak (default, the north star's layout) = configs 2 and 4 whole on every GPU, "
                         "the verify over every rank's sequences with the lm_head vocab-sharded; strong = the "
                         "1-GPU job split tensor-parallel")
    ap.add_argument("--profile-case", choices=["verify", "rms", "attention", "fp8", "verify_rank8_weak",
                                               "verify_rank8_strong"], default=None,
                    help="call one operator at its benchmark config --steps times (the workload of the ncu "
                         "captures in profiles/)")
    ap.add_argument("--sweep-only", default="",
                    help="with --sweep: comma-separated section names to run (config1..config5, "
                         "ref_bench_fusion_verify, operators; prefixes match), so sections can run in separate "
                         "processes")
    ap.add_argument("--compare", action="store_true",
                    help="with --sweep: every GEMM config under both schedules, the single-query lines under "
                         "both decode kernels")
    ap.add_argument("--gemm-schedule", choices=["dp", "streamk"], default="dp",
                    help="tensor-core GEMM schedule: whole tiles per CTA, or stream-K where it is faster")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.profile_case:
        run_profile_case(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.sweep:
        run_sweep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
