"""Randomised interleaving models of synchronisation protocols, used by
tests/test_protocol_models.py (test infrastructure, CPU only).

Each kernel role is a Python generator; the asynchronous engines (TMA copy
completions, the in-order tcgen05 pipe, NVLink stores in flight) are event
queues; a scheduler picks a random runnable step.  Every parity wait carries
the completion it is meant to observe, and buffers carry tags, so a wait
that passes early or a read of stale data raises Violation.
"""

import random


class Bar:
    """An mbarrier: `count` arrivals plus outstanding transaction bytes
    complete a phase; test(parity) is try_wait.parity."""

    def __init__(self, name, count):
        self.name, self.count, self.pending, self.done = name, count, count, 0
        self.tx = 0

    def arrive(self):
        self.pending -= 1
        self._maybe()

    def expect_tx(self, n):
        self.tx += n
        self.pending -= 1  # arrive.expect_tx
        self._maybe()

    def complete_tx(self, n):
        self.tx -= n
        self._maybe()

    def _maybe(self):
        if self.pending == 0 and self.tx == 0:
            self.done += 1
            self.pending = self.count

    def test(self, parity):
        return (self.done & 1) != parity


class Violation(Exception):
    pass

# --------------------------------------------------------------------------- #
# verify_exchange_chain_kernel (csrc/mtp_verify.cuh).  Each rank runs E calls.
# Call e: par = e & 1; push the local keys (tagged (rank, e)) into slot
# [par][rank] of every peer (stores land at any later time before this rank's
# fence completes); fence; release flag [par][rank] = e in every peer; wait
# until its own flags [par][p] >= e for all p; read slots [par][p] -- each must
# hold (p, e).
# --------------------------------------------------------------------------- #


def run_exchange(seed, W, E, parities=2):
    rnd = random.Random(seed)
    slots = [[[None] * W for _ in range(2)] for _ in range(W)]   # slots[owner][par][src]
    flags = [[[0] * W for _ in range(2)] for _ in range(W)]      # flags[owner][par][src]
    inflight = []  # pending stores: (owner, par, src, value)

    def rank_proc(r):
        for e in range(1, E + 1):
            par = e & 1 if parities == 2 else 0
            for p in range(W):
                inflight.append((p, par, r, (r, e)))
                yield "step"
            # fence: wait until this rank's stores have landed
            while any(x[2] == r for x in inflight):
                yield "blocked"
            for p in range(W):
                flags[p][par][r] = e
                yield "step"
            for p in range(W):
                while flags[r][par][p] < e:
                    yield "blocked"
            for p in range(W):
                v = slots[r][par][p]
                if v != (p, e):
                    raise Violation(f"rank {r} call {e} reads slot {p}: {v}")
                yield "step"

    procs = [rank_proc(r) for r in range(W)]
    alive = list(procs)
    steps = 0
    while alive or inflight:
        steps += 1
        if steps > 10 ** 6:
            raise Violation("no progress")
        opts = [("p", x) for x in alive] + ([("s", None)] if inflight else [])
        kind, x = rnd.choice(opts)
        if kind == "s":
            i = rnd.randrange(len(inflight))
            owner, par, src, val = inflight.pop(i)
            slots[owner][par][src] = val
        else:
            try:
                next(x)
            except StopIteration:
                alive.remove(x)




# --------------------------------------------------------------------------- #
# mtp_verify_shard_fused (csrc/mtp_gemm_sk.cuh, FIN_CHAIN_PEERS).  Each rank
# runs E calls of a GEMM with n_tiles tiles.  Call e: par = e & 1; every tile
# sends its key (here the value e * 1000 + rank * 10 + tile) to keys[par] of
# every rank by atomic max (remote ones land at any later time before the
# rank's fence); the last CTA fences, releases flag [par][rank] = e in every
# rank, waits for its own flags [par][p] >= e, reads keys[par] -- which must be
# the maximum over all ranks' keys of call e -- and puts it back to rest.
# --------------------------------------------------------------------------- #
def run_fused_exchange(seed, W, E, n_tiles=3, parities=2):
    rnd = random.Random(seed)
    REST = -1
    keys = [[REST] * 2 for _ in range(W)]                      # keys[owner][par] (one row)
    flags = [[[0] * W for _ in range(2)] for _ in range(W)]   # flags[owner][par][src]
    inflight = []  # (owner, par, src, value)

    def rank_proc(r):
        for e in range(1, E + 1):
            par = e & 1 if parities == 2 else 0
            for t in range(n_tiles):
                v = e * 1000 + r * 10 + t
                for p in range(W):
                    inflight.append((p, par, r, v))
                yield "step"
            while any(x[2] == r for x in inflight):   # fence before the ticket / flags
                yield "blocked"
            for p in range(W):
                flags[p][par][r] = e
                yield "step"
            for p in range(W):
                while flags[r][par][p] < e:
                    yield "blocked"
            want = e * 1000 + (W - 1) * 10 + (n_tiles - 1)
            if keys[r][par] != want:
                raise Violation(f"rank {r} call {e} decodes {keys[r][par]}, want {want}")
            keys[r][par] = REST
            yield "step"

    alive = [rank_proc(r) for r in range(W)]
    steps = 0
    while alive or inflight:
        steps += 1
        if steps > 10 ** 6:
            raise Violation("no progress")
        opts = [("p", x) for x in alive] + ([("s", None)] if inflight else [])
        kind, x = rnd.choice(opts)
        if kind == "s":
            owner, par, src, val = inflight.pop(rnd.randrange(len(inflight)))
            keys[owner][par] = max(keys[owner][par], val)
        else:
            try:
                next(x)
            except StopIteration:
                alive.remove(x)


# --------------------------------------------------------------------------- #
# gemm_tc_kernel (csrc/mtp_gemm_tc.cuh): TMA producer into a STAGES-deep ring,
# single-thread MMA issuer (in-order tcgen05 pipe, commits to empty[stage]
# and tfull[acc]) and the epilogue (waits tfull[acc], reads the accumulator,
# arrives tempty[acc] -- modelled as 4 warps).  acc_bufs = 2: accumulators
# double-buffered (128-row tiles); 1: one accumulator per tile (256-row
# tiles fill TMEM).  phase_rule "kernel" is the kernel's formula; "double"
# applies the double-buffer phases to a single buffer (a control that must
# be flagged).
# --------------------------------------------------------------------------- #


def run_gemm(seed, n_tiles, num_kb, stages, acc_bufs, phase_rule="kernel"):
    rnd = random.Random(seed)
    bars = {}

    def B(name, count=1):
        bars[name] = Bar(name, count)

    for s in range(stages):
        B(f"full{s}"), B(f"empty{s}")
    for a in range(2):
        B(f"tfull{a}"), B(f"tempty{a}", 4)

    smem = [None] * stages            # (tile, kb, consumed)
    acc = [None] * 2                  # (tile, K blocks accumulated) or ("free", tile drained)
    tma_q, pipe = [], []

    def acc_of(local):
        if acc_bufs == 2:
            return local & 1, (local >> 1) & 1
        if phase_rule == "double":
            return 0, (local >> 1) & 1
        return 0, local & 1

    def wait(bar, parity, want_done):
        while not bars[bar].test(parity):
            yield "blocked"
        if bars[bar].done < want_done:
            raise Violation(f"{bar}: parity {parity} passed with {bars[bar].done} completions, wanted {want_done}")

    def uses(local):
        """Completions of the accumulator buffer of tile `local` before it."""
        return local // 2 if acc_bufs == 2 else local

    def producer():
        it = 0
        for t in range(n_tiles):
            for kb in range(num_kb):
                s = it % stages
                yield from wait(f"empty{s}", ((it // stages) & 1) ^ 1, it // stages)
                if smem[s] is not None and not smem[s][2]:
                    raise Violation(f"producer overwrites stage {s} holding {smem[s]}")
                bars[f"full{s}"].expect_tx(1)
                tma_q.append((s, (t, kb)))
                it += 1
                yield "step"

    def mma():
        it = 0
        for t in range(n_tiles):
            a, ph = acc_of(t)
            yield from wait(f"tempty{a}", ph ^ 1, uses(t))
            for kb in range(num_kb):
                s = it % stages
                yield from wait(f"full{s}", (it // stages) & 1, it // stages + 1)
                pipe.append(("mma", s, a, t, kb))
                pipe.append(("commit", f"empty{s}"))
                it += 1
                yield "step"
            pipe.append(("commit", f"tfull{a}"))

    def epilogue(w):
        for t in range(n_tiles):
            a, ph = acc_of(t)
            yield from wait(f"tfull{a}", ph, uses(t) + 1)
            if acc[a] != (t, num_kb):
                raise Violation(f"epilogue w{w} tile {t} reads accumulator {a} = {acc[a]}")
            yield "step"
            if acc[a] != (t, num_kb):
                raise Violation(f"epilogue w{w} tile {t}: accumulator {a} changed to {acc[a]} while read")
            bars[f"tempty{a}"].arrive()
            yield "step"

    alive = [producer(), mma()] + [epilogue(w) for w in range(4)]
    steps = blocked = 0
    while alive or tma_q or pipe:
        steps += 1
        if steps > 400000:
            raise Violation("no progress (livelock)")
        choices = [("role", r) for r in alive] + ([("tma", None)] if tma_q else []) + ([("pipe", None)] if pipe else [])
        kind, what = rnd.choice(choices)
        if kind == "role":
            try:
                st = next(what)
            except StopIteration:
                alive.remove(what)
                continue
            if st == "blocked":
                blocked += 1
                if blocked > 5000 and not tma_q and not pipe:
                    raise Violation("deadlock: " + ", ".join(f"{b.name}:{b.done}" for b in bars.values()))
            else:
                blocked = 0
        elif kind == "tma":
            s, item = tma_q.pop(rnd.randrange(len(tma_q)))
            smem[s] = (item[0], item[1], False)
            bars[f"full{s}"].complete_tx(1)
            blocked = 0
        else:
            op = pipe.pop(0)
            blocked = 0
            if op[0] == "commit":
                if op[1].startswith("empty"):
                    s = int(op[1][5:])
                    smem[s] = (smem[s][0], smem[s][1], True)
                bars[op[1]].arrive()
            else:
                _, s, a, t, kb = op
                if smem[s] is None or smem[s][:2] != (t, kb):
                    raise Violation(f"MMA tile {t} kb {kb} reads stage {s} holding {smem[s]}")
                if kb == 0:
                    if acc[a] is not None and acc[a][1] != num_kb:
                        raise Violation(f"tile {t} starts accumulator {a} over unfinished {acc[a]}")
                    acc[a] = (t, 1)
                else:
                    if acc[a] != (t, kb):
                        raise Violation(f"MMA tile {t} kb {kb} accumulates into {acc[a]}")
                    acc[a] = (t, kb + 1)
    return steps
