"""Randomised interleaving models of two synchronisation protocols, used by
tests/test_protocol_models.py (test infrastructure, CPU only).

Each kernel role is a Python generator; the asynchronous engines (TMA copy
completions, the in-order tcgen05 pipe, NVLink stores in flight) are event
queues; a scheduler picks a random runnable step.  Every parity wait carries
the completion it is meant to observe, and buffers carry tags, so a wait
that passes early or a read of stale data raises Violation.
"""

import random

# --------------------------------------------------------------------------- #
# tree_attention_tc2_kernel (csrc/mtp_attention_tc2.cuh): TMA producer, MMA
# issuer and softmax warps over the K/V ring, the two score buffers per query
# tile (S/P tags) and the O accumulator (set of chunks it holds)
# --------------------------------------------------------------------------- #


class Bar:
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


def run_attn2(seed, n_iter, n_tiles, kNumBuf=9, p_rescale=0.3, final_wait="o_done"):
    rnd = random.Random(seed)
    bars = {}

    def B(name, count=1):
        if name not in bars:
            bars[name] = Bar(name, count)
        return bars[name]

    for i in range(kNumBuf):
        B(f"buf_full{i}"), B(f"buf_empty{i}")
    for t in range(n_tiles):
        for sb in range(2):
            B(f"s_full{t}{sb}"), B(f"p_full{t}{sb}", 4)
        B(f"pv_done{t}"), B(f"o_done{t}")
    B("q_full")

    # state with tags
    smem = [None] * kNumBuf          # item loaded in ring slot
    S = {(t, sb): None for t in range(n_tiles) for sb in range(2)}  # ('S', c) or ('P', c)
    O = {t: set() for t in range(n_tiles)}   # chunks accumulated
    O_scaled_at = {t: [] for t in range(n_tiles)}
    tma_q = []     # pending TMA completions: (slot, item)
    pipe = []      # in-order tcgen05 ops: ('S', t, sb, item, c) | ('PV', t, sb, item, c) | ('commit', bar)
    results = {}

    def wait(bar, parity, want_done):
        """yield until bar passes parity; check it passed for the intended completion."""
        while not bars[bar].test(parity):
            yield "blocked"
        if bars[bar].done < want_done:
            raise Violation(f"{bar}: parity {parity} passed with {bars[bar].done} completions, wanted {want_done}")

    # ------------------------------------------------------------ producer
    def producer():
        # Q
        bars["q_full"].expect_tx(1)
        tma_q.append(("Q", None))
        item = 0
        for c in range(n_iter):
            for kv in range(2):
                buf = item % kNumBuf
                yield from wait(f"buf_empty{buf}", ((item // kNumBuf) & 1) ^ 1, item // kNumBuf)
                if smem[buf] is not None and smem[buf][1] is False:
                    raise Violation(f"producer overwrites slot {buf} holding unconsumed item {smem[buf]}")
                bars[f"buf_full{buf}"].expect_tx(1)
                tma_q.append((buf, item))
                item += 1
                yield "step"

    # ------------------------------------------------------------ MMA issuer
    def mma():
        yield from wait("q_full", 0, 1)

        def wait_item(it):
            yield from wait(f"buf_full{it % kNumBuf}", (it // kNumBuf) & 1, it // kNumBuf + 1)

        for j in range(min(2, n_iter)):
            yield from wait_item(2 * j)
            for t in range(n_tiles):
                pipe.append(("S", t, j, 2 * j, j))
                pipe.append(("commit", f"s_full{t}{j}"))
            pipe.append(("consumed", 2 * j))
            pipe.append(("commit", f"buf_empty{(2 * j) % kNumBuf}"))
            yield "step"
        for i in range(n_iter):
            sb = i & 1
            vitem, knext = 2 * i + 1, 2 * i + 4
            for t in range(n_tiles):
                yield from wait(f"p_full{t}{sb}", (i >> 1) & 1, (i >> 1) + 1)
                if t == 0:
                    yield from wait_item(vitem)
                pipe.append(("PV", t, sb, vitem, i))
                pipe.append(("commit", f"pv_done{t}"))
                if i == n_iter - 1:
                    pipe.append(("commit", f"o_done{t}"))
                if t == n_tiles - 1:
                    pipe.append(("consumed", vitem))
                    pipe.append(("commit", f"buf_empty{vitem % kNumBuf}"))
                if i + 2 < n_iter:
                    if t == 0:
                        yield from wait_item(knext)
                    pipe.append(("S", t, sb, knext, i + 2))
                    pipe.append(("commit", f"s_full{t}{sb}"))
                    if t == n_tiles - 1:
                        pipe.append(("consumed", knext))
                        pipe.append(("commit", f"buf_empty{knext % kNumBuf}"))
                yield "step"

    # ------------------------------------------------------------ softmax warp
    def softmax(t, w):
        for i in range(n_iter):
            sb = i & 1
            yield from wait(f"s_full{t}{sb}", (i >> 1) & 1, (i >> 1) + 1)
            if S[(t, sb)] != ("S", i):
                raise Violation(f"softmax t{t} w{w} chunk {i} reads {S[(t, sb)]}")
            yield "step"  # compute
            if i > 0 and rnd.random() < p_rescale:
                yield from wait(f"pv_done{t}", (i - 1) & 1, i)
                if O[t] != set(range(i)):
                    raise Violation(f"rescale t{t} chunk {i}: O holds {sorted(O[t])}")
                yield "step"
                if O[t] != set(range(i)):
                    raise Violation(f"rescale t{t} chunk {i} (store): O holds {sorted(O[t])}")
            # write P (one warp's quarter: model as the whole buffer once all 4 warps wrote)
            key = (t, sb, i)
            results.setdefault(key, 0)
            results[key] += 1
            if results[key] == 4:
                if S[(t, sb)] != ("S", i):
                    raise Violation(f"P write t{t} chunk {i} over {S[(t, sb)]}")
                S[(t, sb)] = ("P", i)
            bars[f"p_full{t}{sb}"].arrive()
            yield "step"
        if final_wait == "o_done":
            yield from wait(f"o_done{t}", 0, 1)
        else:  # control: a parity wait on the per-PV barrier
            yield from wait(f"pv_done{t}", (n_iter - 1) & 1, n_iter)
        if O[t] != set(range(n_iter)):
            raise Violation(f"final O t{t} holds {sorted(O[t])}")

    roles = [producer(), mma()] + [softmax(t, w) for t in range(n_tiles) for w in range(4)]
    alive = list(roles)

    def engine_steps():
        acts = []
        if tma_q:
            acts.append("tma")
        if pipe:
            acts.append("pipe")
        return acts

    steps = 0
    blocked_rounds = 0
    while alive or tma_q or pipe:
        steps += 1
        if steps > 200000:
            raise Violation("no progress (livelock)")
        choices = [("role", r) for r in alive] + [("eng", e) for e in engine_steps()]
        kind, what = rnd.choice(choices)
        if kind == "role":
            try:
                st = next(what)
            except StopIteration:
                alive.remove(what)
                blocked_rounds = 0
                continue
            if st == "blocked":
                blocked_rounds += 1
                if blocked_rounds > 5000 and not tma_q and not pipe:
                    raise Violation("deadlock: " + ", ".join(f"{b.name}:{b.done}" for b in bars.values()))
            else:
                blocked_rounds = 0
        elif what == "tma":
            k = rnd.randrange(len(tma_q))
            slot, item = tma_q.pop(k)
            if slot == "Q":
                bars["q_full"].complete_tx(1)
            else:
                smem[slot] = (item, False)
                bars[f"buf_full{slot}"].complete_tx(1)
            blocked_rounds = 0
        else:
            op = pipe.pop(0)
            blocked_rounds = 0
            if op[0] == "commit":
                bars[op[1]].arrive()
            elif op[0] == "consumed":
                it = op[1]
                slot = it % kNumBuf
                if smem[slot] is None or smem[slot][0] != it:
                    raise Violation(f"consumed item {it} but slot holds {smem[slot]}")
                smem[slot] = (it, True)
            else:
                kindop, t, sb, item, c = op
                slot = item % kNumBuf
                if smem[slot] is None or smem[slot][0] != item:
                    raise Violation(f"{kindop} t{t} chunk {c} reads slot {slot} holding {smem[slot]}, want {item}")
                if kindop == "S":
                    if S[(t, sb)] is not None and S[(t, sb)] != ("P", c - 2):
                        raise Violation(f"S t{t} chunk {c} overwrites {S[(t, sb)]}")
                    S[(t, sb)] = ("S", c)
                else:
                    if S[(t, sb)] != ("P", c):
                        raise Violation(f"PV t{t} chunk {c} reads {S[(t, sb)]}")
                    O[t].add(c)
    return steps




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
