"""Models of the synchronisation protocols of the cooperating kernels (CPU).

Each model restates, in Python, the control flow of one kernel's cooperating parts --
which unit, stage or tile each part works on, when it issues a copy or a tensor-core
operation, what it waits for and what it signals -- and runs it with the asynchronous
completions (TMA copies, tensor-core operations in issue order) and the parts
interleaved at random.  It checks what the kernel relies on: no deadlock, no mbarrier
waiter two phases behind (the hardware only compares parities), and every buffer read
for the tile it holds, never overwritten before it was read.  The models follow the
CUDA sources by hand and change with them:

* csrc/gemv_dynamic.cu: units fetched from a counter one unit ahead, each warp's
  cp.async ring running across units, waits on the groups committed after the stage
  consumed, the counter reset by the last CTA;
* csrc/attention_tc.cu: Q / K / V loads, S = Q K^T into two TMEM buffers, P V into the
  output accumulator, the four softmax warps (max, rescale, P);
* csrc/gemm_tc_persistent.cu: the TMA ring across tiles and the two TMEM accumulators
  shared by the MMA thread and the four epilogue warps;
* csrc/gemv_attention.cuh (decode attention at the end of attn_in): each CTA's per-head
  count of finished q / k / v tasks (fa_tasks_for_head against a brute-force
  classification of the tasks), one atomic add per head, the head computed by the CTA
  whose add completes it, the counter reset for the next call;
* csrc/decode_layer.cu (one launch per decode layer): the grid barrier between the four
  phases (arrival count reset by the last arrival before it moves the generation) over
  consecutive launches that start early (programmatic dependent launch) and wait for the
  previous launch before touching the barrier; and its all-reduce form over 2-8 ranks at
  different speeds (two fused all-reduces per launch between the barriers);
* csrc/gemv_allreduce.cuh (fused projection + all-reduce, one process per GPU): every
  CTA's partial into every rank's exchange row of slot epoch & 1, the last CTA's flags,
  the wait for every rank's flag, the rank-order read, the tickets and the epoch counter,
  over consecutive calls on ranks running at different speeds (memory sequentially
  consistent; the kernel's fences and release / acquire accesses provide that order);
* csrc/p2p.cu, allreduce_ll_kernel (the low-latency all-reduce): every thread stores each
  of its words, tagged with the call's epoch (one 64-bit store: tag and data land
  together), into row `rank` of slot epoch & 1 of every rank's buffer, then polls its own
  rows until each word carries the epoch; the epoch counter advances when every thread is
  done, and a rank's next call starts only after its previous call completed (the
  programmatic-dependent-launch wait), which is what makes two slots enough.

Removing any wait the data flow needs makes one of these checks fail.
"""

from __future__ import annotations

import random

import pytest

W = 8  # warps


def share(n, w):
    return (w * n) // W, ((w + 1) * n) // W


def simulate(ntasks, ms, S, UT, grid, seed):
    rnd = random.Random(seed)
    n_units = -(-ntasks // UT)
    assert grid <= n_units
    ctr = [0, 0]
    unit_tasks = lambda u: min(UT, ntasks - u * UT)
    done = {}  # (task, piece) -> count

    def fetch():
        v = ctr[0]
        ctr[0] += 1
        return v + grid if 0 <= v < n_units - grid else -1

    # Each CTA simulated as a generator yielding at barriers; CTA interleaving random.
    def cta(b):
        s_unit = [None, None, None]
        tag = [None, None, None]
        s_unit[0], tag[0] = b, 0
        warps = []
        for w in range(W):
            st = dict(ik=0, iu=b, issued=0, consumed=0, groups=[], slots=[None] * S)
            st['is'], st['ihi'] = share(unit_tasks(b) * ms, w)
            warps.append(st)

        def issue_more(w, consumed, known_k):
            st = warps[w]
            while st['issued'] - consumed < S and st['iu'] >= 0:
                if st['is'] == st['ihi']:
                    if st['ik'] + 1 > known_k:
                        break
                    st['ik'] += 1
                    assert tag[st['ik'] % 3] == st['ik'], ("stale unit slot", st['ik'], tag)
                    st['iu'] = s_unit[st['ik'] % 3]
                    if st['iu'] < 0:
                        break
                    st['is'], st['ihi'] = share(unit_tasks(st['iu']) * ms, w)
                    continue
                slot = st['issued'] % S
                # the slot being overwritten must have been consumed
                old = st['slots'][slot]
                assert old is None or old[2] < consumed or old[2] == -1 or old[3], ("overwrite unconsumed", old)
                tl = st['is'] // ms
                st['slots'][slot] = (st['iu'], st['is'], st['issued'], False)
                st['groups'].append(st['issued'])
                st['is'] += 1
                st['issued'] += 1

        for w in range(W):
            issue_more(w, 0, 0)
        yield  # pdl wait / activation staging barrier
        s_unit[1], tag[1] = fetch(), 1
        yield  # __syncthreads before loop
        k = 0
        while True:
            u = s_unit[k % 3]
            assert tag[k % 3] == k, ("stale unit at loop top", k, tag)
            if u < 0:
                break
            for w in range(W):
                st = warps[w]
                lo, hi = share(unit_tasks(u) * ms, w)
                if st['ik'] < k:
                    assert st['issued'] == st['consumed'], "reset with stages in flight"
                    st['ik'], st['iu'], st['is'], st['ihi'] = k, u, lo, hi
                for s_ in range(lo, hi):
                    issue_more(w, st['consumed'], k + 1)
                    pending_allowed = st['issued'] - 1 - st['consumed']
                    assert 0 <= pending_allowed <= 7
                    slot = st['consumed'] % S
                    ent = st['slots'][slot]
                    assert ent is not None and ent[0] == u and ent[1] == s_ and ent[2] == st['consumed'], (ent, u, s_, st['consumed'])
                    st['slots'][slot] = (ent[0], ent[1], ent[2], True)
                    tl = s_ // ms
                    key = (u * UT + tl, s_ - tl * ms)
                    done[key] = done.get(key, 0) + 1
                    st['consumed'] += 1
            yield  # first __syncthreads of the unit
            assert tag[(k + 1) % 3] == k + 1
            s_unit[(k + 2) % 3] = -1 if s_unit[(k + 1) % 3] < 0 else fetch()
            tag[(k + 2) % 3] = k + 2
            yield  # second __syncthreads
            k += 1
        for w in range(W):
            assert warps[w]['issued'] == warps[w]['consumed'], ("leftover issued", w, warps[w])
        ctr[1] += 1
        if ctr[1] == grid:
            ctr[0] = ctr[1] = 0

    gens = [cta(b) for b in range(grid)]
    live = list(range(grid))
    while live:
        i = rnd.choice(live)
        try:
            next(gens[i])
        except StopIteration:
            live.remove(i)
    assert ctr == [0, 0], ctr
    for t in range(ntasks):
        for p in range(ms):
            assert done.get((t, p)) == 1, ("missing/dup", t, p, done.get((t, p)))
    assert len(done) == ntasks * ms


class Deadlock(Exception):
    pass


EVENTS = [0]


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.arrived, self.tx, self.done = name, count, 0, 0, 0

    def arrive(self, tx=0):
        EVENTS[0] += 1
        self.arrived += 1
        self.tx += tx
        self._check()

    def complete_tx(self, n):
        EVENTS[0] += 1
        self.tx -= n
        assert self.tx >= 0, (self.name, "tx underflow")
        self._check()

    def _check(self):
        if self.arrived == self.count and self.tx == 0:
            self.done += 1
            self.arrived = 0

    def ready(self, k):
        """waiting for the k-th completion (parity k & 1)"""
        if self.done >= k + 2:
            raise AssertionError(f"{self.name}: waiter for completion {k} is two phases behind ({self.done})")
        return self.done == k + 1


class Sim:
    def __init__(self, seed):
        self.rnd = random.Random(seed)
        self.pending = []  # async ops: (callable)
        self.mma_q = []    # in-order tensor ops of the issuing thread: (callable) ; commits appended as markers

    def run(self, roles, max_steps=10 ** 6):
        live = list(roles)
        steps = 0
        while live or self.pending or self.mma_q:
            steps += 1
            assert steps < max_steps
            choices = []
            if live:
                choices.append("role")
            if self.pending:
                choices.append("async")
            if self.mma_q:
                choices.append("mma")
            c = self.rnd.choice(choices)
            if c == "async":
                op = self.pending.pop(self.rnd.randrange(len(self.pending)))
                op()
            elif c == "mma":
                op = self.mma_q.pop(0)  # tensor ops complete in issue order
                op()
            else:
                progressed = False
                before = (EVENTS[0], len(self.pending), len(self.mma_q))
                order = list(live)
                self.rnd.shuffle(order)
                for r in order:
                    try:
                        res = next(r)
                    except StopIteration:
                        live.remove(r)
                        progressed = True
                        break
                    if res != "blocked":
                        progressed = True
                        break
                if (before != (EVENTS[0], len(self.pending), len(self.mma_q))):
                    progressed = True
                if not progressed and not self.pending and not self.mma_q:
                    raise Deadlock(f"all roles blocked: {WAITING}")


WAITING = {}


def wait(bar, k, who="?"):
    while not bar.ready(k):
        WAITING[who] = (bar.name, k, bar.done, bar.arrived)
        yield "blocked"
    WAITING.pop(who, None)


# --------------------------------------------------------------------------------------
# attention_tc.cu
# --------------------------------------------------------------------------------------
def sim_attention(n, seed, wait_for_p=True):
    sim = Sim(seed)
    q_full = Bar("q_full", 1)
    kv_full = [Bar(f"kv_full{s}", 1) for s in range(2)]
    kv_empty = [Bar(f"kv_empty{s}", 1) for s in range(2)]
    s_full = [Bar(f"s_full{s}", 1) for s in range(2)]
    s_free = [Bar(f"s_free{s}", 4) for s in range(2)]
    p_full, o_full, o_free = Bar("p_full", 4), Bar("o_full", 1), Bar("o_free", 4)
    # buffer contents: which tile each holds
    kv = [None, None]      # stage -> tile loaded
    S = [None, None]       # TMEM S buffer -> tile
    P = [None]             # smem P -> tile
    O = {"tiles": [], "rescaled_for": -1}  # tiles accumulated
    log = []

    def producer():
        sim.pending.append(lambda: q_full.complete_tx(1))
        q_full.arrive(tx=1)
        for j in range(n):
            s = j & 1
            if j >= 2:
                yield from wait(kv_empty[s], (j >> 1) - 1, "producer")
            kv_full[s].arrive(tx=1)

            def land(s=s, j=j):
                kv[s] = j
                kv_full[s].complete_tx(1)
            sim.pending.append(land)
            yield "ok"

    def mma():
        yield from wait(q_full, 0, "mma")
        for j in range(n + 1):
            if j < n:
                s = j & 1
                yield from wait(kv_full[s], j >> 1, "mma")
                if j >= 2:
                    yield from wait(s_free[s], (j >> 1) - 1, "mma")
                assert kv[s] == j, ("S reads wrong K", kv[s], j)

                def s_mma(s=s, j=j):
                    assert kv[s] == j, ("K overwritten before S MMA ran", kv[s], j)
                    S[s] = j
                sim.mma_q.append(s_mma)
                sim.mma_q.append(lambda s=s: s_full[s].arrive())
            if j >= 1:
                i = j - 1
                s = i & 1
                if wait_for_p:
                    yield from wait(p_full, i, "mma")
                if i >= 1:
                    yield from wait(o_free, i - 1, "mma")

                def pv(s=s, i=i):
                    assert P[0] == i, ("PV reads wrong P", P[0], i)
                    assert kv[s] == i, ("V overwritten before PV ran", kv[s], i)
                    assert O["rescaled_for"] == i or i == 0, ("O not rescaled before PV", O, i)
                    O["tiles"].append(i)
                sim.mma_q.append(pv)
                sim.mma_q.append(lambda: o_full.arrive())
                sim.mma_q.append(lambda s=s: kv_empty[s].arrive())
            yield "ok"

    def softmax(w):
        for j in range(n):
            s = j & 1
            yield from wait(s_full[s], j >> 1, f"sm{w}")
            assert S[s] == j, ("softmax reads wrong S", S[s], j)
            yield "ok"  # pass 1
            if j >= 1:
                yield from wait(o_full, j - 1, f"sm{w}")
                assert O["tiles"][-1] == j - 1
                if w == 0:
                    O["rescaled_for"] = j  # (every warp rescales its own rows)
                o_free.arrive()
            assert S[s] == j, ("S overwritten during pass 2", S[s], j)
            if w == 0:
                P[0] = j
            yield "ok"
            s_free[s].arrive()
            p_full.arrive()
        yield from wait(o_full, n - 1, f"sm{w}")
        assert O["tiles"] == list(range(n)), O

    sim.run([producer(), mma()] + [softmax(w) for w in range(4)])


# --------------------------------------------------------------------------------------
# gemm_tc_persistent.cu
# --------------------------------------------------------------------------------------
def sim_persistent(tiles, nkb, stages, seed):
    sim = Sim(seed)
    full = [Bar(f"full{s}", 1) for s in range(stages)]
    empty = [Bar(f"empty{s}", 1) for s in range(stages)]
    acc_full = [Bar(f"acc_full{b}", 1) for b in range(2)]
    acc_empty = [Bar(f"acc_empty{b}", 4) for b in range(2)]
    stage = [None] * stages
    acc = [None, None]
    out = []

    def producer():
        g = 0
        for t in range(tiles):
            for kb in range(nkb):
                s = g % stages
                if g >= stages:
                    yield from wait(empty[s], g // stages - 1)
                full[s].arrive(tx=1)

                def land(s=s, t=t, kb=kb):
                    stage[s] = (t, kb)
                    full[s].complete_tx(1)
                sim.pending.append(land)
                g += 1
                yield "ok"

    def mma():
        g = 0
        for i in range(tiles):
            b = i & 1
            if i >= 2:
                yield from wait(acc_empty[b], i // 2 - 1)
            for kb in range(nkb):
                s = g % stages
                yield from wait(full[s], g // stages)

                def op(s=s, i=i, kb=kb, b=b):
                    assert stage[s] == (i, kb), ("MMA reads wrong stage", stage[s], (i, kb))
                    if kb == 0:
                        assert acc[b] is None or acc[b][1] == "read", ("accumulator overwritten unread", acc[b])
                        acc[b] = (i, "partial")
                sim.mma_q.append(op)
                sim.mma_q.append(lambda s=s: empty[s].arrive())
                g += 1
                yield "ok"

            def fin(b=b, i=i):
                acc[b] = (i, "full")
            sim.mma_q.append(fin)
            sim.mma_q.append(lambda b=b: acc_full[b].arrive())

    def epilogue(w):
        for i in range(tiles):
            b = i & 1
            yield from wait(acc_full[b], i // 2)
            assert acc[b] == (i, "full") or acc[b] == (i, "read"), ("epilogue reads wrong tile", acc[b], i)
            if w == 3:
                acc[b] = (i, "read")
                out.append(i)
            yield "ok"
            acc_empty[b].arrive()

    sim.run([producer(), mma()] + [epilogue(w) for w in range(4)])
    assert out == list(range(tiles))



# --------------------------------------------------------------------------------------
# gemv_allreduce.cuh
# --------------------------------------------------------------------------------------


def simulate_allreduce(nranks, ctas, calls, seed, skew=True):
    rnd = random.Random(seed)
    # per rank device state
    counter = [0] * nranks
    tickets = [[0, 0] for _ in range(nranks)]
    flags = [[[0] * nranks for _ in range(2)] for _ in range(nranks)]     # flags[rank][slot][src]
    data = [[[None] * nranks for _ in range(2)] for _ in range(nranks)]   # data[rank][slot][src] = (call, src)
    results = [[None] * calls for _ in range(nranks)]

    def cta(rank, call, cid, state):
        # epoch read after pdl_wait: the previous call on this rank is complete
        epoch = counter[rank] + 1
        assert epoch == call + 1, (rank, call, epoch)
        slot = epoch & 1
        yield
        # ar_push: this CTA's share of the partial to every rank's buffer (row `rank`)
        for q in range(nranks):
            data[q][slot][rank] = (call, rank)
            yield
        # ticket 0; the last CTA raises this rank's flag everywhere
        tickets[rank][0] += 1
        if tickets[rank][0] == ctas:
            for q in range(nranks):
                flags[q][slot][rank] = epoch
                yield
        yield
        # wait for every rank's flag (bounded in the kernel; here: until set)
        for r in range(nranks):
            spins = 0
            while flags[rank][slot][r] != epoch:
                assert flags[rank][slot][r] < epoch, ("flag ahead", rank, slot, r, flags[rank][slot][r], epoch)
                spins += 1
                assert spins < 10 ** 6
                yield "spin"
        # read the rows in rank order
        got = []
        for r in range(nranks):
            got.append(data[rank][slot][r])
            yield
        assert got == [(call, r) for r in range(nranks)], ("stale or overwritten rows", rank, call, got)
        state["got"] = got
        tickets[rank][1] += 1
        if tickets[rank][1] == ctas:
            tickets[rank][0] = tickets[rank][1] = 0
            counter[rank] = epoch
        yield

    # each rank runs its calls in order; a call's CTAs start when the previous call is complete
    rank_call = [0] * nranks
    running = {r: [] for r in range(nranks)}
    done_ctas = {r: 0 for r in range(nranks)}

    def start(r):
        c = rank_call[r]
        running[r] = [cta(r, c, i, {}) for i in range(ctas)]
        done_ctas[r] = 0

    for r in range(nranks):
        start(r)
    steps = 0
    while any(rank_call[r] < calls for r in range(nranks)):
        steps += 1
        assert steps < 10 ** 7, "no progress"
        live = [(r, g) for r in range(nranks) for g in running[r]]
        r, g = rnd.choice(live)
        if skew and rnd.random() < 0.5 and r == 0:
            continue  # rank 0 slower
        try:
            next(g)
        except StopIteration:
            running[r].remove(g)
            done_ctas[r] += 1
            if done_ctas[r] == ctas:
                rank_call[r] += 1
                if rank_call[r] < calls:
                    start(r)
    assert all(t == [0, 0] for t in tickets)
    assert counter == [calls] * nranks


def simulate_allreduce_ll(nranks, threads, words, calls, seed, pdl_wait=True):
    """allreduce_ll_kernel over `calls` consecutive calls; returns nothing, raises on a
    word read after it was overwritten, a wrong value, or no progress."""
    rnd = random.Random(seed)
    counter = [0] * nranks
    # buf[rank][slot][src][word] = (epoch, value); the zero-filled buffer has epoch 0
    buf = [[[[(0, None)] * words for _ in range(nranks)] for _ in range(2)] for _ in range(nranks)]
    done_threads = [[0] * calls for _ in range(nranks)]

    def thread(rank, call, tid):
        epoch = counter[rank] + 1 if pdl_wait else call + 1
        assert epoch == call + 1, (rank, call, epoch)
        slot = epoch & 1
        mine = range(tid, words, threads)
        yield
        for i in mine:  # 1. push: one tagged 64-bit store per word and peer
            for p in range(nranks):
                buf[p][slot][rank][i] = (epoch, (call, rank, i))
                yield
        for i in mine:  # 2. poll each rank's word, sum in rank order
            for q in range(nranks):
                spins = 0
                while buf[rank][slot][q][i][0] != epoch:
                    tag = buf[rank][slot][q][i][0]
                    assert tag < epoch, ("overwritten before it was read", rank, call, q, i, tag)
                    spins += 1
                    assert spins < 10 ** 6, "no progress"
                    yield "spin"
                assert buf[rank][slot][q][i][1] == (call, q, i), ("wrong word", rank, call, q, i)
                yield
        done_threads[rank][call] += 1
        if done_threads[rank][call] == threads:  # after __syncthreads: thread 0 moves the counter
            counter[rank] = epoch
        yield

    rank_call = [0] * nranks
    running = {r: [] for r in range(nranks)}
    for r in range(nranks):
        running[r] = [thread(r, 0, t) for t in range(threads)]
    steps = 0
    while any(running[r] for r in range(nranks)):
        steps += 1
        assert steps < 10 ** 7, "no progress"
        live = [(r, g) for r in range(nranks) for g in running[r]]
        r, g = rnd.choice(live)
        if r == 0 and rnd.random() < 0.6:
            continue  # rank 0 slower
        try:
            next(g)
        except StopIteration:
            running[r].remove(g)
        # the next call of rank r: after its previous call completed (pdl_wait), or, in the
        # variant without that wait, as soon as the previous call's threads have all started
        c = rank_call[r]
        if c + 1 < calls and (not running[r] if pdl_wait else rnd.random() < 0.3):
            rank_call[r] = c + 1
            running[r] = running[r] + [thread(r, c + 1, t) for t in range(threads)]
    assert counter == [calls] * nranks


@pytest.mark.parametrize("seed", range(80))
def test_low_latency_allreduce_protocol(seed):
    r = random.Random(seed)
    simulate_allreduce_ll(r.choice([2, 3, 4, 8]), r.choice([1, 2, 4]), r.choice([1, 3, 8]), r.randint(1, 7), seed)


def test_the_ll_model_needs_the_previous_call_complete():
    """Without the wait for the rank's previous call, a fast rank's call e+2 overwrites a
    word of slot e & 1 that a slow rank's call e has not read yet, in some interleaving."""
    caught = 0
    for seed in range(60):
        try:
            simulate_allreduce_ll(2, 2, 4, 6, seed, pdl_wait=False)
        except AssertionError:
            caught += 1
    assert caught > 0


@pytest.mark.parametrize("seed", range(40))
def test_dynamic_gemv_schedule(seed):
    r = random.Random(seed)
    ntasks = r.choice([7, 40, 300, 512, 4096, 1376])
    ms = r.choice([1, 2, 8, 22, 43])
    S = r.choice([5, 8])
    gr = r.choice([1, 3, 148, 296, 444])
    ut = max(ntasks // (gr * 4), -(-8 // ms))
    gr = min(gr, ntasks, -(-ntasks // ut))
    simulate(ntasks, ms, S, ut, gr, seed)


@pytest.mark.parametrize("seed", range(100))
def test_attention_tc_protocol(seed):
    sim_attention(random.Random(seed).randint(1, 9), seed)


@pytest.mark.parametrize("seed", range(100))
def test_persistent_gemm_protocol(seed):
    r = random.Random(seed)
    sim_persistent(r.randint(1, 9), r.randint(1, 6), 4, seed)


def test_the_model_notices_a_missing_wait():
    """The attention model with the MMA thread no longer waiting for P fails its check."""
    caught = 0
    for seed in range(30):
        try:
            sim_attention(4, seed, wait_for_p=False)
        except AssertionError:
            caught += 1
    assert caught > 0


@pytest.mark.parametrize("seed", range(80))
def test_fused_allreduce_protocol(seed):
    r = random.Random(seed)
    simulate_allreduce(r.choice([2, 3, 4, 8]), r.choice([1, 2, 5]), r.randint(1, 7), seed, skew=r.random() < 0.5)


# --------------------------------------------------------------------------------------
# gemv_attention.cuh
# --------------------------------------------------------------------------------------
def tasks_for_head(hq, hkv, hd, h, lo, hi):
    """fa_tasks_for_head: tasks in [lo, hi) feeding query head h."""
    half = hd // 2
    kvh = h // (hq // hkv)

    def overlap(b0):
        return max(0, min(hi, b0 + half) - max(lo, b0))
    return overlap(h * half) + overlap((hq + kvh) * half) + overlap((hq + hkv + kvh) * half)


def brute_tasks_for_head(hq, hkv, hd, h, lo, hi):
    half = hd // 2
    n = 0
    for t in range(lo, hi):
        blk = t // half
        if blk < hq:
            n += blk == h
        else:
            kv = (blk - hq) % hkv  # k heads, then v heads
            n += kv == h // (hq // hkv)
    return n


def simulate_fused_attention(hq, hkv, hd, ctas, calls, seed):
    rnd = random.Random(seed)
    ntasks = (hq + 2 * hkv) * (hd // 2)
    cnt = [0] * hq
    for _ in range(calls):
        cuts = sorted(rnd.sample(range(1, ntasks), ctas - 1)) if ctas > 1 else []
        ranges = list(zip([0] + cuts, cuts + [ntasks]))
        written = set()
        computed = []
        order = list(range(ctas))
        rnd.shuffle(order)  # CTAs finish in any order
        for c in order:
            lo, hi = ranges[c]
            written.update(range(lo, hi))
            for h in range(hq):
                n = tasks_for_head(hq, hkv, hd, h, lo, hi)
                assert n == brute_tasks_for_head(hq, hkv, hd, h, lo, hi)
                if n > 0:
                    old = cnt[h]
                    cnt[h] += n
                    if old + n == 3 * (hd // 2):
                        cnt[h] = 0
                        # every q / k / v task the head reads is written
                        half = hd // 2
                        kvh = h // (hq // hkv)
                        need = set(range(h * half, (h + 1) * half))
                        need |= set(range((hq + kvh) * half, (hq + kvh + 1) * half))
                        need |= set(range((hq + hkv + kvh) * half, (hq + hkv + kvh + 1) * half))
                        assert need <= written, ("head computed before its inputs", h)
                        computed.append(h)
        assert sorted(computed) == list(range(hq)), computed
        assert cnt == [0] * hq


@pytest.mark.parametrize("seed", range(60))
def test_fused_decode_attention_counting(seed):
    r = random.Random(seed)
    hq, hkv = r.choice([(4, 4), (8, 2), (32, 32), (4, 1), (2, 2)])
    hd = r.choice([64, 128])
    ntasks = (hq + 2 * hkv) * hd // 2
    simulate_fused_attention(hq, hkv, hd, r.randint(1, min(ntasks, 60)), r.randint(1, 3), seed)


# --------------------------------------------------------------------------------------
# decode_layer.cu
# --------------------------------------------------------------------------------------
def simulate_decode_layer(ctas, layers, seed, reset_first=True):
    """Consecutive launches of the layer kernel, each CTA: weight prologue, griddepcontrol
    wait (the previous launch complete), four phases separated by the grid barrier (count
    and generation; the last arrival resets the count, then moves the generation).  The
    next launch's CTAs start once every CTA of the running one has started (the trigger at
    the top of the kernel).  Checks that no CTA reads a phase's input before every CTA
    wrote it, that the barrier words return to (0, 3 * layers) and that nothing deadlocks."""
    rnd = random.Random(seed)
    bar = [0, 0]
    done = [[set() for _ in range(4)] for _ in range(layers)]  # CTAs that finished phase p
    complete = [0] * layers
    started = [0] * layers

    def barrier():
        g = bar[1]
        yield
        old = bar[0]
        bar[0] += 1  # atomicAdd
        if old == ctas - 1:
            yield
            if reset_first:
                bar[0] = 0
                yield
                bar[1] = g + 1
            else:
                bar[1] = g + 1
                yield
                bar[0] = 0
        else:
            while bar[1] == g:
                yield "spin"

    def cta(layer, cid):
        started[layer] += 1
        yield  # prologue: weights only
        while layer > 0 and complete[layer - 1] < ctas:
            yield "spin"  # griddepcontrol.wait
        for p in range(4):
            if p > 0:
                yield from barrier()
                assert done[layer][p - 1] == set(range(ctas)), ("phase input read early", layer, p)
            for _ in range(rnd.randint(1, 3)):
                yield
            done[layer][p].add(cid)

    running = [(0, cta(0, i)) for i in range(ctas)]
    launched = 1
    spins = 0
    while running:
        if launched < layers and started[launched - 1] == ctas:
            running += [(launched, cta(launched, i)) for i in range(ctas)]
            launched += 1
        item = rnd.choice(running)
        try:
            r = next(item[1])
        except StopIteration:
            running.remove(item)
            complete[item[0]] += 1
            spins = 0
            continue
        spins = spins + 1 if r == "spin" else 0
        if spins > 200 * ctas + 1000:
            raise Deadlock(f"layer kernel: no progress ({bar})")
    assert bar == [0, 3 * layers]
    assert all(len(done[l][3]) == ctas for l in range(layers))


@pytest.mark.parametrize("seed", range(60))
def test_decode_layer_grid_barrier(seed):
    r = random.Random(seed)
    simulate_decode_layer(r.choice([1, 2, 3, 7, 16]), r.randint(1, 4), seed)


def test_the_layer_model_notices_a_late_count_reset():
    """Moving the generation before the count is reset loses an early arrival at the next barrier."""
    caught = 0
    for seed in range(40):
        try:
            simulate_decode_layer(4, 2, seed, reset_first=False)
        except (AssertionError, Deadlock):
            caught += 1
    assert caught > 0


def simulate_decode_layer_ar(nranks, ctas, layers, seed, barrier_after_reduce=True, step=False):
    """The layer kernel's all-reduce form over ranks: per launch, phase 1, grid barrier,
    o_proj partials pushed to every rank (epoch counter + 1), the fused all-reduce (ticket,
    flags, wait, rank-order read, ticket reset and counter by the last CTA out), grid
    barrier, mlp, grid barrier, down partials and the all-reduce of epoch counter + 2.  A
    rank's next launch starts when its current one is complete (the trigger sits at the
    end); ranks run at different speeds.  Checks every rank-order read against the epoch
    it belongs to, the barrier and ticket words at rest after the last launch, and that
    nothing deadlocks."""
    rnd = random.Random(seed)
    bar = [[0, 0] for _ in range(nranks)]
    counter = [0] * nranks
    tickets = [[0, 0] for _ in range(nranks)]
    flags = [[[0] * nranks for _ in range(2)] for _ in range(nranks)]
    data = [[[None] * nranks for _ in range(2)] for _ in range(nranks)]
    written = [set() for _ in range(nranks)]  # (epoch, cta): that CTA's columns of the sum are out

    def barrier(rank):
        g = bar[rank][1]
        yield
        old = bar[rank][0]
        bar[rank][0] += 1
        if old == ctas - 1:
            yield
            bar[rank][0] = 0
            yield
            bar[rank][1] = g + 1
        else:
            while bar[rank][1] == g:
                yield "spin"

    def allreduce(rank, epoch, cid):
        slot = epoch & 1
        for q in range(nranks):  # this CTA's partials into every rank's row `rank`
            data[q][slot][rank] = (epoch, rank)
            yield
        tickets[rank][0] += 1
        if tickets[rank][0] == ctas:
            for q in range(nranks):
                flags[q][slot][rank] = epoch
                yield
        yield
        for r in range(nranks):
            while flags[rank][slot][r] != epoch:
                assert flags[rank][slot][r] < epoch, ("flag ahead", rank, r, epoch)
                yield "spin"
        for r in range(nranks):
            assert data[rank][slot][r] == (epoch, r), ("stale or overwritten row", rank, epoch, data[rank][slot])
            yield
        written[rank].add((epoch, cid))
        tickets[rank][1] += 1
        if tickets[rank][1] == ctas:
            tickets[rank][0] = tickets[rank][1] = 0
            counter[rank] = epoch

    def one_layer(rank, e1, cid):
        yield
        yield from barrier(rank)  # attention -> o_proj
        yield from allreduce(rank, e1, cid)
        if barrier_after_reduce:
            yield from barrier(rank)  # o_proj -> mlp
        assert all((e1, c) in written[rank] for c in range(ctas)), ("mlp_in reads h early", rank, e1)
        yield
        yield from barrier(rank)  # mlp -> down
        yield from allreduce(rank, e1 + 1, cid)

    def cta(rank, layer, cid):
        base = counter[rank] + 1  # read after griddepcontrol.wait
        assert base == 2 * layer + 1, (rank, layer, base)
        if not step:
            yield from one_layer(rank, base, cid)
            return
        for l in range(layers):  # the whole-step kernel: every layer in one launch
            yield from one_layer(rank, base + 2 * l, cid)
            if l + 1 < layers:
                yield from barrier(rank)  # layer l's output -> layer l + 1
                assert all((base + 2 * l + 1, c) in written[rank] for c in range(ctas)), ("next layer early", rank)

    launch = [0] * nranks
    running = {r: [cta(r, 0, i) for i in range(ctas)] for r in range(nranks)}
    spins = 0
    while any(running.values()):
        r = rnd.choice([q for q in range(nranks) if running[q]])
        if nranks > 1 and r == 0 and rnd.random() < 0.4:
            continue  # rank 0 slower
        g = rnd.choice(running[r])
        try:
            got = next(g)
        except StopIteration:
            running[r].remove(g)
            spins = 0
            if not running[r]:
                launch[r] += 1
                if launch[r] < (1 if step else layers):
                    running[r] = [cta(r, launch[r], i) for i in range(ctas)]
            continue
        spins = spins + 1 if got == "spin" else 0
        if spins > 400 * ctas * nranks + 2000:
            raise Deadlock("layer kernel (all-reduce form): no progress")
    assert all(b[0] == 0 for b in bar) and all(t == [0, 0] for t in tickets)
    assert counter == [2 * layers] * nranks


@pytest.mark.parametrize("seed", range(60))
def test_decode_layer_allreduce_form(seed):
    r = random.Random(seed)
    simulate_decode_layer_ar(r.choice([2, 3, 4, 8]), r.choice([1, 2, 5]), r.randint(1, 4), seed)


@pytest.mark.parametrize("seed", range(40))
def test_decode_step_allreduce_form(seed):
    """The whole-step kernel: every layer's two all-reduces in one launch, a grid barrier
    between layers."""
    r = random.Random(seed)
    simulate_decode_layer_ar(r.choice([1, 2, 4, 8]), r.choice([1, 3, 5]), r.randint(1, 5), seed, step=True)


def test_the_layer_model_needs_the_barrier_after_the_first_all_reduce():
    """Without it a CTA starts the mlp phase before every CTA wrote its columns of h."""
    caught = 0
    for seed in range(60):
        try:
            simulate_decode_layer_ar(2, 4, 2, seed, barrier_after_reduce=False)
        except (AssertionError, Deadlock):
            caught += 1
    assert caught > 0
