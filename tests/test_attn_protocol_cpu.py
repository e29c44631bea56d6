"""The hand-offs inside one attention CTA (csrc/attn.cu, attn_fwd_kernel), checked on a CPU model under
random interleavings of its warps, its TMA copies and the tensor pipe.

Agents, in the kernel's roles: the K and V TMA producers, the Q.K^T issuer, the P.V issuer, four softmax
warps per Q tile (one per tensor-memory lane quarter) and four correction warps. They meet on mbarriers
with the kernel's arrival counts (a warp's 32 threads arrive together, so a count of 128 threads is 4
warps here). The tensor pipe completes MMAs in issue order, at random times; a commit arrives once every
MMA its thread issued before it has completed. TMA copies land at random times.

What is checked, on every interleaving:
- S of a tile is overwritten (the next Q.K^T) only after all four softmax warps read it and all four
  correction warps refilled it, and the softmax reads S only once its Q.K^T completed;
- O is rescaled only while no P.V on it is in flight;
- the softmax writes a P buffer only when no P.V that reads it is in flight — with no wait of its own for
  that buffer: the kernel relies on the correction warps' order (the refill for tile j + 1 after every O
  stage of tile j - 1) for it;
- no barrier is ever polled two phases past the phase waited for (the kernel's parity waits would alias);
- no state without a runnable agent (a deadlock).
Broken variants must fail: refills taken as soon as S was read, and two P buffers instead of three.
"""
import random

import pytest

K_STAGES = 2


class Bar:
    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0      # phase = phases completed

    def arrive(self):
        self.pending -= 1
        assert self.pending >= 0
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count


class Model:
    def __init__(self, seed, ns, p_bufs=3, eager_refill=False):
        self.rng = random.Random(seed)
        self.ns, self.n, self.p_bufs, self.eager_refill = ns, len(ns), p_bufs, eager_refill
        B = Bar
        self.k_full, self.k_empty = [B(1) for _ in range(K_STAGES)], [B(1) for _ in range(K_STAGES)]
        self.v_full, self.v_empty = [B(1) for _ in range(K_STAGES)], [B(1) for _ in range(K_STAGES)]
        self.s_full, self.s_read, self.s_free = [B(1), B(1)], [B(4), B(4)], [B(4), B(4)]
        self.p_full = [[B(4) for _ in range(p_bufs)] for _ in range(2)]
        self.o_ready, self.o_done = [B(4), B(4)], [B(1), B(1)]
        self.mma = []            # in-order tensor pipe: [issuer, kind, tile, key tile, callbacks]
        self.tma = []            # copies in flight: barriers to arrive on
        self.commits = []        # (barrier, issuer, index of the issuer's last MMA at the commit)
        self.issued = {"qk": 0, "pv": 0}
        self.done_mmas = {"qk": 0, "pv": 0}
        self.s_holds = [("magic", -1), ("magic", -1)]   # per tile: what S holds
        self.s_readers = [set(), set()]                 # softmax warps that read S's current scores
        self.s_refilled = [set(), set()]                # correction warps that refilled S since the read
        self.pv_reading = [dict(), dict()]              # tile -> {P buffer: P.V in flight}
        self.p_writes = [dict(), dict()]                # tile -> {P buffer: (key tile, warps that wrote it)}
        self.o_busy = [0, 0]                            # P.V in flight on O_t

    # ---------------------------------------------------------------- mechanisms
    def wait(self, bar, k):
        """A parity wait for phase k of `bar` (complete once phase k completed)."""
        while True:
            assert bar.phase <= k + 1, "polled two phases past the waited phase: parity waits alias"
            if bar.phase > k:
                return
            yield

    def issue(self, who, kind, t, j, callbacks):
        self.mma.append([who, kind, t, j, callbacks])
        self.issued[who] += 1

    def commit(self, bar, who):
        self.commits.append((bar, who, self.issued[who]))
        self.fire_commits()

    def fire_commits(self):
        keep = []
        for bar, who, upto in self.commits:
            if self.done_mmas[who] >= upto:
                bar.arrive()
            else:
                keep.append((bar, who, upto))
        self.commits = keep

    def complete_mma(self):
        who, kind, t, j, callbacks = self.mma.pop(0)
        for cb in callbacks:
            cb()
        self.done_mmas[who] += 1
        self.fire_commits()

    # ---------------------------------------------------------------- roles
    def producer(self, full, empty):
        for i in range(self.n):
            s = i % K_STAGES
            if i >= K_STAGES:
                yield from self.wait(empty[s], i // K_STAGES - 1)
            self.tma.append(full[s])

    def qk_issuer(self):
        for k in range(self.n):
            s = k % K_STAGES
            yield from self.wait(self.k_full[s], k // K_STAGES)
            for t in range(2):
                yield from self.wait(self.s_free[t], k)
                assert self.s_holds[t] == ("magic", k - 1) and len(self.s_refilled[t]) == 4, \
                    f"Q.K^T {k} of tile {t} issued onto S that was not read and refilled"

                def qk_done(t=t, k=k):
                    self.s_holds[t] = ("scores", k)
                    self.s_readers[t], self.s_refilled[t] = set(), set()
                self.issue("qk", "qk", t, k, [qk_done])
                self.commit(self.s_full[t], "qk")
            self.commit(self.k_empty[s], "qk")

    def pv_issuer(self):
        u = 0
        for j in range(self.n):
            s = j % K_STAGES
            yield from self.wait(self.v_full[s], j // K_STAGES)
            for hh in range(self.ns[j]):
                for t in range(2):
                    yield from self.wait(self.o_ready[t], u)
                    pb = j % self.p_bufs
                    assert self.p_writes[t].get(pb) == (j, 4), f"P.V {j} of tile {t} issued before P was written"
                    self.pv_reading[t][pb] = self.pv_reading[t].get(pb, 0) + 1
                    self.o_busy[t] += 1

                    def pv_done(t=t, pb=pb):
                        self.pv_reading[t][pb] -= 1
                        self.o_busy[t] -= 1
                    self.issue("pv", "pv", t, j, [pv_done])
                    self.commit(self.o_done[t], "pv")
                u += 1
            self.commit(self.v_empty[s], "pv")

    def softmax(self, t, w):
        for j in range(self.n):
            yield from self.wait(self.s_full[t], j)
            assert self.s_holds[t] == ("scores", j), f"softmax {t}.{w} read S before Q.K^T {j} completed"
            self.s_readers[t].add(w)
            self.s_read[t].arrive()
            yield
            pb = j % self.p_bufs
            assert self.pv_reading[t].get(pb, 0) == 0, f"P buffer {pb} of tile {t} written under a P.V"
            prev = self.p_writes[t].get(pb, (j, 0))
            self.p_writes[t][pb] = (j, prev[1] + 1 if prev[0] == j else 1)
            self.p_full[t][pb].arrive()
            yield

    def refill(self, t, w):
        assert len(self.s_readers[t]) == 4, "S refilled before every softmax warp read it"
        self.s_refilled[t].add(w)
        if len(self.s_refilled[t]) == 4:
            self.s_holds[t] = ("magic", self.s_holds[t][1])
        self.s_free[t].arrive()

    def correction(self, w):
        for t in range(2):                               # the initial fill
            self.s_refilled[t].add(w)
            self.s_free[t].arrive()
        u = 0
        for j in range(self.n):
            if j + 1 < self.n and not self.eager_refill:
                for t in range(2):
                    yield from self.wait(self.s_read[t], j)
                    self.refill(t, w)
            for hh in range(self.ns[j]):
                for t in range(2):
                    if hh == 0:
                        yield from self.wait(self.p_full[t][j % self.p_bufs], j // self.p_bufs)
                    if u > 0:
                        yield from self.wait(self.o_done[t], u - 1)
                        assert self.o_busy[t] == 0, "O rescaled under a P.V"
                    self.o_ready[t].arrive()
                    yield
                u += 1

    def eager_refiller(self, w):
        """Broken variant: each S refill taken as soon as the softmax read S."""
        for j in range(self.n - 1):
            for t in range(2):
                yield from self.wait(self.s_read[t], j)
                self.refill(t, w)

    # ---------------------------------------------------------------- scheduler
    def run(self):
        agents = [self.producer(self.k_full, self.k_empty), self.producer(self.v_full, self.v_empty),
                  self.qk_issuer(), self.pv_issuer()]
        agents += [self.softmax(t, w) for t in range(2) for w in range(4)]
        agents += [self.correction(w) for w in range(4)]
        if self.eager_refill:
            agents += [self.eager_refiller(w) for w in range(4)]
        live = list(agents)
        steps = 0
        while live or self.mma or self.tma:
            steps += 1
            assert steps < 200000, "no progress"
            moves = []
            if self.mma:
                moves.append(("mma", None))
            if self.tma:
                moves.append(("tma", None))
            moves += [("agent", a) for a in live]
            kind, a = self.rng.choice(moves)
            if kind == "mma":
                self.complete_mma()
            elif kind == "tma":
                self.tma.pop(self.rng.randrange(len(self.tma))).arrive()
            else:
                try:
                    next(a)
                except StopIteration:
                    live.remove(a)
        assert all(not c for c in self.commits)


def _tiles(rng):
    n = rng.randint(1, 9)
    ns = [2] * n
    if n > 2 and rng.random() < 0.5:
        ns[rng.randrange(n - 1)] = 1                  # a code segment ending on a 64-key half
    if rng.random() < 0.5:
        ns[-1] = 1
    return ns


@pytest.mark.parametrize("seed", range(60))
def test_attention_handoffs_hold(seed):
    rng = random.Random(1000 + seed)
    Model(seed, _tiles(rng)).run()


def _fails(**kw):
    failures = 0
    for seed in range(80):
        try:
            Model(seed, [2] * 8, **kw).run()
        except AssertionError:
            failures += 1
    return failures


def test_eager_refills_break_the_p_buffer_reuse():
    assert _fails(eager_refill=True) > 0


def test_two_p_buffers_are_not_enough():
    assert _fails(p_bufs=2) > 0
