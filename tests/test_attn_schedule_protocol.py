"""The barrier protocol of the persistent attention schedule (attn_fwd_persistent_kernel, csrc/attn.cu),
checked on a CPU model under random interleavings.

The model restates the kernel's synchronisation, not its arithmetic:
- Roles: the TMA producer, the tcgen05 issuer, and two softmax warpgroups of 4 warps each.
- They run as generators over mbarriers with the hardware's parity rule: a phase completes after `count`
  arrivals, and try_wait.parity(P) succeeds while the current phase's parity differs from P.
- TMA loads and MMAs complete asynchronously, MMAs in issue order; tcgen05.commit arrives once every
  earlier MMA has completed.

Buffer contents are tracked (Q, the K/V stages, S, the two P buffers, O), so a read of stale or
overwritten data fails an assertion, and a schedule with no runnable role is a deadlock. The same model
with the protocol deliberately broken must fail, which shows that the checks have teeth.
"""
import random

import pytest

STAGES = 3          # K/V stages of the kernel (kStages)


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.arrived, self.phase = name, count, 0, 0

    def arrive(self):
        self.arrived += 1
        assert self.arrived <= self.count, f"{self.name}: more arrivals than its count"
        if self.arrived == self.count:
            self.phase += 1
            self.arrived = 0

    def ready(self, parity):
        return (self.phase & 1) != parity


class Always(Bar):
    """A wait that is always satisfied: a point where the scheduler may run other roles."""

    def __init__(self):
        super().__init__("yield", 1)

    def ready(self, parity):
        return True


class Model:
    """One CTA: `n_tiles[k]` key tiles for its k-th work item. `early_q_release` and `local_p_parity`
    break the protocol, `shared_staging` stages the key-range epilogue in 8 KB per warp across the P
    buffers (the single-item kernel's layout) instead of each warp's own P rows (for the sensitivity
    tests)."""

    def __init__(self, n_tiles, seed, early_q_release=False, local_p_parity=False, shared_staging=False):
        self.rng = random.Random(seed)
        self.n_tiles = n_tiles
        self.early_q_release, self.local_p_parity = early_q_release, local_p_parity
        self.shared_staging = shared_staging
        self.rows = {}                         # (tile t, P buffer, warp's 32-row block) -> last writer
        self.q_full, self.q_empty = Bar("q_full", 1), Bar("q_empty", 1)
        self.k_full = [Bar(f"k_full{s}", 1) for s in range(STAGES)]
        self.k_empty = [Bar(f"k_empty{s}", 1) for s in range(STAGES)]
        self.v_full = [Bar(f"v_full{s}", 1) for s in range(STAGES)]
        self.v_empty = [Bar(f"v_empty{s}", 1) for s in range(STAGES)]
        self.s_full = [Bar(f"s_full{t}", 1) for t in range(2)]
        self.s_free = [Bar(f"s_free{t}", 4) for t in range(2)]
        self.p_full = [Bar(f"p_full{t}", 4) for t in range(2)]
        self.o_done = [Bar(f"o_done{t}", 1) for t in range(2)]
        self.o_free = [Bar(f"o_free{t}", 4) for t in range(2)]
        self.tma, self.mma = [], []            # pending asynchronous work, completed in order
        self.q = None                          # item whose Q tiles are in shared memory
        self.stage_k, self.stage_v = [None] * STAGES, [None] * STAGES
        self.s = ["magic", "magic"]            # tile whose scores S_t holds, or the refill constant
        self.p = [[None, None], [None, None]]  # P_t[buffer] = (tile, warps that wrote their rows)
        self.o = [None, None]                  # (item, last tile accumulated) in O_t
        self.o_read = [None, None]             # item whose O_t every epilogue warp has read

    # ---------------------------------------------------------------- roles
    def producer(self):
        g = 0
        for k, n in enumerate(self.n_tiles):
            if k > 0:
                yield self.q_empty, (k - 1) & 1
            assert not any(getattr(op, "reads_q", False) for op in self.mma), "Q reloaded under a Q.K^T"
            self.tma.append(lambda k=k: (setattr(self, "q", k), self.q_full.arrive()))
            for _ in range(n):
                s, ph = g % STAGES, (g // STAGES) & 1
                yield self.k_empty[s], ph ^ 1
                self.tma.append(lambda s=s, g=g: (self.stage_k.__setitem__(s, g), self.k_full[s].arrive()))
                yield self.v_empty[s], ph ^ 1
                self.tma.append(lambda s=s, g=g: (self.stage_v.__setitem__(s, g), self.v_full[s].arrive()))
                g += 1

    def issuer(self):
        g = 0
        for k, n in enumerate(self.n_tiles):
            yield self.q_full, k & 1
            yield self.k_full[g % STAGES], (g // STAGES) & 1
            for t in range(2):
                yield self.s_free[t], g & 1
                self.qk(t, g, k)
            self.commit(self.k_empty[g % STAGES])
            if self.early_q_release:
                self.commit(self.q_empty)
            for j in range(n):
                s, more = g % STAGES, j + 1 < n
                if more:
                    yield self.k_full[(g + 1) % STAGES], ((g + 1) // STAGES) & 1
                yield self.v_full[s], (g // STAGES) & 1
                if not more and not self.early_q_release:
                    self.commit(self.q_empty)
                for t in range(2):
                    if more:
                        yield self.s_free[t], (g + 1) & 1
                        self.qk(t, g + 1, k)
                    if j == 0 and k > 0:
                        yield self.o_free[t], (k - 1) & 1
                    yield self.p_full[t], g & 1
                    self.pv(t, g, k, first=j == 0, buf=(j & 1) if self.local_p_parity else (g & 1))
                self.commit(self.v_empty[s])
                if more:
                    self.commit(self.k_empty[(g + 1) % STAGES])
                g += 1

    def staging(self, t, w):
        """The P-row blocks warp w stages its 32 rows of the partial in (16 KB P buffers of 4 blocks)."""
        if self.shared_staging:                # bytes [8K*w, 8K*w + 8K) of the tile's two buffers
            return [(t, w // 2, 2 * (w % 2)), (t, w // 2, 2 * (w % 2) + 1)]
        return [(t, 0, w), (t, 1, w)]          # its own rows in both buffers

    def softmax_warp(self, t, w):
        g = 0
        self.s_free[t].arrive()                 # S_t starts as the refill constant
        for k, n in enumerate(self.n_tiles):
            for i in range(n):
                yield self.s_full[t], g & 1
                assert self.s[t] == g, f"softmax {t}: S holds {self.s[t]}, tile {g} expected"
                self.s_free[t].arrive()
                if self.s_free[t].arrived == 0:      # every warp has refilled S_t
                    self.s[t] = "magic"
                self.rows[(t, g & 1, w)] = ("P", g)
                tile, warps = self.p[t][g & 1] or (None, 0)
                self.p[t][g & 1] = (g, warps + 1 if tile == g else 1)
                if i > 0:
                    yield self.o_done[t], (g - 1) & 1
                self.p_full[t].arrive()
                g += 1
            yield self.o_done[t], (g - 1) & 1
            assert self.o[t] == (k, g - 1), f"epilogue {t}: O holds {self.o[t]}, item {k} expected"
            self.o_read[t] = k
            for block in self.staging(t, w):       # key-range epilogue: stage, then copy out
                self.rows[block] = ("stage", w, k)
            for _ in range(16):                      # the copy's 16 store iterations
                yield Always(), 0
                for block in self.staging(t, w):
                    assert self.rows[block] == ("stage", w, k), \
                        f"epilogue {t}.{w}: staged rows {block} overwritten by {self.rows[block]}"
            self.o_free[t].arrive()

    # ---------------------------------------------------------------- asynchronous work
    def commit(self, bar):
        self.mma.append(bar.arrive)

    def qk(self, t, g, k):
        s = g % STAGES

        def run():
            assert self.q == k, f"Q.K^T({t}, {g}): Q of item {self.q}, item {k} expected"
            assert self.stage_k[s] == g, f"Q.K^T({t}, {g}): stage {s} holds K of tile {self.stage_k[s]}"
            assert self.s[t] == "magic", f"Q.K^T({t}, {g}): S_{t} not refilled"
            self.s[t] = g
        run.reads_q = True
        self.mma.append(run)
        self.commit(self.s_full[t])

    def pv(self, t, g, k, first, buf):
        s = g % STAGES

        def run():
            assert self.stage_v[s] == g, f"P.V({t}, {g}): stage {s} holds V of tile {self.stage_v[s]}"
            assert self.p[t][buf] == (g, 4), f"P.V({t}, {g}): P buffer {buf} holds {self.p[t][buf]}"
            if first:
                prev = self.o[t]
                assert prev is None or self.o_read[t] == prev[0], f"P.V({t}, {g}): O overwritten before read"
            else:
                assert self.o[t] == (k, g - 1), f"P.V({t}, {g}): O holds {self.o[t]}"
            self.o[t] = (k, g)
        self.mma.append(run)
        self.commit(self.o_done[t])

    # ---------------------------------------------------------------- scheduler
    def run(self, max_steps=500_000):
        roles = [self.producer(), self.issuer()] + [self.softmax_warp(t, w) for t in range(2) for w in range(4)]
        wait = [None] * len(roles)
        done = [False] * len(roles)
        for _ in range(max_steps):
            if all(done) and not self.tma and not self.mma:
                return
            runnable = [r for r in range(len(roles)) if not done[r] and (wait[r] is None or wait[r][0].ready(wait[r][1]))]
            if not runnable and not self.tma and not self.mma:
                raise RuntimeError("deadlock: " + ", ".join(f"role {r} on {wait[r][0].name}"
                                                            for r in range(len(roles)) if not done[r]))
            if runnable and (self.rng.random() < 0.7 or not (self.tma or self.mma)):
                r = self.rng.choice(runnable)
                try:
                    wait[r] = next(roles[r])
                except StopIteration:
                    done[r], wait[r] = True, None
            else:
                queue = self.tma if self.tma and (not self.mma or self.rng.random() < 0.5) else self.mma
                queue.pop(0)()
        raise RuntimeError("step limit")


def _schedules(count, seed):
    rng = random.Random(seed)
    for trial in range(count):
        yield [rng.randint(1, 7) for _ in range(rng.randint(1, 4))], trial


def test_random_schedules_complete_without_hazards():
    for n_tiles, trial in _schedules(300, 1):
        Model(n_tiles, seed=trial).run()


@pytest.mark.parametrize("mutation", ["early_q_release", "local_p_parity", "shared_staging"])
def test_the_model_catches_a_broken_protocol(mutation):
    caught = 0
    for n_tiles, trial in _schedules(100, 7):
        if len(n_tiles) < 2:
            n_tiles = n_tiles + [3]
        try:
            Model(n_tiles, seed=trial, **{mutation: True}).run()
        except (AssertionError, RuntimeError):
            caught += 1
    assert caught >= 50, f"{mutation}: only {caught} of 100 schedules failed"
