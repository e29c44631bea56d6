"""The cross-rank protocols of the sequence splits, checked on a CPU model under random interleavings:
the key-range split (lingbot_b200.split.KeySplitAttention over csrc/peer.cu and the key-range attention
kernel) and, below, the query split (SplitAttention).

Every rank runs the calls of a pass sequence on two streams (main and side) joined by events, exactly in
the order KeySplitAttention.__call__ launches them:
- main stream: block stats, totals push, window totals, the quantizers, peer wait, attention, peer wait,
  merge;
- side stream, forked at the call start: query quantizer and query push; then, for persisting calls and
  after the window totals, the bf16 share push.

The model follows the device mechanisms:
- the totals travel as tagged words in parity-double-buffered slots;
- the data signals are monotonic counters that the receiver compares with its own "seen" count;
- a push or the attention raises the other ranks' counters after all its writes.

Writes land one destination at a time, and reads re-check what they read. So a reader that could see
another call's data fails an assertion, and a state with no runnable stream is a deadlock. Three broken
variants must fail, to show the checks have teeth: a query push not ordered after the previous call's
merge, a merge that does not wait for the partials, and a push that signals before writing.
"""
import random

import pytest


class Rank:
    def __init__(self, n):
        self.q_rows = [-1] * n          # call whose query codes rank r's rows hold here
        self.recv = [-1] * n            # call whose partial slot s holds here
        self.cache = [-1] * n           # call whose bf16 share of rank s the chunk region holds
        self.slots = [[(-1, -1)] * n for _ in range(2)]   # [parity][sender] = (tag, call)
        self.flags = [0] * n            # data signals raised by each sender
        self.seen = [0] * n             # data signals consumed
        self.calls = 0                  # window totals completed (tag - 1)
        self.events = set()             # recorded stream events ("fork", c), ("totals", c), ("join", c)


class SplitModel:
    def __init__(self, n, persist, seed, unordered_q_push=False, no_partial_wait=False, signal_before_write=False):
        self.n, self.persist = n, persist
        self.rng = random.Random(seed)
        self.unordered_q_push, self.no_partial_wait = unordered_q_push, no_partial_wait
        self.signal_before_write = signal_before_write
        self.ranks = [Rank(n) for _ in range(n)]

    def wait(self, cond):
        """Yield until cond() holds (a device-side poll or a stream-event wait)."""
        while not cond():
            yield

    def signal(self, r):
        for p in range(self.n):
            if p != r:
                self.ranks[p].flags[r] += 1

    def push(self, r, write):
        """A push kernel: its writes land one destination at a time, then one signal per other rank."""
        order = list(range(self.n))
        self.rng.shuffle(order)
        if self.signal_before_write:
            self.signal(r)
        for p in order:
            write(p)
            yield
        if not self.signal_before_write:
            self.signal(r)

    def peer_wait(self, r, signals):
        me = self.ranks[r]
        targets = {t: me.seen[t] + signals for t in range(self.n) if t != r}
        yield from self.wait(lambda: all(me.flags[t] >= v for t, v in targets.items()))
        for t, v in targets.items():
            me.seen[t] = v

    def main(self, r):
        me = self.ranks[r]
        for c, persist in enumerate(self.persist):
            me.events.add(("fork", c))
            # totals push: tagged words into every rank's slot for this call's parity
            for p in range(self.n):
                self.ranks[p].slots[c & 1][r] = (c + 1, c)
                yield
            # window totals: poll until every rank's words carry this call's tag, then read them
            par = me.calls & 1
            yield from self.wait(lambda: all(w[0] == me.calls + 1 for w in me.slots[par]))
            yield
            assert all(w == (c + 1, c) for w in me.slots[par]), f"rank {r} call {c}: totals overwritten"
            me.calls += 1
            me.events.add(("totals", c))
            yield                                    # the quantizers (local)
            yield from self.wait(lambda: ("join", c) in me.events)
            yield from self.peer_wait(r, 1 + int(persist))
            # attention: reads every rank's query rows, then stores its partials at the row owners
            assert all(v == c for v in me.q_rows), f"rank {r} call {c}: query rows {me.q_rows}"
            yield
            assert all(v == c for v in me.q_rows), f"rank {r} call {c}: query rows changed under attention"
            yield from self.push(r, lambda p: self.ranks[p].recv.__setitem__(r, c))
            if not self.no_partial_wait:
                yield from self.peer_wait(r, 1)
            # merge: reads every rank's partial for this rank's rows
            assert all(v == c for v in me.recv), f"rank {r} call {c}: partials {me.recv}"
            yield
            assert all(v == c for v in me.recv), f"rank {r} call {c}: partials changed under the merge"

    def side(self, r):
        me = self.ranks[r]
        for c, persist in enumerate(self.persist):
            if not self.unordered_q_push:
                yield from self.wait(lambda: ("fork", c) in me.events)
            yield from self.push(r, lambda p: self.ranks[p].q_rows.__setitem__(r, c))
            if persist:
                # the bf16 share lands in the chunk region of every rank's cache, which no rank reads
                # during a call; it still follows the window totals
                yield from self.wait(lambda: ("totals", c) in me.events)
                yield from self.push(r, lambda p: self.ranks[p].cache.__setitem__(r, c))
            me.events.add(("join", c))

    def run(self, max_steps=2_000_000):
        gens = [g for r in range(self.n) for g in (self.main(r), self.side(r))]
        live = list(range(len(gens)))
        stalled = 0
        for _ in range(max_steps):
            if not live:
                return
            i = self.rng.choice(live)
            before = self.state()
            try:
                next(gens[i])
            except StopIteration:
                live.remove(i)
                stalled = 0
                continue
            stalled = stalled + 1 if self.state() == before else 0
            if stalled > 200 * len(gens):
                raise RuntimeError("deadlock: no stream makes progress")
        raise RuntimeError("step limit")

    def state(self):
        return tuple((tuple(x.q_rows), tuple(x.recv), tuple(x.flags), tuple(x.seen), x.calls, len(x.events),
                      tuple(tuple(s) for s in x.slots)) for x in self.ranks)


@pytest.mark.parametrize("n", [2, 3, 4, 8])
def test_key_split_protocol_random_interleavings(n):
    rng = random.Random(n)
    for trial in range(40 if n < 8 else 15):
        persist = [rng.random() < 0.3 for _ in range(rng.randint(2, 6))]
        SplitModel(n, persist, seed=trial).run()


@pytest.mark.parametrize("mutation", ["unordered_q_push", "no_partial_wait", "signal_before_write"])
def test_the_model_catches_a_broken_protocol(mutation):
    caught = 0
    for trial in range(40):
        persist = [True, False, True, True]
        try:
            SplitModel(3, persist, seed=trial, **{mutation: True}).run()
        except (AssertionError, RuntimeError):
            caught += 1
    assert caught >= 10, f"{mutation}: only {caught} of 40 schedules failed"


class QuerySplitModel(SplitModel):
    """The query split (lingbot_b200.split.SplitAttention) in its launch order:
    - main stream: block stats, totals push, window totals, then the fork; the memory quantizer; join,
      peer wait, attention;
    - side stream, after the fork: this rank's share quantized into its own code buffer and pushed into
      every other rank's, the bf16 share push for persisting calls, and the query quantizer.

    `codes[s]` on a rank is the call whose chunk codes of rank s its buffer holds; the attention reads
    all of them. `early_fork` forks the side stream before the window totals (a broken variant)."""

    def __init__(self, n, persist, seed, early_fork=False, **kw):
        super().__init__(n, persist, seed, **kw)
        self.early_fork = early_fork
        for x in self.ranks:
            x.codes = [-1] * n

    def main(self, r):
        me = self.ranks[r]
        for c, persist in enumerate(self.persist):
            if self.early_fork:
                me.events.add(("fork", c))
            for p in range(self.n):
                self.ranks[p].slots[c & 1][r] = (c + 1, c)
                yield
            par = me.calls & 1
            yield from self.wait(lambda: all(w[0] == me.calls + 1 for w in me.slots[par]))
            yield
            assert all(w == (c + 1, c) for w in me.slots[par]), f"rank {r} call {c}: totals overwritten"
            me.calls += 1
            me.events.add(("fork", c))
            yield                                    # the memory quantizer (local)
            yield from self.wait(lambda: ("join", c) in me.events)
            yield from self.peer_wait(r, 1 + int(persist))
            assert all(v == c for v in me.codes), f"rank {r} call {c}: chunk codes {me.codes}"
            yield
            assert all(v == c for v in me.codes), f"rank {r} call {c}: chunk codes changed under attention"

    def side(self, r):
        me = self.ranks[r]
        for c, persist in enumerate(self.persist):
            yield from self.wait(lambda: ("fork", c) in me.events)
            yield from self.push(r, lambda p: self.ranks[p].codes.__setitem__(r, c))
            if persist:
                yield from self.push(r, lambda p: self.ranks[p].cache.__setitem__(r, c))
            me.events.add(("join", c))

    def state(self):
        return super().state() + tuple(tuple(x.codes) for x in self.ranks)


@pytest.mark.parametrize("n", [2, 4, 8])
def test_query_split_protocol_random_interleavings(n):
    rng = random.Random(100 + n)
    for trial in range(40 if n < 8 else 15):
        persist = [rng.random() < 0.3 for _ in range(rng.randint(2, 6))]
        QuerySplitModel(n, persist, seed=trial).run()


@pytest.mark.parametrize("mutation", ["early_fork", "signal_before_write"])
def test_the_query_split_model_catches_a_broken_protocol(mutation):
    caught = 0
    for trial in range(40):
        try:
            QuerySplitModel(3, [True, False, False, True], seed=trial, **{mutation: True}).run()
        except (AssertionError, RuntimeError):
            caught += 1
    assert caught >= 10, f"{mutation}: only {caught} of 40 schedules failed"
