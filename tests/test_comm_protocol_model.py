"""Host-side model check of the all-reduce kernels' flag protocol (``csrc/comm.cu``).

A Python model of the per-rank barriers, run under many random interleavings of every CTA
of every rank, for a mix of one-shot and two-shot calls:

* entry barrier: every CTA reads the call number from the rank's counter; CTA 0 publishes it
  to every rank's flag slot, waits until every rank's flag has reached it, then releases its
  rank's other CTAs through the local go word;
* data phase: one-shot reads every peer's IN buffer (three buffers in rotation, refilled by
  the previous kernel); two-shot reads every peer's single IN buffer and writes every peer's
  OUT rows;
* exit: the last CTA of a rank (a done counter) runs the two-shot exit exchange, then
  advances the counter;
* kernels of one rank run in stream order, and between two all-reduces the rank's GEMM
  refills the IN buffer the next call uses.

Checked: no interleaving deadlocks; every read sees the peer's data of the same call (never an
older or newer fill); when a two-shot call completes on a rank, every peer has finished
writing that rank's OUT rows.
"""
import random


class Rank:
    def __init__(self, r, world):
        self.r = r
        self.flags = {slot: [0] * world for slot in ("one", "A", "B")}
        self.calls = 0
        self.go = 0
        self.done = 0
        self.in_ver = [0, 0, 0]   # one-shot rotation buffers: call number of the data they hold (up to 3)
        self.in2_ver = 0           # two-shot IN buffer
        self.out_writes = {}       # call -> set of ranks that wrote this rank's OUT rows


def reached(v, e):
    return v >= e


def run(kinds, world=2, ctas=2, seed=0, nbuf=3):
    rng = random.Random(seed)
    ranks = [Rank(r, world) for r in range(world)]
    # per rank: index of the current call, and per-CTA program counters
    call_idx = [0] * world
    state = {}

    def start_call(r):
        k = call_idx[r]
        kind = kinds[k]
        rk = ranks[r]
        # the previous kernel (the GEMM) fills the IN buffer this call reads
        if kind == "one":
            rk.in_ver[(k + 1) % nbuf] = k + 1
        else:
            rk.in2_ver = k + 1
        state[r] = {"kind": kind, "pc": [0] * ctas, "epoch": [None] * ctas, "finished": 0}

    for r in range(world):
        start_call(r)

    steps = 0
    while any(call_idx[r] < len(kinds) for r in range(world)):
        steps += 1
        assert steps < 200000, "no progress"
        runnable = []
        for r in range(world):
            if call_idx[r] >= len(kinds):
                continue
            st, rk = state[r], ranks[r]
            k = call_idx[r]
            slot = "one" if st["kind"] == "one" else "A"
            for c in range(ctas):
                pc = st["pc"][c]
                e = st["epoch"][c]
                if pc == 0:
                    runnable.append((r, c))
                elif pc == 1:  # CTA 0 publishes, the others wait for go
                    if c == 0 or reached(rk.go, e):
                        runnable.append((r, c))
                elif pc == 2:  # CTA 0 waits for every rank's flag
                    if all(reached(v, e) for v in rk.flags[slot]):
                        runnable.append((r, c))
                elif pc in (3, 4):
                    runnable.append((r, c))
                elif pc == 5:  # two-shot exit exchange by the last CTA
                    if all(reached(v, e) for v in rk.flags["B"]):
                        runnable.append((r, c))
        assert runnable, "deadlock"
        r, c = rng.choice(runnable)
        st, rk = state[r], ranks[r]
        k = call_idx[r]
        pc = st["pc"][c]
        if pc == 0:
            st["epoch"][c] = rk.calls + 1
            assert st["epoch"][c] == k + 1, "CTAs of one call disagree on the call number"
            st["pc"][c] = 1
        elif pc == 1:
            e = st["epoch"][c]
            slot = "one" if st["kind"] == "one" else "A"
            if c == 0:
                for p in ranks:
                    p.flags[slot][r] = e
                st["pc"][c] = 2
            else:
                st["pc"][c] = 3
        elif pc == 2:
            rk.go = st["epoch"][c]
            st["pc"][c] = 3
        elif pc == 3:  # data phase
            e = st["epoch"][c]
            for p in ranks:
                if st["kind"] == "one":
                    assert p.in_ver[e % nbuf] == e, f"rank {r} read rank {p.r}'s IN of call {p.in_ver[e % nbuf]} for {e}"
                else:
                    assert p.in2_ver == e, f"rank {r} read rank {p.r}'s two-shot IN of call {p.in2_ver} for {e}"
                    p.out_writes.setdefault(e, set()).add((r, c))
            st["pc"][c] = 4
        elif pc == 4:  # exit
            e = st["epoch"][c]
            rk.done += 1
            if rk.done == ctas:
                if st["kind"] == "two":
                    for p in ranks:
                        p.flags["B"][r] = e
                    st["pc"][c] = 5
                    continue
                rk.done = 0
                rk.calls = e
            st["pc"][c] = 6
        elif pc == 5:
            rk.done = 0
            rk.calls = st["epoch"][c]
            st["pc"][c] = 6
        if all(x == 6 for x in st["pc"]):
            e = k + 1
            if st["kind"] == "two":
                # every rank's CTAs have written this rank's OUT rows before the call completes here
                assert len(rk.out_writes.get(e, ())) == world * ctas, "two-shot call completed before all stores"
            call_idx[r] += 1
            if call_idx[r] < len(kinds):
                start_call(r)
    return steps


def test_protocol_random_interleavings():
    mixes = [["one"] * 7, ["two"] * 5, ["one", "two", "one", "one", "two", "two", "one"]]
    for kinds in mixes:
        for world, ctas in ((2, 1), (2, 3), (3, 2), (4, 2)):
            for seed in range(150):
                run(kinds, world=world, ctas=ctas, seed=seed)


def test_model_catches_a_missing_rotation():
    # one-shot with a single IN buffer (no rotation): a rank that finished call k refills the
    # buffer for call k + 1 while a slower peer may still read call k.  The model must find it.
    found = False
    for seed in range(400):
        try:
            run(["one"] * 6, world=2, ctas=2, seed=seed, nbuf=1)
        except AssertionError as e:
            assert "read rank" in str(e)
            found = True
            break
    assert found
