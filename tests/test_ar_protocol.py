"""Protocol model of the fused all-reduce's synchronisation, checked over interleavings (CPU).

The device kernel (csrc/kernels/allreduce.cu) relies on three facts:
  * each call's partial goes into slot (call % 2) of the writer's symmetric buffer;
  * one epoch barrier per call: a rank raises flag[rank] = call + 1 in every peer, waits until
    every peer's flag in its own buffer reached call + 1, then reads all peers' slots;
  * a rank's next GEMM (which overwrites a slot) starts only after its previous all-reduce ended
    (stream order).
This model executes those steps for several ranks under adversarial schedules (hypothesis picks
which rank moves next) and checks that no read ever sees a slot being overwritten or a stale
version. The same checker must find a violation when the partials use a single slot, which shows
the schedules are strong enough to exercise the race the double buffer prevents.
"""
from hypothesis import given, settings, strategies as st


def run_protocol(world, calls, schedule, slots=2):
    """Returns None if the schedule ran without violation, else a description of the first one."""
    ops = []
    for i in range(calls):
        ops += [("w_start", i), ("w_end", i), ("signal", i), ("wait", i), ("r_start", i), ("r_end", i)]
    pc = [0] * world
    flags = [[0] * world for _ in range(world)]          # flags[owner][src]
    version = [[-1] * slots for _ in range(world)]       # last completed write per (rank, slot)
    writing = [[False] * slots for _ in range(world)]
    readers = {}                                          # (rank, slot) -> set of readers
    k = 0
    while any(p < len(ops) for p in pc):
        movable = [r for r in range(world) if pc[r] < len(ops) and not (
            ops[pc[r]][0] == "wait" and min(flags[r]) < ops[pc[r]][1] + 1)]
        if not movable:
            return "deadlock"
        r = movable[schedule[k % len(schedule)] % len(movable)] if schedule else movable[0]
        k += 1
        op, i = ops[pc[r]]
        s = i % slots
        if op == "w_start":
            if readers.get((r, s)):
                return f"rank {r} overwrites slot {s} (call {i}) while {sorted(readers[(r, s)])} read it"
            writing[r][s] = True
        elif op == "w_end":
            writing[r][s] = False
            version[r][s] = i
        elif op == "signal":
            for p in range(world):
                flags[p][r] = i + 1
        elif op == "r_start":
            for p in range(world):
                if writing[p][s]:
                    return f"rank {r} reads slot {s} of rank {p} during a write"
                readers.setdefault((p, s), set()).add(r)
        elif op == "r_end":
            for p in range(world):
                if version[p][s] != i:
                    return f"rank {r} read version {version[p][s]} of rank {p} slot {s}, wanted {i}"
                readers[(p, s)].discard(r)
        pc[r] += 1
    return None


@settings(max_examples=400, deadline=None)
@given(world=st.integers(2, 8), calls=st.integers(1, 6),
       schedule=st.lists(st.integers(0, 63), min_size=1, max_size=200))
def test_double_buffered_epoch_barrier_has_no_race(world, calls, schedule):
    assert run_protocol(world, calls, schedule) is None


def test_single_slot_protocol_is_caught():
    """Without the second slot a fast rank overwrites a partial a slow peer is still reading."""
    import random
    found = None
    for seed in range(2000):
        rng = random.Random(seed)
        sched = [rng.randrange(64) for _ in range(64)]
        found = run_protocol(2, 3, sched, slots=1)
        if found:
            break
    assert found is not None


# ------------------------------------------------------------------------------------------------
# The decode GEMM with the all-reduce in its own launch (gemm_tcgen05.cu, ar_tail).
#
# Per rank, launch i runs `ctas` CTAs at once; each CTA pushes its part of every token row into
# the owner rank's push slot (i % slots), then raises its own phase-0 flag = i + 1 in every rank.
# The owner's reducing CTA waits for the phase-0 flags of every CTA of every rank, reads all
# sources' parts of its row, writes the normed row into every rank and raises its phase-1 flag
# everywhere (a rank that owns no row has no reducing CTA and raises nothing). CTA 0 waits for the
# phase-1 flags of every rank's reducing CTAs; the launch ends when all CTAs finished, and then the
# next kernel (the consumer) reads the normed rows before launch i + 1 starts.
# ------------------------------------------------------------------------------------------------
def run_gemm_ar_protocol(world, ctas, rows, calls, schedule, slots=2, wait0=True, wait1=True):
    owner_of = [r for r in range(rows)]                   # rank r owns row r (rows <= world)
    slot = [[[[-1] * ctas for _ in range(world)] for _ in range(slots)] for _ in range(world)]
    normed = [[-1] * rows for _ in range(world)]           # normed[rank][row] = call that wrote it
    # flags[rank][phase][src][cta] = last epoch raised there
    flags = [[[[0] * ctas for _ in range(world)] for _ in range(2)] for _ in range(world)]
    reading_slot = [set() for _ in range(world)]           # slots a rank's reducer is reading
    reading_normed = [False] * world
    call = [0] * world
    progs, pcs = {}, {}
    reducers = lambda r: 1 if r < rows else 0  # noqa: E731  (one reducing CTA per owned row here)

    def program(r, c):
        p = [("push",), ("signal", 0)]
        if c < reducers(r):
            p += ([("wait", 0)] if wait0 else []) + [("read_start",), ("read_end",), ("write_normed",),
                                                   ("signal", 1)]
        if c == 0:
            p += [("wait", 1)] if wait1 else []
        return p

    def ready(r, phase, e):
        if phase == 0:
            return all(flags[r][0][src][c] >= e for src in range(world) for c in range(ctas))
        return all(flags[r][1][src][c] >= e for src in range(world) for c in range(reducers(src)))

    def start_launch(r):
        for c in range(ctas):
            progs[(r, c)] = program(r, c)
            pcs[(r, c)] = 0
        progs[(r, "consumer")] = None

    for r in range(world):
        start_launch(r)
    k = 0
    while True:
        live = [key for key, p in progs.items() if p is not None and pcs.get(key, 0) < len(p)]
        # a rank whose CTAs are all done runs its consumer, then the next launch
        for r in range(world):
            if call[r] >= calls:
                continue
            if all(pcs[(r, c)] >= len(progs[(r, c)]) for c in range(ctas)) and progs[(r, "consumer")] is None:
                progs[(r, "consumer")] = [("cread_start",), ("cread_end",)]
                pcs[(r, "consumer")] = 0
                live.append((r, "consumer"))
        if not live:
            break
        movable = []
        for key in live:
            op = progs[key][pcs[key]]
            r = key[0]
            if op[0] == "wait" and not ready(r, op[1], call[r] + 1):
                continue
            movable.append(key)
        if not movable:
            return "deadlock"
        key = movable[schedule[k % len(schedule)] % len(movable)] if schedule else movable[0]
        k += 1
        r, c = key
        i = call[r]
        e = i + 1
        s = i % slots
        op = progs[key][pcs[key]]
        if op[0] == "push":
            for d in range(world):
                if s in reading_slot[d]:
                    return f"rank {r} cta {c} pushes call {i} into slot {s} of rank {d} during its read"
                slot[d][s][r][c] = i
        elif op[0] == "signal":
            for d in range(world):
                flags[d][op[1]][r][c] = e
        elif op[0] == "read_start":
            for src in range(world):
                for cc in range(ctas):
                    if slot[r][s][src][cc] != i:
                        return f"rank {r} reduces call {i} but slot {s} holds call {slot[r][s][src][cc]} of {src}"
            reading_slot[r].add(s)
        elif op[0] == "read_end":
            reading_slot[r].discard(s)
        elif op[0] == "write_normed":
            for d in range(world):
                if reading_normed[d]:
                    return f"rank {r} writes normed row (call {i}) into rank {d} while its consumer reads"
                normed[d][owner_of.index(r)] = i
        elif op[0] == "cread_start":
            for row in range(rows):
                if normed[r][row] != i:
                    return f"consumer of rank {r} reads row {row} from call {normed[r][row]}, wanted {i}"
            reading_normed[r] = True
        elif op[0] == "cread_end":
            reading_normed[r] = False
            call[r] += 1
            progs[(r, "consumer")] = None
            if call[r] < calls:
                start_launch(r)
            else:
                for cc in range(ctas):
                    progs[(r, cc)] = None
            continue
        pcs[key] += 1
    return None


@settings(max_examples=300, deadline=None)
@given(world=st.integers(1, 8), ctas=st.integers(1, 3), rows_frac=st.integers(0, 8), calls=st.integers(1, 4),
       slots=st.integers(1, 2), schedule=st.lists(st.integers(0, 63), min_size=1, max_size=300))
def test_gemm_allreduce_two_phase_protocol_has_no_race(world, ctas, rows_frac, calls, slots, schedule):
    """No race with two push slots, nor with one: phase 1 already keeps the next launch's pushes
    away from a slot that is still being read."""
    rows = max(1, min(world, rows_frac))
    assert run_gemm_ar_protocol(world, ctas, rows, calls, schedule, slots=slots) is None


def _find_violation(**kw):
    import random
    for seed in range(3000):
        rng = random.Random(seed)
        sched = [rng.randrange(64) for _ in range(120)]
        v = run_gemm_ar_protocol(3, 2, 2, 3, sched, **kw)
        if v:
            return v
    return None


def test_gemm_allreduce_protocol_without_phase0_wait_is_caught():
    """A reducer that does not wait for every rank's pushes reads an incomplete row."""
    assert _find_violation(wait0=False) is not None


def test_gemm_allreduce_protocol_without_phase1_wait_is_caught():
    """Without CTA 0's final wait the consumer can read normed rows a peer has not written yet."""
    assert _find_violation(wait1=False) is not None
