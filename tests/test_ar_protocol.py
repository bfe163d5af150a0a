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
