"""Tile-ring protocol of the persistent attention kernel, simulated on the host.

attn_flat_gqa8_kernel (tinybrain_b200/csrc/tb_attention.cu) streams each chunk's
tiles (K of pages 0..np-1, then V of pages 0..np-1) through a ring of R data
slots; consumer warp w takes pages w, w + 4, ... in both passes, and a barrier
between the passes orders them.  A consumer waits for tile j with an mbarrier
parity wait, which only sees the parity of the barrier's phase count: it returns
as soon as the phase count differs in parity from the awaited one.  With one
full barrier per slot, a warp that is ahead may wait for tile j while tile
j - R (same slot) is still in flight; the barrier's phase count then has the
parity that tile j - 2R left, and the wait returns before tile j has landed.
The kernel therefore keeps 2R full barriers (tile j completes barrier j % 2R).

This test replays random schedules of that protocol and checks that with 2R
barriers no consumer ever passes a wait before its tile landed, and that with R
barriers some schedule does (the failure the 2R barriers remove).
"""
import random


def simulate(ring, nbar, np_pages, chunks, seed, warps=4):
    """Random interleaving of producer, copy engine and consumers.
    Returns the number of waits that passed before their tile had landed."""
    rng = random.Random(seed)
    # the consumer tile order of every warp, chunk by chunk, and barrier points
    order = [[] for _ in range(warps)]
    base = 0
    for _ in range(chunks):
        for w in range(warps):
            order[w].append(("tiles", [base + i for i in range(w, np_pages, warps)]))
            order[w].append(("bar", None))
            order[w].append(("tiles", [base + np_pages + i for i in range(w, np_pages, warps)]))
            order[w].append(("bar", None))
        base += 2 * np_pages
    total = base
    flat = [[] for _ in range(warps)]
    for w in range(warps):
        for kind, tiles in order[w]:
            if kind == "bar":
                flat[w].append(("bar", None))
            else:
                flat[w].extend(("tile", j) for j in tiles)
    pos = [0] * warps
    phases = [0] * nbar           # completed phases of each full barrier
    landed = [False] * total
    released = [False] * total
    issued = 0                    # tiles handed to the copy engine
    in_flight = []
    at_bar = set()
    bad = 0
    while any(pos[w] < len(flat[w]) for w in range(warps)) or in_flight:
        actors = []
        if issued < total and (issued < ring or released[issued - ring]):
            actors.append("produce")
        if in_flight:
            actors.append("land")
        for w in range(warps):
            if pos[w] < len(flat[w]) and w not in at_bar:
                kind, j = flat[w][pos[w]]
                if kind == "bar":
                    actors.append(("bar", w))
                else:
                    b = j % nbar
                    want = (j // nbar) & 1
                    if (phases[b] & 1) != want:  # the parity wait returns
                        actors.append(("take", w))
        if not actors:
            raise AssertionError("protocol deadlock")
        a = rng.choice(actors)
        if a == "produce":
            in_flight.append(issued)
            issued += 1
        elif a == "land":
            j = in_flight.pop(rng.randrange(len(in_flight)))
            landed[j] = True
            phases[j % nbar] += 1
        elif a[0] == "bar":
            at_bar.add(a[1])
            if len(at_bar) == warps:
                for w in range(warps):
                    pos[w] += 1
                at_bar.clear()
        else:
            w = a[1]
            j = flat[w][pos[w]][1]
            if not landed[j]:
                bad += 1
                landed[j] = True  # count it once; the kernel would read a stale slot
            released[j] = True
            pos[w] += 1
    return bad


def test_two_barriers_per_slot_never_pass_early():
    for seed in range(300):
        assert simulate(ring=10, nbar=20, np_pages=16, chunks=3, seed=seed) == 0


def test_one_barrier_per_slot_can_pass_early():
    # the schedule that stalled the kernel: some random interleaving passes a
    # wait before the tile landed when only R barriers exist
    def early(seed):
        try:
            return simulate(ring=10, nbar=10, np_pages=16, chunks=3, seed=seed) > 0
        except AssertionError:  # a stall counts too
            return True
    assert any(early(s) for s in range(300))
