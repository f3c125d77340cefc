"""Row maps of the peer-memory expert-parallel exchange, checked against a direct simulation."""
import numpy as np

from rl_project_b200.parallel.expert_p2p import ALIGN, build_maps


def test_maps_route_every_slot_to_its_expert_and_back():
    rng = np.random.default_rng(0)
    world, El = 4, 3
    E = world * El
    cnt = rng.integers(0, 200, size=(world, E))
    cnt[1, 4] = 0
    cnt[:, 7] = 0  # an expert nobody routes to
    maps = [build_maps(cnt, r, El) for r in range(world)]
    # every source's slots, expert-sorted, tagged (source, expert, index)
    slots = [[(s, e, i) for e in range(E) for i in range(cnt[s, e])] for s in range(world)]
    for o, m in enumerate(maps):
        R = len(m["d_rank"])
        assert R % ALIGN == 0 and R == m["seg_len"].sum() and m["tile_group"].size == R // ALIGN
        for row in range(R):
            j = np.searchsorted(np.cumsum(m["seg_len"]), row, side="right")
            if m["d_rank"][row] < 0:
                continue
            s, e, _ = slots[m["d_rank"][row]][m["d_row"][row]]
            assert e == o * El + j  # the row sits in its expert's segment
            assert m["tile_group"][row // ALIGN] == j
        got = sorted(slots[m["d_rank"][r]][m["d_row"][r]] for r in range(R) if m["d_rank"][r] >= 0)
        want = sorted(t for s in range(world) for t in slots[s] if t[1] // El == o)
        assert got == want  # every slot of the owner's experts arrives exactly once
    for s in range(world):
        m = maps[s]
        assert len(m["c_rank"]) == len(slots[s])
        for i, (src, e, idx) in enumerate(slots[s]):
            o, row = m["c_rank"][i], m["c_row"][i]
            assert o == e // El
            assert (maps[o]["d_rank"][row], maps[o]["d_row"][row]) == (s, i)  # combine inverts dispatch
