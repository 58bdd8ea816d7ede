"""Host-side check of the stream-K tail's schedule (CPU).

A restatement, in Python, of the planner (`plan_stream_k` in csrc/ce_linear.cu)
and of the per-cluster unit lists (`Sched::cluster_units`, `sched_unit` in
csrc/tc_gemm.cuh), with the same integer formulas. It checks the invariants
the kernel relies on, for many shapes: every k block of every tile lies in
exactly one unit; a cluster holds at most one earlier part (one partial slot
per cluster); each finishing part's slot range [fix_lo, fix_hi) is exactly the
clusters holding that tile's earlier parts, in k order; within a cluster the
earlier part comes before the finishing part (a cluster publishes before it
waits, and waits only on lower clusters). The GPU tests check the kernel
itself (tests/test_gpu_stream_k.py).
"""

import random

MAX_PARTS = 3     # kSkMaxParts
MIN_SAVED = 24    # the default of soup_gemm_set_stream_k_min_saved


def plan(tiles, kb, max_cl, min_saved=MIN_SAVED, slots=74):
    """(sk_tiles, sk_clusters, clusters launched) or None when the tail stays a partial wave."""
    if tiles % max_cl == 0:
        return None
    sk = tiles % max_cl if tiles > max_cl else tiles
    iters = sk * kb
    skc = min(max_cl, sk * MAX_PARTS, iters)
    if skc <= sk or skc > slots or (iters + 1) * (skc + 1) >= 2 ** 31:
        return None
    if (iters + skc - 1) // skc + min_saved > kb:
        return None
    return sk, skc, (max_cl if tiles > max_cl else skc)


def units(tiles, kb, sk, skc, n_clusters):
    """Per cluster: [(tile, kb0, kb1, role, fix_lo, fix_hi)] in processing order."""
    s = sk * kb
    t_whole = tiles - sk
    out = {}
    for c in range(n_clusters):
        lst = []
        g0, g1 = (s * c // skc, s * (c + 1) // skc) if c < skc else (0, 0)
        n_sk = 0 if g1 <= g0 else (2 if g0 // kb != (g1 - 1) // kb else 1)
        for i in range(n_sk):
            t0 = g0 // kb
            if n_sk == 2 and i == 0:
                t, lo, hi = t0 + 1, (t0 + 1) * kb, g1
            elif n_sk == 2:
                t, lo, hi = t0, g0, (t0 + 1) * kb
            else:
                t, lo, hi = t0, g0, g1
            k0, k1 = lo - t * kb, hi - t * kb
            role, fl, fh = "whole", 0, 0
            if k1 < kb:
                role = "part"
            elif k0 > 0:
                role, fl, fh = "finish", ((t * kb + 1) * skc - 1) // s, c
            lst.append((t_whole + t, k0, k1, role, fl, fh))
        n = (t_whole - c + n_clusters - 1) // n_clusters if c < t_whole else 0
        lst += [(c + i * n_clusters, 0, kb, "whole", 0, 0) for i in range(n)]
        out[c] = lst
    return out


def check(tiles, kb, max_cl=74, min_saved=MIN_SAVED):
    p = plan(tiles, kb, max_cl, min_saved)
    if p is None:
        return None
    sk, skc, n_clusters = p
    lists = units(tiles, kb, sk, skc, n_clusters)
    covered, parts = {}, {}
    for c, lst in lists.items():
        assert sum(u[3] == "part" for u in lst) <= 1, (tiles, kb, c)
        finished = False
        for t, k0, k1, role, fl, fh in lst:
            for k in range(k0, k1):
                assert (t, k) not in covered, (tiles, kb, t, k)
                covered[(t, k)] = c
            if role == "part":
                assert not finished, "an earlier part after the finishing part"
                parts.setdefault(t, []).append((k0, c))
            finished |= role == "finish"
    assert len(covered) == tiles * kb
    finishers = []
    for c, lst in lists.items():
        for t, k0, k1, role, fl, fh in lst:
            if role == "finish":
                finishers.append(t)
                ordered = sorted(parts.get(t, []))
                assert [c2 for _, c2 in ordered] == list(range(fl, fh)), (tiles, kb, t)
                assert ordered[0][0] == 0 and fh == c
    assert sorted(finishers) == sorted(parts), (tiles, kb)
    return max(sum(u[2] - u[1] for u in lst) for lst in lists.values())


def test_schedule_invariants_at_the_qlora_shapes():
    # 256 x 256 pair tiles at 8192 tokens: K = 8960 / 17920 (141 / 281 k blocks) take the tail
    for tiles, kb in ((192, 141), (192, 281)):
        longest = check(tiles, kb)
        assert longest is not None and longest < 3 * kb  # shorter than the third, partial wave
    # K = 1536 (25 k blocks): the tail would save too little, the partial wave stays
    assert check(192, 25) is None and check(256, 25) is None and check(2240, 25) is None


def test_schedule_invariants_for_random_shapes_with_every_tail_forced():
    rng = random.Random(0)
    for _ in range(400):
        check(rng.randint(1, 600), rng.randint(1, 120), min_saved=0)
