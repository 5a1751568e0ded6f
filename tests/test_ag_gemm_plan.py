"""Gather / tile order of the fused all-gather + GEMM (host side, CPU)."""

from dtensor_muon_b200.parallel.ag_gemm import gather_plan


def _src(rows, world):
    out = []
    for n in rows:
        for r in range(0, n, 128):
            out.append(r // (n // world))
    return out


def test_plan_local_first_then_next_ranks():
    rows = [4096, 1024, 1024]  # q, k, v of Llama-3-8B
    for world in (1, 2, 4, 8):
        src = _src(rows, world)
        for rank in range(world):
            order, tiles, local = gather_plan(rows, rank, world)
            assert sorted(order) == list(range(len(src)))
            assert sorted(tiles) == list(range(len(src) // 2))
            dist_ = [(src[c] - rank) % world for c in order]
            assert dist_ == sorted(dist_), "chunks must come own rank first, then rank + 1, ..."
            assert local == sum(1 for s in src if s == rank)
            assert all(src[c] == rank for c in order[:local])
            pos = {c: i for i, c in enumerate(order)}
            keys = [max(pos[2 * t], pos[2 * t + 1]) for t in tiles]
            assert keys == sorted(keys)
