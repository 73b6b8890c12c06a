"""CPU tier: the stream-K work schedule of the tcgen05 GEMM, restated in Python.

The persistent kernels (TcWorkIter in matrixflash_pro_b200/csrc/tc_kernel.cuh) deal the
first tiles out whole and cut the K blocks of the last sk_tiles tiles into one contiguous
range per worker; shared tiles leave partial sums in slot 2w (first tile of worker w's
range) or 2w + 1 (its last), and the fix-up kernel (streamk_reduce_kernel, gemm_tc.cu)
finds a tile's workers with tc_sk_owner and adds their slots in K order. These checks pin
the arithmetic both sides rely on: every (tile, K block) is computed exactly once, no two
shares of one launch use the same slot, and the fix-up's view of a tile's shares is the
workers' own. The GPU parity tests run the kernels themselves."""
import pytest


def owner(i, iters, workers):
    return ((i + 1) * workers - 1) // iters


def units(worker, workers, tiles, sk_tiles, kb):
    """The work units of one worker, as TcWorkIter::next yields them."""
    out = []
    dp = tiles - sk_tiles
    t = worker
    while t < dp:
        out.append((t, 0, kb, -1))
        t += workers
    iters = sk_tiles * kb
    i, e = iters * worker // workers, iters * (worker + 1) // workers
    first_rel = i // kb if kb else 0
    while i < e:
        rel = i // kb
        base = rel * kb
        kb0, kb1 = i - base, min(e - base, kb)
        whole = kb0 == 0 and kb1 == kb
        out.append((dp + rel, kb0, kb1, -1 if whole else (2 * worker if rel == first_rel else 2 * worker + 1)))
        i = base + kb
    return out


def streamk_tiles(tiles, workers, kb, min_blocks=8):
    """The host policy of gemm_tc.cu (streamk_tiles)."""
    if workers <= 1 or tiles <= 0 or kb <= 0:
        return 0
    if tiles < workers and tiles * 10 > workers * 6:
        return 0
    waves = -(-tiles // workers)
    if tiles * 10 >= waves * workers * 9:
        return 0
    full = tiles // workers
    sk = tiles - (full - 1) * workers if full >= 1 else tiles
    return 0 if sk * kb < min_blocks * workers else sk


def reduce_view(r, workers, sk_tiles, kb):
    """(workers, slots) the fix-up kernel adds for stream-K tile r, or None if one worker owns it."""
    iters = sk_tiles * kb
    w0, w1 = owner(r * kb, iters, workers), owner((r + 1) * kb - 1, iters, workers)
    if w0 == w1:
        return None
    slots = []
    for w in range(w0, w1 + 1):
        first_rel = (iters * w // workers) // kb
        slots.append(2 * w if r == first_rel else 2 * w + 1)
    return list(range(w0, w1 + 1)), slots


CASES = [(64, 74, 64), (128, 148, 64), (4, 74, 2048), (16, 148, 2048), (3, 148, 40), (200, 148, 30),
         (1376, 74, 128), (150, 148, 9), (90, 74, 13), (1, 148, 5000)]


@pytest.mark.parametrize("tiles,workers,kb", CASES)
def test_every_k_block_once_and_slots_distinct(tiles, workers, kb):
    sk = streamk_tiles(tiles, workers, kb)
    for forced in sorted({sk, min(tiles, workers), tiles}):
        if forced * kb < workers:
            continue  # a share of less than one K block per worker is never scheduled
        seen = {}
        slots = {}
        for w in range(workers):
            for (t, kb0, kb1, slot) in units(w, workers, tiles, forced, kb):
                assert 0 <= kb0 < kb1 <= kb and 0 <= t < tiles
                for k in range(kb0, kb1):
                    assert (t, k) not in seen, (t, k)
                    seen[(t, k)] = w
                if slot >= 0:
                    assert slot not in slots, f"slot {slot} used twice"
                    assert slot // 2 == w
                    slots[slot] = (t, kb0, kb1)
        assert len(seen) == tiles * kb
        # The fix-up kernel finds exactly the shares the workers stored, in K order.
        dp = tiles - forced
        for r in range(forced):
            view = reduce_view(r, workers, forced, kb)
            shares = sorted((v[1], s) for s, v in slots.items() if v[0] == dp + r)
            if view is None:
                assert not shares
                continue
            ws, ss = view
            assert [s for _, s in shares] == ss
            assert shares[0][0] == 0 and all(slots[s][0] == dp + r for s in ss)
            # consecutive shares meet: the K ranges tile [0, kb)
            ranges = [slots[s][1:] for s in ss]
            assert ranges[0][0] == 0 and ranges[-1][1] == kb
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))


def test_policy_picks_shapes_that_leave_workers_idle():
    # 2048^3 on 74 SM pairs: 64 tiles of 256 x 256 fill 86% of the pairs -> whole tiles
    # (measured faster than sharing); on 148 SMs with 128 x 128 tiles (1.73 waves) -> shared
    assert streamk_tiles(64, 74, 64) == 0
    assert streamk_tiles(256, 148, 64) == 256
    # 4096^3 on pairs: 256 tiles, 3.46 waves -> the last 1.46 waves' worth shared
    assert streamk_tiles(256, 74, 128) == 256 - 2 * 74
    # the linear layer 8192 x 11008 on pairs: 1376 tiles, 18.6 waves -> data parallel
    assert streamk_tiles(1376, 74, 128) == 0
    # 1.2 waves: the last ~1.2 waves are shared, earlier waves stay whole
    assert streamk_tiles(178, 148, 64) == 178
    assert streamk_tiles(3 * 148 + 20, 148, 64) == 148 + 20
    # too little K per worker: stay data parallel
    assert streamk_tiles(16, 74, 32) == 0
    assert streamk_tiles(4, 74, 2048) == 4


def test_split_of_the_2048_cube_on_pairs():
    # 4096 K blocks over 74 pairs: ~55 each, so every tile is shared by two or three pairs
    iters = 64 * 64
    spans = [owner((r + 1) * 64 - 1, iters, 74) - owner(r * 64, iters, 74) + 1 for r in range(64)]
    assert max(spans) == 3 and min(spans) == 2
