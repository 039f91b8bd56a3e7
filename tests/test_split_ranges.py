"""The split-KV decode kernel's tile ranges (vllm_quantpack_b200/csrc/qp_decode.cu, decode_kernel: win_lo, tile_lo,
tps, tile0, ntl; qp_paged_decode: the tokens_after_keys clamp), restated on the host: over random contexts, query
token counts, sliding windows, tokens after the keys and split counts, every key a query row may see lies in exactly
one split's tiles, and a split holds no tile past the context. A tile outside every split is never read, so a key
missing here would silently drop out of the attention. Also the fact the kernel's row states rely on: a row with no
key in the first tile of its split meets its first key in a tile the kernel computes with both bounds."""
import numpy as np

TILE = 128


def kernel_ranges(n, qlen, window, after, splits):
    """(vis_base, win_hi, [(tile0, ntl)] per split) as decode_kernel computes them."""
    after = min(after, qlen + window)                      # qp_paged_decode's clamp (window 0: qlen)
    vis_base = n - qlen + after
    win_lo = max(0, vis_base - window + 1) if window > 0 else 0
    tile_lo = win_lo // TILE
    n_tiles = (n + TILE - 1) // TILE
    tps = max(0, -(-(n_tiles - tile_lo) // splits))
    ranges = []
    for s in range(splits):
        tile0 = tile_lo + s * tps
        ranges.append((tile0, max(0, min(tile0 + tps, n_tiles) - tile0)))
    win_hi = vis_base + qlen - window if window > 0 else -1
    return vis_base, win_hi, ranges


def visible(n, qlen, window, after, i):
    """Keys token i of the call sees: causal (its position is n - qlen + i + after) and inside its window."""
    last = min(n - 1, n - qlen + i + after)
    first = max(0, n - qlen + i + after - window + 1) if window > 0 else 0
    return first, last


def test_every_visible_key_is_in_exactly_one_split():
    rng = np.random.default_rng(0)
    for _ in range(3000):
        n = int(rng.integers(1, 6000))
        qlen = int(rng.integers(1, 5)) if rng.random() < 0.7 else int(rng.integers(1, 33))
        qlen = min(qlen, n + 32)
        window = 0 if rng.random() < 0.2 else int(rng.integers(1, 3000))
        after = 0 if rng.random() < 0.6 else int(rng.integers(0, 4000))
        splits = int(rng.integers(1, 40))
        vis_base, win_hi, ranges = kernel_ranges(n, qlen, window, after, splits)
        owner = np.full(-(-n // TILE) + 1, -1)
        for s, (t0, ntl) in enumerate(ranges):
            assert t0 >= 0 and (ntl == 0 or t0 + ntl <= -(-n // TILE)), (n, qlen, window, after, splits)
            for t in range(t0, t0 + ntl):
                assert owner[t] == -1, "a tile in two splits"
                owner[t] = s
        for i in range(qlen):
            first, last = visible(n, qlen, window, after, i)
            if first > last:
                continue
            for t in range(first // TILE, last // TILE + 1):
                assert owner[t] >= 0, (n, qlen, window, after, splits, i, t)
            # the window's masked tiles reach every token's first key (before clamping to the context's start)
            if window > 0:
                assert win_hi >= vis_base + i - window + 1, "the last token's first key bounds every token's"


def test_a_row_opens_in_a_tile_computed_with_both_bounds():
    """With a window, a row whose first key lies beyond the first tile of its split opens in a tile that starts at
    or before win_hi (the last token's first key), which the kernel computes on its masked path."""
    rng = np.random.default_rng(1)
    for _ in range(3000):
        n = int(rng.integers(129, 6000))
        qlen = int(rng.integers(1, 33))
        window = int(rng.integers(1, 3000))
        after = 0 if rng.random() < 0.6 else int(rng.integers(0, 400))
        splits = int(rng.integers(1, 40))
        vis_base, win_hi, ranges = kernel_ranges(n, qlen, window, after, splits)
        for t0, ntl in ranges:
            if ntl == 0:
                continue
            for i in range(qlen):
                first, last = visible(n, qlen, window, after, i)
                if first > last or first < (t0 + 1) * TILE or first >= (t0 + ntl) * TILE:
                    continue
                assert (first // TILE) * TILE <= win_hi, (n, qlen, window, after, splits, i)
