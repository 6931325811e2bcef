"""The forward main kernel's work decomposition, on the CPU.

Restates the host's unit parameters (csrc/capi.cpp: `make_layout`, `enqueue_main`) and
the kernel's decode (csrc/swa_kernels.cu: `decode_unit`, `tile_of`) over a sweep of
shapes: whole sequences (plain, causal, a radius per head) and sequence shards.  It checks
the properties the kernel relies on:

* an active query tile has at least one member key tile.  Without one, its softmax warps
  wait for an accumulator that no P*V fills; the barrier model in test_fwd_protocol.py
  assumes this;
* every key a query row must see in the band (inside the keys the problem holds) lies in a
  member band tile of the row's query tile;
* the global-row units' splits cover every key tile of the shard exactly once, each split
  holding at least one tile;
* no band tile lies wholly outside the keys the problem holds;
* in a shard, every band tile lies wholly in the left halo, the shard or the right halo.
  A tile may straddle the shard's end only in the last shard, where the part past the end
  is zero-filled.
"""
import pytest

from long_context_attention.distributed import shard_bounds

T = 128              # query rows / keys per tile (BM = BN = kTileRows)
MIN_GROW_UNITS = 148


def cdiv(a, b):
    assert a >= 0 and b > 0
    return (a + b - 1) // b


def params(n, window, G, bh, q_off=0, n_total=None, world=1, causal=False, head_window=()):
    sharded = world > 1
    n_total = n if n_total is None else n_total
    window = min(window, n_total)                      # the host clamps radii to the sequence
    head_window = [min(h, n_total) for h in head_window]
    lead = cdiv(window, T) * T if sharded else window
    p = dict(n=n, q_off=q_off, n_total=n_total, sharded=sharded, window=window, lead=lead, bh=bh, G=G,
             causal=causal, head_window=list(head_window), halo=window if sharded else 0)
    if sharded:
        p["key_lo"], p["key_hi"] = max(0, q_off - window), min(n_total, q_off + n + window)
    else:
        p["key_lo"], p["key_hi"] = 0, n
    p["gk_lo"], p["gk_n"] = q_off, n
    p["q_tiles"] = cdiv(n, T)
    p["q_pairs"] = (p["q_tiles"] + 1) // 2
    p["g_tiles"] = p["n_splits"] = p["split_tiles"] = p["n_grow_units"] = 0
    if G > 0:
        g_tiles = cdiv(G, T)
        key_tiles = cdiv(n, T)
        band_tiles = (lead + window + 2 * T - 1) // T + g_tiles
        split = max(4, min(64, 4 * band_tiles))
        while split > 2 and bh * g_tiles * cdiv(key_tiles, split) < MIN_GROW_UNITS:
            split -= 2
        split += split & 1
        p.update(g_tiles=g_tiles, split_tiles=split, n_splits=cdiv(key_tiles, split),
                 n_grow_units=bh * g_tiles * cdiv(key_tiles, split))
    p["n_band_units"] = bh * p["q_pairs"]
    return p


def band_unit(p, t):
    pair, bh = t % p["q_pairs"], t // p["q_pairs"]
    q0 = pair * 2 * T
    active = [True, q0 + T < p["n"]]
    hw = p["head_window"]
    w = hw[bh % len(hw)] if hw else p["window"]
    lead = w if hw else p["lead"]
    kstart = p["q_off"] + q0 - lead
    nA = (lead + T - 1) // T + 1 if p["causal"] else (lead + w + T + T - 1) // T
    p_first = (p["key_lo"] - kstart) // T if kstart < p["key_lo"] else 0
    p_last = nA if active[1] else nA - 1
    assert p["key_hi"] - 1 - kstart >= 0
    p_last = min(p_last, (p["key_hi"] - 1 - kstart) // T)
    num_band = p_last - p_first + 1
    tiles = []
    for j in range(num_band + p["g_tiles"]):
        if j < num_band:
            pp = p_first + j
            tiles.append(dict(row0=kstart + pp * T, global_key=False, mem=[pp <= nA - 1, active[1] and pp >= 1]))
        else:
            tiles.append(dict(row0=(j - num_band) * T, global_key=True, mem=[True, active[1]]))
    return dict(q0=q0, active=active, w=w, tiles=tiles, num_band=num_band)


def grow_unit(p, t):
    split, rest = t % p["n_splits"], t // p["n_splits"]
    k0 = p["gk_lo"] + split * p["split_tiles"] * T
    rem = cdiv(p["gk_lo"] + p["gk_n"] - k0, T)
    ntiles = min(rem, p["split_tiles"])
    return dict(active=[True, ntiles >= 2], split=split, gt=rest % p["g_tiles"], bh=rest // p["g_tiles"],
                tiles=[dict(row0=k0 + j * T, mem=[j % 2 == 0, j % 2 == 1]) for j in range(ntiles)])


def check(p):
    for t in range(p["n_band_units"]):
        un = band_unit(p, t)
        w = un["w"]
        for x in range(2):
            if not un["active"][x]:
                assert not any(tl["mem"][x] for tl in un["tiles"])
                continue
            assert any(tl["mem"][x] for tl in un["tiles"]), f"active query tile {x} of unit {t} has no member tile"
            starts = sorted(tl["row0"] for tl in un["tiles"] if tl["mem"][x] and not tl["global_key"])
            # the member band tiles are one contiguous run, so the band of every row of the
            # query tile is covered once the first and last keys of its first and last rows are
            assert starts == list(range(starts[0], starts[-1] + 1, T)) if starts else True
            lo_row = p["q_off"] + un["q0"] + x * T
            hi_row = min(lo_row + T, p["q_off"] + p["n"]) - 1
            for i in (lo_row, hi_row):
                keys_lo = max(i - w, p["key_lo"])
                keys_hi = min(i if p["causal"] else i + w, p["key_hi"] - 1)
                for key in {keys_lo, keys_hi} if keys_hi >= keys_lo else ():
                    assert any(s <= key < s + T for s in starts), f"key {key} of row {i} in no member tile"
        for tl in un["tiles"]:
            if not tl["global_key"]:
                assert tl["row0"] < p["key_hi"] and tl["row0"] + T > p["key_lo"], "band tile outside the keys held"
        if p["sharded"]:
            lo, hi = p["q_off"], p["q_off"] + p["n"]
            for tl in un["tiles"]:
                if tl["global_key"]:
                    continue
                s = tl["row0"]
                assert (s - lo) % T == 0, "band tile not aligned to the shard start"
                if s < lo:
                    assert s + T <= lo
                elif s < hi:
                    assert s + T <= hi or hi == p["n_total"], "band tile straddles the shard's end"
                else:
                    assert s < hi + p["halo"]
    seen = {}
    for t in range(p["n_grow_units"]):
        un = grow_unit(p, t)
        assert un["tiles"], "empty split"
        for tl in un["tiles"]:
            assert sum(tl["mem"]) == 1
            seen.setdefault((un["bh"], un["gt"]), []).append(tl["row0"])
    assert len(seen) == p["bh"] * p["g_tiles"]
    for rows in seen.values():
        assert sorted(rows) == [p["gk_lo"] + i * T for i in range(cdiv(p["n"], T))], "splits do not tile the keys"


NS = [1, 5, 127, 128, 129, 255, 256, 257, 300, 700, 1000, 4096]
WINDOWS = [0, 1, 17, 64, 127, 128, 129, 255, 256, 300, 1000, 5000]


@pytest.mark.parametrize("n", NS)
def test_whole_sequence_units(n):
    for w in WINDOWS:
        for G in (0, 1, 65, 200):
            if G > n:
                continue
            for bh in (1, 3):
                check(params(n, w, G, bh))
                check(params(n, w, G, bh, causal=True))
        check(params(n, w, 3, 4, head_window=(w, max(0, w // 3), w + 70, 1)))


@pytest.mark.parametrize("n_total,world", [(1000, 2), (4096, 2), (4096, 3), (4096, 4), (65536, 8), (131072, 8),
                                           (5000, 4), (2177, 3), (129, 2), (300, 2)])
def test_sequence_shard_units(n_total, world):
    for w in (0, 1, 64, 127, 128, 129, 256, 512, 700):
        for G in (0, 16, 65):
            if G > n_total:
                continue
            for off, ln in shard_bounds(n_total, world):
                check(params(ln, w, G, 2, q_off=off, n_total=n_total, world=world))
