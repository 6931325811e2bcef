"""The backward's work decomposition, on the CPU: every visible (query, key) pair reaches
dQ of its query and dK / dV of its key exactly once.

Restates the host's unit parameters (csrc/capi.cpp: `make_bwd_layout`, the BwdParams of
`lca_swa_backward`) and the kernel's unit decode and per-column masks
(csrc/swa_backward.cu: `bwd_decode`, `tile_row0`, the P / dS warps' [lo, hi] range and
global-row bitmap, the epilogue's write rule and `lca_bwd_reduce`):

* band units (outer tile against its band's inner tiles, global inner rows masked, plus the
  compact global tiles) write the outer rows that are not global tokens;
* global units (compact global outer rows against one split of all inner rows) write
  partials that the reduce sums into the global tokens' rows.

The count of each (query, key) pair in what is written must equal the reference's mask
(python/long_context_attention/__init__.py:46-47) as an 0/1 matrix.
"""
import numpy as np
import pytest

BM, BN = 128, 64  # outer tile rows, inner tile rows


def cdiv(a, b):
    return (a + b - 1) // b


def layout(n, w, G):
    p = dict(n=n, w=w, G=G, n_tiles=cdiv(n, BM), g_tiles=0, gi_tiles=0, split_tiles=0, n_splits=0)
    if G > 0:
        p["g_tiles"], p["gi_tiles"] = cdiv(G, BM), cdiv(G, BN)
        band_tiles = (2 * w + BM + 2 * BN - 1) // BN + p["gi_tiles"]
        p["split_tiles"] = max(16, min(128, 2 * band_tiles))
        p["n_splits"] = cdiv(cdiv(n, BN), p["split_tiles"])
    p["n_band_units"] = p["n_tiles"]                       # one (batch, head)
    p["n_units"] = p["n_band_units"] + p["g_tiles"] * p["n_splits"]
    return p


def decode(p, u):
    n_all = p["n_units"] - p["n_band_units"]
    if u < n_all:
        split, rest = u % p["n_splits"], u // p["n_splits"]
        inner0 = split * p["split_tiles"] * BN
        return dict(all=True, outer0=(rest % p["g_tiles"]) * BM, inner0=inner0,
                    n_cont=min(cdiv(p["n"] - inner0, BN), p["split_tiles"]), n_comp=0)
    b = u - n_all
    outer0 = b * BM
    lo, hi = max(0, outer0 - p["w"]), min(p["n"] - 1, outer0 + BM - 1 + p["w"])
    return dict(all=False, outer0=outer0, inner0=lo, n_cont=(hi - lo + BN) // BN, n_comp=p["gi_tiles"])


def counts(n, w, gl):
    """(cnt_q, cnt_k): cnt_q[i, j] counts pair (query i, key j) in what the dQ kernel writes
    for row i; cnt_k[i, j] the same for the dK / dV kernel's row j."""
    G = len(gl)
    p = layout(n, w, G)
    is_g = np.zeros(n + 64, dtype=bool)
    is_g[gl] = True
    gidx = np.asarray(gl, dtype=np.int64)
    out = []
    for km in (False, True):
        cnt = np.zeros((n, n), dtype=np.int64)
        for u in range(p["n_units"]):
            un = decode(p, u)
            r = np.arange(BM)
            orow = un["outer0"] + r
            row_ok = orow < (G if un["all"] else n)
            # the epilogue: band units write outer rows that are not global; global units write
            # partials for their compact rows, which the reduce adds to the global tokens' rows
            if un["all"]:
                writes, target = row_ok, np.where(row_ok, gidx[np.minimum(orow, max(G - 1, 0))] if G else 0, 0)
            else:
                writes, target = row_ok & ~is_g[np.minimum(orow, n - 1)], orow
            for t in range(un["n_cont"] + un["n_comp"]):
                cont = t < un["n_cont"]
                tile0 = un["inner0"] + t * BN if cont else (t - un["n_cont"]) * BN
                c = np.arange(BN)
                if un["all"]:
                    lo, hi = np.zeros(BM, np.int64), np.where(row_ok, n - 1 - tile0, -1)
                elif cont:
                    lo = orow - tile0 - w
                    hi = np.minimum(orow - tile0 + w, n - 1 - tile0)
                    hi = np.where(row_ok, hi, -1)
                else:
                    lo, hi = np.zeros(BM, np.int64), np.where(row_ok, G - 1 - tile0, -1)
                vis = (c[None, :] >= lo[:, None]) & (c[None, :] <= hi[:, None])
                if cont and not un["all"] and G > 0:
                    vis &= ~is_g[tile0 + c][None, :]          # global inner rows: counted elsewhere
                vis &= writes[:, None]
                rr, cc = np.nonzero(vis)
                inner = (tile0 + cc) if cont else gidx[tile0 + cc]
                outer = target[rr]
                q, k = (inner, outer) if km else (outer, inner)
                np.add.at(cnt, (q, k), 1)
        out.append(cnt)
    return out


def mask(n, w, gl):
    i = np.arange(n)
    m = np.abs(i[:, None] - i[None, :]) <= w
    g = np.zeros(n, dtype=bool)
    g[gl] = True
    return (m | g[None, :] | g[:, None]).astype(np.int64)


CASES = [(1, 0, []), (5, 1, [2]), (63, 3, [0, 62]), (64, 64, [10]), (65, 17, []), (127, 0, [126]),
         (128, 30, [0, 5, 127]), (129, 128, [128]), (200, 17, list(range(0, 200, 7))), (300, 100, [0, 299]),
         (511, 63, list(range(3, 511, 4))), (640, 40, list(range(0, 640, 4))), (700, 1000, [1, 350]),
         (700, 256, list(range(0, 700, 10)))]


@pytest.mark.parametrize("n,w,gl", CASES)
def test_every_visible_pair_reaches_each_gradient_once(n, w, gl):
    w = min(w, n)  # the host clamps the radius to the sequence
    cnt_q, cnt_k = counts(n, w, sorted(set(gl)))
    want = mask(n, w, sorted(set(gl)))
    assert np.array_equal(cnt_q, want), "dQ"
    assert np.array_equal(cnt_k, want), "dK / dV"
