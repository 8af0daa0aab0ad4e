"""Host restatement of the decode GEMM's work decomposition
(cuda_optimazation_b200/csrc/gemm_skinny.cu, UnitRange / SegCursor): every
(tile, K-block) unit is computed exactly once, each CTA has at most two
partially owned ("split") tiles -- the two fp32 partial slices the workspace
holds per CTA -- whole tiles are walked last, and the contributor formula the
epilogue uses names exactly the CTAs that own a split tile's units."""
import pytest


def unit_range(T, nkb, c, G):
    wn = T // G
    split_tiles = T - wn * G
    if split_tiles > 0 and split_tiles * nkb < G:  # too few split units: all stream-K
        wn, split_tiles = 0, T
    su = split_tiles * nkb
    return dict(nkb=nkb, wn=wn, split_tiles=split_tiles, su=su,
                su0=su * c // G, su1=su * (c + 1) // G, wt0=split_tiles + c * wn)


def segments(r):
    nkb, su0, su1 = r["nkb"], r["su0"], r["su1"]
    segs = []
    if su1 > su0:
        lo, hi = su0 // nkb, (su1 - 1) // nkb
        order = [lo] if lo == hi else [hi, lo] + list(range(lo + 1, hi))
        for t in order:
            kb_lo = su0 - t * nkb if t == lo else 0
            kb_hi = su1 - t * nkb if t == hi else nkb
            segs.append((t, kb_lo, kb_hi, True))
    for t in range(r["wt0"], r["wt0"] + r["wn"]):
        segs.append((t, 0, nkb, False))
    return segs


def contributor(u, G, su):
    return ((u + 1) * G - 1) // su


@pytest.mark.parametrize("T,nkb,G", [(224, 16, 148), (224, 32, 148), (3, 16, 48), (296, 16, 148),
                                     (100, 1, 148), (7, 2, 5), (224, 16, 1), (449, 16, 148),
                                     (156, 16, 148), (150, 16, 148), (149, 1, 148)])
def test_schedule(T, nkb, G):
    G = min(G, T * nkb)  # the host never launches more CTAs than units
    seen = {}
    owners = {}
    for c in range(G):
        r = unit_range(T, nkb, c, G)
        segs = segments(r)
        partial = [s for s in segs if s[3] and (s[2] - s[1]) < nkb]
        assert len(partial) <= 2
        # whole tiles after all split segments
        flags = [s[3] for s in segs]
        assert flags == sorted(flags, reverse=True)
        assert sum(s[2] - s[1] for s in segs) == (r["su1"] - r["su0"]) + r["wn"] * nkb
        for t, a, b, split in segs:
            for kb in range(a, b):
                assert (t, kb) not in seen
                seen[(t, kb)] = c
                owners.setdefault(t, set()).add(c)
    assert len(seen) == T * nkb
    r0 = unit_range(T, nkb, 0, G)
    for t, cs in owners.items():
        if t < r0["split_tiles"]:
            cf = contributor(t * nkb, G, r0["su"])
            cl = contributor((t + 1) * nkb - 1, G, r0["su"])
            assert set(range(cf, cl + 1)) == cs
        else:
            assert len(cs) == 1
