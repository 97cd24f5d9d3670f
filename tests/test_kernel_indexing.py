"""CPU replay of the Q4_K decode GEMV's request cursor
(go-infer_b200/csrc/gemv.cu, gemv_q4k_kernel): the weight addresses it
advances in place, across tiles of one matrix by dt * 15 rows, must equal
the direct address of every unit (matrix, 16-row tile with clamped last
rows, column block) for every CTA and warp, over matrix boundaries,
ragged row counts, the interleaved SwiGLU tiles and warps-per-CTA both
above and below the column-block count; and the warp-local activation
staging and slot zeroing of the same kernel."""
import pytest


def direct(rows, nku, T, u_lku, g, swiglu, tstart, base):
    if swiglu:
        m, lt = T & 1, T >> 1
    else:
        m = sum(T >= s for s in tstart[1:len(rows)])
        lt = T - tstart[m]
    r0, rl, rowb = lt * 16, rows[m] - 1, nku * 144
    return (base[m] + min(r0 + g, rl) * rowb + u_lku * 144, base[m] + min(r0 + g + 8, rl) * rowb + u_lku * 144)


def replay(rows, nku, W, ctas, swiglu=False):
    tiles = [(r + 15) // 16 for r in rows]
    tstart = [0]
    for k in tiles:
        tstart.append(tstart[-1] + k)
    ntiles = tstart[-1]
    base = [10 ** 9 * (m + 1) for m in range(len(rows))]
    rowb = nku * 144
    gran = 2 if swiglu else 1
    nun = ntiles // gran
    checked = 0
    for c in range(ctas):
        T0, T1 = gran * (nun * c // ctas), gran * (nun * (c + 1) // ctas)
        n = (T1 - T0) * nku
        for warp in range(W):
            for g in range(8):
                ltile, lku = warp // nku, warp % nku
                nxt, fast_end = warp, 0
                pa = pb = None

                def seek():
                    nonlocal pa, pb, fast_end
                    T = T0 + ltile
                    pa, pb = direct(rows, nku, T, lku, g, swiglu, tstart, base)
                    if swiglu:
                        fast_end = 0
                    else:
                        m = sum(T >= s for s in tstart[1:len(rows)])
                        fast_end = tstart[m] + (rows[m] >> 4)

                if nxt < n:
                    seek()
                while nxt < n:
                    want = direct(rows, nku, T0 + nxt // nku, nxt % nku, g, swiglu, tstart, base)
                    assert (pa, pb) == want, (rows, nku, W, ctas, c, warp, g, nxt)
                    checked += 1
                    nxt += W
                    lku += W
                    pa += W * 144
                    pb += W * 144
                    if lku >= nku:
                        dt = 0
                        while lku >= nku:
                            lku -= nku
                            dt += 1
                        ltile += dt
                        if nxt < n:
                            if T0 + ltile < fast_end:
                                pa += dt * 15 * rowb
                                pb += dt * 15 * rowb
                            else:
                                seek()
    return checked


@pytest.mark.parametrize("rows,nku,W,ctas", [
    ([11008, 11008], 16, 16, 148),   # gate + up, config 2
    ([4096], 43, 16, 148),           # down, config 2
    ([4096], 16, 8, 296),
    ([100, 37], 8, 16, 5),           # ragged tails, nku < W
    ([4100, 256], 3, 8, 7),
    ([40, 48, 24], 5, 16, 3),        # three matrices
    ([17], 1, 16, 1),
])
def test_cursor_matches_direct_addressing(rows, nku, W, ctas):
    assert replay(rows, nku, W, ctas) > 0


def test_cursor_swiglu_interleave():
    assert replay([96, 96], 4, 8, 3, swiglu=True) > 0
    assert replay([100, 100], 16, 16, 5, swiglu=True) > 0


def q6m_replay(rows, nku, W, ctas):
    """The Q6_K tensor-core kernel's request cursor (gemv.cu, q6m): lane L
    copies row L/2 of a unit from src = row start + ((210 lku) & ~15); within
    a tile src moves by the difference of those rounded offsets, and a new
    tile re-seeks (clamping rows past the end).  Every unit's source must be
    the direct one, 16-byte aligned, and its 224 bytes must end inside the
    matrix."""
    ntiles = (rows + 15) // 16
    rowb = 210 * nku
    checked = 0
    for c in range(ctas):
        T0, T1 = ntiles * c // ctas, ntiles * (c + 1) // ctas
        n = (T1 - T0) * nku
        for warp in range(W):
            for crow in range(16):
                ltile, lku, nxt = warp // nku, warp % nku, warp
                src = None

                def seek():
                    return min((T0 + ltile) * 16 + crow, rows - 1) * rowb + ((210 * lku) & ~15)
                if nxt < n:
                    src = seek()
                while nxt < n:
                    want = min((T0 + ltile) * 16 + crow, rows - 1) * rowb + ((210 * lku) & ~15)
                    assert src == want
                    assert src % 16 == 0 and src + 224 <= rows * rowb
                    checked += 1
                    nxt += W
                    lku += W
                    if lku < nku:
                        src += ((210 * lku) & ~15) - ((210 * (lku - W)) & ~15)
                    else:
                        while lku >= nku:
                            lku -= nku
                            ltile += 1
                        if nxt < n:
                            src = seek()
    return checked


@pytest.mark.parametrize("rows,nku,W,ctas", [(16, 8, 16, 1), (17, 8, 16, 2), (300, 16, 16, 19), (2000, 32, 16, 125),
                                             (4100, 8, 8, 148), (40, 16, 8, 3)])
def test_q6m_request_cursor(rows, nku, W, ctas):
    assert q6m_replay(rows, nku, W, ctas) > 0


def staged_by(nku, W):
    """stage_x (csrc/q4k.cuh): warp w stages the column blocks
    u0 + k W, u0 = w, w + 4W, ..., k < 4 -- block u by warp u % W.  The
    Q8_0 and Q6_K tensor-core kernels' stage_x (csrc/gemv.cu: u = w, w + W,
    ...) assign the same owners."""
    owner = {}
    for w in range(W):
        for u0 in range(w, nku, 4 * W):
            for k in range(4):
                u = u0 + k * W
                if u < nku:
                    assert u not in owner
                    owner[u] = w
    assert sorted(owner) == list(range(nku))
    assert owner == {u: w for w in range(W) for u in range(w, nku, W)}
    return owner


def computed_blocks(nku, W, ntl, warp):
    """The compute cursor of gemv_q4k_kernel: units warp, warp + W, ... of
    the CTA's ntl * nku units; (ctile, cku) advanced in place as the
    kernel does.  Returns the (tile, column block) of each unit."""
    ctile, cku = warp // nku, warp % nku
    out = []
    for i in range(warp, ntl * nku, W):
        assert (ctile, cku) == divmod(i, nku)
        out.append((ctile, cku))
        cku += W
        while cku >= nku:
            cku -= nku
            ctile += 1
    return out


@pytest.mark.parametrize("W", [8, 16])
@pytest.mark.parametrize("nku", [1, 3, 4, 8, 16, 32, 43, 48, 112])
def test_warp_local_staging(nku, W):
    """The kernel skips the CTA barrier after staging exactly when
    nku % W == 0; then every block a warp computes is one it staged itself
    (on any number of tiles per CTA).  Otherwise some warp needs a block
    another warp staged, and the barrier is required."""
    owner = staged_by(nku, W)
    foreign = False
    for ntl in (1, 2, 3, 5):
        for warp in range(W):
            for _tile, cku in computed_blocks(nku, W, ntl, warp):
                if owner[cku] != warp:
                    foreign = True
                    assert nku % W != 0, (nku, W, ntl, warp, cku)
    assert foreign == (nku % W != 0)


def test_warp_local_slot_zeroing():
    """Each warp zeroes slots[(t * W + warp) * 16 + j] for its CTA's ntl
    tiles: together the warps cover the whole [ntl][W][16] array once, and
    every slot a warp writes at the end of a tile is one it zeroed."""
    for W in (8, 16):
        for ntl in (1, 2, 7):
            seen = []
            for warp in range(W):
                mine = set()
                for i in range(ntl * 16):  # lanes i = lane, lane + 32, ...
                    s = ((i >> 4) * W + warp) * 16 + (i & 15)
                    mine.add(s)
                    seen.append(s)
                for nku in (3, 16, 43):
                    for tile, _ in computed_blocks(nku, W, ntl, warp):
                        assert {(tile * W + warp) * 16 + j for j in range(16)} <= mine
            assert sorted(seen) == list(range(ntl * W * 16))


@pytest.mark.parametrize("nku,W", [(43, 16), (43, 8), (3, 8), (112, 16), (5, 16)])
def test_single_tile_ctas_read_only_their_own_blocks(nku, W):
    """A CTA with one tile computes unit i on block i, which warp i % W
    staged -- for any column-block count -- and with two tiles of the
    config-2 down shape (43 blocks, 16 warps) every warp first streams 2-3
    units of its own blocks (the room a split barrier would have)."""
    owner = staged_by(nku, W)
    for warp in range(W):
        assert all(owner[c] == warp for _t, c in computed_blocks(nku, W, 1, warp))
    if (nku, W) == (43, 16):
        lead = []
        for warp in range(W):
            blocks = computed_blocks(nku, W, 2, warp)
            lead.append(next(i for i, (_t, c) in enumerate(blocks) if owner[c] != warp))
        assert lead == [3] * 11 + [2] * 5
