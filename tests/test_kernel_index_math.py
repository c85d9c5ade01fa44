"""Host restatements of the GEMM kernels' tile / piece index arithmetic (csrc/tc_gemm.cu), checked
for exact coverage on the shapes the library runs: every output tile is visited once, the fused
all-gather pulls every piece of every shard once and fills every panel counter to its target,
and the panel / segment maps stay inside their buffers."""
import itertools

import pytest

BM, BN, BK, PANEL = 128, 256, 64, 128


def tile_coords(t, tiles_m, tiles_n, band, symmetric, tiles_per_batch, pair=False):
    """tile_coords / tile_coords_pair of tc_gemm.cu."""
    b, r = divmod(t, tiles_per_batch)
    if not symmetric:
        span = band * tiles_m
        bi, rr = divmod(r, span)
        w = min(band, tiles_n - bi * band)
        return b, rr // w, bi * band + rr % w
    i = 0
    while True:
        cnt = tiles_n - (i if pair else i >> 1)
        if r < cnt:
            return b, i, (i if pair else i >> 1) + r
        r -= cnt
        i += 1


def host_band(units, tiles_m, tiles_n):
    band = (units + tiles_m - 1) // tiles_m
    return max(1, min(band, tiles_n))


@pytest.mark.parametrize("M,N,batch,pair", [(4096, 4096, 1, False), (4096, 14336, 3, False), (1024, 4096, 2, False),
                                            (128, 256, 1, False), (4096, 14336, 2, True), (512, 768, 1, True)])
def test_banded_tiles_cover_every_output_tile_once(M, N, batch, pair):
    bm = 256 if pair else BM
    tiles_m, tiles_n = M // bm, N // BN
    band = host_band(74 if pair else 148, tiles_m, tiles_n)
    per = tiles_m * tiles_n
    seen = [tile_coords(t, tiles_m, tiles_n, band, False, per) for t in range(per * batch)]
    assert sorted(seen) == sorted(itertools.product(range(batch), range(tiles_m), range(tiles_n)))


@pytest.mark.parametrize("M,pair", [(4096, False), (1024, False), (4096, True), (1536, True), (256, True)])
def test_symmetric_tiles_cover_the_upper_triangle_once(M, pair):
    bm = 256 if pair else BM
    tiles_m, tiles_n = M // bm, M // BN
    per = sum(tiles_n - (i if pair else i >> 1) for i in range(tiles_m))  # host count (launch())
    seen = [tile_coords(t, tiles_m, tiles_n, 1, True, per, pair)[1:] for t in range(per)]
    # every tile touching the upper triangle (row block end > column block start), exactly once
    want = [(i, j) for i in range(tiles_m) for j in range(tiles_n) if (j + 1) * BN > i * bm]
    assert sorted(seen) == sorted(want)


@pytest.mark.parametrize("N,K,ws", [(4096, 4096, 8), (1024, 4096, 8), (14336, 4096, 8), (4096, 14336, 8),
                                    (14336, 4096, 2), (1024, 4096, 4), (2304, 768, 2), (3072, 768, 8)])
def test_all_gather_gemm_schedule(N, K, ws):
    """ag_gemm_kernel: rotated tiles, panel sources, and the puller's piece assignment."""
    assert N % (PANEL * ws) == 0 and N % BN == 0
    rows = N // ws
    pps, ppp = rows // PANEL, K // BK
    tiles_m, tiles_n = 4096 // BM, N // BN
    band = host_band(148, tiles_m, tiles_n)
    for rank in range(ws):
        rot = (rank * rows) // BN
        tiles = set()
        for t in range(tiles_m * tiles_n):
            _, tm, tn = tile_coords(t, tiles_m, tiles_n, band, False, tiles_m * tiles_n)
            tn = (tn + rot) % tiles_n
            tiles.add((tm, tn))
            for h in range(2):  # the two 128-row panels of the B tile
                panel = 2 * tn + h
                owner = panel // pps
                lrow = (panel - owner * pps) * PANEL
                assert 0 <= owner < ws and 0 <= lrow <= rows - PANEL
                assert owner * rows + lrow == panel * PANEL  # G row of that panel
        assert len(tiles) == tiles_m * tiles_n
        # the first tile column visited contains the first row of this rank's own shard
        _, _, tn0 = tile_coords(0, tiles_m, tiles_n, band, False, tiles_m * tiles_n)
        start = ((tn0 + rot) % tiles_n) * BN
        assert start <= rank * rows < start + BN
        # pullers: piece gi goes to CTA gi % grid; every (shard, panel, k-block) exactly once,
        # shards in ring order starting at rank + 1, own shard last
        grid = min(148, tiles_m * tiles_n)
        per_shard = pps * ppp
        counts = {}
        order = []
        for cta in range(grid):
            for gi in range(cta, ws * per_shard, grid):
                step, rem = divmod(gi, per_shard)
                src = (rank + 1 + step) % ws
                lp, kb = divmod(rem, ppp)
                counts[(src, lp, kb)] = counts.get((src, lp, kb), 0) + 1
                order.append((gi, src))
        assert len(counts) == ws * per_shard and set(counts.values()) == {1}
        srcs_in_order = [s for _, s in sorted(order)]
        ring = [(rank + 1 + s) % ws for s in range(ws)]
        assert [srcs_in_order[i * per_shard] for i in range(ws)] == ring
        panel_pieces = {}
        for (src, lp, _), c in counts.items():
            panel_pieces[src * pps + lp] = panel_pieces.get(src * pps + lp, 0) + c
        assert len(panel_pieces) == N // PANEL and set(panel_pieces.values()) == {ppp}


@pytest.mark.parametrize("N,ws", [(4096, 8), (14336, 2), (1024, 4), (768, 2)])
def test_weight_gradient_segments(N, ws):
    """wgrad_out: row r of dW goes to segment r // seg_rows at row r - seg * seg_rows."""
    seg_rows = N // ws
    for r in range(N):
        seg = r // seg_rows
        assert 0 <= seg < ws and 0 <= r - seg * seg_rows < seg_rows
