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


# ----------------------------------------------------------------- attention (csrc/attention.cu)
QB = KB = 128


def swz_offset(row, col):
    chunk, c = col >> 6, col & 63
    unit = (c >> 3) ^ (row & 7)
    return chunk * (128 * 128) + row * 128 + unit * 16 + (c & 7) * 2


def _bwd_unit_elements(ping):
    """(warp, lane) -> the (key row, query column, dS^T byte offset, P^T TMEM column) each thread
    handles for one 64-query unit of half h, as the plain (8 warps x 32 queries) and the ping-pong
    (one warpgroup x 64 queries in two passes) elementwise code computes them."""
    out = {}
    for h in range(2):
        items = []
        warps = range(2, 6) if (ping and h == 0) else range(6, 10) if ping else range(2, 10)
        for warp in warps:
            q = warp & 3
            for lane in range(32):
                kr = q * 32 + lane
                passes = [0, 32] if ping else [((warp - 2) >> 2) * 32]
                for c0 in passes:
                    for g in range(4):
                        for e in range(8):
                            qu = c0 + g * 8 + e                       # query column in the unit
                            items.append((kr, h * 64 + qu, swz_offset(kr, c0 + g * 8) + 2 * e, c0 + g * 4 + e // 2))
        out[h] = items
    return out


def test_attention_bwd_ping_pong_covers_each_unit_like_the_plain_layout():
    """Each (key, query) element of a unit is produced exactly once, at the same dS^T smem byte
    and the same packed-P^T TMEM column in both layouts, so the MMA side needs no change."""
    plain, ping = _bwd_unit_elements(False), _bwd_unit_elements(True)
    for h in range(2):
        assert sorted(plain[h]) == sorted(ping[h])
        keys = {(kr, qc) for kr, qc, _, _ in ping[h]}
        assert len(keys) == len(ping[h]) == 128 * 64
        offs = [o for _, _, o, _ in ping[h]]
        assert len(set(offs)) == len(offs) and max(offs) < 16384  # one 16 KB dS^T buffer per half
        # the dV MMA reads query k-step kk (16 queries) from TMEM column (kk >> 1) * 32 + (kk & 1) * 8
        for kr, qc, _, col in ping[h]:
            qu = qc - h * 64
            kk = qu // 16
            assert col == (kk >> 1) * 32 + (kk & 1) * 8 + (qu % 16) // 2


def test_attention_bwd_ping_pong_statistics_and_mask():
    """Warpgroup wg stages -lse*log2e / -delta of queries wg*64 .. wg*64+63 at [0, 64) / [64, 128)
    of its own 128 floats; the packed mask (qc < kr per pair) equals the plain one."""
    for wg in range(2):
        staged = {}
        for wt in range(128):
            src = "lse" if wt < 64 else "delta"
            staged[wt] = (src, wg * 64 + (wt & 63))
        for qu in range(64):
            assert staged[qu] == ("lse", wg * 64 + qu) and staged[64 + qu] == ("delta", wg * 64 + qu)
        assert 0 <= wg * 128 and wg * 128 + 127 < 256  # inside the 1 KB statistics region
    for h in range(2):
        for kr in range(128):
            for qu in range(0, 64, 2):
                qc = h * 64 + qu
                plain = [qc + t < kr for t in range(2)]
                packed = [qc < kr, qc + 1 < kr]
                assert plain == packed


def test_attention_forward_packed_mask_and_exponent():
    """Forward v2: keys past the query row are masked with e > qi - k0, and exp2(s*c - m) with m the
    scaled max equals exp2(s*c - max(s*c)) because c > 0."""
    import math
    import random

    for qb in range(3):
        for j in range(qb + 1):
            for r in range(0, 128, 7):
                qi = qb * QB + r
                for hf in range(2):
                    k0 = j * KB + hf * 64
                    for e in range(64):
                        assert (e > qi - k0) == (j * KB + hf * 64 + e > qi)
    rnd = random.Random(0)
    c = 0.088 * 1.4426950408889634
    s = [rnd.uniform(-30, 30) for _ in range(128)]
    m_scaled = max(s) * c
    assert abs(m_scaled - max(x * c for x in s)) < 1e-12
    ref = [2 ** (x * c - max(y * c for y in s)) for x in s]
    got = [2 ** (math.fma(x, c, -m_scaled) if hasattr(math, "fma") else x * c - m_scaled) for x in s]
    assert max(abs(a - b) for a, b in zip(ref, got)) < 1e-12


def test_attention_fwd3_register_split():
    """attn_fwd3_kernel: 384 threads launched at 168 registers; WG0 drops to 56, the two softmax
    warpgroups rise to 224.  The block's pool and each sub-partition's 16384 registers suffice."""
    launch, ctrl, soft = 168, 56, 224
    assert 128 * ctrl + 256 * soft <= 384 * launch
    # warp w runs on sub-partition w % 4: one WG0 warp and two softmax warps each
    for sp in range(4):
        warps = [w for w in range(12) if w % 4 == sp]
        regs = sum((ctrl if w < 4 else soft) * 32 for w in warps)
        assert regs <= 16384
    assert all(r % 8 == 0 for r in (launch, ctrl, soft)) and 24 <= ctrl and soft <= 256
