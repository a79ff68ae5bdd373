"""The index arithmetic of the opt-in kernels, restated in Python and checked on the CPU.

Each mirror follows its kernel's loops line for line (grid, warps, lanes, loop bounds and
guards) and records what every thread would load and store; the checks are that every
output element is produced exactly once, that every load is in bounds and 16-byte
aligned, and that the units / rows / K ranges the threads cover tile the problem with
no gap and no overlap.  Kernels: gemv_kernel (csrc/gemv.cu), two_shot_norm16mw_kernel
(csrc/allreduce_norm.cuh), two_shot16s_kernel (csrc/allreduce_staged.cuh).
"""
import itertools

import pytest

K_SEG, K_WARPS, K_ROWS = 256, 8, 4  # gemv.cu: kSeg, kWarps, kRows
UNIT16, WARPS16 = 512, 8            # common.cuh kUnit16, allreduce.cuh kWarps16
STAGE_OFF = 512                     # workspace.h kStageBlockOff


def gemv_mirror(M, N_out, K, ldx, ldw, swiglu):
    """Returns (per output (m, col): list of (weight row, k range) summed, loads)."""
    I = N_out if swiglu else 0
    RW = 2 * K_ROWS if swiglu else K_ROWS
    grid = (N_out + K_ROWS - 1) // K_ROWS
    MT = 1 if M <= 1 else 2 if M <= 2 else 4 if M <= 4 else 8
    sums = {}
    loads = []
    for blk in range(grid):
        n0 = blk * K_ROWS
        wrow = []
        for r in range(RW):
            col = n0 + (r % K_ROWS)
            n = col if col < N_out else 0
            wrow.append(I + n if (swiglu and r >= K_ROWS) else n)
        part = {}  # (warp, r) -> list of k ranges
        nseg = (K + K_SEG - 1) // K_SEG
        for warp in range(K_WARPS):
            for s in range(warp, nseg, K_WARPS):
                for lane in range(32):
                    k0 = s * K_SEG + lane * 8
                    if k0 >= K:
                        continue
                    for r in range(RW):
                        loads.append(("w", wrow[r] * ldw + k0))
                        part.setdefault(r, []).append((k0, k0 + 8))
                    for m in range(MT):
                        if m < M:
                            loads.append(("x", m * ldx + k0))
        for t in range(K_ROWS * MT):
            r, m = t // MT, t % MT
            col = n0 + r
            if m < M and col < N_out:
                key = (m, col)
                assert key not in sums, f"output {key} written twice"
                sums[key] = {"gate": (wrow[r], sorted(part.get(r, [])))}
                if swiglu:
                    sums[key]["up"] = (wrow[K_ROWS + r], sorted(part.get(K_ROWS + r, [])))
    return sums, loads


@pytest.mark.parametrize("M,N,K,swiglu", [(1, 256, 64, False), (3, 300, 1000, False), (4, 1280, 8192, False),
                                          (8, 4096, 4096, False), (5, 9, 2056, False), (1, 128, 64, True),
                                          (4, 3584, 8192, True), (7, 1376, 4096, True), (2, 5, 24, True)])
def test_gemv_index_math(M, N, K, swiglu):
    ldx, ldw = K, K  # contiguous rows, as the tests and the model use
    rows_w = 2 * N if swiglu else N
    sums, loads = gemv_mirror(M, N, K, ldx, ldw, swiglu)
    assert set(sums) == {(m, c) for m in range(M) for c in range(N)}
    full = [(k, k + 8) for k in range(0, K, 8)]
    for (m, col), parts in sums.items():
        assert parts["gate"][0] == col and parts["gate"][1] == full, (m, col)
        if swiglu:
            assert parts["up"][0] == N + col and parts["up"][1] == full, (m, col)
    for kind, off in loads:
        assert off % 8 == 0  # 8 bf16 = 16 bytes from a 16-byte aligned base
        limit = (rows_w if kind == "w" else M) * K
        assert 0 <= off and off + 8 <= limit, (kind, off)


def norm_mw_mirror(M, W, H, G, wpr):
    """Rows and units each (rank, CTA, warp) touches in the three phases of the kernel."""
    RG = WARPS16 // wpr
    R = (M + W - 1) // W
    upr = H // UNIT16
    p1, p2, p3 = [], [], []
    for rank, b, warp in itertools.product(range(W), range(G), range(WARPS16)):
        rg, q = warp // wpr, warp % wpr
        row_step, row0 = G * RG, b + G * rg
        for rr in range(row0, R, row_step):
            for jj in range(W):  # phase 1
                j = (rank + 1 + jj) % W
                g = j * R + rr
                if g >= M:
                    continue
                for u in range(q, upr, wpr):
                    p1.append((rank, j, rr * upr + u))
            g = rank * R + rr  # phase 2
            if g < M:
                for u in range(q, upr, wpr):
                    p2.append((rank, rr * upr + u))
            for jj in range(1, W):  # phase 3
                j = (rank + jj) % W
                g = j * R + rr
                if g < M:
                    for u in range(q, upr, wpr):
                        p3.append((rank, j, rr * upr + u))
    return R, upr, p1, p2, p3


@pytest.mark.parametrize("M,W,H,wpr", [(8192, 8, 4096, 4), (1000, 4, 4096, 2), (300, 8, 2048, 4), (77, 3, 512, 4),
                                        (130, 1, 1024, 2), (1024, 8, 8192, 8)])
def test_norm_multi_warp_index_math(M, W, H, wpr):
    rows_per_cta = WARPS16 // wpr
    R = (M + W - 1) // W
    G = min((R + rows_per_cta - 1) // rows_per_cta, 444 // W if W > 1 else 444)  # the launch's cap
    R, upr, p1, p2, p3 = norm_mw_mirror(M, W, H, G, wpr)
    own = lambda j: [rr for rr in range(R) if j * R + rr < M]  # noqa: E731
    # phase 1: every rank sends every valid unit of every row block exactly once
    want1 = sorted((rank, j, rr * upr + u) for rank in range(W) for j in range(W) for rr in own(j) for u in range(upr))
    assert sorted(p1) == want1
    # phase 2: every rank reduces each unit of its own rows exactly once
    assert sorted(p2) == sorted((rank, rr * upr + u) for rank in range(W) for rr in own(rank) for u in range(upr))
    # phase 3: every rank gathers every unit of every other rank's rows exactly once
    want3 = sorted((rank, j, rr * upr + u) for rank in range(W) for j in range(W) if j != rank for rr in own(j)
                   for u in range(upr))
    assert sorted(p3) == want3


@pytest.mark.parametrize("n_units,G", [(8192, 444), (16384, 444), (37, 5), (1, 1), (9, 2), (1000, 128)])
def test_staged_two_shot_unit_split(n_units, G):
    """Per warp, stage 0 takes [0, half) and stage 1 [half, my_units) of its unit list;
    together the (CTA, warp, stage) lists cover every unit of a chunk exactly once, and
    stage-1 flag blocks stay inside the flag array."""
    wpb = WARPS16
    ustride = G * wpb
    seen = []
    assert G <= STAGE_OFF and G + STAGE_OFF <= 1024
    for b, warp in itertools.product(range(G), range(wpb)):
        u0 = b * wpb + warp
        my_units = (n_units - 1 - u0) // ustride + 1 if u0 < n_units else 0
        half = (my_units + 1) // 2
        for s, (lo, hi) in enumerate([(0, half), (half, my_units)]):
            for i in range(lo, hi):
                seen.append(u0 + i * ustride)
    assert sorted(seen) == list(range(n_units))
