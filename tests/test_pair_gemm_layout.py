"""Index maps of the paired projection GEMM (``flux_b200/csrc/tc_gemm.cu``,
``tc_gemm_pair_kernel`` and ``tf32_split_swiglu_rows_kernel``), restated on
the host:

* the persistent tile walk t = pair + u * pairs covers every (W block, X
  block) once, and each CTA of a pair stages its own 96 W rows and 128 X rows;
* the fused-SwiGLU row order of the packed gate/up weight is a permutation
  whose blocks hold 48 gate rows and then their 48 up rows per epilogue half,
  so that the epilogue's column q and 48 + q are the gate and up of one
  feature, written to act column (tile_n0 + c0) / 2 + q;
* with that order, silu(gate) * up per epilogue thread equals the reference's
  packed SwiGLU on the [gate | up] layout.

No GPU is needed."""

from __future__ import annotations

import numpy as np
import pytest

PAIR_N = 192          # W rows per pair tile (96 per CTA)
HALF = PAIR_N // 2    # 96: the epilogue half a thread holds
INTER = 1536
HIDDEN = 576


def swiglu_row_source(r: int, inter: int = INTER) -> int:
    """Source row of destination row r (tf32_split_swiglu_rows_kernel)."""
    b, c = divmod(r, PAIR_N)
    f = HALF * b + (PAIR_N // 4) * (c // HALF) + c % (PAIR_N // 4)
    return f if c % HALF < PAIR_N // 4 else inter + f


def test_swiglu_row_order_is_a_permutation():
    src = [swiglu_row_source(r) for r in range(2 * INTER)]
    assert sorted(src) == list(range(2 * INTER))


@pytest.mark.parametrize("c0", [0, HALF])
def test_epilogue_halves_pair_gate_with_up(c0):
    for b in range(2 * INTER // PAIR_N):
        tile_n0 = b * PAIR_N
        for q in range(PAIR_N // 4):
            gate = swiglu_row_source(tile_n0 + c0 + q)
            up = swiglu_row_source(tile_n0 + c0 + PAIR_N // 4 + q)
            feature = (tile_n0 + c0) // 2 + q           # the act column the thread writes
            assert gate == feature and up == INTER + feature


def test_fused_swiglu_matches_packed_layout():
    rng = np.random.default_rng(3)
    rows = 5
    packed = rng.standard_normal((rows, 2 * INTER)).astype(np.float32)   # [gate | up] per row
    silu = lambda g: g / (1.0 + np.exp(-g))  # noqa: E731
    ref = silu(packed[:, :INTER]) * packed[:, INTER:]
    # the GEMM with permuted weight rows produces D[:, r] = packed[:, src(r)]
    perm = np.array([swiglu_row_source(r) for r in range(2 * INTER)])
    d = packed[:, perm]
    act = np.empty_like(ref)
    for b in range(2 * INTER // PAIR_N):
        for c0 in (0, HALF):
            cols = d[:, b * PAIR_N + c0: b * PAIR_N + c0 + HALF]
            g, u = cols[:, :HALF // 2], cols[:, HALF // 2:]
            act[:, (b * PAIR_N + c0) // 2: (b * PAIR_N + c0) // 2 + HALF // 2] = silu(g) * u
    np.testing.assert_array_equal(act, ref)


@pytest.mark.parametrize("m,n,pairs", [(8192, 3072, 74), (8192, 960, 74), (8192, 576, 74), (2048, 576, 70),
                                       (2500, 192, 3)])
def test_persistent_pair_walk_covers_every_tile_once(m, n, pairs):
    nblocks = n // PAIR_N
    tiles = nblocks * ((m + 255) // 256)
    pairs = min(pairs, tiles)
    seen = {}
    for pair in range(pairs):
        mine = (tiles - 1 - pair) // pairs + 1 if pair < tiles else 0
        for u in range(mine):
            t = pair + u * pairs
            n0, m0 = t % nblocks * PAIR_N, t // nblocks * 256
            for rank in (0, 1):
                w_rows = (n0 + rank * HALF, n0 + rank * HALF + HALF)      # this CTA's B half
                x_rows = (m0 + rank * 128, m0 + rank * 128 + 128)         # this CTA's A half and D rows
                assert w_rows[1] <= n
                seen.setdefault((n0, m0), []).append((rank, w_rows, x_rows))
    assert len(seen) == tiles
    assert all(len(v) == 2 for v in seen.values())
