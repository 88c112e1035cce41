"""The decode step's tile-ring rule (``flux_b200/csrc/step_kernel.cu``, the
producer loop), simulated on the host against an in-order consumer: tile k of
``size`` bytes (rounded to 128) starts at the byte-stream position, moved to
the next lap when it would straddle the ring's end; it may be written once
every tile whose bytes it reuses has been released and at most ``ahead``
tiles are in flight; tile k uses barrier pair k % 12.  Checked over random
tile sequences with the step's tile sizes: no tile overwrites bytes of a tile
still in flight, no barrier pair is reused before its tile was released, the
depth never exceeds ``ahead``, and the producer never waits for a tile it has
not issued (no deadlock)."""

from __future__ import annotations

import random

import pytest

RING = 7 * 27648
BARS = 12
MAX_TILE = 27648


def simulate(sizes: list[int], ahead: int, consume_lag: random.Random) -> None:
    pos, freed, nxt = 0, 0, 0
    spans: dict[int, tuple[int, int]] = {}  # tile -> [start, end) in the byte stream
    released = 0  # tiles the consumer has released (in order)
    for k, raw in enumerate(sizes):
        size = (raw + 127) // 128 * 128
        assert 0 < size <= MAX_TILE
        if pos % RING + size > RING:
            pos += RING - pos % RING
        end = pos + size
        while nxt < k and (freed < end - RING or nxt <= k - ahead):
            # the producer waits for tile `nxt`'s release: the consumer gets there
            assert nxt < k, "waiting for a tile that was never issued"
            released = max(released, nxt + 1)
            freed = spans[nxt][1]
            nxt += 1
        # the bytes [pos, end) of this lap are free of every tile still in flight
        for j in range(released, k):
            s, e = spans[j]
            assert e <= pos or s >= end, (k, j)  # the stream spans of live tiles never collide ...
            assert e - RING <= pos and pos + size - RING <= s, (k, j)  # ... nor their ring positions
        assert k - released < ahead or nxt == k
        if k >= BARS:
            assert released >= k - BARS + 1, "barrier pair reused before its tile was released"
        spans[k] = (pos, end)
        pos = end
        # the consumer releases some tiles at its own pace (never ahead of the issued ones)
        released = max(released, min(k + 1, released + consume_lag.randint(0, 2)))
        if released > nxt:
            nxt, freed = released, spans[released - 1][1]


def step_tile_sizes(rng: random.Random, layers: int = 30) -> list[int]:
    """A step's sequence: per layer A (norm + 6-8 QKV rows), 0-4 cache tiles
    (54 rows of K and V, the last shorter), misc (norm + 1-2 o_proj strip
    pairs), gate, up, down; then the final norm and 12-row LM-head tiles."""
    row, strip = 2304, 3 * 3072
    n_att = rng.choice([0, 1, 1, 2, 4])
    last = rng.randint(1, 54)
    sizes = []
    for _ in range(layers):
        sizes.append(row * (1 + 2 * rng.choice([3, 4])))
        sizes += [54 * 512] * max(0, n_att - 1) + ([last * 512] if n_att else [])
        sizes.append(row + strip * rng.choice([1, 2]))
        nf = rng.choice([8, 12])
        sizes += [nf * row, nf * row, (nf // 4) * strip]
    sizes.append(row)
    sizes += [12 * row] * rng.randint(20, 40)
    return sizes


@pytest.mark.parametrize("ahead", [7, 12])
def test_ring_rule_never_overwrites_live_tiles(ahead):
    rng = random.Random(ahead)
    for trial in range(200):
        simulate(step_tile_sizes(rng), ahead, random.Random(trial))


def test_ring_rule_extremes():
    for ahead in (7, 12):
        simulate([MAX_TILE] * 100, ahead, random.Random(1))          # every tile the largest
        simulate([128] * 100, ahead, random.Random(2))               # many tiny tiles: the depth cap binds
        simulate([MAX_TILE, 128] * 60, ahead, random.Random(3))      # alternating: laps with skipped tails
