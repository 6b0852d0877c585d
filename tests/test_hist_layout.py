"""The histogram's row-chunk lane mapping (silvic_b200/csrc/hist_device.cuh: chunk_period, ChunkLane, FixedChunk,
add_fixed, hist_rows), restated on the host: for every unit of F full tiles, in every load and step of a 32-row
batch, the 32 lanes' shared-memory atomics fall in 32 different banks, every (row, feature) of the batch is added
exactly once, and the per-lane byte selection (words swapped by r / 4, then byte (s ^ r) mod 4) reads byte s ^ r of
the chunk. Bit-exact histograms on the GPU are tested in test_gpu_parity.py; these are the layout properties the
kernel's speed and correctness rest on."""

from __future__ import annotations

import pytest


def chunk_period(f: int) -> int:
    return 8 if f == 3 else 2 * f


def lane_steps(f: int):
    """Yield (load g, step s, [(lane, row, tile, feature lane) of the active lanes])."""
    c_per = chunk_period(f)
    rows_per_load = 32 // c_per
    for g in range(c_per):
        for s in range(16):
            out = []
            for k in range(32):
                c, ri = k % c_per, k // c_per
                row = g * rows_per_load + ri
                if c >= 2 * f or row >= 32:
                    continue  # F = 3: lanes of chunks 6 and 7 are idle
                r = k >> 1
                out.append((k, row, c >> 1, (c & 1) * 16 + (s ^ r)))
            yield g, s, out


@pytest.mark.parametrize("f", [1, 2, 3, 4])
def test_every_step_hits_distinct_banks(f):
    for g, s, lanes in lane_steps(f):
        # slot (bin, feature lane) of a tile is word bin * 32 + feature lane, each tile's array 128-byte aligned:
        # the bank is the feature lane, whatever the bins and tiles
        banks = [fl for _, _, _, fl in lanes]
        assert len(set(banks)) == len(banks), (f, g, s, banks)


@pytest.mark.parametrize("f", [1, 2, 3, 4])
def test_every_row_and_feature_is_added_once(f):
    seen = {}
    for _, _, lanes in lane_steps(f):
        for _, row, tile, fl in lanes:
            seen[(row, tile, fl)] = seen.get((row, tile, fl), 0) + 1
    assert len(seen) == 32 * f * 32 and set(seen.values()) == {1}


@pytest.mark.parametrize("f", [1, 2, 3, 4])
def test_a_lane_keeps_one_tile(f):
    """FixedChunk needs a lane's chunk, and with it its tile, to be the same in every load of a batch."""
    tiles = {}
    for _, _, lanes in lane_steps(f):
        for k, _, tile, _ in lanes:
            tiles.setdefault(k, set()).add(tile)
    assert all(len(t) == 1 for t in tiles.values())


def test_byte_selection_reads_byte_s_xor_r():
    """add_fixed: words swapped to position j ^ (r / 4), then __byte_perm(word[s / 4], 0, bsel[s % 4]) with
    bsel[q] = ((q ^ r) & 3) | 0x4440 extracts byte (s ^ r) of the chunk's 16 bytes."""
    chunk = list(range(100, 116))  # byte i of the chunk holds 100 + i
    words = [chunk[4 * j:4 * j + 4] for j in range(4)]
    for r in range(16):
        wq = r >> 2
        swapped = [words[j ^ wq] for j in range(4)]
        for s in range(16):
            sel = ((s & 3) ^ r) & 3
            assert swapped[s >> 2][sel] == chunk[s ^ r], (r, s)
