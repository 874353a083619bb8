"""The TMA tile maps land in the tcgen05 operand layout (host-side arithmetic, no GPU).

The value tiles of the forward walk and of the chunk-parallel kernels, and the dO tiles of the
backward walk, are loaded by one 5-D tensor copy each, with dims (c % 8, token % 8, c / 8,
row / 8, head [or 2 head + r]) and a box of (8, 8, 8, 8, 1).  A tensor copy writes the box to
shared memory with dim 0 fastest.  These checks restate that traversal and the kernels'
K-major, no-swizzle operand index (umma.cuh kmaj: 8 x 8 core matrices of 128 bytes, K groups of
a row group adjacent) and confirm that every element of a 64-token x 64-channel tile lands where
the products read it, and comes from the element the cp.async path copies.
"""
import numpy as np


def kmaj(r, k, kt):
    """umma.cuh kmaj: element (row r, K index k) of a K-major operand with kt K elements."""
    return (((r >> 3) * (kt >> 3) + (k >> 3)) << 6) + ((r & 7) << 3) + (k & 7)


def _box_smem_offset(a0, a1, a2, a3, a4):
    """Shared-memory element offset of box coordinate (a0..a4), box (8, 8, 8, 8, 1), dim 0 fastest."""
    return (((a4 * 8 + a3) * 8 + a2) * 8 + a1) * 8 + a0


def test_value_tile_lands_in_operand_layout():
    st, sh, T, H, V = 2048, 64, 4096, 16, 64     # (B, T, H, V) bf16, contiguous: st = H V
    b, h, t0 = 3, 5, 640
    row0 = b * T + t0
    x3 = row0 // 8
    for a0 in range(8):
        for a1 in range(8):
            for a2 in range(8):
                for a3 in range(8):
                    j, v = 8 * a3 + a1, 8 * a2 + a0         # token within the chunk, value column
                    assert _box_smem_offset(a0, a1, a2, a3, 0) == kmaj(j, v, 64)
                    # global element: dims strides (1, st, 8, 8 st, sh) in elements
                    g = a0 + a1 * st + a2 * 8 + (x3 + a3) * 8 * st + h * sh
                    assert g == (b * T + t0 + j) * st + h * sh + v   # what pf_values copies


def test_dO_tiles_land_in_operand_layout():
    T, H, V, R = 4096, 16, 128, 2                # dO (B, T, H, 2, V) bf16 contiguous
    sr, sh, st = V, R * V, H * R * V
    b, h, t0, vb0 = 1, 7, 1984, 64
    x2, x3 = vb0 // 8, (b * T + t0) // 8
    doa = np.full(R * 64 * 64, -1, np.int64)     # DOA: rows (r, i), 64 value columns
    for r in range(R):
        base = r * 64 * 64                       # second read column: the 64-row half after the first
        for a0 in range(8):
            for a1 in range(8):
                for a2 in range(8):
                    for a3 in range(8):
                        g = a0 + a1 * st + (x2 + a2) * 8 + (x3 + a3) * 8 * st + (R * h + r) * sr
                        doa[base + _box_smem_offset(a0, a1, a2, a3, 0)] = g
    for r in range(R):
        for i in range(64):
            for v in range(64):
                want = (b * T + t0 + i) * st + h * sh + r * sr + vb0 + v   # pf_dO's source element
                assert doa[kmaj(r * 64 + i, v, 64)] == want
