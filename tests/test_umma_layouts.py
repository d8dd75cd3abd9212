"""Layout contract of the tcgen05 prefill kernel (csrc/paged_prefill_tc.cu):
the shared-memory matrix descriptors it builds address exactly the bytes the
TMA boxes (128-byte swizzle) and the Q staging wrote.

Canonical sm_100 layouts, in 16-byte units with the 128-byte swizzle applied
to the byte address (16-byte chunk bits [4,7) XOR row bits [7,10)):
  K-major  ((8, n), 2) : ((8, SBO), 1)          Q (A operand) and K (B operand)
  N-major  ((8, n), (8, k)) : ((1, LBO), (8, SBO))   V (B operand of P.V)
The kernel's choices restated here: K step of 16 elements = +32 B of the
start address inside a 64-column slab, slabs of 128 rows (Q) or 64 rows
(K/V) x 128 B, SBO = 1024 B (8 rows), LBO = the 64-column slab size for V, a
16-key step of V = +2048 B.  No GPU is involved.
"""


def _swz(addr: int) -> int:
    return addr ^ (((addr >> 7) & 7) << 4)


def _tma(base: int, slab: int, row: int, col: int) -> int:
    """Byte of element (row, col) of a [rows][D] tile written as 64-column
    slabs of 128-byte rows with the 128-byte swizzle."""
    hb, c = divmod(col, 64)
    chunk, within = divmod(c, 8)
    return base + hb * slab + row * 128 + ((chunk ^ (row & 7)) << 4) + within * 2


def _k_major(start: int, sbo: int, mn: int, k: int) -> int:
    i, r = divmod(mn, 8)
    u, within = divmod(k, 8)
    return _swz(start + r * 128 + i * sbo + u * 16) + within * 2


def _n_major(start: int, lbo: int, sbo: int, mn: int, k: int) -> int:
    i, rest = divmod(mn, 64)
    u, within = divmod(rest, 8)
    t, r = divmod(k, 8)
    return _swz(start + u * 16 + i * lbo + r * 128 + t * sbo) + within * 2


def test_q_and_k_descriptors_match_the_staged_tiles():
    for D in (64, 128):
        for rows in (128, 64):          # Q tile (M = 128), K tile (N = 64 keys)
            slab = rows * 128
            base = 4096                 # any 1024-aligned stage address
            for kk in range(D // 16):
                start = base + (kk >> 2) * slab + (kk & 3) * 32
                for mn in range(rows):
                    for k in range(16):
                        assert _k_major(start, 1024, mn, k) == _tma(base, slab, mn, kk * 16 + k)


def test_v_descriptor_matches_the_staged_tile():
    for D in (64, 128):
        base, slab = 8192, 64 * 128
        for kt in range(4):             # 16-key steps of a 64-key tile
            start = base + kt * 2048
            for n in range(D):
                for k in range(16):
                    assert _n_major(start, slab, 1024, n, k) == _tma(base, slab, kt * 16 + k, n)
