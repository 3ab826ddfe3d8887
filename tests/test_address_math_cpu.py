"""CPU checks of the pipelined kernel's address arithmetic (csrc/quantize_tma.cu),
restated here in Python, over every alignment the kernel can meet.

1. Row path: X rows that are not 16-byte aligned are read through one tensor
   map per row phase f = row % 8: base = row f's address rounded down to 16
   bytes, d_f = its misalignment in elements, extent k + d_f columns by the
   phase's rows, row stride 16 * ld_x bytes; a tile loads 136-column boxes at
   column 128 * ct.  Checked: every byte a box can read lies in the 16-byte
   chunks holding that row's own elements; the 64 columns a thread re-aligns
   from its box row are the row's columns; the misalignment the kernel
   computes in 32-bit arithmetic equals 2 * d_f.
2. Any-offset stores (store_row_any): a row segment of seg bytes at any
   address is written as aligned 16-byte chunks (byte-shifted chunk pairs)
   plus the head and tail bytes.  Checked: every byte of the segment is
   written exactly once with its value, each store is aligned to its size,
   and nothing outside the segment is touched.
"""

import numpy as np
import pytest

PHASES, PHASE_ROWS, BOX_COLS = 8, 16, 136


def phase_maps(x_addr, m, ld_x, k):
    """(base, d, rows) of each phase map, as encode_x_maps builds them."""
    maps = []
    for f in range(min(m, PHASES)):
        row0 = x_addr + 2 * f * ld_x
        base = row0 & ~15
        maps.append((base, (row0 - base) // 2, (m - f + PHASES - 1) // PHASES))
    return maps


def check_row_path(m, k, ld_x, x_off, rng):
    x_addr = 0x7F0000000000 + 2 * x_off
    vals = rng.integers(0, 1 << 16, size=(m, k))
    maps = phase_maps(x_addr, m, ld_x, k)
    stride = 16 * ld_x
    for f, (base, d, rows) in enumerate(maps):
        assert base % 16 == 0 and d < 8 and stride % 16 == 0 and stride >= 2 * (k + d)
        for j in range(rows):
            r = PHASES * j + f
            assert r < m
            lo_ok = (x_addr + 2 * r * ld_x) & ~15                      # first chunk of row r
            hi_ok = (x_addr + 2 * (r * ld_x + k) + 15) & ~15           # end of its last chunk
            for ct in range(-(-k // 128)):
                e0, e1 = 128 * ct, min(128 * ct + BOX_COLS, k + d)     # map columns a box reads
                if e0 >= e1:
                    continue
                assert lo_ok <= base + stride * j + 2 * e0 and base + stride * j + 2 * e1 <= hi_ok
                # the kernel's misalignment: low 4 bits of X's address of (r, 128 ct), in 32-bit arithmetic
                off = ((x_addr & 0xFFFFFFFF) + 2 * ((r * ld_x) & 0xFFFFFFFF) + 2 * 128 * ct) & 15
                assert off == 2 * d
                for h in range(2):
                    cf = 128 * ct + 64 * h
                    if cf >= k:
                        continue
                    cols = np.arange(cf, cf + 64)
                    box_idx = off // 2 + 64 * h + np.arange(64)          # element of the box row
                    src_col = 128 * ct + box_idx - d                      # row column it holds
                    got = np.where(cols < k, vals[r, np.minimum(src_col, k - 1)], 0)
                    want = np.where(cols < k, vals[r, np.minimum(cols, k - 1)], 0)
                    assert np.array_equal(got, want)


@pytest.mark.parametrize("m,k,ld_x,x_off", [(1, 1, 1, 1), (3, 5, 5, 1), (7, 33, 37, 3), (8, 255, 255, 0),
                                            (9, 129, 131, 5), (130, 300, 301, 2), (257, 1000, 1003, 7),
                                            (77, 520, 777, 1), (40, 8191, 8191, 0), (17, 4097, 4099, 6)])
def test_row_path_maps_read_only_the_rows_own_chunks(m, k, ld_x, x_off):
    check_row_path(m, k, ld_x, x_off, np.random.default_rng(m * 1000 + k))


def test_row_path_maps_random_layouts():
    rng = np.random.default_rng(5)
    for _ in range(40):
        k = int(rng.integers(1, 700))
        ld_x = k + int(rng.integers(0, 20))
        m = int(rng.integers(1, 300))
        check_row_path(m, k, ld_x, int(rng.integers(0, 8)), rng)


def funnel_r(lo, hi, sh):
    return ((hi << 32 | lo) >> sh) & 0xFFFFFFFF


def bytes_from(a, b, h):
    """bytes_from in stores.cuh: 16 bytes from byte h of the 32 bytes a | b,
    a and b given as 4 little-endian words each."""
    w = list(a) + list(b)
    q, sh = h >> 2, 8 * (h & 3)
    return [funnel_r(w[q + t], w[q + t + 1], sh) for t in range(4)]


def store_row_any(dst, seg, words):
    """The stores store_row_any issues for one row segment: (address, size,
    value), from the chunks each lane loads (its own and the next) and the
    boundary bytes it reads from the staging row."""
    stores = []
    d = dst & 15
    chunk = [words[4 * i:4 * i + 4] for i in range(8)]
    seg_bytes = b"".join(w.to_bytes(4, "little") for w in words)
    for c in range(8):
        if d & 3 == 0:                                   # 4-byte aligned row: each lane's own chunk
            if 16 * c < seg:
                a = dst + 16 * c
                width = 16 if a % 16 == 0 else 8 if a % 8 == 0 else 4
                for o in range(0, 16, width):
                    i = (16 * c + o) // 4
                    stores.append((a + o, width, sum(words[i + t] << (32 * t) for t in range(width // 4))))
            continue
        v, vn = chunk[c], chunk[min(c + 1, 7)]
        h = 16 - d
        if 16 * (c + 1) < seg:                           # aligned chunk c + 1
            out = bytes_from(v, vn, h)
            stores.append((dst - d + 16 * (c + 1), 16, sum(out[t] << (32 * t) for t in range(4))))
        for j in (c, c + 8):                             # boundary slots: head bytes, then tail bytes
            o = j if j < h else seg - 16 + j
            stores.append((dst + o, 1, seg_bytes[o]))
    return stores


@pytest.mark.parametrize("seg", [32, 64, 96, 128])
def test_any_offset_row_store_writes_each_byte_once(seg):
    rng = np.random.default_rng(seg)
    for start in range(256, 256 + 16):                   # every offset within a 16-byte chunk
        data = rng.integers(0, 256, size=128, dtype=np.uint8)
        data[seg:] = 0
        words = [int.from_bytes(data[4 * i:4 * i + 4].tobytes(), "little") for i in range(32)]
        count = np.zeros(1024, dtype=int)
        mem = np.zeros(1024, dtype=np.uint8)
        for addr, size, value in store_row_any(start, seg, words):
            assert addr % size == 0, (start, seg, addr, size)
            for b in range(size):
                mem[addr + b] = (value >> (8 * b)) & 0xFF
                count[addr + b] += 1
        assert np.array_equal(mem[start:start + seg], data[:seg]), (start, seg)
        assert (count[start:start + seg] == 1).all(), (start, seg)
        assert count[:start].sum() == 0 and count[start + seg:].sum() == 0, (start, seg)
