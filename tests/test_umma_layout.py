"""CPU check of the tcgen05 operand layouts used by the chunked-prefill kernel.

The kernel writes Q, K, V and P into shared memory with ``sw128_offset`` (128-byte rows, 16-byte
unit u of row r stored at unit u ^ (r % 8), 64 columns per 16 KiB region) and describes them to
``tcgen05.mma`` with 64-bit shared-memory descriptors.  This test restates both sides:

* the descriptor bit packing (start>>4 at bits 0-13, LBO>>4 at 16-29, SBO>>4 at 32-45, version 1 at
  46, swizzle mode 2 = 128B at 61-63) and the instruction descriptor (f32 accumulate, bf16 A/B,
  majors, N>>3 at 17-22, M>>4 at 24-28);
* the canonical SW128 layouts the hardware reads: K-major ((8,m),(8,2)):((128B,SBO),(2B,16B)) and
  MN-major ((64,m),(8,k)):((2B,LBO),(128B,SBO)), each followed by the 128-byte XOR swizzle of
  address bits [4:6] with bits [7:9];

and checks that every element each of the 8 + 8 MMAs of a tile reads sits exactly where the
writer put it, and that no read leaves the operand's 32 KiB buffer.
"""

REGION = 16384
TILE = 32768


def sw128_offset(row, unit16):
    return (unit16 >> 3) * REGION + row * 128 + (((unit16 & 7) ^ (row & 7)) << 4)


def writer_addr(row, col):
    """Byte offset of element (row, col) of a 128 x 128 16-bit operand as the kernel writes it."""
    return sw128_offset(row, col // 8) + (col % 8) * 2


def swizzle(addr):
    return addr ^ (((addr >> 7) & 7) << 4)


def desc(start, lbo, sbo):
    return (start >> 4) & 0x3FFF | (lbo >> 4) << 16 | (sbo >> 4) << 32 | 1 << 46 | 2 << 61


def decode(d):
    return dict(start=(d & 0x3FFF) << 4, lbo=((d >> 16) & 0x3FFF) << 4, sbo=((d >> 32) & 0x3FFF) << 4,
                version=(d >> 46) & 3, layout=(d >> 61) & 7)


def kmajor_read(d, m, k):
    """Address the MMA reads for element (m, k), k in [0, 16), of a K-major SW128 operand."""
    f = decode(d)
    return swizzle(f["start"] + (m // 8) * f["sbo"] + (m % 8) * 128 + k * 2)


def mnmajor_read(d, n, k):
    """Address the MMA reads for element (n, k), n along N (contiguous), k in [0, 16)."""
    f = decode(d)
    return swizzle(f["start"] + (n // 64) * f["lbo"] + (k // 8) * f["sbo"] + (k % 8) * 128 + (n % 64) * 2)


def idesc(bf16, b_mn, m, n):
    return 1 << 4 | bf16 << 7 | bf16 << 10 | b_mn << 16 | (n >> 3) << 17 | (m >> 4) << 24


def test_descriptor_fields():
    f = decode(desc(0x1A400, 16, 1024))
    assert f == dict(start=0x1A400, lbo=16, sbo=1024, version=1, layout=2)
    f = decode(desc(0x28000, REGION, 1024))
    assert f["lbo"] == REGION and f["sbo"] == 1024
    i = idesc(1, 1, 128, 128)
    assert (i >> 4) & 3 == 1 and (i >> 7) & 7 == 1 and (i >> 10) & 7 == 1
    assert (i >> 15) & 1 == 0 and (i >> 16) & 1 == 1
    assert (i >> 17) & 0x3F == 16 and (i >> 24) & 0x1F == 8


def test_qk_operands_read_what_the_writer_stored():
    base_q, base_k = 0, 1024 * 64  # any 1024-aligned buffers
    for s in range(8):  # k-steps over head_dim
        off = (s >> 2) * REGION + (s & 3) * 32
        dq, dk = desc(base_q + off, 16, 1024), desc(base_k + off, 16, 1024)
        for m in range(128):
            for k in range(16):
                col = s * 16 + k
                a = kmajor_read(dq, m, k)
                assert a == base_q + writer_addr(m, col)
                assert base_q <= a < base_q + TILE
                assert kmajor_read(dk, m, k) == base_k + writer_addr(m, col)


def test_pv_operands_read_what_the_writer_stored():
    base_p, base_v = 4 * TILE, 5 * TILE
    for s in range(8):  # k-steps over the 128 KV positions of the tile
        poff = (s >> 2) * REGION + (s & 3) * 32
        dp = desc(base_p + poff, 16, 1024)
        dv = desc(base_v + s * 2048, REGION, 1024)
        for k in range(16):
            kv = s * 16 + k
            for m in range(128):
                assert kmajor_read(dp, m, k) == base_p + writer_addr(m, kv)
            for n in range(128):  # N = head_dim column of V
                a = mnmajor_read(dv, n, k)
                assert a == base_v + writer_addr(kv, n)
                assert base_v <= a < base_v + TILE


def test_smem_budget():
    # Q + 2 K + 2 V + P tiles + barriers + alignment slack must fit the 227 KiB opt-in limit
    assert 6 * TILE + 64 + 1024 <= 227 * 1024
