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

Q_REGION = 128 * 128  # Q: 128 rows x 128 columns -> two 16 KiB regions
KV_REGION = 64 * 128  # K, V: 64 rows x 128 columns -> two 8 KiB regions
P_REGION = 128 * 128  # P: 128 rows x 64 columns -> one 16 KiB region (written into the K buffer)


def sw128_offset(row, unit16, region):
    return (unit16 >> 3) * region + row * 128 + (((unit16 & 7) ^ (row & 7)) << 4)


def writer_addr(row, col, region):
    """Byte offset of element (row, col) of a 16-bit operand as the kernel writes it."""
    return sw128_offset(row, col // 8, region) + (col % 8) * 2


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
    f = decode(desc(0x8000, KV_REGION, 1024))
    assert f["lbo"] == KV_REGION and f["sbo"] == 1024
    i = idesc(1, 1, 128, 128)
    assert (i >> 4) & 3 == 1 and (i >> 7) & 7 == 1 and (i >> 10) & 7 == 1
    assert (i >> 15) & 1 == 0 and (i >> 16) & 1 == 1
    assert (i >> 17) & 0x3F == 16 and (i >> 24) & 0x1F == 8
    assert (idesc(1, 0, 128, 64) >> 17) & 0x3F == 8


def test_qk_operands_read_what_the_writer_stored():
    base_q, base_k = 0, 32768  # Q at 0, first K buffer right after (both 1024-aligned)
    for s in range(8):  # k-steps over head_dim
        dq = desc(base_q + (s >> 2) * Q_REGION + (s & 3) * 32, 16, 1024)
        dk = desc(base_k + (s >> 2) * KV_REGION + (s & 3) * 32, 16, 1024)
        for k in range(16):
            col = s * 16 + k
            for m in range(128):  # M = 128 query rows
                a = kmajor_read(dq, m, k)
                assert a == base_q + writer_addr(m, col, Q_REGION)
                assert base_q <= a < base_q + 2 * Q_REGION
            for n in range(64):  # N = 64 KV rows
                a = kmajor_read(dk, n, k)
                assert a == base_k + writer_addr(n, col, KV_REGION)
                assert base_k <= a < base_k + 2 * KV_REGION


def test_pv_operands_read_what_the_writer_stored():
    base_p, base_v = 32768, 65536  # P lives in the tile's K buffer; V in its own buffer
    for s in range(4):  # k-steps over the 64 KV positions of the tile
        dp = desc(base_p + s * 32, 16, 1024)
        dv = desc(base_v + s * 2048, KV_REGION, 1024)
        for k in range(16):
            kv = s * 16 + k
            for m in range(128):
                a = kmajor_read(dp, m, k)
                assert a == base_p + writer_addr(m, kv, P_REGION)
                assert base_p <= a < base_p + P_REGION  # P fits the 16 KiB K buffer
            for n in range(128):  # N = head_dim column of V
                a = mnmajor_read(dv, n, k)
                assert a == base_v + writer_addr(kv, n, KV_REGION)
                assert base_v <= a < base_v + 2 * KV_REGION


PAIR, STAGES = 2, 4  # row tiles per CTA; depth of the K and of the V ring


def test_smem_budget_one_cta_per_sm():
    q = PAIR * 2 * Q_REGION
    kv = 2 * STAGES * (2 * KV_REGION)
    per_cta = q + kv + 256 + 65 * 8 + 1024  # + barriers, page ids, alignment slack
    assert per_cta <= 227 * 1024
    assert 2 * (per_cta + 1024) > 228 * 1024  # never two CTAs on one SM: each allocates all 512 TMEM columns
    barriers = 1 + 4 * STAGES + 2 * PAIR * 2 + 2 * PAIR
    assert barriers * 8 + 4 <= 256


def test_tmem_columns():
    s_cols = [(g * 128 + st * 64, g * 128 + st * 64 + 64) for g in range(PAIR) for st in range(2)]
    o_cols = [(256 + g * 128, 256 + g * 128 + 128) for g in range(PAIR)]
    spans = sorted(s_cols + o_cols)
    assert spans[0][0] == 0 and spans[-1][1] == 512
    assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:]))  # disjoint
    # P(i) of row tile g: 32 columns (64 16-bit values per row) at the start of its S buffer; the
    # 4 PV k-steps read 8 columns each
    for g in range(PAIR):
        for st in range(2):
            lo = g * 128 + st * 64
            assert all(lo <= lo + ks * 8 and lo + ks * 8 + 8 <= lo + 32 for ks in range(4))
