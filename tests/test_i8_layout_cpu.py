"""The int8 operand layout of the prompt pass's kind::i8 GEMM (csrc/grouped_mma.cuh), restated in integers: the
staging kernel's writes of a row's int8 codes (lane l of the row's warp holds columns 256 q + 8 l .. + 7) and the
converters' writes of a weight row's codes (16 columns per 16-byte piece) must both put column c of row r where a
K-major, 128-byte-swizzled operand block of 128-column chunks holds it: chunk c // 128, 16-byte piece
(c % 128) // 16 stored at position piece ^ (r % 8) of the row, byte c % 16 within it. Then every MMA K step (32
bytes) pairs the same columns of A and B."""
GM_B_BYTES = 128 * 128  # one 128-column int8 chunk of 128 rows


def sw128_offset(r, c):
    """Byte offset of 16-byte piece c of row r in a K-major block with the 128-byte swizzle (8-row atoms of 1024 B)."""
    return (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)


def canonical(r, col):
    """(chunk, byte offset in the chunk's block) of column col of row r."""
    return col // 128, sw128_offset(r, (col % 128) // 16) + col % 16


def staged_byte(r, q, lane, u):
    """Where the staging kernel writes byte u (0..7) of lane `lane`'s 8 columns of 256-column group q, row r."""
    chunk = 2 * q + (lane >> 4)
    return chunk, sw128_offset(r, (lane & 15) >> 1) + 8 * (lane & 1) + u


def converted_byte(r, h, g, i):
    """Where a converter writes byte i of 16-column group g (0..7) of the chunk h of weight row r."""
    return h, sw128_offset(r, g) + i


def test_staged_activation_bytes_sit_where_the_mma_reads_them():
    seen = set()
    for r in range(128):
        for q in range(8):  # K = 2048
            for lane in range(32):
                for u in range(8):
                    col = 256 * q + 8 * lane + u
                    pos = staged_byte(r, q, lane, u)
                    assert pos == canonical(r, col)
                    seen.add((r,) + pos)
    assert len(seen) == 128 * 2048  # every byte of the 16 chunk blocks written once


def test_converted_weight_bytes_sit_where_the_mma_reads_them():
    for r in range(128):
        for h in range(16):
            for g in range(8):
                for i in range(16):
                    assert converted_byte(r, h, g, i) == canonical(r, 128 * h + 16 * g + i)


def test_k_steps_pair_the_same_columns():
    """K step s of a chunk reads bytes 32 s .. 32 s + 31 of each row (the descriptor's start advanced by 32 bytes
    within the swizzle atom): the same 32 columns for A and B."""
    for r in range(16):
        for s in range(4):
            cols = [c for c in range(128) if 32 * s <= c < 32 * s + 32]
            a = sorted(canonical(r, c)[1] for c in cols)
            b = sorted(staged_byte(r, 0, lane, u)[1] for lane in range(16) for u in range(8)
                       if 32 * s <= 8 * lane + u < 32 * s + 32)
            assert a == b
    assert GM_B_BYTES == 16384
