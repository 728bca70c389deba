"""The partition arithmetic of the fused single-token kernel, restated on the CPU.

minimax-rs_b200/csrc/decode.cu splits one token's MoE block over the grid: `decode_configure`
derives the per-CTA sizes (gate/up slots, output rows, rows per copy unit, stage size),
`gu_range` gives each CTA a whole number of 32-row Q8_1 blocks of the computed (position, row)
pairs, and `table_structure` cuts a CTA's range into copy units, one producer lane per chunk.
Expert parallelism drops the slots another rank owns before the split, so a rank may compute
anywhere from 0 to 8 positions of a token.  These tests restate that arithmetic and check, for
every position count and several grid sizes, that each row is computed exactly once and that
every bound the kernel's fixed tables rely on holds (one lane per chunk: at most 32 chunks;
units within kMaxUnits; partial-sum rows within act_slots; a unit within a stage).
"""
from __future__ import annotations

import pytest

QK_K, TOPK, K_MAX_UNITS, K_CONSUMER_THREADS = 256, 8, 80, 384
Q4K, Q5K = 1, 4
BLOCK_BYTES = {Q4K: 144, Q5K: 176}


def row_bytes(t: int, k: int) -> int:
    return (k // QK_K) * BLOCK_BYTES[t]


def configure(H: int, I: int, gu: int, dn: int, sms: int) -> dict:
    """decode_configure's derived sizes (stage count aside: it depends on shared memory)."""
    act_slots = 32 * ((TOPK * I // 32 + sms - 1) // sms) + 1
    res_slots = (H + sms - 1) // sms + 1
    gu_row, dn_stage = row_bytes(gu, H), row_bytes(dn, I) * (res_slots - 1)
    gu_unit_rows = max(4, dn_stage // gu_row)
    max_chunks = (act_slots + gu_unit_rows - 1) // gu_unit_rows + TOPK
    ok = (H // QK_K <= K_CONSUMER_THREADS and TOPK * (I // QK_K) <= K_CONSUMER_THREADS and max_chunks <= 32
          and 2 * max_chunks + TOPK <= K_MAX_UNITS)
    stage_bytes = (max(gu_row * gu_unit_rows, dn_stage) + 127) // 128 * 128
    return dict(act_slots=act_slots, res_slots=res_slots, gu_unit_rows=gu_unit_rows, stage_bytes=stage_bytes,
                supported=ok, gu_row=gu_row, dn_row=row_bytes(dn, I))


def gu_range(cta: int, G: int, nvs: int, I: int) -> tuple[int, int]:
    nblk = nvs * I // 32
    return 32 * (cta * nblk // G), 32 * ((cta + 1) * nblk // G)


def table_structure(cta: int, G: int, nv: int, I: int, U: int):
    """The chunks (position, first row, rows, offset in the range) of a CTA, in lane order."""
    p0, p1 = gu_range(cta, G, nv, I)
    chunks, q, pos = [], p0, p0 // I
    while q < p1:
        seg_end = min(p1, (pos + 1) * I)
        for r in range(q, seg_end, U):
            chunks.append((pos, r - pos * I, min(U, seg_end - r), r - p0))
        q, pos = seg_end, pos + 1
    return p0, p1, chunks


SHAPES = [
    (3072, 1536, Q4K, Q5K),  # MiniMax-M2.7, one GPU or expert parallel
    (3072, 768, Q4K, Q5K),   # a TP = 2 rank's shard
    (1024, 512, Q4K, Q5K),   # smoke test shape
    (512, 512, Q4K, Q5K),    # multi-GPU test shape
    (512, 512, Q5K, Q4K),
]


@pytest.mark.parametrize("H,I,gu,dn", SHAPES)
@pytest.mark.parametrize("sms", [148, 132, 160])
def test_every_row_once_within_the_tables(H, I, gu, dn, sms):
    c = configure(H, I, gu, dn, sms)
    assert c["supported"]
    U = c["gu_unit_rows"]
    assert c["stage_bytes"] >= c["gu_row"] * U and c["stage_bytes"] >= c["dn_row"] * (c["res_slots"] - 1)
    for nvs in range(0, TOPK + 1):  # expert parallel: 0..8 positions computed on this rank
        seen = [0] * (nvs * I)
        for cta in range(sms):
            p0, p1, chunks = table_structure(cta, sms, nvs, I, U)
            assert p0 % 32 == 0 and p1 % 32 == 0  # whole Q8_1 blocks: the CTA quantises its own act
            cnt = p1 - p0
            assert cnt <= c["act_slots"] - 1  # partial-sum rows and row map entries (2 act_slots)
            assert len(chunks) <= 32  # one producer lane per chunk
            n_units = 2 * len(chunks) + nvs
            assert n_units <= K_MAX_UNITS
            off = 0
            for pos, row0, n, o in chunks:
                assert o == off and 0 < n <= U and 0 <= row0 and row0 + n <= I  # never across a position
                for r in range(n):
                    seen[pos * I + row0 + r] += 1
                off += n
            assert off == cnt
        assert seen == [1] * (nvs * I)


@pytest.mark.parametrize("H", [3072, 1024, 512])
@pytest.mark.parametrize("sms", [148, 132, 160])
def test_output_rows_partition(H, sms):
    """Each CTA reduces and writes its contiguous output rows [cta H / G, (cta + 1) H / G)."""
    res_slots = (H + sms - 1) // sms + 1
    rows = []
    for cta in range(sms):
        r0, r1 = cta * H // sms, (cta + 1) * H // sms
        assert r1 - r0 <= res_slots - 1
        rows.extend(range(r0, r1))
    assert rows == list(range(H))


def test_rank_with_no_expert_computes_nothing():
    """A rank that owns none of the token's eight experts (nvs = 0): empty ranges, no gate/up
    units, no down units; it only adds its zero rows to the exchange."""
    c = configure(3072, 1536, Q4K, Q5K, 148)
    for cta in range(148):
        p0, p1, chunks = table_structure(cta, 148, 0, 1536, c["gu_unit_rows"])
        assert (p0, p1, chunks) == (0, 0, [])


def test_expert_parallel_slot_compaction():
    """Slots whose expert another rank owns (e % W != rank) are dropped; the kept ones become
    positions 0..nvs-1 in slot order, and every slot is computed by exactly one rank."""
    import itertools
    ids = [3, 17, 42, 64, 101, 130, 200, 255]
    for W in (2, 4, 8):
        owners = [[] for _ in range(W)]
        for rank in range(W):
            kept = [k for k, e in enumerate(ids) if e % W == rank]
            posof = {k: i for i, k in enumerate(kept)}
            for k in range(TOPK):
                assert (k in posof) == (ids[k] % W == rank)
            owners[rank] = kept
        assert sorted(itertools.chain(*owners)) == list(range(TOPK))
