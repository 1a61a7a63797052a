"""CPU: host-side step planning, chunking, packing and the KV page allocator."""

from __future__ import annotations

import numpy as np
import pytest

from imba_chess_b200 import _native
from imba_chess_b200.plan import StepPlan, build_chunks


def test_chunks_cover_every_row_once_grouped_and_bounded():
    rng = np.random.default_rng(0)
    for _ in range(50):
        G = int(rng.integers(1, 20))
        R = int(rng.integers(0, 400))
        row_group = rng.integers(0, G, R)
        perm, cg, co, cn = build_chunks(row_group, G)
        assert sorted(perm.tolist()) == list(range(R))
        assert (cn >= 1).all() and (cn <= _native.CHUNK_ROWS).all()
        assert int(cn.sum()) == R
        for c in range(len(cg)):
            rows = perm[co[c] : co[c] + cn[c]]
            assert (row_group[rows] == cg[c]).all()
        # within a group rows keep their original order (prefill causality relies on it)
        for g in range(G):
            rows = perm[np.isin(perm, np.nonzero(row_group == g)[0])]
            assert (np.diff(rows) > 0).all()


def test_group_with_many_rows_is_split_evenly():
    perm, cg, co, cn = build_chunks(np.zeros(130, np.int64), 1)
    assert cn.tolist() == [26] * 5
    perm, cg, co, cn = build_chunks(np.zeros(130, np.int64), 1, max_rows=64)
    assert cn.tolist() == [43, 43, 44]


def test_chunks_listed_longest_prefix_first():
    rng = np.random.default_rng(2)
    G = 9
    row_group = rng.integers(0, G, 300)
    group_vis = rng.integers(1, 400, G)
    row_vis = group_vis[row_group]
    perm, cg, co, cn = build_chunks(row_group, G, row_vis=row_vis)
    cost = [int(row_vis[perm[o : o + n]].max()) for o, n in zip(co, cn)]
    assert cost == sorted(cost, reverse=True)
    assert int(cn.sum()) == 300 and (cn <= 32).all()
    for c in range(len(cg)):
        assert (row_group[perm[co[c] : co[c] + cn[c]]] == cg[c]).all()


def test_prefill_steps_take_64_row_chunks_and_decode_steps_32():
    """Steps without extra keys (prefills) are chunked by 64 rows (one
    prefill-attention unit stacks a chunk's rows for two heads in a 128-row
    tile); steps with extra keys by 32 (one decode-attention item)."""
    from imba_chess_b200.kvpool import KVPool, KVSequence
    from imba_chess_b200.steps import root_plan
    from imba_chess_b200 import synth

    dims = synth.ModelDims(128, 1, 2)
    import torch

    pool = KVPool(num_layers=1, num_heads=2, attention_dim=64, linear_dim=64, num_pages=64, dtype=torch.float32,
                  device=torch.device("cpu"))
    seqs = [KVSequence(pool) for _ in range(2)]
    rng = np.random.default_rng(4)
    plan, _ = root_plan(seqs, [synth.random_tokens(rng, n, dims) for n in (150, 40)])
    plan.finalize()
    _, cg, co, cn = plan.chunks
    assert int(cn.max()) > 32 and int(cn.max()) <= 64 and int(cn.sum()) == 190
    decode = _plan(70)
    decode.row_extra_off = np.arange(71, dtype=np.int32)
    decode.extra_slot = np.arange(70, dtype=np.int32)
    decode.extra_pos = np.arange(70, dtype=np.int32)
    decode.finalize()
    assert int(decode.chunks[3].max()) <= 32


def _plan(R=5):
    rng = np.random.default_rng(1)
    return StepPlan(
        piece_ids=rng.integers(0, 13, (R, 64)).astype(np.uint8),
        side_ids=rng.integers(0, 9, (R, 7)).astype(np.int32),
        positions=np.arange(R, dtype=np.int32),
        row_group=np.zeros(R, np.int32),
        row_vis=np.arange(1, R + 1, dtype=np.int32),
        row_extra_off=np.zeros(R + 1, np.int32),
        extra_slot=np.zeros(0, np.int32),
        extra_pos=np.zeros(0, np.int32),
        row_dst_slot=np.arange(R, dtype=np.int32),
        group_page_off=np.array([0, 1], np.int32),
        group_pages=np.array([0], np.int32),
        legal_off=np.array([0, 2, 2, 5, 6, 6], np.int32),
        legal_ids=np.array([3, 4, 5, 6, 7, 8], np.int32),
    )


def test_pack_round_trips_every_section():
    p = _plan()
    buf, layout = p.pack()
    arrs = p.arrays()
    R = p.num_rows
    assert np.array_equal(buf.view(np.uint8)[: R * 64], p.piece_ids.reshape(-1))
    for name, a in arrs.items():
        off, n = layout[name]
        assert off % 4 == 0  # 16-byte aligned sections
        assert np.array_equal(buf[off : off + n], a)
    c = p.counts()
    assert c["num_rows"] == 5 and c["num_legal"] == 6 and c["num_chunks"] == 1


def test_kv_sequence_slots_and_refcounts():
    torch = pytest.importorskip("torch")
    from imba_chess_b200.kvpool import KVPool, KVPoolExhausted, KVSequence

    pool = KVPool(num_layers=1, num_heads=1, attention_dim=8, linear_dim=8, num_pages=6,
                  dtype=torch.float32, device=torch.device("cpu"))
    a = KVSequence(pool)
    s0 = a.reserve(20)  # 2 pages
    assert len(a.pages) == 2 and a.length == 20
    assert np.array_equal(s0, np.concatenate([a.pages[0] * 16 + np.arange(16), a.pages[1] * 16 + np.arange(4)]))
    s1 = a.reserve(12)  # fills page 2, spills to a third
    assert len(a.pages) == 2 + 0 or len(a.pages) == 2  # 32 tokens fit in exactly two pages
    assert np.array_equal(s1, a.slots(20, 32))
    b = a.retain()
    a.release()
    assert pool.free_pages == 4  # still held by the snapshot
    b.release()
    assert pool.free_pages == 6
    c = KVSequence(pool)
    with pytest.raises(KVPoolExhausted):
        c.reserve(16 * 7)


def test_reserve_many_matches_sequential_reserves():
    """KVSequence.reserve_many (one vectorised pass, used by the wave planner)
    gives the same slots, page lists and lengths as calling reserve() on each
    sequence in turn, including a sequence listed more than once."""
    torch = pytest.importorskip("torch")
    from imba_chess_b200.kvpool import KVPool, KVSequence

    rng = np.random.default_rng(3)
    for _ in range(20):
        pools = [KVPool(num_layers=1, num_heads=1, attention_dim=8, linear_dim=8, num_pages=400,
                        dtype=torch.float32, device=torch.device("cpu")) for _ in range(2)]
        pre = [int(x) for x in rng.integers(0, 40, 4)]
        order = [int(x) for x in rng.integers(0, 4, 7)]
        counts = [int(x) for x in rng.integers(0, 35, 7)]
        out = []
        for k, pool in enumerate(pools):
            seqs = [KVSequence(pool) for _ in range(4)]
            for s, n in zip(seqs, pre):
                s.reserve(n)
            listed = [seqs[i] for i in order]
            if k == 0:
                slots = np.concatenate([s.reserve(c) for s, c in zip(listed, counts)])
            else:
                slots = KVSequence.reserve_many(listed, counts)
            out.append((slots, [s.pages for s in seqs], [s.length for s in seqs]))
        assert np.array_equal(out[0][0], out[1][0])
        assert out[0][1] == out[1][1] and out[0][2] == out[1][2]
