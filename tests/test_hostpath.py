"""CPU: the C++ host path of the wave service (request packing and response
rows) against a plain-Python restatement of the same conversions."""

from __future__ import annotations

import numpy as np
import pytest

from imba_chess_b200 import _hostpath, synth
from imba_chess_b200.protocol import WaveRequest, WaveRow
from imba_chess_b200.steps import ids_csr

FIELDS = ("turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id")
NO_PARENT = -(2**63)


def _requests(seed=5, n_req=7):
    rng = np.random.default_rng(seed)
    reqs = []
    node = 0
    for g in range(n_req):
        k = int(rng.integers(0, 9))  # includes a request without rows
        tok = synth.random_tokens(rng, k, synth.D256)
        rows = []
        for i in range(k):
            bs = {"piece_ids": tok["piece_ids"][i].tolist(), **{f: int(tok[f][i]) for f in FIELDS}}
            legal = synth.random_legal_ids(rng, int(rng.integers(0, 40)), 1970).tolist()
            parent = None if rng.random() < 0.5 else int(rng.integers(0, 1000))
            rows.append(WaveRow(node_id=node, parent_id=parent, prev_move_vocab_id=int(tok["prev_move_id"][i]),
                                board_state=bs, legal_vocab_ids=legal))
            node += 1
        reqs.append(WaveRequest(worker_id=g, turn_id=0, rows=rows))
    return reqs


def test_pack_matches_python_restatement():
    reqs = _requests()
    rows = [r for q in reqs for r in q.rows]
    R = len(rows)
    piece = np.empty((R, 64), np.uint8)
    side = np.zeros((R, 7), np.int32)
    n, loff_b, lids_b, node_b, parent_b = _hostpath.pack_wave_rows(reqs, piece, side)
    assert n == R
    assert np.array_equal(piece, np.array([r.board_state["piece_ids"] for r in rows], np.uint8))
    exp_side = np.array([[0] + [r.board_state[f] for f in FIELDS] + [r.prev_move_vocab_id] for r in rows], np.int32)
    assert np.array_equal(side[:, 1:], exp_side[:, 1:])
    off, ids = ids_csr([r.legal_vocab_ids for r in rows])
    assert np.array_equal(np.frombuffer(loff_b, np.int32), off)
    assert np.array_equal(np.frombuffer(lids_b, np.int32), ids)
    assert np.frombuffer(node_b, np.int64).tolist() == [r.node_id for r in rows]
    assert np.frombuffer(parent_b, np.int64).tolist() == [NO_PARENT if r.parent_id is None else r.parent_id for r in rows]


def test_pack_rejects_bad_boards():
    reqs = _requests(seed=6, n_req=3)
    rows = [r for q in reqs for r in q.rows]
    piece = np.empty((len(rows), 64), np.uint8)
    side = np.empty((len(rows), 7), np.int32)
    rows[0].board_state["piece_ids"][5] = 13
    with pytest.raises(ValueError, match=r"\[0, 12\]"):
        _hostpath.pack_wave_rows(reqs, piece, side)
    rows[0].board_state["piece_ids"][5] = 0
    rows[0].board_state["piece_ids"].append(0)
    with pytest.raises(ValueError, match="64 piece_ids"):
        _hostpath.pack_wave_rows(reqs, piece, side)
    rows[0].board_state["piece_ids"].pop()
    del rows[0].board_state["turn_id"]
    with pytest.raises(KeyError):
        _hostpath.pack_wave_rows(reqs, piece, side)
    with pytest.raises(ValueError, match="too small"):
        _hostpath.pack_wave_rows(reqs, piece[:0], side)


def test_responses_match_python_restatement():
    rng = np.random.default_rng(9)
    counts = [3, 0, 5, 1]
    R = sum(counts)
    lens = rng.integers(0, 6, R)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    vals = rng.standard_normal(R).astype(np.float32)
    legal = rng.standard_normal(int(off[-1])).astype(np.float32)
    got = _hostpath.wave_responses(counts, vals, legal, off)
    exp, r = [], 0
    for n in counts:
        exp.append([(float(vals[i]), legal[off[i] : off[i + 1]].tolist()) for i in range(r, r + n)])
        r += n
    assert got == exp
    with pytest.raises(TypeError):
        _hostpath.wave_responses(counts, vals.astype(np.float64), legal, off)
    with pytest.raises(ValueError):
        _hostpath.wave_responses([R + 1], vals, legal, np.zeros(R + 1, np.int32))


def test_ids_csr_matches_python_restatement():
    rng = np.random.default_rng(3)
    rows = [synth.random_legal_ids(rng, int(rng.integers(0, 40)), 1970).tolist() for _ in range(50)]
    rows[7] = []
    rows[11] = tuple(rows[11])
    rows[13] = np.asarray(rows[13], dtype=np.int64)  # numpy integers take the general conversion
    off, ids = ids_csr(rows)
    want_off = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    want_ids = np.asarray([int(v) for r in rows for v in r], dtype=np.int32)
    assert off.dtype == np.int32 and ids.dtype == np.int32
    np.testing.assert_array_equal(off, want_off)
    np.testing.assert_array_equal(ids, want_ids)
    off, ids = ids_csr([])
    assert off.tolist() == [0] and ids.size == 0
    with pytest.raises(TypeError):
        ids_csr([[1, 2.5]])
    with pytest.raises(TypeError):
        ids_csr([3])
