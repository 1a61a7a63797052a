"""CPU: worker-side chess (the C++ ``_chess`` extension behind
``imba_chess_b200.worker_chess``): move generation, the static move
vocabulary, the UCI-sorted legal-id projection and the board-state encoding.

python-chess and cozy-chess are not installed here, so the move generator is
pinned by perft counts -- the number of leaf nodes of the legal move tree,
published for the six positions the reference's own tests use as edge cases
(tests/test_cozy_bridge.py:15-22: the start position, "Kiwipete" and the
other standard perft positions, with castling, en passant, promotions,
pins and checks) -- and the vocabulary and encoding by the facts the
reference's tests/test_move_vocab.py and tests/test_board_state.py assert.
"""

from __future__ import annotations

import numpy as np
import pytest

from imba_chess_b200 import worker_chess as wc

START = "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1"
# tests/test_cozy_bridge.py:15-22 of the reference
EDGE_FENS = [
    START,
    "r3k2r/p1ppqpb1/bn2pnp1/3PN3/1p2P3/2N2Q1p/PPPBBPPP/R3K2R w KQkq - 0 1",
    "8/2p5/3p4/KP5r/1R3p1k/8/4P1P1/8 w - - 0 1",
    "r3k2r/Pppp1ppp/1b3nbN/nP6/BBP1P3/q4N2/Pp1P2PP/R2Q1RK1 w kq - 0 1",
    "rnbq1k1r/pp1Pbppp/2p5/8/2B5/8/PPP1NnPP/RNBQK2R w KQ - 1 8",
    "r4rk1/1pp1qppp/p1np1n2/2b1p1B1/2B1P1b1/P1NP1N2/1PP1QPPP/R4RK1 w - - 0 10",
]
# Published perft leaf counts of those positions, depths 1..3 (and 4 for the
# three cheapest).
PERFT = [
    [20, 400, 8902, 197281],
    [48, 2039, 97862],
    [14, 191, 2812, 43238],
    [6, 264, 9467, 422333],
    [44, 1486, 62379],
    [46, 2079, 89890],
]


@pytest.mark.parametrize("i", range(len(EDGE_FENS)))
def test_perft_matches_published_counts(i):
    for depth, want in enumerate(PERFT[i], start=1):
        assert wc.perft(EDGE_FENS[i], depth) == want, (EDGE_FENS[i], depth)


def test_static_vocab_layout():
    v = wc.static_move_vocab()
    assert len(v) == 1970
    assert v["<pad>"] == 0 and v["<start>"] == 1
    toks = list(v)
    assert toks[2:5] == ["a1b1", "a1c1", "a1d1"]  # a1's queen / knight targets in square order
    assert toks[-176:][:4] == ["a7a8q", "a7a8r", "a7a8b", "a7a8n"]
    assert toks[-1] == "h2h1n"
    for u in ("e2e4", "a7a8q", "h2h1n", "e1g1", "g1f3"):
        assert u in v
    assert "a1h2" not in v


@pytest.mark.parametrize("fen", EDGE_FENS + [
    "r3k2r/pppq1ppp/2npbn2/1B2p3/3PP3/2N1BN2/PPP1QPPP/R3K2R w KQkq - 0 1",
    "rnbq1bnr/ppPppk1p/8/8/8/8/PP1PPpPP/RNBQKBNR w KQ - 0 1",
])
def test_projection_is_every_legal_move_sorted_by_uci(fen):
    ids, ucis = wc.legal_vocab_projection(fen)
    v = wc.static_move_vocab()
    assert len(ucis) == wc.perft(fen, 1)  # every legal move is in the vocabulary
    assert ucis == sorted(ucis) and len(set(ucis)) == len(ucis)
    assert ids == [v[u] for u in ucis]


def test_start_position_projection_and_castling_uci():
    ids, ucis = wc.legal_vocab_projection(START)
    assert ucis[:4] == ["a2a3", "a2a4", "b1a3", "b1c3"] and len(ucis) == 20
    _, ucis = wc.legal_vocab_projection(EDGE_FENS[1])
    assert "e1g1" in ucis and "e1c1" in ucis  # castling as the king's two-square move


def test_encoding_matches_reference_tests():
    enc = wc.BoardStateEncoder()
    s = enc.encode_fen(START)
    assert len(s.piece_ids) == 64
    assert (s.turn_id, s.castle_id, s.ep_file_id, s.halfmove_bucket_id, s.fullmove_bucket_id) == (0, 15, 0, 0, 0)
    assert s.piece_ids[0] == 4 and s.piece_ids[4] == 6 and s.piece_ids[60] == 12 and s.piece_ids[56] == 10
    s = enc.encode_fen("8/8/8/8/8/8/8/K6k w - - 0 1")
    assert s.piece_ids[0] == 6 and s.piece_ids[7] == 12 and sum(1 for x in s.piece_ids if x) == 2
    assert enc.encode_fen("r3k2r/8/8/8/8/8/8/R3K2R w Kq - 0 1").castle_id == 9
    after_e4 = "rnbqkbnr/pppppppp/8/8/4P3/8/PPPP1PPP/RNBQKBNR b KQkq e3 0 1"
    assert wc.BoardStateEncoder(wc.BoardTokenConfig(en_passant="legal")).encode_fen(after_e4).ep_file_id == 0
    assert wc.BoardStateEncoder(wc.BoardTokenConfig(en_passant="fen")).encode_fen(after_e4).ep_file_id == 5
    s = enc.encode_fen("8/8/8/8/8/8/8/K6k w - - 150 500")
    assert s.halfmove_bucket_id == 50 and s.fullmove_bucket_id == 100


def test_en_passant_modes_with_a_capturer():
    # Black just played d7d5 next to the e5 pawn: a legal capture exists.
    fen = "rnbqkbnr/ppp1pppp/8/3pP3/8/8/PPPP1PPP/RNBQKBNR w KQkq d6 0 3"
    for mode in ("legal", "fen", "xfen"):
        assert wc.BoardStateEncoder(wc.BoardTokenConfig(en_passant=mode)).encode_fen(fen).ep_file_id == 4
    assert "e5d6" in wc.legal_vocab_projection(fen)[1]
    # The capturing pawn is pinned against its king: pseudo-legal only.
    pinned = "4k3/8/8/K2pP2r/8/8/8/8 w - d6 0 1"
    assert "e5d6" not in wc.legal_vocab_projection(pinned)[1]
    assert wc.BoardStateEncoder(wc.BoardTokenConfig(en_passant="legal")).encode_fen(pinned).ep_file_id == 0
    assert wc.BoardStateEncoder(wc.BoardTokenConfig(en_passant="xfen")).encode_fen(pinned).ep_file_id == 4


def test_push_uci_and_expand():
    fen = wc.push_uci(START, "e2e4")
    assert fen == "rnbqkbnr/pppppppp/8/8/4P3/8/PPPP1PPP/RNBQKBNR b KQkq - 0 1"
    fen = wc.push_uci(wc.push_uci(fen, "c7c5"), "g1f3")
    assert fen.endswith("b KQkq - 1 2")
    with pytest.raises(ValueError):
        wc.push_uci(START, "e2e5")
    piece, side, loff, lids = wc.expand(EDGE_FENS)
    assert piece.shape == (6, 64) and side.shape == (6, 5)
    assert np.diff(loff).tolist() == [p[0] for p in PERFT]
    for i, fen in enumerate(EDGE_FENS):
        ids, _ = wc.legal_vocab_projection(fen)
        assert lids[loff[i]:loff[i + 1]].tolist() == ids
        s = wc.BoardStateEncoder().encode_fen(fen)
        assert piece[i].tolist() == s.piece_ids
        assert side[i].tolist() == [s.turn_id, s.castle_id, s.ep_file_id, s.halfmove_bucket_id, s.fullmove_bucket_id]


def test_bad_input_raises():
    with pytest.raises(ValueError):
        wc.perft("not a fen", 1)
    with pytest.raises(ValueError):
        wc.BoardStateEncoder(wc.BoardTokenConfig(en_passant="bogus"))


def test_random_games_self_consistent():
    """Random playouts: at every position the two-ply leaf count computed
    inside the generator equals the sum of one-ply counts of the children
    reached through FEN text (push_uci writes the FEN, the child is parsed
    back), so FEN writing and parsing keep castling rights, en passant,
    counters and side to move; every legal move is in the vocabulary; each
    side keeps one king."""
    rng = np.random.default_rng(11)
    for _ in range(8):
        fen = START
        for _ in range(int(rng.integers(20, 100))):
            _, ucis = wc.legal_vocab_projection(fen)
            assert len(ucis) == wc.perft(fen, 1)
            if not ucis:
                break
            assert wc.perft(fen, 2) == sum(wc.perft(wc.push_uci(fen, u), 1) for u in ucis)
            s = wc.BoardStateEncoder().encode_fen(fen)
            assert s.piece_ids.count(6) == 1 and s.piece_ids.count(12) == 1
            fen = wc.push_uci(fen, ucis[int(rng.integers(0, len(ucis)))])
