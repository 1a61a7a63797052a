"""Worker-side chess for the search actors, backed by the C++ ``_chess``
extension (``host/chess.cpp``): the work each search worker does per expanded
node before it sends a wave -- legal move generation, the UCI-sorted
legal-id projection onto the static move vocabulary, and the board-state
encoding the model consumes.

Reference counterparts (same names where a Python function exists there):

* ``legal_vocab_projection``: ``_legal_vocab_projection``
  (src/imba_chess/eval/actor_worker.py:230-264), on a FEN instead of a cozy
  board; returns (vocab ids, UCIs) sorted by UCI, castling as the king's
  two-square move (cozy_bridge.py:91-100);
* ``BoardStateEncoder.encode_fen``: ``BoardStateEncoder.encode`` /
  ``encode_cozy`` (src/imba_chess/data/board_state.py:94-166) with the same
  ``BoardTokenConfig`` fields and en-passant modes ("legal", "fen", "xfen");
* ``static_move_vocab``: ``MoveVocab.build_static``
  (src/imba_chess/data/move_vocab.py:76-79, :124-155), token -> id;
* ``expand``: a batch of positions packed straight into a wave's arrays
  (piece ids, side ids, legal-id CSR).

Positions are FEN strings; ``push_uci`` applies a legal move.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _chess


@dataclass(frozen=True)
class BoardTokenConfig:
    en_passant: str = "legal"
    halfmove_max: int = 100
    halfmove_bucket_size: int = 2
    fullmove_max: int = 200
    fullmove_bucket_size: int = 2

    def kwargs(self) -> dict:
        return dict(en_passant=self.en_passant, halfmove_max=self.halfmove_max,
                    halfmove_bucket_size=self.halfmove_bucket_size, fullmove_max=self.fullmove_max,
                    fullmove_bucket_size=self.fullmove_bucket_size)


@dataclass(frozen=True)
class BoardState:
    piece_ids: list[int]
    turn_id: int
    castle_id: int
    ep_file_id: int
    halfmove_bucket_id: int
    fullmove_bucket_id: int


class BoardStateEncoder:
    def __init__(self, config: BoardTokenConfig | None = None) -> None:
        self.config = config or BoardTokenConfig()
        if self.config.halfmove_bucket_size <= 0:
            raise ValueError("halfmove_bucket_size must be > 0")
        if self.config.fullmove_bucket_size <= 0:
            raise ValueError("fullmove_bucket_size must be > 0")
        if self.config.en_passant not in ("legal", "fen", "xfen"):
            raise ValueError(f"Unsupported en_passant mode: {self.config.en_passant}")

    def encode_fen(self, fen: str) -> BoardState:
        ids, turn, castle, ep, half, full = _chess.encode(fen, **self.config.kwargs())
        return BoardState(ids, turn, castle, ep, half, full)


def legal_vocab_projection(fen: str) -> tuple[list[int], list[str]]:
    return _chess.legal_projection(fen)


def static_move_vocab() -> dict[str, int]:
    return {tok: i for i, tok in enumerate(_chess.vocab())}


def push_uci(fen: str, uci: str) -> str:
    return _chess.push_uci(fen, uci)


def perft(fen: str, depth: int) -> int:
    return _chess.perft(fen, depth)


def expand(fens: list[str], config: BoardTokenConfig | None = None):
    """(piece_ids uint8 [N, 64], side int32 [N, 5] = turn, castle, ep file,
    halfmove bucket, fullmove bucket; legal_off int32 [N + 1]; legal_ids
    int32), every row's legal ids UCI-sorted."""
    cfg = config or BoardTokenConfig()
    pb, sb, ob, lb = _chess.expand(list(fens), **cfg.kwargs())
    n = len(fens)
    return (np.frombuffer(pb, dtype=np.uint8).reshape(n, 64), np.frombuffer(sb, dtype=np.int32).reshape(n, 5),
            np.frombuffer(ob, dtype=np.int32), np.frombuffer(lb, dtype=np.int32))
