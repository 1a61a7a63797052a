"""Wire messages between torch-free eval workers and the inference server.

Field-for-field the interface of the reference's
src/imba_chess/eval/actor_protocol.py:28-208 (kept identical because workers
build and read these objects).  When the reference package is importable its
own classes are used, so a reference worker's pickled requests and this
server's responses are the same types; otherwise these equivalent
definitions stand in.
"""

from __future__ import annotations

from dataclasses import dataclass

try:  # pragma: no cover - exercised only where the reference package is installed
    from imba_chess.eval.actor_protocol import (  # type: ignore
        GameDone,
        RootEvalRequest,
        RootEvalResponse,
        WaveRequest,
        WaveResponse,
        WaveRow,
        WorkerFinished,
    )
except Exception:  # noqa: BLE001

    @dataclass(kw_only=True)
    class RootEvalRequest:
        """worker -> server: a game-turn's root evaluation.  FULL form
        (``batch_arrays``: the whole game so far, a single jagged document)
        or INCREMENTAL form (``incremental_tokens``: the tokens added since the
        previous root request, with ``prefix_len_before`` for the desync
        check).  Exactly one of the two is set."""

        worker_id: int
        turn_id: int
        legal_vocab_ids: list[int]
        batch_arrays: dict | None = None
        incremental_tokens: dict | None = None
        prefix_len_before: int | None = None

        def __post_init__(self) -> None:
            has_full = self.batch_arrays is not None
            has_inc = self.incremental_tokens is not None
            if has_full == has_inc:
                raise ValueError(
                    "RootEvalRequest must set exactly ONE of batch_arrays (full forward) or "
                    "incremental_tokens (incremental root extension)"
                )
            if has_inc and self.prefix_len_before is None:
                raise ValueError("RootEvalRequest.incremental_tokens requires prefix_len_before")

    @dataclass
    class RootEvalResponse:
        """server -> worker: value and raw legal-move logits (request order)."""

        turn_id: int
        value_stm: float
        legal_logits: list[float]

    @dataclass
    class WaveRow:
        """One search node to decode: ``parent_id`` None hangs it off the
        turn's root prefix; ``board_state`` holds the encoded BoardState
        fields."""

        node_id: int
        parent_id: int | None
        prev_move_vocab_id: int
        board_state: dict
        legal_vocab_ids: list[int]

    @dataclass
    class WaveRequest:
        worker_id: int
        turn_id: int
        rows: list

    @dataclass
    class WaveResponse:
        rows: list

    @dataclass
    class GameDone:
        worker_id: int
        game_idx: int
        summary_fragment: dict

    @dataclass
    class WorkerFinished:
        worker_id: int


def is_root_request(obj) -> bool:
    return type(obj).__name__ == "RootEvalRequest" and hasattr(obj, "incremental_tokens")


def is_wave_request(obj) -> bool:
    return type(obj).__name__ == "WaveRequest" and hasattr(obj, "rows")


__all__ = [
    "GameDone",
    "RootEvalRequest",
    "RootEvalResponse",
    "WaveRequest",
    "WaveResponse",
    "WaveRow",
    "WorkerFinished",
    "is_root_request",
    "is_wave_request",
]
