"""Seeded synthetic weights, token streams and search-wave workloads.

No checkpoint or dataset is available to this package's benchmarks and
tests, so every model here is random-initialised with the reference's
parameter names and shapes (``HSTUChessModel.state_dict()``,
src/imba_chess/model/hstu_model.py:185-273) and every input is drawn from a
seeded generator with the value ranges of the reference's ``BoardState``
encoding (src/imba_chess/data/board_state.py:8-45, data/models.py:17-23):
piece ids 0..12, turn 0..1, castle bitmask 0..15, en-passant file 0..8,
halfmove/fullmove buckets 0..50 / 0..100, previous-move ids over the
1,970-token move vocab.

Two weight profiles:

* ``"reference"`` mirrors the reference's own initialisers (embeddings
  N(0,1), ``_uvqk`` N(0,0.02), ``_o`` Xavier-uniform, ``_ps_w`` N(0,0.02),
  ``nn.Linear`` defaults U(+-1/sqrt(fan_in)), LayerNorm 1/0, position table
  truncated-normal with std sqrt(1/d)).  Used for throughput runs and for the
  precision budget of the bf16 path.
* ``"sharp"`` scales the projections and the relative-bias table up so that
  attention weights are far from uniform and bias-index mistakes change the
  output visibly; LayerNorm affine parameters are perturbed.  Used by the
  parity tests.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, asdict

import numpy as np

BOARD_DIM = 64
BOARD_HEADS = 4
BOARD_LAYERS = 2
PIECE_SQUARE_ROWS = 13 * 64
MOVE_VOCAB_SIZE = 1970
EVENT_TOKEN_ID = 0
BOS_TOKEN_ID = 1
TOKEN_FIELDS = (
    "piece_ids",
    "seq_token_id",
    "turn_id",
    "castle_id",
    "ep_file_id",
    "halfmove_bucket_id",
    "fullmove_bucket_id",
    "prev_move_id",
)


@dataclass(frozen=True)
class ModelDims:
    """Architecture hyper-parameters of one HSTU chess model
    (``HSTUChessConfig``, src/imba_chess/model/hstu_model.py:18-43)."""

    model_dim: int
    num_layers: int
    num_heads: int
    attention_dim: int = 64
    linear_dim: int = 64
    vocab: int = MOVE_VOCAB_SIZE
    max_pos: int = 513
    halfmove_vocab: int = 128
    fullmove_vocab: int = 128
    value_head: bool = True

    @property
    def uvqk_dim(self) -> int:
        return 2 * self.num_heads * self.linear_dim + 2 * self.num_heads * self.attention_dim

    def as_dict(self) -> dict:
        return asdict(self)


# Named model shapes used by the tests and the benchmark.
TINY = ModelDims(32, 2, 2, 8, 8, vocab=32, max_pos=64)          # reference unit-test model
SMALL = ModelDims(128, 2, 2, 64, 64, vocab=MOVE_VOCAB_SIZE, max_pos=48)
D256 = ModelDims(256, 4, 4, max_pos=513)                        # fp32 CPU-runnable model
D512 = ModelDims(512, 8, 8, max_pos=513)                        # grouped-decode model
D512_LONG = ModelDims(512, 8, 8, max_pos=1024)                  # long-prefix workloads
D1024 = ModelDims(1024, 16, 16, max_pos=1024)                   # stress model


def state_dict_shapes(dims: ModelDims) -> dict[str, tuple[int, ...]]:
    """Parameter names and shapes, in the reference's registration order."""
    d = dims.model_dim
    shapes: dict[str, tuple[int, ...]] = {
        "piece_square_embedding.weight": (PIECE_SQUARE_ROWS, BOARD_DIM)
    }
    for b in range(BOARD_LAYERS):
        p = f"board_encoder.blocks.{b}."
        shapes[p + "attn_norm.weight"] = (BOARD_DIM,)
        shapes[p + "attn_norm.bias"] = (BOARD_DIM,)
        shapes[p + "qkv.weight"] = (3 * BOARD_DIM, BOARD_DIM)
        shapes[p + "attn_out.weight"] = (BOARD_DIM, BOARD_DIM)
        shapes[p + "mlp_norm.weight"] = (BOARD_DIM,)
        shapes[p + "mlp_norm.bias"] = (BOARD_DIM,)
        shapes[p + "mlp.0.weight"] = (2 * BOARD_DIM, BOARD_DIM)
        shapes[p + "mlp.0.bias"] = (2 * BOARD_DIM,)
        shapes[p + "mlp.2.weight"] = (BOARD_DIM, 2 * BOARD_DIM)
        shapes[p + "mlp.2.bias"] = (BOARD_DIM,)
    shapes["board_encoder.final_norm.weight"] = (BOARD_DIM,)
    shapes["board_encoder.final_norm.bias"] = (BOARD_DIM,)
    shapes["board_encoder.out_proj.weight"] = (d, BOARD_DIM)
    shapes["board_encoder.out_proj.bias"] = (d,)
    shapes["seq_token_embedding.weight"] = (2, d)
    shapes["turn_embedding.weight"] = (2, d)
    shapes["castle_embedding.weight"] = (16, d)
    shapes["ep_embedding.weight"] = (9, d)
    shapes["halfmove_embedding.weight"] = (dims.halfmove_vocab, d)
    shapes["fullmove_embedding.weight"] = (dims.fullmove_vocab, d)
    shapes["prev_move_embedding.weight"] = (dims.vocab, d)
    shapes["position_embedding.embedding.weight"] = (dims.max_pos, d)
    for l in range(dims.num_layers):
        p = f"layers.{l}."
        shapes[p + "_ps_w"] = (dims.num_heads, 2 * dims.max_pos - 1)
        shapes[p + "_uvqk.weight"] = (dims.uvqk_dim, d)
        shapes[p + "_o.weight"] = (d, dims.num_heads * dims.linear_dim)
        shapes[p + "_o.bias"] = (d,)
    shapes["final_norm.weight"] = (d,)
    shapes["final_norm.bias"] = (d,)
    shapes["prediction_head.weight"] = (dims.vocab, d)
    if dims.value_head:
        shapes["value_head.0.weight"] = (d // 2, d)
        shapes["value_head.0.bias"] = (d // 2,)
        shapes["value_head.2.weight"] = (3, d // 2)
        shapes["value_head.2.bias"] = (3,)
    shapes["moves_left_head.0.weight"] = (d // 2, d)
    shapes["moves_left_head.0.bias"] = (d // 2,)
    shapes["moves_left_head.2.weight"] = (1, d // 2)
    shapes["moves_left_head.2.bias"] = (1,)
    return shapes


def make_state_dict(dims: ModelDims, seed: int, profile: str = "reference") -> dict[str, np.ndarray]:
    """Deterministic float32 weights keyed like the reference's state_dict.

    ``prediction_head.weight`` is tied to ``prev_move_embedding.weight``
    (src/imba_chess/model/hstu_model.py:249): both keys hold the same array.
    """
    if profile not in ("reference", "sharp"):
        raise ValueError(f"unknown weight profile {profile!r}")
    sharp = profile == "sharp"
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    for name, shape in state_dict_shapes(dims).items():
        if name == "prediction_head.weight":
            out[name] = out["prev_move_embedding.weight"]
            continue
        if name.endswith("norm.weight"):
            arr = 1.0 + (0.1 * rng.standard_normal(shape) if sharp else np.zeros(shape))
        elif name.endswith("norm.bias"):
            arr = 0.1 * rng.standard_normal(shape) if sharp else np.zeros(shape)
        elif name.endswith("_ps_w"):
            arr = rng.standard_normal(shape) * (0.5 if sharp else 0.02)
        elif name.endswith("_uvqk.weight"):
            std = 1.5 / math.sqrt(shape[1]) if sharp else 0.02
            arr = rng.standard_normal(shape) * std
        elif name.endswith("_o.weight"):
            bound = math.sqrt(6.0 / (shape[0] + shape[1]))
            arr = rng.uniform(-bound, bound, shape)
        elif name == "position_embedding.embedding.weight":
            std = math.sqrt(1.0 / dims.model_dim)
            arr = np.clip(rng.standard_normal(shape), -2.0, 2.0) * std
        elif name.endswith("embedding.weight"):
            arr = rng.standard_normal(shape)
        elif name.endswith(".weight"):
            bound = 1.0 / math.sqrt(shape[1])
            if sharp and name.startswith("board_encoder") and "qkv" in name:
                bound *= 2.0
            arr = rng.uniform(-bound, bound, shape)
        elif name.endswith(".bias"):
            fan_in = state_dict_shapes(dims)[name[: -len("bias")] + "weight"][1]
            bound = 1.0 / math.sqrt(fan_in)
            arr = rng.uniform(-bound, bound, shape)
        else:  # pragma: no cover - every key is covered above
            raise AssertionError(name)
        out[name] = np.ascontiguousarray(arr, dtype=np.float32)
    return out


def random_board(rng: np.random.Generator, n: int) -> np.ndarray:
    """[n, 64] piece ids with roughly middlegame occupancy (about 40%)."""
    occupied = rng.random((n, 64)) < 0.4
    pieces = rng.integers(1, 13, size=(n, 64))
    return np.where(occupied, pieces, 0).astype(np.int64)


def random_tokens(rng: np.random.Generator, n: int, dims: ModelDims) -> dict[str, np.ndarray]:
    """n decode tokens with every id field in its encoded range."""
    return {
        "piece_ids": random_board(rng, n),
        "seq_token_id": np.full(n, EVENT_TOKEN_ID, dtype=np.int64),
        "turn_id": rng.integers(0, 2, n).astype(np.int64),
        "castle_id": rng.integers(0, 16, n).astype(np.int64),
        "ep_file_id": rng.integers(0, 9, n).astype(np.int64),
        "halfmove_bucket_id": rng.integers(0, 51, n).astype(np.int64),
        "fullmove_bucket_id": rng.integers(0, 101, n).astype(np.int64),
        "prev_move_id": rng.integers(2, dims.vocab, n).astype(np.int64),
    }


def game_tokens(rng: np.random.Generator, n_plies: int, dims: ModelDims) -> dict[str, np.ndarray]:
    """A game prefix of ``n_plies`` plies as the reference lays it out: a BOS
    token (empty board, ``prev_move`` = start id 1), then one EVENT token per
    position including the current one, ``n_plies + 2`` tokens in all
    (src/imba_chess/eval/position_evaluator.py:25-111,
    src/imba_chess/data/event_builder.py:41-102)."""
    t = n_plies + 2
    tok = random_tokens(rng, t, dims)
    tok["seq_token_id"][0] = BOS_TOKEN_ID
    tok["piece_ids"][0] = 0
    for key in ("turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id"):
        tok[key][0] = 0
    tok["prev_move_id"][0] = 1
    tok["turn_id"][1:] = np.arange(t - 1) % 2
    tok["fullmove_bucket_id"][1:] = np.minimum(np.arange(t - 1) // 4, 100)
    return tok


def concat_tokens(parts: list[dict[str, np.ndarray]]) -> dict[str, np.ndarray]:
    return {k: np.concatenate([p[k] for p in parts], axis=0) for k in TOKEN_FIELDS}


def slice_tokens(tok: dict[str, np.ndarray], idx) -> dict[str, np.ndarray]:
    return {k: tok[k][idx] for k in TOKEN_FIELDS}


def random_legal_ids(rng: np.random.Generator, count: int, vocab: int) -> np.ndarray:
    """``count`` distinct move ids in a random (stand-in for UCI-sorted) order."""
    count = min(count, vocab - 2)
    return (rng.permutation(vocab - 2)[:count] + 2).astype(np.int64)


@dataclass
class GroupedWave:
    """One grouped-decode wave: ``G`` parents, each with a game prefix, and
    ``B`` sibling rows (depth-0 children of their parent's prefix)."""

    prefix_tokens: list[dict[str, np.ndarray]]  # per parent, [P_g] tokens
    row_tokens: dict[str, np.ndarray]           # [B] tokens
    group_index: np.ndarray                     # [B] int64
    legal_ids: list[np.ndarray]                 # per row

    @property
    def prefix_lens(self) -> list[int]:
        return [int(p["piece_ids"].shape[0]) for p in self.prefix_tokens]

    @property
    def num_rows(self) -> int:
        return int(self.group_index.shape[0])


def grouped_wave(
    dims: ModelDims,
    *,
    n_parents: int,
    plies: tuple[int, int],
    siblings: tuple[int, int],
    legal: tuple[int, int] = (20, 40),
    seed: int = 1234,
) -> GroupedWave:
    """Parents ``g`` use seed ``seed + g``: prefix of U[plies] plies, then
    U[siblings] depth-0 children each carrying U[legal] legal move ids."""
    prefixes, rows, groups, legal_ids = [], [], [], []
    for g in range(n_parents):
        rng = np.random.default_rng(seed + g)
        n_plies = int(rng.integers(plies[0], plies[1] + 1))
        prefixes.append(game_tokens(rng, n_plies, dims))
        k = int(rng.integers(siblings[0], siblings[1] + 1))
        child = random_tokens(rng, k, dims)
        child["turn_id"][:] = (n_plies + 1) % 2
        rows.append(child)
        groups.append(np.full(k, g, dtype=np.int64))
        for _ in range(k):
            legal_ids.append(random_legal_ids(rng, int(rng.integers(legal[0], legal[1] + 1)), dims.vocab))
    return GroupedWave(prefixes, concat_tokens(rows), np.concatenate(groups), legal_ids)


# ----------------------------------------------------------------------
# Real chess positions from seeded uniformly-random legal play
# ----------------------------------------------------------------------
START_FEN = "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1"
_SIDE_FIELDS = ("turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id")


@dataclass
class ChessGame:
    """A game played by uniformly random legal moves from the start position:
    its token prefix (BOS, then one EVENT token per position from the start
    position to the current one, ``plies + 2`` tokens), the current FEN and
    the current position's UCI-sorted legal moves (vocab ids and UCIs)."""

    tokens: dict[str, np.ndarray]
    fen: str
    legal_ids: list[int]
    legal_ucis: list[str]

    @property
    def plies(self) -> int:
        return int(self.tokens["piece_ids"].shape[0]) - 2


def _position_token(state, prev_move_id: int) -> dict[str, int | list[int]]:
    return {"piece_ids": list(state.piece_ids), "seq_token_id": EVENT_TOKEN_ID, "prev_move_id": int(prev_move_id),
            **{k: int(getattr(state, k)) for k in _SIDE_FIELDS}}


def chess_game(seed: int, n_plies: int) -> ChessGame:
    """``n_plies`` uniformly random legal moves from the start position with
    ``numpy.random.default_rng(seed)`` (fewer when the game ends first),
    tokenised like the reference's sequence history: BOS with the start id as
    previous move, then each observed position with the move that reached it
    (src/imba_chess/eval/position_evaluator.py:25-111).  Uses the worker-side
    chess extension for move generation and the board-state encoding."""
    from . import worker_chess as wc

    rng = np.random.default_rng(seed)
    enc = wc.BoardStateEncoder()
    vocab = wc.static_move_vocab()
    fen = START_FEN
    toks = [{"piece_ids": [0] * 64, "seq_token_id": BOS_TOKEN_ID, "prev_move_id": 1,
             **{k: 0 for k in _SIDE_FIELDS}}]
    prev = 1  # the vocabulary's start id
    ids, ucis = wc.legal_vocab_projection(fen)
    for _ in range(n_plies):
        toks.append(_position_token(enc.encode_fen(fen), prev))
        if not ucis:
            break
        u = ucis[int(rng.integers(len(ucis)))]
        fen = wc.push_uci(fen, u)
        prev = vocab[u]
        ids, ucis = wc.legal_vocab_projection(fen)
    toks.append(_position_token(enc.encode_fen(fen), prev))
    tokens = {k: np.asarray([t[k] for t in toks], dtype=np.int64) for k in TOKEN_FIELDS}
    return ChessGame(tokens, fen, list(ids), list(ucis))


def chess_grouped_wave(*, n_parents: int, plies: tuple[int, int], seed: int = 1234,
                       max_children: int | None = None) -> GroupedWave:
    """A grouped-decode wave over real positions: parent ``g`` is a
    random-legal-play game (seed ``seed + g``, U[plies] plies, drawn with that
    seed's generator), and its rows are the depth-0 children reached by each
    of its legal moves (``max_children`` caps them: the first ones in UCI
    order), each carrying the child's own UCI-sorted legal move ids."""
    from . import worker_chess as wc

    enc = wc.BoardStateEncoder()
    vocab = wc.static_move_vocab()
    prefixes, rows, groups, legal_ids = [], [], [], []
    for g in range(n_parents):
        n_plies = int(np.random.default_rng(seed + g).integers(plies[0], plies[1] + 1))
        game = chess_game(seed + g, n_plies)
        prefixes.append(game.tokens)
        kids = game.legal_ucis if max_children is None else game.legal_ucis[:max_children]
        toks = []
        for u in kids:
            child = wc.push_uci(game.fen, u)
            toks.append(_position_token(enc.encode_fen(child), vocab[u]))
            legal_ids.append(np.asarray(wc.legal_vocab_projection(child)[0], dtype=np.int64))
        if toks:
            rows.append({k: np.asarray([t[k] for t in toks], dtype=np.int64) for k in TOKEN_FIELDS})
        groups.append(np.full(len(toks), g, dtype=np.int64))
    row_tokens = concat_tokens(rows) if rows else empty_tokens()
    return GroupedWave(prefixes, row_tokens, np.concatenate(groups), legal_ids)


def empty_tokens() -> dict[str, np.ndarray]:
    """Zero tokens, with every field's shape and dtype."""
    return {k: np.zeros((0, 64) if k == "piece_ids" else (0,), dtype=np.int64) for k in TOKEN_FIELDS}


def root_batch_arrays(tok: dict[str, np.ndarray], game_id: str = "g") -> dict:
    """A game prefix as the wire form of a full ``RootEvalRequest``
    (``batch_arrays``: plain lists, one jagged document), with every field
    the reference's ``_tensorize_root_batch`` reads
    (src/imba_chess/eval/actor_server.py:120-133; built like
    ``_SequenceHistory._build_single_batch``, position_evaluator.py:80-100)."""
    n = int(tok["piece_ids"].shape[0])
    ba = {k: np.asarray(tok[k]).tolist() for k in TOKEN_FIELDS}
    ba.update(game_id=[game_id], num_games=1, total_tokens=n, seq_lens=[n], seq_offsets=[0, n],
              game_result_white=[0], target_move_id=[-100] * n, played_by_elo=[0] * n)
    return ba
