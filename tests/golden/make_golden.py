"""Generate the golden fixtures in this directory by running the REFERENCE
imba-chess implementation (imported from its source tree through
``ref_shims``) on seeded weights and inputs.

    python tests/golden/make_golden.py

Outputs (committed; the GPU box never needs the reference):

* ``tiny.npz``   - reference unit-test model shape (d=32, 2 layers, 2 heads,
  head dims 8/8, max_pos 64, vocab 32): prefill over three documents, a
  grouped decode wave with interleaved group indices and mixed suffix depths,
  and a single-prefix decode.
* ``small.npz``  - kernel-shaped model (d=128, 2 layers, 2 heads, head dims
  64/64, max_pos 48, vocab 1970): prefill including a 60-token document (past
  max_pos, so both position clamps fire), grouped decode with an empty-prefix
  group and a group with no rows, legal-id gathers, log-priors and values.
* ``server_session.json`` - a scripted ``ActorInferenceServer`` session on
  the small model: merged full roots, decode waves at depths 0-3 across two
  workers, an incremental root mixed with a full root, turn release; with
  every response and the per-turn node chains (arena row ids).

Weights come from ``imba_chess_b200.synth.make_state_dict`` (seeded numpy),
so tests rebuild them bit-identically without storing them.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

# The reference's source tree (read-only); override with IMBA_REFERENCE_SRC.
REFERENCE_SRC = os.environ.get("IMBA_REFERENCE_SRC", "/root/reference/src")

from oracle import ref_shims  # noqa: E402

ref_shims.install(REFERENCE_SRC)

import torch  # noqa: E402

from imba_chess_b200 import synth  # noqa: E402

TINY_SEED = 7
SMALL_SEED = 11


def ref_model(dims: synth.ModelDims, seed: int):
    from imba_chess.config import ModelConfig
    from imba_chess.model import HSTUChessModel, build_hstu_chess_config

    cfg = build_hstu_chess_config(
        ModelConfig(
            model_dim=dims.model_dim,
            linear_hidden_dim=dims.linear_dim,
            attention_dim=dims.attention_dim,
            num_heads=dims.num_heads,
            num_layers=dims.num_layers,
            dropout=0.0,
            max_position_embeddings=dims.max_pos,
            halfmove_vocab_size=dims.halfmove_vocab,
            fullmove_vocab_size=dims.fullmove_vocab,
            enable_value_head=dims.value_head,
        ),
        move_vocab_size=dims.vocab,
    )
    model = HSTUChessModel(cfg).eval()
    sd = synth.make_state_dict(dims, seed, profile="sharp")
    model.load_state_dict({k: torch.from_numpy(v.copy()) for k, v in sd.items()}, strict=True)
    return model


def t(x):
    return torch.from_numpy(np.asarray(x))


def full_batch(tok: dict, offsets: list[int]) -> dict:
    n = int(tok["piece_ids"].shape[0])
    batch = {k: t(v) for k, v in tok.items()}
    batch.update(
        {
            "total_tokens": n,
            "seq_offsets": torch.tensor(offsets, dtype=torch.long),
            "target_move_id": torch.full((n,), -100, dtype=torch.long),
        }
    )
    return batch


def prefill_case(model, dims, rng, doc_lens, out, tag):
    parts = [synth.random_tokens(rng, n, dims) for n in doc_lens]
    tok = synth.concat_tokens(parts)
    offsets = [0] + list(np.cumsum(doc_lens))
    with torch.no_grad():
        res = model(full_batch(tok, offsets), return_loss=False, return_kv=True)
    for k, v in tok.items():
        out[f"{tag}/tok/{k}"] = v
    out[f"{tag}/seq_offsets"] = np.asarray(offsets, dtype=np.int64)
    out[f"{tag}/logits"] = res["logits"].numpy()
    out[f"{tag}/value_logits"] = res["value_logits"].numpy()
    for l, (k, v) in enumerate(res["kv_caches"]):
        out[f"{tag}/kv/{l}/k"] = k.numpy()
        out[f"{tag}/kv/{l}/v"] = v.numpy()
    return tok, offsets, res["kv_caches"]


def grouped_case(model, dims, rng, prefix_kv_list, group_index, depths, out, tag, legal=False):
    """prefix_kv_list: per group, per layer (k [H,T,d], v [H,T,d])."""
    L, H = dims.num_layers, dims.num_heads
    lens = [kv[0][0].shape[1] for kv in prefix_kv_list]
    max_p = max(max(lens), 1)
    grouped = []
    for l in range(L):
        ks, vs = [], []
        for kv in prefix_kv_list:
            k, v = kv[l]
            pad = max_p - k.shape[1]
            ks.append(torch.nn.functional.pad(k, (0, 0, 0, pad)))
            vs.append(torch.nn.functional.pad(v, (0, 0, 0, pad)))
        grouped.append((torch.stack(ks), torch.stack(vs)))
    B = len(group_index)
    s_max = max(depths)
    tok = synth.random_tokens(rng, B, dims)
    positions = np.array([lens[g] + d for g, d in zip(group_index, depths)], dtype=np.int64)
    suffix_kv = suffix_pos = suffix_mask = None
    if s_max > 0:
        suffix_kv = []
        for l in range(L):
            sk = rng.standard_normal((B, H, s_max, dims.attention_dim)).astype(np.float32) * 0.5
            sv = rng.standard_normal((B, H, s_max, dims.linear_dim)).astype(np.float32)
            for r, d in enumerate(depths):  # padded slots hold zeros, as the server's do
                sk[r, :, d:] = 0.0
                sv[r, :, d:] = 0.0
            suffix_kv.append((t(sk), t(sv)))
        suffix_pos = np.zeros((B, s_max), dtype=np.int64)
        suffix_mask = np.zeros((B, s_max), dtype=bool)
        for r, (g, d) in enumerate(zip(group_index, depths)):
            suffix_pos[r] = lens[g] + np.arange(s_max)
            suffix_mask[r, :d] = True
    with torch.no_grad():
        res = model.forward_decode_grouped(
            new_token_batch={k: t(v) for k, v in tok.items()},
            positions=t(positions),
            group_index=t(np.asarray(group_index, dtype=np.int64)),
            prefix_kv_grouped=grouped,
            prefix_lens=torch.tensor(lens, dtype=torch.long),
            prefix_lens_list=list(lens),
            suffix_kv=suffix_kv,
            suffix_positions=None if suffix_pos is None else t(suffix_pos),
            suffix_mask=None if suffix_mask is None else t(suffix_mask),
        )
    for k, v in tok.items():
        out[f"{tag}/tok/{k}"] = v
    out[f"{tag}/positions"] = positions
    out[f"{tag}/group_index"] = np.asarray(group_index, dtype=np.int64)
    out[f"{tag}/prefix_lens"] = np.asarray(lens, dtype=np.int64)
    for l in range(L):
        out[f"{tag}/prefix/{l}/k"] = grouped[l][0].numpy()
        out[f"{tag}/prefix/{l}/v"] = grouped[l][1].numpy()
        if suffix_kv is not None:
            out[f"{tag}/suffix/{l}/k"] = suffix_kv[l][0].numpy()
            out[f"{tag}/suffix/{l}/v"] = suffix_kv[l][1].numpy()
        out[f"{tag}/kv/{l}/k"] = res["kv"][l][0].numpy()
        out[f"{tag}/kv/{l}/v"] = res["kv"][l][1].numpy()
    if suffix_pos is not None:
        out[f"{tag}/suffix_positions"] = suffix_pos
        out[f"{tag}/suffix_mask"] = suffix_mask
    out[f"{tag}/logits"] = res["logits"].numpy()
    out[f"{tag}/value_logits"] = res["value_logits"].numpy()
    if legal:
        from imba_chess.eval.actor_server import _batched_value_stm, _gather_legal_logits
        from imba_chess.eval.actor_worker import _log_softmax_f32

        ids = [synth.random_legal_ids(rng, int(rng.integers(1, 45)), dims.vocab).tolist() for _ in range(B)]
        ids[1] = []  # a row with no mapped legal move
        gathered = _gather_legal_logits(res["logits"], ids)
        offs = np.cumsum([0] + [len(i) for i in ids])
        out[f"{tag}/legal_off"] = offs.astype(np.int64)
        out[f"{tag}/legal_ids"] = np.asarray([x for i in ids for x in i], dtype=np.int64)
        out[f"{tag}/legal_logits"] = np.asarray([x for g in gathered for x in g], dtype=np.float32)
        out[f"{tag}/legal_logprob"] = np.asarray(
            [x for g in gathered for x in _log_softmax_f32(g)], dtype=np.float32
        )
        out[f"{tag}/value_stm"] = np.asarray(_batched_value_stm(res["value_logits"]), dtype=np.float32)


def split_prefix(kv_caches, offsets, doc):
    a, b = offsets[doc], offsets[doc + 1]
    return [(k[:, a:b].clone(), v[:, a:b].clone()) for k, v in kv_caches]


def make_tiny():
    dims = synth.TINY
    model = ref_model(dims, TINY_SEED)
    rng = np.random.default_rng(100)
    out: dict[str, np.ndarray] = {}
    _, offsets, kv = prefill_case(model, dims, rng, [9, 5, 12], out, "prefill")
    prefixes = [split_prefix(kv, offsets, d) for d in range(3)]
    grouped_case(model, dims, rng, prefixes, [0, 2, 1, 0, 2, 2, 1], [0, 1, 2, 0, 0, 3, 1], out, "grouped")
    grouped_case(model, dims, rng, [prefixes[0]], [0, 0, 0, 0], [0, 2, 1, 0], out, "single")
    np.savez_compressed(os.path.join(HERE, "tiny.npz"), **out)


def make_small():
    dims = synth.SMALL
    model = ref_model(dims, SMALL_SEED)
    rng = np.random.default_rng(200)
    out: dict[str, np.ndarray] = {}
    _, offsets, kv = prefill_case(model, dims, rng, [17, 60, 7], out, "prefill")
    prefixes = [split_prefix(kv, offsets, d) for d in range(3)]
    empty = [(k[:, :0].clone(), v[:, :0].clone()) for k, v in prefixes[0]]
    prefixes = prefixes + [prefixes[2], empty]  # group 3 gets no rows; group 4 has P=0
    group_index = [1, 0, 4, 2, 1, 0, 0, 2, 4, 1, 1, 0, 2]
    depths = [0, 2, 1, 0, 3, 0, 1, 2, 0, 1, 0, 3, 1]
    grouped_case(model, dims, rng, prefixes, group_index, depths, out, "grouped", legal=True)
    np.savez_compressed(os.path.join(HERE, "small.npz"), **out)


# ----------------------------------------------------------------------
# Scripted actor-server session.
# ----------------------------------------------------------------------
def _batch_arrays(tok: dict) -> dict:
    n = int(tok["piece_ids"].shape[0])
    ba = {k: np.asarray(v).tolist() for k, v in tok.items()}
    ba.update(
        {
            "game_id": ["g"],
            "num_games": 1,
            "total_tokens": n,
            "seq_lens": [n],
            "seq_offsets": [0, n],
            "game_result_white": [0],
            "target_move_id": [-100] * n,
            "played_by_elo": [0] * n,
        }
    )
    return ba


def _wave_row(rng, dims, node_id, parent_id):
    tok = synth.random_tokens(rng, 1, dims)
    return {
        "node_id": node_id,
        "parent_id": parent_id,
        "prev_move_vocab_id": int(tok["prev_move_id"][0]),
        "board_state": {
            "piece_ids": tok["piece_ids"][0].tolist(),
            "turn_id": int(tok["turn_id"][0]),
            "castle_id": int(tok["castle_id"][0]),
            "ep_file_id": int(tok["ep_file_id"][0]),
            "halfmove_bucket_id": int(tok["halfmove_bucket_id"][0]),
            "fullmove_bucket_id": int(tok["fullmove_bucket_id"][0]),
        },
        "legal_vocab_ids": synth.random_legal_ids(rng, int(rng.integers(3, 40)), dims.vocab).tolist(),
    }


def session_script(dims) -> list[dict]:
    """A list of steps; each step is ``{"service": [requests]}`` or
    ``{"release_turn": [w, t]}`` / ``{"release_game": w}``."""
    rng = np.random.default_rng(300)
    legal = lambda: synth.random_legal_ids(rng, int(rng.integers(5, 40)), dims.vocab).tolist()  # noqa: E731
    game_a = synth.game_tokens(rng, 18, dims)  # 20 tokens
    game_b = synth.game_tokens(rng, 31, dims)  # 33 tokens
    game_c = synth.game_tokens(rng, 7, dims)   # 9 tokens
    inc = synth.random_tokens(rng, 2, dims)
    W = lambda w, tn, rows: {"type": "wave", "worker_id": w, "turn_id": tn, "rows": rows}  # noqa: E731
    R = lambda w, tn, **kw: {"type": "root", "worker_id": w, "turn_id": tn, "legal_vocab_ids": legal(), **kw}  # noqa: E731
    row = lambda n, p: _wave_row(rng, dims, n, p)  # noqa: E731
    steps = [
        {"service": [R(0, 0, batch_arrays=_batch_arrays(game_a)), R(1, 0, batch_arrays=_batch_arrays(game_b))]},
        {"service": [W(0, 0, [row(i, None) for i in range(1, 6)]), W(1, 0, [row(i, None) for i in range(1, 5)])]},
        {"service": [W(1, 0, [row(5, 1), row(6, 4)]), W(0, 0, [row(6, 2), row(7, 3), row(8, None)])]},
        {"service": [W(0, 0, [row(9, 6), row(10, 8), row(11, 7)]), W(1, 0, [row(7, 6)])]},
        {"release_turn": [0, 0]},
        {
            "service": [
                R(0, 1, incremental_tokens={k: np.asarray(v).tolist() for k, v in inc.items()}, prefix_len_before=20),
                R(2, 0, batch_arrays=_batch_arrays(game_c)),
            ]
        },
        {"service": [W(0, 1, [row(1, None), row(2, None)]), W(1, 0, [row(8, 7), row(9, 5)]), W(2, 0, [row(1, None)])]},
        {"service": [W(0, 1, [row(3, 1), row(4, 2), row(5, None)])]},
        {"release_game": 1},
    ]
    return steps


def to_request(d):
    from imba_chess.eval.actor_protocol import RootEvalRequest, WaveRequest, WaveRow

    if d["type"] == "root":
        kw = {k: v for k, v in d.items() if k != "type"}
        return RootEvalRequest(**kw)
    return WaveRequest(worker_id=d["worker_id"], turn_id=d["turn_id"], rows=[WaveRow(**r) for r in d["rows"]])


def make_session():
    from imba_chess.eval.actor_protocol import RootEvalResponse
    from imba_chess.eval.actor_server import ActorInferenceServer

    dims = synth.SMALL
    model = ref_model(dims, SMALL_SEED)
    server = ActorInferenceServer(model=model, device=torch.device("cpu"), dtype=torch.float32)
    steps = session_script(dims)
    results = []
    for step in steps:
        if "service" in step:
            resps = server.service([to_request(r) for r in step["service"]])
            enc = []
            for r in resps:
                if isinstance(r, RootEvalResponse):
                    enc.append({"type": "root", "turn_id": r.turn_id, "value_stm": r.value_stm, "legal_logits": r.legal_logits})
                else:
                    enc.append({"type": "wave", "rows": [[v, ll] for v, ll in r.rows]})
            results.append(enc)
        elif "release_turn" in step:
            server.release_turn(*step["release_turn"])
            results.append(None)
        else:
            server.release_game(step["release_game"])
            results.append(None)
    chains = {
        f"{w},{tn}": {str(n): c for n, c in ts.node_chains.items()} for (w, tn), ts in server._turns.items()
    }
    arena_sizes = {f"{w},{tn}": (ts.arena.size if ts.arena is not None else 0) for (w, tn), ts in server._turns.items()}
    game_lens = {str(w): g.prefix_len for w, g in server._games.items()}
    doc = {
        "model": {"dims": dims.as_dict(), "seed": SMALL_SEED, "profile": "sharp"},
        "steps": steps,
        "responses": results,
        "node_chains": chains,
        "arena_sizes": arena_sizes,
        "game_prefix_lens": game_lens,
    }
    with open(os.path.join(HERE, "server_session.json"), "w") as f:
        json.dump(doc, f)


if __name__ == "__main__":
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    make_tiny()
    make_small()
    make_session()
    for name in ("tiny.npz", "small.npz", "server_session.json"):
        print(name, os.path.getsize(os.path.join(HERE, name)), "bytes")
