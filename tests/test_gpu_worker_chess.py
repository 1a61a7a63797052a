"""GPU: real chess positions from the worker-side chess module through the
server.  A turn's wave holds the start position's 20 children: their board
states, the move that reached each one (its vocabulary id) and each child's
UCI-sorted legal vocabulary ids all come from ``worker_chess``, as a search
worker would send them.  ``ActorInferenceServer.service()`` (fp32 model)
must match the oracle's grouped decode of the same rows over the same prefix
(max abs 1e-4 on every legal logit and on v)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from imba_chess_b200 import synth
from imba_chess_b200 import worker_chess as wc
from imba_chess_b200.model import B200HSTUChessModel
from imba_chess_b200.protocol import RootEvalRequest, WaveRequest, WaveRow
from imba_chess_b200.server import ActorInferenceServer
from oracle.hstu_np import OracleModel, value_stm

pytestmark = pytest.mark.gpu

START = "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1"
SIDE = ("turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id")


def test_chess_wave_through_server_matches_oracle():
    dims = synth.SMALL
    sd = synth.make_state_dict(dims, 4, profile="sharp")
    model = B200HSTUChessModel(sd, dtype=torch.float32, device="cuda:0")
    server = ActorInferenceServer(model=model, device="cuda:0", dtype=torch.float32, kv_pool_pages=64)
    oracle = OracleModel(sd, dims)

    rng = np.random.default_rng(3)
    tok = synth.game_tokens(rng, 9, dims)
    T = int(tok["piece_ids"].shape[0])
    ba = {k: v.tolist() for k, v in tok.items()}
    ba.update(total_tokens=T, seq_offsets=[0, T])
    server.service([RootEvalRequest(worker_id=0, turn_id=0, legal_vocab_ids=[2, 3], batch_arrays=ba)])

    vocab = wc.static_move_vocab()
    _, ucis = wc.legal_vocab_projection(START)
    rows, new, legal = [], {k: [] for k in ("piece_ids", "seq_token_id", "prev_move_id", *SIDE)}, []
    for i, u in enumerate(ucis):
        child = wc.push_uci(START, u)
        s = wc.BoardStateEncoder().encode_fen(child)
        ids, _ = wc.legal_vocab_projection(child)
        bs = {"piece_ids": s.piece_ids, **{k: getattr(s, k) for k in SIDE}}
        rows.append(WaveRow(node_id=i, parent_id=None, prev_move_vocab_id=vocab[u], board_state=bs,
                            legal_vocab_ids=ids))
        new["piece_ids"].append(s.piece_ids)
        new["seq_token_id"].append(synth.EVENT_TOKEN_ID)
        new["prev_move_id"].append(vocab[u])
        for k in SIDE:
            new[k].append(getattr(s, k))
        legal.append(ids)
    [resp] = server.service([WaveRequest(worker_id=0, turn_id=0, rows=rows)])

    ref_kv = oracle.forward(tok, np.array([0, T]))["kv_caches"]
    B = len(rows)
    ref = oracle.forward_decode_grouped(
        new_token_batch={k: np.asarray(v, dtype=np.int64) for k, v in new.items()},
        positions=np.full(B, T), group_index=np.zeros(B, dtype=np.int64),
        prefix_kv_grouped=[(k[None], v[None]) for k, v in ref_kv], prefix_lens_list=[T],
    )
    v_ref = value_stm(ref["value_logits"])
    assert len(resp.rows) == B
    for i, (v, ll) in enumerate(resp.rows):
        assert len(ll) == len(legal[i]) > 0
        assert abs(v - float(v_ref[i])) <= 1e-4
        assert np.abs(np.asarray(ll) - ref["logits"][i, legal[i]]).max() <= 1e-4
