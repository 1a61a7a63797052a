"""GPU: a reference-format checkpoint file loaded by
``B200HSTUChessModel.from_checkpoint`` and served on the device.

The file is an Ignite checkpoint (the state dict under ``"model"``, keys
prefixed with ``module._orig_mod.`` as a DDP-wrapped compiled model saves
them), read like the reference's ``load_hstu_checkpoint``
(src/imba_chess/eval/position_evaluator.py:118-181).  The served model must
match the fp32 oracle built from the same tensors: a prefill through the
model API and a grouped-decode wave through ``ActorInferenceServer``, max abs
1e-4 on logits, value logits, legal logits and v.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from imba_chess_b200 import synth
from imba_chess_b200.model import B200HSTUChessModel
from imba_chess_b200.protocol import RootEvalRequest, WaveRequest, WaveRow
from imba_chess_b200.server import ActorInferenceServer
from oracle.hstu_np import OracleModel, value_stm

pytestmark = pytest.mark.gpu

ATOL = 1e-4


def test_ignite_checkpoint_served_matches_oracle(tmp_path):
    dims = synth.D256
    sd = synth.make_state_dict(dims, 17, profile="reference")
    path = tmp_path / "checkpoint_1000.pt"
    torch.save({"model": {"module._orig_mod." + k: torch.from_numpy(v) for k, v in sd.items()},
                "optimizer": {}, "trainer": {"iteration": 1000}}, path)
    model = B200HSTUChessModel.from_checkpoint(path, dtype=torch.float32, device="cuda:0", require_value_head=True)
    orc = OracleModel(sd, dims)

    # prefill of three real games through the model API
    games = [synth.chess_game(40 + g, n) for g, n in enumerate((12, 47, 90))]
    tok = synth.concat_tokens([g.tokens for g in games])
    lens = [int(g.tokens["piece_ids"].shape[0]) for g in games]
    offsets = np.concatenate([[0], np.cumsum(lens)])
    batch = {k: torch.from_numpy(v) for k, v in tok.items()}
    batch["seq_offsets"] = torch.from_numpy(offsets)
    batch["total_tokens"] = int(offsets[-1])
    out = model.forward(batch, return_loss=False, return_kv=False)
    ref = orc.forward(tok, offsets)
    assert float(np.abs(out["logits"].cpu().numpy() - ref["logits"]).max()) <= ATOL
    assert float(np.abs(out["value_logits"].cpu().numpy() - ref["value_logits"]).max()) <= ATOL

    # a wave of every legal child of each game through the server
    wave = synth.chess_grouped_wave(n_parents=3, plies=(12, 90), seed=40)
    server = ActorInferenceServer(model=model, device="cuda:0", dtype=torch.float32, kv_pool_pages=256)
    roots = []
    for g, pt in enumerate(wave.prefix_tokens):
        T = int(pt["piece_ids"].shape[0])
        ba = {k: v.tolist() for k, v in pt.items()}
        ba.update(total_tokens=T, seq_offsets=[0, T])
        roots.append(RootEvalRequest(worker_id=g, turn_id=0, legal_vocab_ids=[2], batch_arrays=ba))
    server.service(roots)
    keys = ("turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id")
    rt = wave.row_tokens
    reqs, order = [], []
    for g in range(3):
        rows = []
        for i in np.nonzero(wave.group_index == g)[0]:
            bs = {"piece_ids": rt["piece_ids"][i].tolist(), **{k: int(rt[k][i]) for k in keys}}
            rows.append(WaveRow(node_id=int(i), parent_id=None, prev_move_vocab_id=int(rt["prev_move_id"][i]),
                                board_state=bs, legal_vocab_ids=wave.legal_ids[i].tolist()))
            order.append(int(i))
        reqs.append(WaveRequest(worker_id=g, turn_id=0, rows=rows))
    got = [row for r in server.service(reqs) for row in r.rows]
    order = np.asarray(order)
    pl = wave.prefix_lens
    pref = [orc.forward(pt, [0, n])["kv_caches"] for pt, n in zip(wave.prefix_tokens, pl)]
    max_p = max(pl)
    grouped = [(np.stack([np.pad(p[l][0], ((0, 0), (0, max_p - p[l][0].shape[1]), (0, 0))) for p in pref]),
                np.stack([np.pad(p[l][1], ((0, 0), (0, max_p - p[l][1].shape[1]), (0, 0))) for p in pref]))
               for l in range(dims.num_layers)]
    gi = wave.group_index[order]
    rd = orc.forward_decode_grouped(new_token_batch=synth.slice_tokens(rt, order), positions=np.asarray(pl)[gi],
                                    group_index=gi, prefix_kv_grouped=grouped, prefix_lens_list=pl)
    v_ref = value_stm(rd["value_logits"])
    assert len(got) == order.size > 0
    for j, (v, ll) in enumerate(got):
        ids = wave.legal_ids[order[j]]
        assert abs(v - float(v_ref[j])) <= ATOL
        if len(ids):
            assert float(np.abs(np.asarray(ll) - rd["logits"][j, ids]).max()) <= ATOL
