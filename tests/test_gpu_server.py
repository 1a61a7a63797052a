"""GPU: the B200 ActorInferenceServer replays the reference server's scripted
session (tests/golden/server_session.json, produced by the reference's own
``ActorInferenceServer`` on CPU fp32) and must give the same responses
(max abs 1e-4) and the same arena row ids / node chains (exactly)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from imba_chess_b200 import synth
from imba_chess_b200.model import B200HSTUChessModel
from imba_chess_b200.protocol import RootEvalRequest, WaveRequest, WaveRow
from imba_chess_b200.server import ActorInferenceServer
from tests import golden_io

pytestmark = pytest.mark.gpu

ATOL = 1e-4


def _request(d):
    if d["type"] == "root":
        return RootEvalRequest(**{k: v for k, v in d.items() if k != "type"})
    return WaveRequest(worker_id=d["worker_id"], turn_id=d["turn_id"], rows=[WaveRow(**r) for r in d["rows"]])


def _server(dtype=torch.float32, pages=512):
    doc = golden_io.load_session()
    dims = synth.ModelDims(**doc["model"]["dims"])
    sd = synth.make_state_dict(dims, doc["model"]["seed"], profile=doc["model"]["profile"])
    model = B200HSTUChessModel(sd, dtype=dtype, device="cuda:0")
    return doc, ActorInferenceServer(model=model, device="cuda:0", dtype=dtype, kv_pool_pages=pages)


def _replay(doc, server, check=True):
    captured = []
    for step, expected in zip(doc["steps"], doc["responses"]):
        if "service" in step:
            got = server.service([_request(r) for r in step["service"]])
            captured.append(got)
            if not check:
                continue
            assert len(got) == len(expected)
            for g, e in zip(got, expected):
                if e["type"] == "root":
                    assert g.turn_id == e["turn_id"]
                    assert abs(g.value_stm - e["value_stm"]) <= ATOL
                    assert len(g.legal_logits) == len(e["legal_logits"])
                    assert np.abs(np.asarray(g.legal_logits) - np.asarray(e["legal_logits"])).max(initial=0) <= ATOL
                else:
                    assert len(g.rows) == len(e["rows"])
                    for (gv, gl), (ev, el) in zip(g.rows, e["rows"]):
                        assert abs(gv - ev) <= ATOL
                        assert len(gl) == len(el)
                        assert np.abs(np.asarray(gl) - np.asarray(el)).max(initial=0) <= ATOL
        elif "release_turn" in step:
            server.release_turn(*step["release_turn"])
        else:
            server.release_game(step["release_game"])
    return captured


def test_server_session_matches_reference_fp32():
    doc, server = _server()
    _replay(doc, server)
    chains = {f"{w},{t}": {str(n): c for n, c in ts.node_chains.items()} for (w, t), ts in server._turns.items()}
    assert chains == doc["node_chains"]
    sizes = {f"{w},{t}": (ts.arena.length if ts.arena is not None else 0) for (w, t), ts in server._turns.items()}
    assert sizes == doc["arena_sizes"]
    assert {str(w): g.prefix_len for w, g in server._games.items()} == doc["game_prefix_lens"]


def test_arena_payload_persists_bit_exact():
    """Every node's k/v, read back from its arena slot after later waves,
    roots and releases, is bit-identical to what was written when the node
    was evaluated (no page reuse while a turn is live)."""
    doc, server = _server()
    snapshots = {}
    model = server._model
    for step in doc["steps"]:
        if "service" in step:
            server.service([_request(r) for r in step["service"]])
            for (w, t), ts in server._turns.items():
                if ts.arena is None:
                    continue
                for node, chain in ts.node_chains.items():
                    key = (w, t, node)
                    if key in snapshots:
                        continue
                    slot = torch.from_numpy(ts.arena.slots_of([chain[-1]]).astype(np.int32)).cuda()
                    snapshots[key] = [tuple(x.clone() for x in model.kv_gather(server.pool, l, slot))
                                      for l in range(model.dims.num_layers)]
        elif "release_turn" in step:
            server.release_turn(*step["release_turn"])
            snapshots = {k: v for k, v in snapshots.items() if (k[0], k[1]) != tuple(step["release_turn"])}
        else:
            server.release_game(step["release_game"])
    assert snapshots
    for (w, t, node), layers in snapshots.items():
        ts = server._turns[(w, t)]
        slot = torch.from_numpy(ts.arena.slots_of([ts.node_chains[node][-1]]).astype(np.int32)).cuda()
        for l, (k0, v0) in enumerate(layers):
            k1, v1 = model.kv_gather(server.pool, l, slot)
            assert torch.equal(k0, k1) and torch.equal(v0, v1)


def test_server_errors_match_reference():
    doc, server = _server()
    steps = doc["steps"]
    with pytest.raises(TypeError):
        server.service([object()])
    with pytest.raises(KeyError):  # wave for an unregistered turn
        server.service([_request(steps[1]["service"][0])])
    with pytest.raises(KeyError):  # incremental root without a game
        server.service([_request(steps[5]["service"][0])])
    assert server.service([]) == []
    server.service([_request(r) for r in steps[0]["service"]])
    inc = dict(steps[5]["service"][0])
    bad = dict(inc, prefix_len_before=inc["prefix_len_before"] + 1)
    with pytest.raises(RuntimeError):  # desync
        server.service([_request(bad)])
    over = dict(inc, incremental_tokens={k: v * 40 for k, v in inc["incremental_tokens"].items()})
    with pytest.raises(RuntimeError):  # past max_position_embeddings
        server.service([_request(over)])
    zero = dict(inc, incremental_tokens={k: [] for k in inc["incremental_tokens"]})
    with pytest.raises(ValueError):
        server.service([_request(zero)])
    server.release_turn(123, 456)  # idempotent no-ops
    server.release_game(789)


def test_value_head_guard():
    dims = synth.ModelDims(64, 1, 1, 64, 64, vocab=40, max_pos=32, value_head=False)
    sd = synth.make_state_dict(dims, 1, profile="sharp")
    model = B200HSTUChessModel(sd, dtype=torch.float32, device="cuda:0")
    with pytest.raises(ValueError):
        ActorInferenceServer(model=model, device="cuda:0", dtype=torch.float32, kv_pool_pages=64)
    server = ActorInferenceServer(model=model, device="cuda:0", dtype=torch.float32, kv_pool_pages=64,
                                  require_value_head=False)
    rng = np.random.default_rng(0)
    tok = synth.game_tokens(rng, 5, dims)
    ba = {k: v.tolist() for k, v in tok.items()}
    ba.update(total_tokens=7, seq_offsets=[0, 7])
    [resp] = server.service([RootEvalRequest(worker_id=0, turn_id=0, legal_vocab_ids=[3, 4, 5], batch_arrays=ba)])
    assert resp.value_stm == 0.0  # documented zero placeholder
    assert len(resp.legal_logits) == 3
