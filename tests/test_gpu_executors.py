"""GPU: the paged executors for the rollout scheduler (imba_chess_b200.executors)
against the fp32 oracle, and the dense model API reusing its scratch pool.

The reference's rollout path merges every live game's request of a tick into
one call (src/imba_chess/eval/merged_executors.py:124-135, :300-346), padding
and stacking every game's prefix KV per decode wave.  The paged executors keep
each game's prefix and node arena in the model's pool instead.  Checked here
on real random-legal-play games (fp32 model, max abs 1e-4): a merged root eval
of three games, then two decode waves (depth-0 children of each game, then one
child per depth-0 node whose suffix is its parent's arena row), with the arena
rows numbered like ``_KVArena.append``.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from imba_chess_b200 import synth
from imba_chess_b200.executors import PagedDecodeRequest, make_decode_wave_executor, make_root_eval_executor
from imba_chess_b200.model import B200HSTUChessModel
from oracle.hstu_np import OracleModel, value_stm

pytestmark = pytest.mark.gpu

ATOL = 1e-4


def _stack(kv_list, L):
    max_p = max(p[0][0].shape[1] for p in kv_list)
    return [(np.stack([np.pad(p[l][0], ((0, 0), (0, max_p - p[l][0].shape[1]), (0, 0))) for p in kv_list]),
             np.stack([np.pad(p[l][1], ((0, 0), (0, max_p - p[l][1].shape[1]), (0, 0))) for p in kv_list]))
            for l in range(L)]


def test_paged_executors_match_oracle():
    dims = synth.D256
    sd = synth.make_state_dict(dims, 6, profile="reference")
    model = B200HSTUChessModel(sd, dtype=torch.float32, device="cuda:0")
    orc = OracleModel(sd, dims)
    pool = model.new_pool(512)
    games = [synth.chess_game(300 + g, n) for g, n in enumerate((14, 41, 77))]
    games = [g for g in games if g.legal_ucis]
    root = make_root_eval_executor(model=model, pool=pool)
    res = root([dict(g.tokens, legal_ids=g.legal_ids) for g in games])
    pref = []
    for g, r in zip(games, res):
        o = orc.forward(g.tokens, [0, g.tokens["piece_ids"].shape[0]])
        pref.append(o["kv_caches"])
        assert abs(r["value_stm"] - float(value_stm(o["value_logits"][-1:])[0])) <= ATOL
        assert np.abs(r["legal_logits"] - o["logits"][-1, g.legal_ids]).max() <= ATOL
        assert r["game"].prefix_len == g.tokens["piece_ids"].shape[0]
    paged = [r["game"] for r in res]
    lens = [p.prefix_len for p in paged]
    decode = make_decode_wave_executor(model=model, pool=pool)
    rng = np.random.default_rng(8)
    node_kv = {}  # (game, arena row) -> oracle per-layer (k [H, d], v [H, d])
    prev_rows = [[] for _ in games]
    for depth in range(2):
        reqs, toks, chains, legal = [], [], [], []
        for gi, g in enumerate(games):
            n = 5 if depth == 0 else len(prev_rows[gi])
            tok = synth.random_tokens(rng, n, dims)
            ch = [[] for _ in range(n)] if depth == 0 else [[r] for r in prev_rows[gi]]
            ids = [synth.random_legal_ids(rng, int(rng.integers(1, 30)), dims.vocab).tolist() for _ in range(n)]
            reqs.append(PagedDecodeRequest(game=paged[gi], tokens=tok, parent_rows=ch, legal_ids=ids))
            toks.append(tok)
            chains.append(ch)
            legal.append(ids)
        out = decode(reqs)
        # oracle: grouped decode of all rows, suffix = the parent's KV from the oracle
        gi_all = np.concatenate([np.full(len(c), gi) for gi, c in enumerate(chains)])
        tok_all = synth.concat_tokens(toks)
        kw = {}
        if depth:
            flat_chains = [c for cs in chains for c in cs]
            sk = [np.stack([np.stack([node_kv[(gi_all[i], r)][l][0] for r in c], axis=1)
                            for i, c in enumerate(flat_chains)]) for l in range(dims.num_layers)]
            sv = [np.stack([np.stack([node_kv[(gi_all[i], r)][l][1] for r in c], axis=1)
                            for i, c in enumerate(flat_chains)]) for l in range(dims.num_layers)]
            kw = dict(suffix_kv=list(zip(sk, sv)), suffix_positions=np.asarray(lens)[gi_all][:, None],
                      suffix_mask=np.ones((len(gi_all), 1), dtype=bool))
        rd = orc.forward_decode_grouped(new_token_batch=tok_all, positions=np.asarray(lens)[gi_all] + depth,
                                        group_index=gi_all, prefix_kv_grouped=_stack(pref, dims.num_layers),
                                        prefix_lens_list=lens, **kw)
        v_ref = value_stm(rd["value_logits"])
        i = 0
        for gi, o in enumerate(out):
            n = len(chains[gi])
            # arena rows: consecutive per game, in wave order
            assert o["arena_rows"] == list(range(depth * 5, depth * 5 + n))
            for j in range(n):
                assert abs(float(o["value_stm"][j]) - float(v_ref[i])) <= ATOL
                if legal[gi][j]:
                    assert np.abs(o["legal_logits"][j] - rd["logits"][i, legal[gi][j]]).max() <= ATOL
                node_kv[(gi, o["arena_rows"][j])] = [(rd["kv"][l][0][i, :, 0], rd["kv"][l][1][i, :, 0])
                                                     for l in range(dims.num_layers)]
                i += 1
            prev_rows[gi] = o["arena_rows"]


def test_dense_decode_api_reuses_its_scratch_pool():
    """Consecutive forward_decode_grouped calls on the dense API stage into
    one scratch pool (no pool allocation per call) and stay correct."""
    dims = synth.SMALL
    sd = synth.make_state_dict(dims, 5, profile="sharp")
    model = B200HSTUChessModel(sd, dtype=torch.float32, device="cuda:0")
    orc = OracleModel(sd, dims)
    rng = np.random.default_rng(1)
    lens = [9, 20, 13]
    docs = [synth.game_tokens(rng, n - 2, dims) for n in lens]
    pref = [orc.forward(d, [0, n])["kv_caches"] for d, n in zip(docs, lens)]
    grouped = [(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()) for k, v in _stack(pref, dims.num_layers)]
    pools = []
    for call in range(3):
        gi = rng.integers(0, 3, size=7)
        new = synth.random_tokens(rng, 7, dims)
        pos = np.asarray(lens)[gi]
        out = model.forward_decode_grouped(new_token_batch={k: torch.from_numpy(v) for k, v in new.items()},
                                           positions=torch.from_numpy(pos), group_index=torch.from_numpy(gi),
                                           prefix_kv_grouped=grouped, prefix_lens=torch.tensor(lens),
                                           prefix_lens_list=lens)
        ref = orc.forward_decode_grouped(new_token_batch=new, positions=pos, group_index=gi,
                                         prefix_kv_grouped=_stack(pref, dims.num_layers), prefix_lens_list=lens)
        assert float(np.abs(out["logits"].cpu().numpy() - ref["logits"]).max()) <= ATOL
        pools.append(model._scratch)
    assert pools[0] is pools[1] is pools[2]
