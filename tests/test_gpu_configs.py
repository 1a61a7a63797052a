"""GPU parity at the benchmark configurations, through the product API,
against the fp32 CPU oracle.

The reference's own contracts are the model (grouped decode == per-game
decode, decode == full forward: tests/test_grouped_decode.py:137-481 and
tests/test_prefix_decode.py:198-291 of the reference) and the actor server
(tests/test_actor_server.py).  Here they are checked at the sizes the
benchmark runs, on real positions from seeded uniformly-random legal play:

* config 1, exactly as stated: fp32, d256 / 4 layers / 4 heads, 64 games of
  U[10, 120] plies; jagged prefill (``forward(return_kv=True)``), then one
  decode token per game (``forward_decode_grouped`` over the padded prefix
  stack) and the same through ``ActorInferenceServer.service()``.  Bar: max
  abs error 1e-4 on logits and value logits.
* config 2 at full size: bf16, d512 / 8 layers / 8 heads, 256 parents of
  U[20, 200] plies, every legal move of each parent as a sibling row, one
  ``service()`` wave.  Bars against the fp32 oracle: max abs 3e-2 on the
  legal logits (and on their log-softmax), top-1 legal-move agreement >=
  99.9 % (asserted only on >= 1,000 rows), |delta v| <= 0.02.
* config 3, seeded subset: bf16, d512 / 8 / 8 with max_pos 1024, 200 games of
  log-uniform [1, 300] plies prefilled as one packed jagged batch, then 5
  single-token decode + KV-append steps per game (incremental roots); the
  same bf16 bars over the 1,200 evaluated positions; the persisted prefix
  lengths are checked exactly.
* config 4, seeded subset: bf16, d512 / 8 / 8 with max_pos 1024, 36 games of
  U[40, 250] plies, sequential-halving rounds of 16 / 8 / 4 / 2 arms whose
  rows carry their arms' suffix chains (1,080 rows).
* config 5, seeded subset: bf16, d1024 / 16 layers / 16 heads, 26 parents of
  U[300, 600] plies with K = 40 sibling rows each (1,040 rows).

Set IMBA_PARITY_REPORT to a file path to append each case's measured errors
as one JSON line.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from imba_chess_b200 import synth
from imba_chess_b200.model import B200HSTUChessModel
from imba_chess_b200.protocol import RootEvalRequest, WaveRequest, WaveRow
from imba_chess_b200.server import ActorInferenceServer
from oracle.hstu_np import OracleModel, log_softmax_f32, value_stm

pytestmark = pytest.mark.gpu

FP32_ATOL = 1e-4
BF16_ATOL = 3e-2
BF16_TOP1 = 0.999
BF16_DV = 0.02
TOP1_MIN_ROWS = 1000
SIDE = ("turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id")


def _report(case: str, **stats) -> None:
    path = os.environ.get("IMBA_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"case": case, **stats}) + "\n")


def _pool_pages(lens, rows, extra=64):
    return sum(-(-n // 16) for n in lens) + 2 * len(lens) + 2 * (-(-rows // 16)) + extra


def _roots(prefixes, turn_id=0):
    reqs = []
    for g, pt in enumerate(prefixes):
        T = int(pt["piece_ids"].shape[0])
        ba = {k: v.tolist() for k, v in pt.items()}
        ba.update(total_tokens=T, seq_offsets=[0, T])
        reqs.append(RootEvalRequest(worker_id=g, turn_id=turn_id, legal_vocab_ids=[2, 3], batch_arrays=ba))
    return reqs


def _wave_requests(wave, turn_id=0):
    """One WaveRequest per parent with rows (request order = parent order)."""
    rt = wave.row_tokens
    reqs, order = [], []
    for g in range(len(wave.prefix_tokens)):
        idx = np.nonzero(wave.group_index == g)[0]
        if idx.size == 0:
            continue
        rows = []
        for i in idx:
            bs = {"piece_ids": rt["piece_ids"][i].tolist(), **{k: int(rt[k][i]) for k in SIDE}}
            rows.append(WaveRow(node_id=int(i), parent_id=None, prev_move_vocab_id=int(rt["prev_move_id"][i]),
                                board_state=bs, legal_vocab_ids=[int(x) for x in wave.legal_ids[i]]))
            order.append(int(i))
        reqs.append(WaveRequest(worker_id=g, turn_id=turn_id, rows=rows))
    return reqs, np.asarray(order, dtype=np.int64)


def _stack(kv_list, L):
    """Per-prefix oracle KV -> the reference's padded [G, H, maxP, d] stack."""
    max_p = max(p[0][0].shape[1] for p in kv_list)
    out = []
    for l in range(L):
        ks = np.stack([np.pad(p[l][0], ((0, 0), (0, max_p - p[l][0].shape[1]), (0, 0))) for p in kv_list])
        vs = np.stack([np.pad(p[l][1], ((0, 0), (0, max_p - p[l][1].shape[1]), (0, 0))) for p in kv_list])
        out.append((ks, vs))
    return out


def _oracle_wave(orc, wave, rows):
    """The oracle's grouped decode of ``rows`` (indices into the wave)."""
    lens = wave.prefix_lens
    pref = [orc.forward(pt, [0, lens[g]])["kv_caches"] for g, pt in enumerate(wave.prefix_tokens)]
    gi = wave.group_index[rows]
    tok = synth.slice_tokens(wave.row_tokens, rows)
    return orc.forward_decode_grouped(new_token_batch=tok, positions=np.asarray(lens)[gi], group_index=gi,
                                      prefix_kv_grouped=_stack(pref, orc.L), prefix_lens_list=lens)


def _compare_rows(got_rows, ref_logits, ref_value_logits, legal):
    """got_rows: (v, legal logits) per row; reference logits [n, V] and value
    logits [n, 3]; legal: per-row ids.  Returns the measured errors."""
    ref_v = value_stm(ref_value_logits)
    max_dl = max_dlp = max_dv = 0.0
    agree = 0
    for j, (v_got, ll_got) in enumerate(got_rows):
        ids = np.asarray(legal[j], dtype=np.int64)
        ll_got = np.asarray(ll_got, dtype=np.float64)
        ll_ref = ref_logits[j, ids].astype(np.float64)
        assert ll_got.shape == ll_ref.shape
        max_dv = max(max_dv, abs(float(v_got) - float(ref_v[j])))
        if ids.size == 0:
            agree += 1
            continue
        max_dl = max(max_dl, float(np.abs(ll_got - ll_ref).max()))
        max_dlp = max(max_dlp, float(np.abs(log_softmax_f32(ll_got) - log_softmax_f32(ll_ref)).max()))
        agree += int(np.argmax(ll_got) == np.argmax(ll_ref))
    n = len(got_rows)
    return {"rows": n, "max_dlogit": max_dl, "max_dlogprob": max_dlp, "max_dv": max_dv, "top1": agree / n}


def _assert_bf16(stats):
    assert stats["max_dlogit"] <= BF16_ATOL, stats
    assert stats["max_dlogprob"] <= BF16_ATOL, stats
    assert stats["max_dv"] <= BF16_DV, stats
    if stats["rows"] >= TOP1_MIN_ROWS:
        assert stats["top1"] >= BF16_TOP1, stats


# ----------------------------------------------------------------------
# config 1: fp32 d256 / 4 layers / 4 heads, 64 games, prefill + one decode token
# ----------------------------------------------------------------------
def _cfg1_games():
    """64 games of U[10, 120] random legal plies that are still in progress
    (a game that ended in mate or stalemate has no decode token to add; the
    next seed takes its place)."""
    rng = np.random.default_rng(1234)
    games, seed = [], 1234
    while len(games) < 64:
        g = synth.chess_game(seed, int(rng.integers(10, 121)))
        seed += 1
        if g.legal_ucis:
            games.append(g)
    return games


def test_config1_prefill_then_decode_fp32_model_api():
    dims = synth.D256
    sd = synth.make_state_dict(dims, 2, profile="reference")
    model = B200HSTUChessModel(sd, dtype=torch.float32, device="cuda:0")
    orc = OracleModel(sd, dims)
    games = _cfg1_games()
    tok = synth.concat_tokens([g.tokens for g in games])
    lens = [int(g.tokens["piece_ids"].shape[0]) for g in games]
    offsets = np.concatenate([[0], np.cumsum(lens)])
    batch = {k: torch.from_numpy(v) for k, v in tok.items()}
    batch["seq_offsets"] = torch.from_numpy(offsets)
    batch["total_tokens"] = int(offsets[-1])
    out = model.forward(batch, return_loss=False, return_kv=True)
    ref = orc.forward(tok, offsets)
    d_pre = float(np.abs(out["logits"].cpu().numpy() - ref["logits"]).max())
    d_pre_v = float(np.abs(out["value_logits"].cpu().numpy() - ref["value_logits"]).max())
    d_kv = max(float(np.abs(k.cpu().numpy() - rk).max()) for (k, _), (rk, _) in zip(out["kv_caches"], ref["kv_caches"]))
    # one decode token per game: the position after the first of its legal moves
    from imba_chess_b200 import worker_chess as wc

    enc, vocab = wc.BoardStateEncoder(), wc.static_move_vocab()
    new = {k: [] for k in synth.TOKEN_FIELDS}
    for g in games:
        u = g.legal_ucis[0]
        s = enc.encode_fen(wc.push_uci(g.fen, u))
        new["piece_ids"].append(s.piece_ids)
        new["seq_token_id"].append(synth.EVENT_TOKEN_ID)
        new["prev_move_id"].append(vocab[u])
        for k in SIDE:
            new[k].append(getattr(s, k))
    new = {k: np.asarray(v, dtype=np.int64) for k, v in new.items()}
    G = len(games)
    # the reference's merge: pad every game's prefix KV to max length and stack
    max_p = max(lens)
    grouped = []
    for k, v in out["kv_caches"]:
        ks, vs = [], []
        for g in range(G):
            a, b = int(offsets[g]), int(offsets[g + 1])
            ks.append(torch.nn.functional.pad(k[:, a:b], (0, 0, 0, max_p - (b - a))))
            vs.append(torch.nn.functional.pad(v[:, a:b], (0, 0, 0, max_p - (b - a))))
        grouped.append((torch.stack(ks), torch.stack(vs)))
    gi = np.arange(G)
    res = model.forward_decode_grouped(
        new_token_batch={k: torch.from_numpy(v) for k, v in new.items()}, positions=torch.tensor(lens),
        group_index=torch.from_numpy(gi), prefix_kv_grouped=grouped, prefix_lens=torch.tensor(lens),
        prefix_lens_list=lens)
    ref_pk = [[(k[:, a:b], v[:, a:b]) for k, v in ref["kv_caches"]] for a, b in zip(offsets[:-1], offsets[1:])]
    rd = orc.forward_decode_grouped(new_token_batch=new, positions=np.asarray(lens), group_index=gi,
                                    prefix_kv_grouped=_stack(ref_pk, dims.num_layers), prefix_lens_list=lens)
    d_dec = float(np.abs(res["logits"].cpu().numpy() - rd["logits"]).max())
    d_dec_v = float(np.abs(res["value_logits"].cpu().numpy() - rd["value_logits"]).max())
    d_dec_kv = max(float(np.abs(k.cpu().numpy() - rk).max()) for (k, _), (rk, _) in zip(res["kv"], rd["kv"]))
    _report("config1_model_api", games=G, prefill_tokens=int(offsets[-1]), prefill_max_dlogit=d_pre,
            prefill_max_dvalue_logit=d_pre_v, prefill_max_dk=d_kv, decode_max_dlogit=d_dec,
            decode_max_dvalue_logit=d_dec_v, decode_max_dk=d_dec_kv)
    assert d_pre <= FP32_ATOL and d_pre_v <= FP32_ATOL and d_kv <= FP32_ATOL
    assert d_dec <= FP32_ATOL and d_dec_v <= FP32_ATOL and d_dec_kv <= FP32_ATOL


def test_config1_through_server_fp32():
    """The same 64 games through ``service()``: full roots, then one wave of
    one row per game (every legal move id of the child), at 1e-4."""
    dims = synth.D256
    sd = synth.make_state_dict(dims, 2, profile="reference")
    model = B200HSTUChessModel(sd, dtype=torch.float32, device="cuda:0")
    orc = OracleModel(sd, dims)
    games = _cfg1_games()
    wave = synth.GroupedWave([g.tokens for g in games], *_first_children(games))
    server = ActorInferenceServer(model=model, device="cuda:0", dtype=torch.float32,
                                  kv_pool_pages=_pool_pages(wave.prefix_lens, wave.num_rows))
    root_resp = server.service(_roots(wave.prefix_tokens))
    reqs, order = _wave_requests(wave)
    resp = server.service(reqs)
    got = [row for r in resp for row in r.rows]
    ref = _oracle_wave(orc, wave, order)
    stats = _compare_rows(got, ref["logits"], ref["value_logits"], [wave.legal_ids[i] for i in order])
    # root responses: the last prefix token of each game
    pre = [orc.forward(pt, [0, n]) for pt, n in zip(wave.prefix_tokens, wave.prefix_lens)]
    d_root_v = max(abs(r.value_stm - float(value_stm(p["value_logits"][-1:])[0])) for r, p in zip(root_resp, pre))
    _report("config1_server", **stats, root_max_dv=d_root_v)
    assert stats["max_dlogit"] <= FP32_ATOL and stats["max_dv"] <= FP32_ATOL, stats
    assert stats["top1"] == 1.0
    assert d_root_v <= FP32_ATOL


def _first_children(games):
    from imba_chess_b200 import worker_chess as wc

    enc, vocab = wc.BoardStateEncoder(), wc.static_move_vocab()
    toks, legal = [], []
    for g in games:
        u = g.legal_ucis[0]
        child = wc.push_uci(g.fen, u)
        s = enc.encode_fen(child)
        toks.append({"piece_ids": np.asarray([s.piece_ids]), "seq_token_id": np.asarray([synth.EVENT_TOKEN_ID]),
                     "prev_move_id": np.asarray([vocab[u]]), **{k: np.asarray([getattr(s, k)]) for k in SIDE}})
        legal.append(np.asarray(wc.legal_vocab_projection(child)[0], dtype=np.int64))
    rows = {k: np.concatenate([t[k] for t in toks]).astype(np.int64) for k in synth.TOKEN_FIELDS}
    return rows, np.arange(len(games), dtype=np.int64), legal


# ----------------------------------------------------------------------
# config 2 at full size (bf16 d512 / 8 / 8, 256 parents, every legal move)
# ----------------------------------------------------------------------
def _bf16_server_wave(dims, wave, seed):
    sd = synth.make_state_dict(dims, seed, profile="reference")
    model = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    server = ActorInferenceServer(model=model, device="cuda:0", dtype=torch.bfloat16,
                                  kv_pool_pages=_pool_pages(wave.prefix_lens, wave.num_rows))
    server.service(_roots(wave.prefix_tokens))
    reqs, order = _wave_requests(wave)
    resp = server.service(reqs)
    got = [row for r in resp for row in r.rows]
    assert len(got) == order.size == wave.num_rows
    ref = _oracle_wave(OracleModel(sd, dims), wave, order)
    return _compare_rows(got, ref["logits"], ref["value_logits"], [wave.legal_ids[i] for i in order])


def test_config2_full_wave_bf16_through_server():
    wave = synth.chess_grouped_wave(n_parents=256, plies=(20, 200), seed=1234)
    assert wave.num_rows >= TOP1_MIN_ROWS
    stats = _bf16_server_wave(synth.D512, wave, seed=2)
    _report("config2_full_wave", parents=256, **stats)
    _assert_bf16(stats)


# ----------------------------------------------------------------------
# config 5 subset (bf16 d1024 / 16 / 16, long prefixes, K = 40)
# ----------------------------------------------------------------------
def test_config5_subset_bf16_through_server():
    wave = synth.grouped_wave(synth.D1024, n_parents=26, plies=(300, 600), siblings=(40, 40), seed=1234)
    assert wave.num_rows == 1040
    stats = _bf16_server_wave(synth.D1024, wave, seed=2)
    _report("config5_subset", parents=26, **stats)
    _assert_bf16(stats)


# ----------------------------------------------------------------------
# config 4 subset: sequential-halving rounds with suffix chains
# ----------------------------------------------------------------------
def test_config4_halving_subset_bf16_through_server():
    """36 games of U[40, 250] plies, rounds of 16 / 8 / 4 / 2 surviving arms
    (1,080 rows): round r evaluates one node per arm at depth r whose suffix is
    the arm's chain in the turn arena (rounds 1-3 run the pages-only attention
    and the per-row combine pass), against the fp32 oracle fed its own KV of
    the chain nodes as suffix keys."""
    dims = synth.D512_LONG
    sd = synth.make_state_dict(dims, 2, profile="reference")
    model = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    orc = OracleModel(sd, dims)
    rng = np.random.default_rng(1234)
    G, rounds = 36, (16, 8, 4, 2)
    prefixes = [synth.game_tokens(rng, int(rng.integers(40, 251)), dims) for _ in range(G)]
    lens = [int(p["piece_ids"].shape[0]) for p in prefixes]
    server = ActorInferenceServer(model=model, device="cuda:0", dtype=torch.bfloat16,
                                  kv_pool_pages=_pool_pages(lens, G * sum(rounds), extra=256))
    server.service(_roots(prefixes))
    grouped = _stack([orc.forward(pt, [0, lens[g]])["kv_caches"] for g, pt in enumerate(prefixes)], orc.L)
    node_kv = {}  # node id -> per-layer (k [H, d], v [H, d]) from the oracle
    got_all, ref_logits, ref_values, legal_all = [], [], [], []
    for r, K in enumerate(rounds):
        tok = synth.random_tokens(rng, G * K, dims)
        legal = [synth.random_legal_ids(rng, int(rng.integers(20, 41)), dims.vocab) for _ in range(G * K)]
        reqs, nodes, parents = [], [], []
        for g in range(G):
            rows = []
            for a in range(K):
                i = g * K + a
                nid = 10000 * g + 100 * r + a
                pid = None if r == 0 else 10000 * g + 100 * (r - 1) + a
                bs = {"piece_ids": tok["piece_ids"][i].tolist(), **{k: int(tok[k][i]) for k in SIDE}}
                rows.append(WaveRow(node_id=nid, parent_id=pid, prev_move_vocab_id=int(tok["prev_move_id"][i]),
                                    board_state=bs, legal_vocab_ids=legal[i].tolist()))
                nodes.append(nid)
                parents.append(pid)
            reqs.append(WaveRequest(worker_id=g, turn_id=0, rows=rows))
        resp = server.service(reqs)
        got_all += [row for wr in resp for row in wr.rows]
        gi = np.repeat(np.arange(G), K)
        kw = {}
        if r > 0:
            chains = []
            for pid in parents:  # the arm's nodes of rounds 0 .. r - 1
                ch, p = [], pid
                while p is not None:
                    ch.append(p)
                    p = p - 100 if (p % 10000) >= 100 else None
                chains.append(ch[::-1])
            sk = [np.stack([np.stack([node_kv[n][l][0] for n in ch], axis=1) for ch in chains]) for l in range(orc.L)]
            sv = [np.stack([np.stack([node_kv[n][l][1] for n in ch], axis=1) for ch in chains]) for l in range(orc.L)]
            kw = dict(suffix_kv=list(zip(sk, sv)), suffix_positions=np.asarray(lens)[gi][:, None] + np.arange(r)[None, :],
                      suffix_mask=np.ones((G * K, r), dtype=bool))
        ref = orc.forward_decode_grouped(new_token_batch=tok, positions=np.asarray(lens)[gi] + r, group_index=gi,
                                         prefix_kv_grouped=grouped, prefix_lens_list=lens, **kw)
        for i, nid in enumerate(nodes):
            node_kv[nid] = [(ref["kv"][l][0][i, :, 0], ref["kv"][l][1][i, :, 0]) for l in range(orc.L)]
        ref_logits.append(ref["logits"])
        ref_values.append(ref["value_logits"])
        legal_all += legal
    stats = _compare_rows(got_all, np.concatenate(ref_logits), np.concatenate(ref_values), legal_all)
    assert stats["rows"] == G * sum(rounds) >= TOP1_MIN_ROWS
    _report("config4_halving_subset", games=G, rounds=list(rounds), **stats)
    _assert_bf16(stats)


# ----------------------------------------------------------------------
# config 3 subset: packed jagged prefill, then decode + KV append steps
# ----------------------------------------------------------------------
def test_config3_prefill_then_append_steps_bf16():
    from imba_chess_b200 import worker_chess as wc

    dims = synth.D512_LONG
    G, steps = 200, 5
    sd = synth.make_state_dict(dims, 2, profile="reference")
    model = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    orc = OracleModel(sd, dims)
    rng = np.random.default_rng(4321)
    plies = np.exp(rng.uniform(np.log(1), np.log(300), size=G)).astype(int)
    games = [synth.chess_game(5000 + g, int(n)) for g, n in enumerate(plies)]
    # games that ended keep no further moves; the subset keeps the live ones
    games = [g for g in games if len(g.legal_ucis) > 0][:G]
    lens = [int(g.tokens["piece_ids"].shape[0]) for g in games]
    assert sum(lens) <= 32768  # one packed jagged batch
    server = ActorInferenceServer(model=model, device="cuda:0", dtype=torch.bfloat16,
                                  kv_pool_pages=_pool_pages([n + steps for n in lens], 0))
    roots = _roots([g.tokens for g in games])
    for r, g in zip(roots, games):
        r.legal_vocab_ids = list(g.legal_ids)
    got = [(r.value_stm, r.legal_logits) for r in server.service(roots)]
    ref_logits, ref_value, legal = [], [], [list(g.legal_ids) for g in games]
    kv = []
    for g in games:
        o = orc.forward(g.tokens, [0, g.tokens["piece_ids"].shape[0]])
        ref_logits.append(o["logits"][-1])
        ref_value.append(o["value_logits"][-1])
        kv.append([(k.copy(), v.copy()) for k, v in o["kv_caches"]])
    enc, vocab = wc.BoardStateEncoder(), wc.static_move_vocab()
    step_rng = np.random.default_rng(99)
    fens = [g.fen for g in games]
    ucis = [list(g.legal_ucis) for g in games]
    for step in range(steps):
        new = {k: [] for k in synth.TOKEN_FIELDS}
        reqs, step_legal = [], []
        for w, g in enumerate(games):
            if not ucis[w]:  # the game ended: repeat its last position (a legal, if idle, token)
                u, child = None, fens[w]
            else:
                u = ucis[w][int(step_rng.integers(len(ucis[w])))]
                child = wc.push_uci(fens[w], u)
            s = enc.encode_fen(child)
            ids, cu = wc.legal_vocab_projection(child)
            tok = {"piece_ids": [list(s.piece_ids)], "seq_token_id": [synth.EVENT_TOKEN_ID],
                   "prev_move_id": [vocab[u] if u else 1], **{k: [getattr(s, k)] for k in SIDE}}
            for k in synth.TOKEN_FIELDS:
                new[k].append(tok[k][0])
            reqs.append(RootEvalRequest(worker_id=w, turn_id=step + 1, legal_vocab_ids=list(ids),
                                        incremental_tokens=tok, prefix_len_before=lens[w] + step))
            step_legal.append(list(ids))
            fens[w], ucis[w] = child, list(cu)
        resp = server.service(reqs)
        got.extend((r.value_stm, r.legal_logits) for r in resp)
        newt = {k: np.asarray(v, dtype=np.int64) for k, v in new.items()}
        plen = [n + step for n in lens]
        rd = orc.forward_decode_grouped(new_token_batch=newt, positions=np.asarray(plen),
                                        group_index=np.arange(len(games)),
                                        prefix_kv_grouped=_stack(kv, dims.num_layers), prefix_lens_list=plen)
        ref_logits.extend(rd["logits"])
        ref_value.extend(rd["value_logits"])
        legal.extend(step_legal)
        for w in range(len(games)):  # append each game's new token to its oracle prefix KV
            kv[w] = [(np.concatenate([k, rd["kv"][l][0][w]], axis=1), np.concatenate([v, rd["kv"][l][1][w]], axis=1))
                     for l, (k, v) in enumerate(kv[w])]
    # persisted prefix lengths are the reference's: prefix + one token per step
    for w, n in enumerate(lens):
        assert server._games[w].prefix_len == n + steps
        assert server._games[w].seq.length == n + steps
    stats = _compare_rows(got, np.asarray(ref_logits), np.asarray(ref_value), legal)
    _report("config3_prefill_append", games=len(games), steps=steps, prefill_tokens=sum(lens), **stats)
    assert stats["rows"] == len(games) * (steps + 1) >= TOP1_MIN_ROWS
    _assert_bf16(stats)
