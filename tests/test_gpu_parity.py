"""GPU parity: the CUDA path (through the C ABI) against the reference's own
outputs (golden fixtures) and against the CPU oracle.

Tolerances (from the hot-path contract):
  fp32 model: max abs error 1e-4 on logits and value logits (WDL);
  bf16 model: max abs error 3e-2 on logits and WDL, top-1 legal-move
              agreement >= 99.9 %, |delta v| <= 0.02, against the fp32 oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from imba_chess_b200 import synth
from imba_chess_b200.model import B200HSTUChessModel
from oracle.hstu_np import OracleModel, log_softmax_f32, value_stm
from tests import golden_io

pytestmark = pytest.mark.gpu

FP32_ATOL = 1e-4
BF16_ATOL = 3e-2
BF16_TOP1 = 0.999
BF16_DV = 0.02


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x))


def _maxabs(a, b) -> float:
    a = a.detach().float().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
    b = b.detach().float().cpu().numpy() if isinstance(b, torch.Tensor) else np.asarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    return float(np.abs(a.astype(np.float64) - b.astype(np.float64)).max()) if a.size else 0.0


def _model(which: str, dtype=torch.float32):
    dims, sd = getattr(golden_io, f"{which}_weights")()
    return dims, B200HSTUChessModel(sd, dtype=dtype, device="cuda:0")


def _batch(g, tag):
    b = {k: _t(v) for k, v in golden_io.tokens(g, tag).items()}
    b["seq_offsets"] = _t(g[f"{tag}/seq_offsets"])
    b["total_tokens"] = int(g[f"{tag}/seq_offsets"][-1])
    return b


@pytest.mark.parametrize("which", ["tiny", "small"])
def test_prefill_matches_reference_fp32(which):
    dims, m = _model(which)
    g = golden_io.load(f"{which}.npz")
    out = m.forward(_batch(g, "prefill"), return_loss=False, return_kv=True)
    assert _maxabs(out["logits"], g["prefill/logits"]) <= FP32_ATOL
    assert _maxabs(out["value_logits"], g["prefill/value_logits"]) <= FP32_ATOL
    for l, (k, v) in enumerate(out["kv_caches"]):
        assert _maxabs(k, g[f"prefill/kv/{l}/k"]) <= FP32_ATOL
        assert _maxabs(v, g[f"prefill/kv/{l}/v"]) <= FP32_ATOL


def _grouped_call(m, g, tag, layers):
    inp = golden_io.grouped_inputs(g, tag, layers)
    kw = dict(
        new_token_batch={k: _t(v) for k, v in inp["new_token_batch"].items()},
        positions=_t(inp["positions"]),
        group_index=_t(inp["group_index"]),
        prefix_kv_grouped=[(_t(k), _t(v)) for k, v in inp["prefix_kv_grouped"]],
        prefix_lens=_t(np.asarray(inp["prefix_lens_list"])),
        prefix_lens_list=inp["prefix_lens_list"],
    )
    if inp["suffix_kv"] is not None:
        kw.update(
            suffix_kv=[(_t(k), _t(v)) for k, v in inp["suffix_kv"]],
            suffix_positions=_t(inp["suffix_positions"]),
            suffix_mask=_t(inp["suffix_mask"]),
        )
    return m.forward_decode_grouped(**kw)


@pytest.mark.parametrize("which,tag", [("tiny", "grouped"), ("tiny", "single"), ("small", "grouped")])
def test_grouped_decode_matches_reference_fp32(which, tag):
    dims, m = _model(which)
    g = golden_io.load(f"{which}.npz")
    out = _grouped_call(m, g, tag, dims.num_layers)
    assert _maxabs(out["logits"], g[f"{tag}/logits"]) <= FP32_ATOL
    assert _maxabs(out["value_logits"], g[f"{tag}/value_logits"]) <= FP32_ATOL
    for l, (k, v) in enumerate(out["kv"]):
        assert _maxabs(k, g[f"{tag}/kv/{l}/k"]) <= FP32_ATOL
        assert _maxabs(v, g[f"{tag}/kv/{l}/v"]) <= FP32_ATOL


def test_single_prefix_decode_matches_reference_fp32():
    dims, m = _model("tiny")
    g = golden_io.load("tiny.npz")
    inp = golden_io.grouped_inputs(g, "single", dims.num_layers)
    T = inp["prefix_lens_list"][0]
    out = m.forward_decode(
        new_token_batch={k: _t(v) for k, v in inp["new_token_batch"].items()},
        positions=_t(inp["positions"]),
        prefix_kv=[(_t(k[0, :, :T]), _t(v[0, :, :T])) for k, v in inp["prefix_kv_grouped"]],
        suffix_kv=[(_t(k), _t(v)) for k, v in inp["suffix_kv"]],
        suffix_positions=_t(inp["suffix_positions"]),
        suffix_mask=_t(inp["suffix_mask"]),
    )
    assert _maxabs(out["logits"], g["single/logits"]) <= FP32_ATOL


def test_grouped_decode_small_bf16_tracks_reference():
    """bf16 path on the sharp-weight kernel model: a coarse bound (the bf16
    bars are asserted on the reference-initialised models below)."""
    dims, m = _model("small", torch.bfloat16)
    g = golden_io.load("small.npz")
    out = _grouped_call(m, g, "grouped", dims.num_layers)
    ref = g["grouped/logits"]
    got = out["logits"].cpu().numpy()
    assert np.abs(got - ref).max() <= 0.05 * np.abs(ref).max()
    assert (got.argmax(1) == ref.argmax(1)).mean() >= 0.75


def test_guards_raise_like_reference():
    dims, m = _model("tiny")
    g = golden_io.load("tiny.npz")
    inp = golden_io.grouped_inputs(g, "grouped", dims.num_layers)
    base = dict(
        new_token_batch={k: _t(v) for k, v in inp["new_token_batch"].items()},
        positions=_t(inp["positions"]),
        prefix_kv_grouped=[(_t(k), _t(v)) for k, v in inp["prefix_kv_grouped"]],
        prefix_lens=_t(np.asarray(inp["prefix_lens_list"])),
        prefix_lens_list=inp["prefix_lens_list"],
    )
    bad = inp["group_index"].copy()
    bad[0] = 3
    with pytest.raises(ValueError):
        m.forward_decode_grouped(group_index=_t(bad), **base)
    kw = dict(base)
    kw["prefix_lens_list"] = inp["prefix_lens_list"][:2]
    with pytest.raises(ValueError):
        m.forward_decode_grouped(group_index=_t(inp["group_index"]), **kw)
    kw = dict(base)
    kw["prefix_lens"] = _t(np.zeros(0, np.int64))
    kw["prefix_lens_list"] = []
    kw["prefix_kv_grouped"] = [(k[:0], v[:0]) for k, v in base["prefix_kv_grouped"]]
    with pytest.raises(ValueError):  # rows but no groups (hstu_model.py:713-721)
        m.forward_decode_grouped(group_index=_t(inp["group_index"]), **kw)


# ----------------------------------------------------------------------
# bf16 against the fp32 oracle on reference-initialised models.
# ----------------------------------------------------------------------
def _bf16_wave_check(dims, n_parents, plies, siblings, seed):
    from imba_chess_b200.server import ActorInferenceServer
    from imba_chess_b200.protocol import RootEvalRequest, WaveRequest, WaveRow

    sd = synth.make_state_dict(dims, 3, profile="reference")
    wave = synth.grouped_wave(dims, n_parents=n_parents, plies=plies, siblings=siblings, seed=seed)
    model = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    server = ActorInferenceServer(model=model, device="cuda:0", dtype=torch.bfloat16, kv_pool_pages=2048)
    roots = []
    for g, pt in enumerate(wave.prefix_tokens):
        T = int(pt["piece_ids"].shape[0])
        ba = {k: v.tolist() for k, v in pt.items()}
        ba.update(total_tokens=T, seq_offsets=[0, T])
        roots.append(RootEvalRequest(worker_id=g, turn_id=0, legal_vocab_ids=[2, 3], batch_arrays=ba))
    server.service(roots)
    reqs = []
    r = 0
    for g in range(n_parents):
        rows = []
        for i in np.nonzero(wave.group_index == g)[0]:
            bs = {
                "piece_ids": wave.row_tokens["piece_ids"][i].tolist(),
                **{k: int(wave.row_tokens[k][i]) for k in
                   ("turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id")},
            }
            rows.append(WaveRow(node_id=int(i), parent_id=None, prev_move_vocab_id=int(wave.row_tokens["prev_move_id"][i]),
                                board_state=bs, legal_vocab_ids=wave.legal_ids[i].tolist()))
            r += 1
        reqs.append(WaveRequest(worker_id=g, turn_id=0, rows=rows))
    resp = server.service(reqs)
    # Oracle, fp32 throughout.
    orc = OracleModel(sd, dims)
    lens = wave.prefix_lens
    max_p = max(lens)
    L = dims.num_layers
    pref = [orc.forward(pt, [0, int(pt["piece_ids"].shape[0])])["kv_caches"] for pt in wave.prefix_tokens]
    grouped = []
    for l in range(L):
        ks = np.stack([np.pad(p[l][0], ((0, 0), (0, max_p - p[l][0].shape[1]), (0, 0))) for p in pref])
        vs = np.stack([np.pad(p[l][1], ((0, 0), (0, max_p - p[l][1].shape[1]), (0, 0))) for p in pref])
        grouped.append((ks, vs))
    order = np.argsort(wave.group_index, kind="stable")
    tok = synth.slice_tokens(wave.row_tokens, order)
    gi = wave.group_index[order]
    ref = orc.forward_decode_grouped(new_token_batch=tok, positions=np.asarray(lens)[gi], group_index=gi,
                                     prefix_kv_grouped=grouped, prefix_lens_list=lens)
    ref_v = value_stm(ref["value_logits"])
    got_rows = [row for wr in resp for row in wr.rows]
    max_dl, max_dv, agree = 0.0, 0.0, 0
    for j, i in enumerate(order):
        v_got, ll_got = got_rows[j]
        ids = wave.legal_ids[i]
        ll_ref = ref["logits"][j, ids]
        max_dl = max(max_dl, float(np.abs(np.asarray(ll_got) - ll_ref).max()))
        max_dv = max(max_dv, abs(v_got - float(ref_v[j])))
        agree += int(np.argmax(ll_got) == np.argmax(ll_ref))
    n = len(order)
    return max_dl, max_dv, agree / n, n


@pytest.mark.parametrize(
    "dims,n_parents,plies,siblings",
    [(synth.D512, 6, (20, 60), (20, 40)), (synth.D256, 8, (10, 120), (1, 4)),
     (synth.D1024, 3, (300, 420), (8, 12))],
    ids=["d512-grouped", "d256-grouped", "d1024-16h-long-prefix"],
)
def test_bf16_wave_matches_fp32_oracle(dims, n_parents, plies, siblings):
    max_dl, max_dv, top1, n = _bf16_wave_check(dims, n_parents, plies, siblings, seed=1234)
    assert n > 0
    assert max_dl <= BF16_ATOL, max_dl
    assert max_dv <= BF16_DV, max_dv
    assert top1 >= BF16_TOP1, top1


def test_bf16_halving_chains_match_fp32_oracle():
    """Sequential-halving rounds through the server (arms 6 -> 3 -> 2 per
    parent, round r evaluating one node per surviving arm at depth r whose
    suffix is the arm's chain in the turn arena) against the fp32 oracle fed
    the oracle's own KV of the chain nodes as suffix keys."""
    from imba_chess_b200.protocol import RootEvalRequest, WaveRequest, WaveRow
    from imba_chess_b200.server import ActorInferenceServer

    dims = synth.D512
    sd = synth.make_state_dict(dims, 3, profile="reference")
    model = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    server = ActorInferenceServer(model=model, device="cuda:0", dtype=torch.bfloat16, kv_pool_pages=1024)
    orc = OracleModel(sd, dims)
    rng = np.random.default_rng(77)
    G, rounds = 4, (6, 3, 2)
    prefixes = [synth.game_tokens(rng, int(rng.integers(20, 60)), dims) for _ in range(G)]
    lens = [int(p["piece_ids"].shape[0]) for p in prefixes]
    roots = []
    for g, pt in enumerate(prefixes):
        ba = {k: v.tolist() for k, v in pt.items()}
        ba.update(total_tokens=lens[g], seq_offsets=[0, lens[g]])
        roots.append(RootEvalRequest(worker_id=g, turn_id=0, legal_vocab_ids=[2, 3], batch_arrays=ba))
    server.service(roots)
    pref = [orc.forward(pt, [0, lens[g]])["kv_caches"] for g, pt in enumerate(prefixes)]
    max_p = max(lens)
    grouped = []
    for l in range(dims.num_layers):
        ks = np.stack([np.pad(p[l][0], ((0, 0), (0, max_p - p[l][0].shape[1]), (0, 0))) for p in pref])
        vs = np.stack([np.pad(p[l][1], ((0, 0), (0, max_p - p[l][1].shape[1]), (0, 0))) for p in pref])
        grouped.append((ks, vs))
    node_kv = {}  # node id -> per-layer (k [H, d], v [H, d]) from the oracle
    keys = ("turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id")
    max_dl = max_dv = 0.0
    agree = total = 0
    for r, K in enumerate(rounds):
        tok = synth.random_tokens(rng, G * K, dims)
        legal = [synth.random_legal_ids(rng, int(rng.integers(20, 41)), dims.vocab) for _ in range(G * K)]
        reqs, nodes, parents = [], [], []
        for g in range(G):
            rows = []
            for a in range(K):
                i = g * K + a
                nid = 1000 * g + 100 * r + a
                pid = None if r == 0 else 1000 * g + 100 * (r - 1) + a
                bs = {"piece_ids": tok["piece_ids"][i].tolist(), **{k: int(tok[k][i]) for k in keys}}
                rows.append(WaveRow(node_id=nid, parent_id=pid, prev_move_vocab_id=int(tok["prev_move_id"][i]),
                                    board_state=bs, legal_vocab_ids=legal[i].tolist()))
                nodes.append(nid)
                parents.append(pid)
            reqs.append(WaveRequest(worker_id=g, turn_id=0, rows=rows))
        resp = server.service(reqs)
        got = [row for wr in resp for row in wr.rows]
        gi = np.repeat(np.arange(G), K)
        kw = {}
        if r > 0:
            chains = []
            for pid in parents:
                ch, p = [], pid
                while p is not None:  # the arm's nodes of rounds 0 .. r - 1
                    ch.append(p)
                    p = p - 100 if (p % 1000) >= 100 else None
                chains.append(ch[::-1])
            sk = [np.stack([np.stack([node_kv[n][l][0] for n in ch], axis=1) for ch in chains]) for l in range(dims.num_layers)]
            sv = [np.stack([np.stack([node_kv[n][l][1] for n in ch], axis=1) for ch in chains]) for l in range(dims.num_layers)]
            kw = dict(suffix_kv=list(zip(sk, sv)),
                      suffix_positions=np.asarray(lens)[gi][:, None] + np.arange(r)[None, :],
                      suffix_mask=np.ones((G * K, r), dtype=bool))
        ref = orc.forward_decode_grouped(new_token_batch=tok, positions=np.asarray(lens)[gi] + r, group_index=gi,
                                         prefix_kv_grouped=grouped, prefix_lens_list=lens, **kw)
        for i, nid in enumerate(nodes):
            node_kv[nid] = [(ref["kv"][l][0][i, :, 0], ref["kv"][l][1][i, :, 0]) for l in range(dims.num_layers)]
        ref_v = value_stm(ref["value_logits"])
        for i in range(G * K):
            v_got, ll_got = got[i]
            ll_ref = ref["logits"][i, legal[i]]
            max_dl = max(max_dl, float(np.abs(np.asarray(ll_got) - ll_ref).max()))
            max_dv = max(max_dv, abs(v_got - float(ref_v[i])))
            agree += int(np.argmax(ll_got) == np.argmax(ll_ref))
            total += 1
    assert max_dl <= BF16_ATOL, max_dl
    assert max_dv <= BF16_DV, max_dv
    assert agree / total >= BF16_TOP1, agree / total
