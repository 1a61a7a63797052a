"""GPU: kernel-level cross-checks on identical inputs.

Each tensor-core kernel of the bf16 model against the SIMT kernel of the same
component (the handle's SIMT test hook, ``B200HSTUChessModel(simt=...)``), on
a full grouped-decode step: final hidden state, logits, value logits.

* gemm  - tcgen05/TMA GEMMs vs SIMT GEMMs: the same bf16 operands, fp32
          accumulation (the policy GEMM is exact fp32 in SIMT and split bf16 on
          the tensor cores; the uvqk epilogue's SiLU uses the hardware tanh);
* attn  - mma.sync paged attention (TMA-loaded KV pages) vs the SIMT
          attention and the separate gate pass (the tensor-core kernel rounds
          softmax weights to bf16 for P.V); the second wave's rows carry suffix
          chains, so several gathered extra-key tiles per CTA are covered;
* board - the board encoder (tcgen05 projections from TMEM in the mma.sync
          fragment layout, mma.sync attention; bf16 operands) vs the fp32
          SIMT encoder.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from imba_chess_b200 import synth
from imba_chess_b200.kvpool import KVSequence
from imba_chess_b200.model import B200HSTUChessModel
from imba_chess_b200.plan import DeviceStep, piece_ids_from_tokens, side_ids_from_tokens
from imba_chess_b200.steps import WaveGroup, root_plan, wave_plan

pytestmark = pytest.mark.gpu

# (hidden relative to its max magnitude, logits abs, value logits abs).  The
# tensor-core uvqk epilogue computes SiLU through the hardware tanh (relative
# error ~2^-11) where the SIMT epilogue uses the exact exponential form, so
# the gemm bounds cover that as well as accumulation order.
TOL = {"gemm": (2e-4, 5e-3, 2e-3), "attn": (2e-3, 2e-2, 5e-3), "board": (2e-3, 3e-2, 1e-2)}


def _run_wave(model, dims, wave, depth2=True):
    pool = model.new_pool(4096)
    seqs = [KVSequence(pool) for _ in wave.prefix_lens]
    plan0, _ = root_plan(seqs, wave.prefix_tokens)
    model.run(DeviceStep(plan0, model.device), pool)
    order = np.argsort(wave.group_index, kind="stable")
    counts = np.bincount(wave.group_index, minlength=len(seqs))
    arenas = [KVSequence(pool) for _ in seqs]
    tok = synth.slice_tokens(wave.row_tokens, order)
    groups = [WaveGroup(seqs[g], wave.prefix_lens[g], arenas[g], [[]] * int(counts[g])) for g in range(len(seqs))]
    plan, rows = wave_plan(groups, piece_ids_from_tokens(tok), side_ids_from_tokens(tok),
                           [wave.legal_ids[i] for i in order])
    model.run(DeviceStep(plan, model.device), pool)
    if depth2:  # a second wave whose rows have one-token suffix chains
        rng = np.random.default_rng(3)
        tok2 = synth.random_tokens(rng, plan.num_rows, dims)
        groups2 = [WaveGroup(seqs[g], wave.prefix_lens[g], arenas[g], [[r] for r in rows[g]])
                   for g in range(len(seqs))]
        plan, _ = wave_plan(groups2, piece_ids_from_tokens(tok2), side_ids_from_tokens(tok2),
                            [wave.legal_ids[i] for i in order])
    R = plan.num_rows
    out = {
        "logits": torch.empty((R, dims.vocab), device=model.device),
        "value_logits": torch.empty((R, 3), device=model.device),
        "hidden": torch.empty((R, dims.model_dim), device=model.device),
    }
    model.run(DeviceStep(plan, model.device), pool, **out)
    torch.cuda.synchronize()
    model.check_status()
    return out


@pytest.mark.parametrize("component", ["gemm", "attn", "board"])
@pytest.mark.parametrize("dims,parents", [(synth.D512, 6), (synth.SMALL, 4), (synth.D256, 5), (synth.D1024, 2)],
                         ids=["d512", "d128", "d256", "d1024"])
def test_tensor_core_kernel_matches_simt(component, dims, parents):
    sd = synth.make_state_dict(dims, 9, profile="reference")
    plies = (20, 140) if component == "attn" else (20, 45)
    wave = synth.grouped_wave(dims, n_parents=parents, plies=plies, siblings=(20, 40), seed=99)
    model_tc = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    model_simt = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0", simt=(component,))
    a = _run_wave(model_tc, dims, wave)
    b = _run_wave(model_simt, dims, wave)
    th, tl, tv = TOL[component]
    scale = float(b["hidden"].abs().max())
    assert torch.isfinite(a["logits"]).all()
    assert float((a["hidden"] - b["hidden"]).abs().max()) <= th * scale
    assert float((a["logits"] - b["logits"]).abs().max()) <= tl
    assert float((a["value_logits"] - b["value_logits"]).abs().max()) <= tv


def test_attention_result_independent_of_chunking():
    """The C ABI accepts chunks of up to 64 rows; the planner emits <= 32-row
    chunks (one attention work item) for decode steps and 64-row chunks for
    prefills.  Re-chunking the same steps into 32-, 64- and 16-row chunks
    must give bit-identical results (each row's attention depends only on its
    own keys; a 64-row chunk is processed as two decode items or one prefill
    unit)."""
    from imba_chess_b200.plan import build_chunks

    dims = synth.D256
    sd = synth.make_state_dict(dims, 5, profile="reference")
    # groups of 30-60 siblings, so 64-row chunks hold two work items
    wave = synth.grouped_wave(dims, n_parents=4, plies=(20, 140), siblings=(30, 60), seed=17)
    outs = []
    for max_rows in (32, 64, 16):
        model = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
        orig = build_chunks

        def rechunk(row_group, num_groups, max_rows=32, row_vis=None, _m=max_rows):  # noqa: ARG001
            return orig(row_group, num_groups, max_rows=_m, row_vis=row_vis)

        import imba_chess_b200.plan as plan_mod

        plan_mod.build_chunks = rechunk
        try:
            outs.append(_run_wave(model, dims, wave))
        finally:
            plan_mod.build_chunks = orig
    for o in outs[1:]:
        for k in ("hidden", "logits", "value_logits"):
            assert torch.equal(o[k], outs[0][k]), k


def test_attention_positions_past_max_pos():
    """Prefixes longer than max_pos: relative-bias indices clamp at both ends
    and the paged kernel leaves its fast path; TC attention vs SIMT."""
    dims = synth.ModelDims(256, 2, 4, max_pos=96)
    sd = synth.make_state_dict(dims, 21, profile="sharp")
    wave = synth.grouped_wave(dims, n_parents=3, plies=(100, 230), siblings=(20, 40), seed=23)
    model_tc = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    model_simt = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0", simt=("attn",))
    a = _run_wave(model_tc, dims, wave)
    b = _run_wave(model_simt, dims, wave)
    th, tl, tv = TOL["attn"]
    scale = float(b["hidden"].abs().max())
    assert torch.isfinite(a["logits"]).all()
    assert float((a["hidden"] - b["hidden"]).abs().max()) <= th * scale
    assert float((a["logits"] - b["logits"]).abs().max()) <= tl
    assert float((a["value_logits"] - b["value_logits"]).abs().max()) <= tv


def _prefill(model, dims, lens, seed):
    """One packed jagged prefill of documents of the given lengths: every
    row's hidden state, logits and value logits."""
    rng = np.random.default_rng(seed)
    tokens = [synth.random_tokens(rng, n, dims) for n in lens]
    pool = model.new_pool(sum(-(-n // 16) for n in lens) + 8)
    seqs = [KVSequence(pool) for _ in lens]
    plan, _ = root_plan(seqs, tokens)
    R = plan.num_rows
    out = {
        "logits": torch.empty((R, dims.vocab), device=model.device),
        "value_logits": torch.empty((R, 3), device=model.device),
        "hidden": torch.empty((R, dims.model_dim), device=model.device),
    }
    model.run(DeviceStep(plan, model.device), pool, **out)
    torch.cuda.synchronize()
    model.check_status()
    return out


@pytest.mark.parametrize(
    "dims,lens",
    [
        (synth.D512, [1, 2, 17, 31, 32, 33, 63, 64, 65, 130, 300]),
        (synth.SMALL, [5, 47, 48, 64, 100]),  # positions past max_pos 48: bias indices clamp
        (synth.ModelDims(256, 2, 4, max_pos=96), [230, 1, 96, 97, 64]),
        (synth.D1024, [40, 129, 7]),
    ],
    ids=["d512", "d128", "d256-maxpos96", "d1024"],
)
def test_prefill_attention_matches_simt(dims, lens):
    """The jagged prefill attention (tcgen05 S and P.V over 64-row chunks and
    head pairs, fp32 O and a separate norm / gate pass) against the SIMT
    attention on the same packed prefill: documents from one token to several
    pages, chunk and block boundaries on both sides, odd page counts."""
    sd = synth.make_state_dict(dims, 31, profile="reference")
    model_tc = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    model_simt = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0", simt=("attn",))
    a = _prefill(model_tc, dims, lens, 5)
    b = _prefill(model_simt, dims, lens, 5)
    th, tl, tv = TOL["attn"]
    scale = float(b["hidden"].abs().max())
    assert torch.isfinite(a["hidden"]).all() and torch.isfinite(a["logits"]).all()
    assert float((a["hidden"] - b["hidden"]).abs().max()) <= th * scale
    assert float((a["logits"] - b["logits"]).abs().max()) <= tl
    assert float((a["value_logits"] - b["value_logits"]).abs().max()) <= tv


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
@pytest.mark.parametrize("max_rows", [32, 64])
def test_legal_gather_matches_full_projection(dtype, max_rows):
    """Legal logits without the full projection (fp32 dot products of the
    final-LN output with the legal ids' fp32 policy rows) against the same
    entries of the full 1,970-way logits of the same step, and the log-probs
    against a float64 log-softmax of those.  Covers a row without legal ids,
    repeated ids within a row and 64-row chunks."""
    import imba_chess_b200.plan as plan_mod

    dims = synth.D256
    sd = synth.make_state_dict(dims, 13, profile="reference")
    wave = synth.grouped_wave(dims, n_parents=4, plies=(20, 80), siblings=(30, 60), seed=31)
    model = B200HSTUChessModel(sd, dtype=dtype, device="cuda:0")
    orig = plan_mod.build_chunks

    def rechunk(row_group, num_groups, max_rows_=32, row_vis=None, **kw):  # noqa: ARG001
        return orig(row_group, num_groups, max_rows=max_rows, row_vis=row_vis)

    plan_mod.build_chunks = rechunk
    try:
        pool = model.new_pool(4096)
        seqs = [KVSequence(pool) for _ in wave.prefix_lens]
        plan0, _ = root_plan(seqs, wave.prefix_tokens)
        model.run(DeviceStep(plan0, model.device), pool)
        order = np.argsort(wave.group_index, kind="stable")
        counts = np.bincount(wave.group_index, minlength=len(seqs))
        arenas = [KVSequence(pool) for _ in seqs]
        tok = synth.slice_tokens(wave.row_tokens, order)
        legal = [list(wave.legal_ids[i]) for i in order]
        legal[0] = []
        legal[1] = legal[1] + legal[1][:3]
        groups = [WaveGroup(seqs[g], wave.prefix_lens[g], arenas[g], [[]] * int(counts[g])) for g in range(len(seqs))]
        plan, _ = wave_plan(groups, piece_ids_from_tokens(tok), side_ids_from_tokens(tok), legal)
    finally:
        plan_mod.build_chunks = orig
    R, NL = plan.num_rows, int(plan.legal_ids.shape[0])
    dstep = DeviceStep(plan, model.device)
    full = torch.empty((R, dims.vocab), device=model.device)
    ll_a = torch.empty(NL, device=model.device)
    ll_b = torch.empty(NL, device=model.device)
    lp_b = torch.empty(NL, device=model.device)
    model.run(dstep, pool, logits=full, legal_logits=ll_a)
    model.run(dstep, pool, legal_logits=ll_b, legal_logprob=lp_b)
    torch.cuda.synchronize()
    model.check_status()
    off = plan.legal_off.astype(np.int64)
    ids = torch.as_tensor(plan.legal_ids.astype(np.int64), device=model.device)
    rows = torch.as_tensor(np.repeat(np.arange(R), np.diff(off)), device=model.device)
    ref = full[rows, ids]
    atol = 1e-4 if dtype == torch.float32 else 2e-3
    assert torch.equal(ll_a, ref)
    assert float((ll_b - ref).abs().max()) <= atol
    ll = ll_b.double().cpu().numpy()
    for r in range(R):
        a, b = int(off[r]), int(off[r + 1])
        if a == b:
            continue
        z = ll[a:b]
        lse = z.max() + np.log(np.exp(z - z.max()).sum())
        assert np.abs(lp_b[a:b].double().cpu().numpy() - (z - lse)).max() <= 1e-5


@pytest.mark.parametrize("dims", [synth.D512, synth.D1024], ids=["d512", "d1024"])
def test_small_group_steps_match_simt(dims):
    """Steps of one or two rows per group (one token per game): the paged
    attention's work items then hold a single live row block; it must match
    the SIMT attention (the handle's SIMT test hook) on the same steps, including the
    second wave's one-token suffix chains."""
    sd = synth.make_state_dict(dims, 19, profile="reference")
    wave = synth.grouped_wave(dims, n_parents=40 if dims is synth.D512 else 12, plies=(20, 140), siblings=(1, 2),
                              seed=41)
    assert wave.num_rows <= 2 * len(wave.prefix_lens)
    model_tc = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    model_simt = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0", simt=("attn",))
    a = _run_wave(model_tc, dims, wave)
    b = _run_wave(model_simt, dims, wave)
    th, tl, tv = TOL["attn"]
    scale = float(b["hidden"].abs().max())
    assert torch.isfinite(a["logits"]).all()
    assert float((a["hidden"] - b["hidden"]).abs().max()) <= th * scale
    assert float((a["logits"] - b["logits"]).abs().max()) <= tl
    assert float((a["value_logits"] - b["value_logits"]).abs().max()) <= tv
