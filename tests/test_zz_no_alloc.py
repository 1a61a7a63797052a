"""GPU: the allocation-free step entry point, ``imba_step_noalloc``.

Hosts that may not allocate GPU memory at decode time (a runtime whose
allocator owns all device memory, or an engine driver with a footprint fixed
at load time) cannot hand ``imba_step`` a workspace; they call
``imba_step_noalloc``, which runs the same step on a scratch array compiled
into the library.  This test calls it through the C ABI twice in a row, on two
different waves (the second one's rows are children of the first one's), and
checks every output against the regular ``imba_step`` on the same inputs, for
an fp32 model (SIMT kernels) and a bf16 model (tensor-core kernels, whose TMA
tensor maps then point into the library's scratch array).  Both entry points
run the same kernels, so the outputs must agree to within the fp32 parity
tolerance (max abs 1e-4; in practice bit for bit).  Before the compared calls
one allocation-free call runs on a larger, different wave, so the compared
calls start from another wave's leftover scratch contents.  It also checks
that a step too large for the fixed scratch is refused before anything is
launched.

This file is named so that pytest collects it last; it runs alone in a fresh
process as well as after the other tests.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from imba_chess_b200 import _native, synth
from imba_chess_b200.kvpool import KVSequence
from imba_chess_b200.model import B200HSTUChessModel
from imba_chess_b200.plan import DeviceStep, piece_ids_from_tokens, side_ids_from_tokens
from imba_chess_b200.steps import WaveGroup, root_plan, wave_plan

pytestmark = pytest.mark.gpu

ATOL = 1e-4


def _outputs(model, R, NL):
    dev = model.device
    return {
        "logits": torch.full((R, model.dims.vocab), float("nan"), device=dev),
        "value_logits": torch.full((R, 3), float("nan"), device=dev),
        "value_stm": torch.full((R,), float("nan"), device=dev),
        "legal_logits": torch.full((NL,), float("nan"), device=dev),
        "legal_logprob": torch.full((NL,), float("nan"), device=dev),
    }


def _fill(desc, outs, status):
    for k, t in outs.items():
        setattr(desc, k, t.data_ptr())
    desc.hidden = None
    desc.status = status.data_ptr()


def _waves(model, dims, pool, seed):
    """A prefill of three parents, then wave A (depth-0 siblings) and wave B
    (one child per wave-A row, whose suffix chain is its wave-A parent)."""
    wave = synth.grouped_wave(dims, n_parents=3, plies=(5, 30), siblings=(4, 9), seed=seed)
    seqs = [KVSequence(pool) for _ in wave.prefix_lens]
    plan0, _ = root_plan(seqs, wave.prefix_tokens)
    model.run(DeviceStep(plan0, model.device), pool)
    order = np.argsort(wave.group_index, kind="stable")
    counts = np.bincount(wave.group_index, minlength=len(seqs))
    arenas = [KVSequence(pool) for _ in seqs]
    tok_a = synth.slice_tokens(wave.row_tokens, order)
    groups_a = [WaveGroup(seqs[g], wave.prefix_lens[g], arenas[g], [[]] * int(counts[g])) for g in range(len(seqs))]
    plan_a, rows_a = wave_plan(groups_a, piece_ids_from_tokens(tok_a), side_ids_from_tokens(tok_a),
                               [wave.legal_ids[i] for i in order])
    rng = np.random.default_rng(seed + 1)
    tok_b = synth.random_tokens(rng, plan_a.num_rows, dims)
    groups_b = [WaveGroup(seqs[g], wave.prefix_lens[g], arenas[g], [[r] for r in rows_a[g]]) for g in range(len(seqs))]
    legal_b = [synth.random_legal_ids(rng, int(rng.integers(1, 30)), dims.vocab) for _ in range(plan_a.num_rows)]
    plan_b, _ = wave_plan(groups_b, piece_ids_from_tokens(tok_b), side_ids_from_tokens(tok_b), legal_b)
    return plan_a, plan_b


@pytest.mark.parametrize("dims,dtype", [(synth.SMALL, torch.float32), (synth.D256, torch.bfloat16)],
                         ids=["fp32", "bf16"])
def test_noalloc_step_matches_workspace_step_twice(dims, dtype):
    sd = synth.make_state_dict(dims, 21, profile="sharp" if dtype == torch.float32 else "reference")
    model = B200HSTUChessModel(sd, dtype=dtype, device="cuda:0")
    lib = _native.load()
    stream = torch.cuda.current_stream()
    pool = model.new_pool(512)
    plan_a, plan_b = _waves(model, dims, pool, seed=77)

    status = torch.zeros(1, dtype=torch.int32, device=model.device)
    # A larger, unrelated wave first, so the compared calls below find its
    # leftover contents in the shared scratch array.
    big = synth.grouped_wave(dims, n_parents=4, plies=(20, 60), siblings=(20, 30), seed=5)
    big_seqs = [KVSequence(pool) for _ in big.prefix_lens]
    plan_big, _ = root_plan(big_seqs, big.prefix_tokens)
    assert plan_big.num_rows > max(plan_a.num_rows, plan_b.num_rows)
    ds_big = DeviceStep(plan_big, model.device)
    out_big = _outputs(model, plan_big.num_rows, 0)
    del out_big["legal_logits"], out_big["legal_logprob"]
    _fill(ds_big.desc, out_big, status)
    ds_big.desc.legal_logits = None
    ds_big.desc.legal_logprob = None
    assert int(lib.imba_step_workspace_bytes(model._handle, plan_big.num_rows)) <= _native.NOALLOC_SCRATCH_BYTES
    assert lib.imba_step_noalloc(model._handle, ctypes.byref(ds_big.desc), ctypes.byref(pool.desc),
                                 stream.cuda_stream) == _native.IMBA_OK

    steps = []
    for plan in (plan_a, plan_b):
        ds = DeviceStep(plan, model.device)
        R, NL = plan.num_rows, int(plan.legal_ids.shape[0])
        need = int(lib.imba_step_workspace_bytes(model._handle, R))
        assert need <= _native.NOALLOC_SCRATCH_BYTES
        steps.append((ds, _outputs(model, R, NL), _outputs(model, R, NL)))

    # Reference results through the workspace entry point.
    for ds, ref, _ in steps:
        _fill(ds.desc, ref, status)
        ws = model.workspace(ds.desc.num_rows)
        code = lib.imba_step(model._handle, ctypes.byref(ds.desc), ctypes.byref(pool.desc), ws.data_ptr(),
                             ws.numel(), stream.cuda_stream)
        assert code == _native.IMBA_OK
    # Two allocation-free calls in a row.
    for ds, _, got in steps:
        _fill(ds.desc, got, status)
        code = lib.imba_step_noalloc(model._handle, ctypes.byref(ds.desc), ctypes.byref(pool.desc),
                                     stream.cuda_stream)
        assert code == _native.IMBA_OK
    torch.cuda.synchronize()
    assert int(status.item()) == _native.IMBA_OK
    for _, ref, got in steps:
        for k in ref:
            assert torch.isfinite(got[k]).all(), k
            assert float((got[k] - ref[k]).abs().max()) <= ATOL, k


def test_noalloc_step_refuses_more_rows_than_its_scratch():
    dims = synth.SMALL
    sd = synth.make_state_dict(dims, 21, profile="sharp")
    model = B200HSTUChessModel(sd, dtype=torch.float32, device="cuda:0")
    lib = _native.load()
    cap = _native.NOALLOC_SCRATCH_BYTES

    def fits(rows: int) -> bool:
        return int(lib.imba_step_workspace_bytes(model._handle, rows)) <= cap

    lo, hi = 1, cap  # largest row count whose workspace fits the fixed scratch
    while lo < hi:
        mid = (lo + hi + 1) // 2
        lo, hi = (mid, hi) if fits(mid) else (lo, mid - 1)
    assert fits(lo) and not fits(lo + 1)
    pool = _native.PoolDesc(None, 0)
    for rows in (lo + 1, cap):
        desc = _native.StepDesc()  # null pointers: a launch would be refused with IMBA_ERR_ARG instead
        desc.num_rows = rows
        code = lib.imba_step_noalloc(model._handle, ctypes.byref(desc), ctypes.byref(pool), None)
        assert code == _native.IMBA_ERR_OOM
