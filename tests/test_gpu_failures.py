"""GPU: device-side failure paths, without faulting or hanging a GPU.

The reference fails fast and loudly on bad input (src/imba_chess/eval/
actor_server.py:815-822, tests/test_actor_server.py:395-413).  On the device
this library cannot raise; its kernels check every index before using it and
bound every wait, record the first error code in a status word and skip the
offending access.  These tests make each check fire and verify that the
error reaches the caller as ``ImbaError`` with the right code, and that the
next clean step on the same handle and pool is correct:

* an extra-key slot outside the pool and a visible-prefix length above its
  group's page capacity (IMBA_ERR_RANGE), on the bf16 tensor-core path of a
  decode wave and of a jagged prefill;
* a bounded wait that runs out (IMBA_ERR_TIMEOUT): the library's wait on an
  mbarrier nothing arrives at, with a 1 ms limit instead of the production
  2 s (``imba_selftest_wait_timeout``).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from imba_chess_b200 import _native, synth
from imba_chess_b200.kvpool import KVSequence
from imba_chess_b200.model import B200HSTUChessModel
from imba_chess_b200.plan import DeviceStep, piece_ids_from_tokens, side_ids_from_tokens
from imba_chess_b200.steps import WaveGroup, root_plan, wave_plan

pytestmark = pytest.mark.gpu


def _setup(dtype=torch.bfloat16):
    dims = synth.D256
    sd = synth.make_state_dict(dims, 8, profile="reference")
    model = B200HSTUChessModel(sd, dtype=dtype, device="cuda:0")
    wave = synth.grouped_wave(dims, n_parents=4, plies=(20, 60), siblings=(8, 20), seed=55)
    pool = model.new_pool(512)
    seqs = [KVSequence(pool) for _ in wave.prefix_lens]
    model.run(DeviceStep(root_plan(seqs, wave.prefix_tokens)[0], model.device), pool)
    order = np.argsort(wave.group_index, kind="stable")
    counts = np.bincount(wave.group_index, minlength=len(seqs))
    arenas = [KVSequence(pool) for _ in seqs]
    tok = synth.slice_tokens(wave.row_tokens, order)
    groups = [WaveGroup(seqs[g], wave.prefix_lens[g], arenas[g], [[]] * int(counts[g])) for g in range(len(seqs))]
    plan, rows = wave_plan(groups, piece_ids_from_tokens(tok), side_ids_from_tokens(tok),
                           [wave.legal_ids[i] for i in order])
    # a second wave whose rows carry one-key suffix chains (extra keys beyond themselves)
    rng = np.random.default_rng(2)
    tok2 = synth.random_tokens(rng, plan.num_rows, dims)
    groups2 = [WaveGroup(seqs[g], wave.prefix_lens[g], arenas[g], [[r] for r in rows[g]]) for g in range(len(seqs))]
    plan2, _ = wave_plan(groups2, piece_ids_from_tokens(tok2), side_ids_from_tokens(tok2),
                         [wave.legal_ids[i] for i in order])
    return model, pool, plan, plan2


def _run(model, pool, plan):
    R, NL = plan.num_rows, int(plan.legal_ids.shape[0])
    v = torch.empty(R, device=model.device)
    ll = torch.empty(NL, device=model.device)
    model.run(DeviceStep(plan, model.device), pool, value_stm=v, legal_logits=ll)
    torch.cuda.synchronize()
    return v, ll


def test_out_of_range_indices_raise_and_next_step_is_clean():
    model, pool, plan, plan2 = _setup()
    # clean results of the second wave (its own rows' KV slots are rewritten
    # with the same values by every run of the same plan)
    v_ok, ll_ok = _run(model, pool, plan2)
    model.check_status()
    for corrupt in ("extra_slot", "row_vis"):
        bad = DeviceStep(plan2, model.device)
        arr = plan2.extra_slot.copy() if corrupt == "extra_slot" else plan2.row_vis.copy()
        if corrupt == "extra_slot":
            first_chain = int(plan2.row_extra_off[0])  # row 0's chain key (its parent)
            arr[first_chain] = pool.num_pages * 16 + 5
        else:
            arr[0] = arr[0] + 64  # beyond the group's page capacity
        o, n = bad.layout[corrupt]
        bad.buf[o:o + n].copy_(torch.from_numpy(arr.astype(np.int32)))
        v = torch.empty(plan2.num_rows, device=model.device)
        ll = torch.empty(int(plan2.legal_ids.shape[0]), device=model.device)
        model.run(bad, pool, value_stm=v, legal_logits=ll)
        torch.cuda.synchronize()
        with pytest.raises(_native.ImbaError) as ei:
            model.check_status()
        assert ei.value.code == _native.IMBA_ERR_RANGE
        # check_status cleared the word; the same handle and pool run clean again
        v2, ll2 = _run(model, pool, plan2)
        model.check_status()
        assert torch.equal(v2, v_ok) and torch.equal(ll2, ll_ok)


def test_prefill_out_of_range_prefix_raises_and_next_step_is_clean():
    """The jagged prefill attention path: a visible-prefix length above its
    document's page capacity is reported (IMBA_ERR_RANGE) and clamped; a
    clean re-run of the same prefill on the same handle and pool is bit-exact
    with the first."""
    dims = synth.D256
    sd = synth.make_state_dict(dims, 8, profile="reference")
    model = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    rng = np.random.default_rng(6)
    lens = [70, 40, 33, 5]
    tokens = [synth.random_tokens(rng, n, dims) for n in lens]
    pool = model.new_pool(64)
    seqs = [KVSequence(pool) for _ in lens]
    plan, _ = root_plan(seqs, tokens)

    def run(step):
        out = torch.empty((plan.num_rows, dims.vocab), device=model.device)
        model.run(step, pool, logits=out)
        torch.cuda.synchronize()
        return out

    ok = run(DeviceStep(plan, model.device))
    model.check_status()
    bad = DeviceStep(plan, model.device)
    vis = plan.row_vis.copy()
    vis[3] = 16 * pool.num_pages  # beyond its document's pages (row 3 is in the first, 70-token document)
    o, n = bad.layout["row_vis"]
    bad.buf[o:o + n].copy_(torch.from_numpy(vis.astype(np.int32)))
    run(bad)
    with pytest.raises(_native.ImbaError) as ei:
        model.check_status()
    assert ei.value.code == _native.IMBA_ERR_RANGE
    again = run(DeviceStep(plan, model.device))
    model.check_status()
    assert torch.equal(again, ok)


def test_bounded_wait_times_out_with_status_and_context_survives():
    model, pool, plan, _ = _setup()
    lib = _native.load()
    status = torch.zeros(1, dtype=torch.int32, device=model.device)
    stream = torch.cuda.current_stream()
    assert lib.imba_selftest_wait_timeout(1_000_000, status.data_ptr(), stream.cuda_stream) == _native.IMBA_OK
    torch.cuda.synchronize()
    assert int(status.item()) == _native.IMBA_ERR_TIMEOUT
    # invalid limits are refused on the host, nothing launched
    assert lib.imba_selftest_wait_timeout(0, status.data_ptr(), stream.cuda_stream) == _native.IMBA_ERR_ARG
    assert lib.imba_selftest_wait_timeout(1000, None, stream.cuda_stream) == _native.IMBA_ERR_ARG
    # the context is usable: a step after the timeout runs clean
    v, ll = _run(model, pool, plan)
    model.check_status()
    assert torch.isfinite(v).all() and torch.isfinite(ll).all()


def test_server_maps_device_range_error_to_exception():
    """Through the server: a device-side range error surfaces from
    ``service()`` as ImbaError, and the following wave is served normally."""
    from imba_chess_b200.protocol import RootEvalRequest, WaveRequest, WaveRow
    from imba_chess_b200.server import ActorInferenceServer
    import imba_chess_b200.server as server_mod

    dims = synth.D256
    sd = synth.make_state_dict(dims, 8, profile="reference")
    model = B200HSTUChessModel(sd, dtype=torch.bfloat16, device="cuda:0")
    server = ActorInferenceServer(model=model, device="cuda:0", dtype=torch.bfloat16, kv_pool_pages=256)
    rng = np.random.default_rng(1)
    pt = synth.game_tokens(rng, 30, dims)
    T = int(pt["piece_ids"].shape[0])
    ba = {k: v.tolist() for k, v in pt.items()}
    ba.update(total_tokens=T, seq_offsets=[0, T])
    server.service([RootEvalRequest(worker_id=0, turn_id=0, legal_vocab_ids=[2], batch_arrays=ba)])
    tok = synth.random_tokens(rng, 6, dims)
    keys = ("turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id")

    def wave(base):
        return [WaveRequest(worker_id=0, turn_id=0, rows=[
            WaveRow(node_id=base + i, parent_id=None, prev_move_vocab_id=int(tok["prev_move_id"][i]),
                    board_state={"piece_ids": tok["piece_ids"][i].tolist(), **{k: int(tok[k][i]) for k in keys}},
                    legal_vocab_ids=[3, 7, 11]) for i in range(6)])]

    clean = server.service(wave(0))
    orig = server_mod.wave_plan_flat

    def corrupt(*a, **k):
        plan, starts = orig(*a, **k)
        plan.row_vis = plan.row_vis.copy()
        plan.row_vis[0] += 64  # past the prefix's pages
        return plan, starts

    server_mod.wave_plan_flat = corrupt
    try:
        with pytest.raises(_native.ImbaError) as ei:
            server.service(wave(100))
        assert ei.value.code == _native.IMBA_ERR_RANGE
    finally:
        server_mod.wave_plan_flat = orig
    again = server.service(wave(200))
    for (v0, l0), (v1, l1) in zip(clean[0].rows, again[0].rows):
        assert v0 == v1 and l0 == l1
    # the failed wave minted no arena rows: the next wave continues at row 6
    chains = server._turns[(0, 0)].node_chains
    assert [chains[200 + i] for i in range(6)] == [[6 + i] for i in range(6)]
    assert all(100 + i not in chains for i in range(6))
