"""``ActorInferenceServer`` on the B200 library: the reference server's
``service()`` contract (src/imba_chess/eval/actor_server.py:408-925) with
every prefix and every search node's KV resident in one paged device pool.

What changes relative to the reference, and what does not:

* Root requests (full and incremental) of one ``service()`` call run as ONE
  jagged prefill step per form: every game's tokens are appended in place to
  that game's pool sequence (no ``torch.cat`` of the whole prefix per token,
  actor_server.py:749-781).
* A wave of decode requests is ONE grouped step: each request's rows form a
  group over its turn's root prefix (read in place, never padded and
  stacked, merged_executors.py:187-196); each row's suffix is its parent
  chain read straight from the turn's arena pages, plus itself.
* Logical bookkeeping is the reference's: per-turn arena rows are minted
  consecutively in wave order (``_KVArena.append``), ``node_chains[child] =
  chain(parent) + [own_row]``, positions are ``prefix_len + depth``, a turn's
  prefix is a snapshot of its game's prefix at root time.
* Error conventions are the reference's: ``TypeError`` for unsupported
  request types, ``KeyError`` for an unknown turn/game/parent node,
  ``RuntimeError`` for prefix desync or max-position overflow, ``ValueError``
  for empty incremental requests or a model without a value head.
"""

from __future__ import annotations

import gc
import time
from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch

from . import _hostpath, _native
from .kvpool import PAGE, KVPool, KVSequence
from .model import B200HSTUChessModel
from .plan import StepBuffers, StepPlan
from .steps import root_plan, wave_plan_flat
from .protocol import RootEvalResponse, WaveResponse, is_root_request, is_wave_request
from .synth import EVENT_TOKEN_ID, TOKEN_FIELDS

_TOKEN_FIELDS = TOKEN_FIELDS
_NO_PARENT = -(2**63)  # parent id the host path reports for parent_id None


@dataclass
class _GameState:
    """A worker's current game: its prefix sequence and length."""

    seq: KVSequence
    prefix_len: int


@dataclass
class _TurnState:
    """One live (worker_id, turn_id): a snapshot (sequence, length) of the
    game prefix at root time, the turn's node arena and node chains."""

    seq: KVSequence
    prefix_len: int
    arena: KVSequence | None = None
    node_chains: dict[int, list[int]] = field(default_factory=dict)

    def release(self) -> None:
        self.seq.release()
        if self.arena is not None:
            self.arena.release()
            self.arena = None


class ActorInferenceServer:
    """Owns the model and every worker's KV state, keyed like the reference:
    ``(worker_id, turn_id)`` for a turn's search tree, ``worker_id`` for the
    worker's current game prefix."""

    def __init__(self, *, model, device: torch.device | str, dtype: torch.dtype, require_value_head: bool = True,
                 profile_sync: bool = False, kv_pool_pages: int | None = None,
                 kv_pool_bytes: int | None = None) -> None:
        device = torch.device(device)
        if not isinstance(model, B200HSTUChessModel):
            model_dtype = torch.float32 if dtype == torch.float32 else torch.bfloat16
            model = B200HSTUChessModel.from_reference(model, dtype=model_dtype, device=device)
        if require_value_head and getattr(model, "value_head", None) is None:
            raise ValueError(
                "ActorInferenceServer(require_value_head=True) requires a model with an enabled value head: "
                "every response row carries value_stm. Pass require_value_head=False to serve a "
                "value-head-less model (value_stm is then a 0.0 placeholder)."
            )
        self._model = model
        self._device = model.device
        self._dtype = dtype
        self.profile_sync = bool(profile_sync)
        # waves of at least this many rows run as two overlapped steps
        self.split_rows = 2048
        self.stats: dict[str, float] = {
            "root_build_s": 0.0, "root_gpu_s": 0.0, "root_post_s": 0.0,
            "wave_build_s": 0.0, "wave_gpu_s": 0.0, "wave_post_s": 0.0,
            "root_calls": 0, "root_reqs": 0,
            "wave_calls": 0, "wave_reqs": 0, "wave_rows": 0,
            "incremental_root_gpu_s": 0.0,
            "incremental_root_calls": 0, "incremental_root_reqs": 0,
            "incremental_root_tokens": 0,
        }
        if kv_pool_pages is None:
            page_bytes = self._page_bytes()
            budget = kv_pool_bytes
            if budget is None:
                free, _total = torch.cuda.mem_get_info(self._device)
                budget = min(int(free * 0.25), 8 << 30)
            kv_pool_pages = max(64, budget // page_bytes)
        self.pool: KVPool = model.new_pool(int(kv_pool_pages))
        self._turns: dict[tuple[int, int], _TurnState] = {}
        self._games: dict[int, _GameState] = {}
        self._status = torch.zeros(1, dtype=torch.int32, device=self._device)
        # pinned / device step buffers reused by every call (two: a large wave
        # runs as two steps in flight at once)
        self._buffers = StepBuffers(self._device)
        self._buffers2 = StepBuffers(self._device)

    def _page_bytes(self) -> int:
        d = self._model.dims
        esize = 2 if self._model.dtype == torch.bfloat16 else 4
        return d.num_layers * d.num_heads * PAGE * (d.attention_dim + d.linear_dim) * esize

    # ------------------------------------------------------------------
    def register_root(self, worker_id: int, turn_id: int, batch_arrays: dict, legal_vocab_ids: list[int]):
        from .protocol import RootEvalRequest

        req = RootEvalRequest(worker_id=int(worker_id), turn_id=int(turn_id), batch_arrays=batch_arrays,
                              legal_vocab_ids=list(legal_vocab_ids))
        return self._service_roots([req])[0]

    def service(self, requests: list) -> list:
        """Responses in the order of ``requests`` (roots run before waves)."""
        responses: list[Any] = [None] * len(requests)
        root_pos = [i for i, r in enumerate(requests) if is_root_request(r)]
        wave_pos = [i for i, r in enumerate(requests) if is_wave_request(r)]
        if len(root_pos) + len(wave_pos) != len(requests):
            bad = sorted({type(r).__name__ for r in requests if not (is_root_request(r) or is_wave_request(r))})
            raise TypeError(f"ActorInferenceServer.service() got unsupported request type(s): {bad}")
        if root_pos:
            for i, resp in zip(root_pos, self._service_roots([requests[i] for i in root_pos])):
                responses[i] = resp
        if wave_pos:
            for i, resp in zip(wave_pos, self._service_waves([requests[i] for i in wave_pos])):
                responses[i] = resp
        return responses

    def release_turn(self, worker_id: int, turn_id: int) -> None:
        ts = self._turns.pop((int(worker_id), int(turn_id)), None)
        if ts is not None:
            ts.release()

    def release_game(self, worker_id: int) -> None:
        gs = self._games.pop(int(worker_id), None)
        if gs is not None:
            gs.seq.release()

    def _sync_if_profiling(self) -> None:
        if self.profile_sync:
            torch.cuda.synchronize(self._device)

    # ------------------------------------------------------------------
    def _set_turn(self, key: tuple[int, int], game: _GameState) -> None:
        old = self._turns.pop(key, None)
        if old is not None:
            old.release()
        self._turns[key] = _TurnState(seq=game.seq.retain(), prefix_len=game.prefix_len)

    def _launch(self, plan: StepPlan, buffers: StepBuffers):
        """Enqueue one step (its packed plan copied in, its value and legal
        logits and the status word copied out) on the current stream; returns
        a handle for ``_collect``."""
        R = plan.num_rows
        nl = 0 if plan.legal_ids is None else int(plan.legal_ids.shape[0])
        stream = torch.cuda.current_stream(self._device)
        dstep = buffers.stage(plan, stream)
        out, host = buffers.outputs(R + nl + 1)
        self._status.zero_()
        self._model.run(dstep, self.pool, value_stm=out[:R], legal_logits=out[R : R + nl],
                        status=self._status, stream=stream)
        out[R + nl :].copy_(self._status.view(torch.float32))  # before the next step clears it
        host.copy_(out, non_blocking=True)
        done = torch.cuda.Event()
        done.record(stream)
        return done, host, R, nl

    @staticmethod
    def _collect(handle):
        """Wait for a launched step; (value_stm [R], legal_logits flat)."""
        done, host, R, nl = handle
        done.synchronize()
        arr = host.numpy()
        status = int(arr[R + nl :].view(np.int32)[0])
        if status != _native.IMBA_OK:
            raise _native.ImbaError(status, "device-side check")
        return arr[:R].copy(), arr[R : R + nl].copy()

    def _run_rows(self, plan: StepPlan, n_legal_rows: int):
        """Run one step and bring back (value_stm [R], legal_logits flat)."""
        v, ll = self._collect(self._launch(plan, self._buffers))
        return v, ll, None

    def _service_roots(self, requests: list) -> list:
        if not requests:
            return []
        full = [i for i, r in enumerate(requests) if r.batch_arrays is not None]
        inc = [i for i, r in enumerate(requests) if r.incremental_tokens is not None]
        responses: list[Any] = [None] * len(requests)
        if full:
            for i, resp in zip(full, self._service_full_roots([requests[i] for i in full])):
                responses[i] = resp
        if inc:
            for i, resp in zip(inc, self._service_incremental_roots([requests[i] for i in inc])):
                responses[i] = resp
        return responses

    def _root_step(self, seqs: list[KVSequence], tokens: list[dict], legal: list[list[int]]):
        """One step appending ``tokens[g]`` to ``seqs[g]`` (causal within the
        new tokens).  Value and legal logits come from each group's last token."""
        plan, last = root_plan(seqs, tokens, legal)
        value_stm, legal_flat, _ = self._run_rows(plan, len(seqs))
        loff = plan.legal_off
        return [
            (float(value_stm[i]), legal_flat[int(loff[i]) : int(loff[i + 1])].tolist()) for i in last
        ]

    def _service_full_roots(self, requests: list) -> list:
        t0 = time.perf_counter()
        seqs, tokens, legal = [], [], []
        for r in requests:
            ba = r.batch_arrays
            offs = list(ba["seq_offsets"])
            if len(offs) != 2:
                raise ValueError("a full RootEvalRequest must carry exactly one game (seq_offsets [0, T])")
            T = int(ba["total_tokens"])
            if T < 1:
                raise ValueError("a full RootEvalRequest must carry at least one token")
            tokens.append({k: ba[k] for k in _TOKEN_FIELDS})
            seqs.append(KVSequence(self.pool))
            legal.append(list(r.legal_vocab_ids))
        self._sync_if_profiling()
        t1 = time.perf_counter()
        try:
            outs = self._root_step(seqs, tokens, legal)
        except BaseException:
            for s in seqs:
                s.release()
            raise
        t2 = time.perf_counter()
        self.stats["root_build_s"] += t1 - t0
        self.stats["root_gpu_s"] += t2 - t1
        self.stats["root_calls"] += 1
        self.stats["root_reqs"] += len(requests)
        responses = []
        for r, seq, (v, ll) in zip(requests, seqs, outs):
            w = int(r.worker_id)
            old = self._games.pop(w, None)
            if old is not None:
                old.seq.release()
            game = _GameState(seq=seq, prefix_len=seq.length)
            self._games[w] = game
            self._set_turn((w, int(r.turn_id)), game)
            responses.append(RootEvalResponse(turn_id=r.turn_id, value_stm=v, legal_logits=ll))
        self.stats["root_post_s"] += time.perf_counter() - t2
        return responses

    def _service_incremental_roots(self, requests: list) -> list:
        max_pos = int(self._model.position_embedding.max_seq_len)
        seen = set()
        for r in requests:
            w = int(r.worker_id)
            game = self._games.get(w)
            if game is None:
                raise KeyError(
                    f"RootEvalRequest(incremental) for worker={w} has no persisted game prefix -- "
                    "missing/out-of-order full RootEvalRequest, or release_game() already freed it."
                )
            if w in seen:
                raise RuntimeError(f"worker={w}: two incremental root extensions in one service() call")
            seen.add(w)
            if int(r.prefix_len_before) != game.prefix_len:
                raise RuntimeError(
                    f"worker={w}: incremental RootEvalRequest expected prefix_len_before={r.prefix_len_before}, "
                    f"server has {game.prefix_len} -- worker/server prefix desync."
                )
            n_new = len(r.incremental_tokens["piece_ids"])
            if n_new < 1:
                raise ValueError(f"worker={w}: incremental RootEvalRequest carries zero new tokens.")
            if game.prefix_len + n_new > max_pos:
                raise RuntimeError(
                    f"worker={w}: incremental root extension would grow the persisted prefix to "
                    f"{game.prefix_len + n_new} tokens, past this model's max_position_embeddings={max_pos}."
                )
        t0 = time.perf_counter()
        games = [self._games[int(r.worker_id)] for r in requests]
        for g in games:
            if g.seq.length != g.prefix_len:
                raise RuntimeError("game prefix sequence and recorded prefix length disagree")
        outs = self._root_step([g.seq for g in games],
                               [{k: r.incremental_tokens[k] for k in _TOKEN_FIELDS} for r in requests],
                               [list(r.legal_vocab_ids) for r in requests])
        self._sync_if_profiling()
        self.stats["incremental_root_gpu_s"] += time.perf_counter() - t0
        self.stats["incremental_root_calls"] += len(requests)
        self.stats["incremental_root_reqs"] += len(requests)
        responses = []
        for r, game, (v, ll) in zip(requests, games, outs):
            n_new = len(r.incremental_tokens["piece_ids"])
            self.stats["incremental_root_tokens"] += n_new
            game.prefix_len += n_new
            self._set_turn((int(r.worker_id), int(r.turn_id)), game)
            responses.append(RootEvalResponse(turn_id=r.turn_id, value_stm=v, legal_logits=ll))
        return responses

    # ------------------------------------------------------------------
    def _service_waves(self, requests: list) -> list:
        if not requests:
            return []
        # A wave allocates ~R lists and ~R x n_legal floats for its responses;
        # the cyclic collector is paused meanwhile (none of them form cycles).
        paused = gc.isenabled()
        if paused:
            gc.disable()
        try:
            return self._service_waves_impl(requests)
        finally:
            if paused:
                gc.enable()

    def _service_waves_impl(self, requests: list) -> list:
        turns: list[_TurnState] = []
        for req in requests:
            key = (int(req.worker_id), int(req.turn_id))
            turn = self._turns.get(key)
            if turn is None:
                raise KeyError(
                    f"WaveRequest for worker={req.worker_id} turn={req.turn_id} has no registered root eval -- "
                    "missing/out-of-order RootEvalRequest, or release_turn() already freed this turn."
                )
            turns.append(turn)
        counts = [len(req.rows) for req in requests]
        R = sum(counts)
        # A large wave runs as two steps over consecutive request ranges (rows
        # keep their order, so arena rows are minted exactly as for one step):
        # the second part is packed and planned while the GPU runs the first,
        # and the first part's responses are built while the GPU runs the second.
        if R >= self.split_rows and len(requests) >= 2:
            csum = np.cumsum(counts)
            cut = int(np.searchsorted(csum, R / 2)) + 1
            cut = min(max(cut, 1), len(requests) - 1)
            parts = [(0, cut), (cut, len(requests))]
        else:
            parts = [(0, len(requests))]
        for turn in turns:
            if turn.arena is None:
                turn.arena = KVSequence(self.pool)
        # The reference appends a wave's rows to the arena only after its
        # forward succeeded (actor_server.py:904-914); a failed wave is rolled
        # back so later waves mint the same row ids.
        marks = [(t.arena, t.arena.length, len(t.arena.pages)) for t in turns]
        launched = []
        t_build = t_gpu = 0.0
        try:
            for (a, b), bufs in zip(parts, (self._buffers, self._buffers2)):
                t0 = time.perf_counter()
                launched.append((a, b) + self._plan_part(requests[a:b], turns[a:b], counts[a:b], bufs))
                t_build += time.perf_counter() - t0
            self._sync_if_profiling()
            responses: list = []
            t_post = 0.0
            for a, b, handle, loff, starts, node_b, parent_b in launched:
                t1 = time.perf_counter()
                value_stm, legal_flat = self._collect(handle)
                t2 = time.perf_counter()
                t_gpu += t2 - t1
                rows_out = _hostpath.wave_responses(counts[a:b], value_stm, legal_flat, loff)
                responses.extend(WaveResponse(rows=rows_g) for rows_g in rows_out)
                t_post += time.perf_counter() - t2
        except BaseException:
            for h in launched:  # nothing of this wave may still be running when the arenas shrink
                h[2][0].synchronize()
            for arena, length, npages in reversed(marks):
                arena.truncate(length, npages)
            raise
        t3 = time.perf_counter()
        # node_chains[child] = chain(parent) + [own arena row], in wave order
        for a, b, handle, loff, starts, node_b, parent_b in launched:
            _hostpath.record_chains([t.node_chains for t in turns[a:b]], counts[a:b], node_b, parent_b,
                                    starts.tobytes())
        self._sync_if_profiling()
        self.stats["wave_build_s"] += t_build
        self.stats["wave_gpu_s"] += t_gpu
        self.stats["wave_post_s"] += t_post + time.perf_counter() - t3
        self.stats["wave_calls"] += 1
        self.stats["wave_reqs"] += len(requests)
        self.stats["wave_rows"] += R
        return responses

    def _plan_part(self, requests: list, turns: list, counts: list, buffers: StepBuffers):
        """Pack, plan and launch one consecutive range of a wave's requests;
        returns (step handle, legal offsets, first arena row per request,
        node ids, parent ids)."""
        R = sum(counts)
        piece = np.empty((R, 64), dtype=np.uint8)
        side = np.empty((R, 7), dtype=np.int32)
        # Rows in request order, packed by the C++ host path (ids, boards,
        # legal CSR, node / parent ids) in one pass over the wire objects.
        _, loff_b, lids_b, node_b, parent_b = _hostpath.pack_wave_rows(requests, piece, side)
        side[:, 0] = EVENT_TOKEN_ID
        # Parent chains (arena rows of each row's turn) looked up before the
        # wave, as the reference builds its suffix index (actor_server.py:839-850).
        depth_b, chain_b = _hostpath.wave_chains([t.node_chains for t in turns], counts, parent_b)
        plan, starts = wave_plan_flat(
            [t.seq for t in turns], [t.prefix_len for t in turns], [t.arena for t in turns], counts,
            np.frombuffer(depth_b, dtype=np.int64), np.frombuffer(chain_b, dtype=np.int64), piece, side,
            (np.frombuffer(loff_b, dtype=np.int32), np.frombuffer(lids_b, dtype=np.int32)))
        handle = self._launch(plan, buffers)
        return handle, plan.legal_off, starts, node_b, parent_b
