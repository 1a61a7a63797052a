"""Paged executors for the rollout scheduler's merged calls.

The reference's in-process G-game path (``BatchScheduler`` ->
``_make_root_eval_executor`` / ``_make_decode_wave_executor``,
src/imba_chess/eval/merged_executors.py:124-135, :300-346, called from
src/imba_chess/eval/batch_scheduler.py:96-100) merges every live game's
request of one tick into one model call.  Its decode wave pads every game's
prefix KV to the tick's longest and stacks them (``_merge_decode_requests``,
merged_executors.py:151-276) on every call, and its root eval slices each
game's KV back out of the merged prefill (``_split_root_output``, :97-121).

These executors take the same list-of-payloads -> list-of-results shape but
keep every game's KV in place in the model's paged pool:

* ``make_root_eval_executor``: each payload is one game's token prefix; one
  jagged prefill step appends every game's tokens to a fresh pool sequence
  (its ``PagedGame``), returning the last token's value and legal logits.
* ``make_decode_wave_executor``: each payload is one game's
  ``PagedDecodeRequest`` (its rows: tokens, parent chains in the game's
  node arena, legal ids); one grouped step decodes every game's rows against
  its prefix sequence in place (no padding, no stacking, no copy), appends the
  rows' KV to the game's arena and returns each row's value and legal logits
  plus the arena rows it minted (the reference's node chains extend with
  them, merged_executors.py / actor_server.py:904-914).

Everything runs through the C ABI; there is no CPU path.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from itertools import chain
from typing import Any

import numpy as np
import torch

from . import _native
from .kvpool import KVPool, KVSequence
from .plan import StepBuffers, piece_ids_from_tokens, side_ids_from_tokens
from .steps import ids_csr, root_plan, wave_plan_flat


@dataclass
class PagedGame:
    """One game's KV in the pool: its prefix (root) sequence and length, and
    the node arena of its current search turn."""

    prefix: KVSequence
    prefix_len: int
    arena: KVSequence

    def release(self) -> None:
        self.prefix.release()
        self.arena.release()


@dataclass
class PagedDecodeRequest:
    """One game's rows of a decode wave: ``tokens`` holds the token fields
    (``piece_ids`` [n, 64] and the seven side fields [n]); ``parent_rows[i]``
    is row i's parent chain as arena rows (root -> parent; empty for a child
    of the root); ``legal_ids[i]`` are its legal move ids in the order their
    logits are returned."""

    game: PagedGame
    tokens: dict
    parent_rows: list
    legal_ids: list = field(default_factory=list)


class LegalLogits:
    """One game's rows' legal logits as a sequence: item ``i`` is row i's
    float32 logits at its legal ids (a view into the wave's flat result),
    made when it is read."""

    __slots__ = ("_flat", "_off")

    def __init__(self, flat: np.ndarray, off: np.ndarray) -> None:
        self._flat = flat
        self._off = off

    def __len__(self) -> int:
        return len(self._off) - 1

    def __getitem__(self, i: int) -> np.ndarray:
        n = len(self._off) - 1
        if i < 0:
            i += n
        if not 0 <= i < n:
            raise IndexError("row index out of range")
        return self._flat[self._off[i] : self._off[i + 1]]

    def __iter__(self):
        flat, off = self._flat, self._off.tolist()
        return (flat[a:b] for a, b in zip(off[:-1], off[1:]))


def _step(model, pool: KVPool, plan, buffers: StepBuffers, full_logits: bool):
    """Run one step; (value_stm [R], legal logits flat, logits or None)."""
    R = plan.num_rows
    nl = 0 if plan.legal_ids is None else int(plan.legal_ids.shape[0])
    stream = torch.cuda.current_stream(model.device)
    dstep = buffers.stage(plan, stream)
    out, host = buffers.outputs(R + nl + 1)
    status = torch.zeros(1, dtype=torch.int32, device=model.device)
    logits = torch.empty((R, model.dims.vocab), dtype=torch.float32, device=model.device) if full_logits else None
    model.run(dstep, pool, value_stm=out[:R], legal_logits=out[R : R + nl], logits=logits, status=status,
              stream=stream)
    out[R + nl :].copy_(status.view(torch.float32))
    host.copy_(out, non_blocking=True)
    stream.synchronize()
    arr = host.numpy()
    code = int(arr[R + nl :].view(np.int32)[0])
    if code != _native.IMBA_OK:
        raise _native.ImbaError(code, "device-side check")
    return arr[:R].copy(), arr[R : R + nl].copy(), logits


def make_root_eval_executor(*, model, pool: KVPool, stats=None):
    """Executor over root payloads: each a dict with the token fields of one
    game prefix (and optionally ``legal_ids`` of its last position).  Returns
    per payload ``{"game": PagedGame, "value_stm": float, "legal_logits":
    np.ndarray}``."""
    buffers = StepBuffers(model.device)

    def executor(payloads: list[dict[str, Any]]) -> list[dict[str, Any]]:
        seqs = [KVSequence(pool) for _ in payloads]
        legal = [list(p.get("legal_ids", ())) for p in payloads]
        t0 = time.perf_counter()
        try:
            plan, last = root_plan(seqs, [{k: p[k] for k in p if k != "legal_ids"} for p in payloads], legal)
            v, ll, _ = _step(model, pool, plan, buffers, full_logits=False)
        except BaseException:
            for s in seqs:
                s.release()
            raise
        if stats is not None:
            stats.root_eval += time.perf_counter() - t0
        loff = plan.legal_off
        out = []
        for s, i in zip(seqs, last):
            game = PagedGame(prefix=s, prefix_len=s.length, arena=KVSequence(pool))
            out.append({"game": game, "value_stm": float(v[i]), "legal_logits": ll[loff[i] : loff[i + 1]]})
        return out

    return executor


def make_decode_wave_executor(*, model, pool: KVPool, stats=None, full_logits: bool = False):
    """Executor over ``PagedDecodeRequest`` payloads: one grouped decode step
    for every game's rows.  Returns per payload ``{"value_stm": [n],
    "legal_logits": LegalLogits (n arrays), "arena_rows": [n], "logits":
    [n, V] (when ``full_logits``)}``; the rows' KV is appended to each game's arena (rows
    numbered consecutively in payload order, like ``_KVArena.append``)."""
    buffers = StepBuffers(model.device)

    def executor(payloads: list[PagedDecodeRequest]) -> list[dict[str, Any]]:
        games = [p.game for p in payloads]
        counts = np.fromiter((len(p.parent_rows) for p in payloads), dtype=np.int64, count=len(payloads))
        chains_all = [c for p in payloads for c in p.parent_rows]
        depths = np.fromiter(map(len, chains_all), dtype=np.int64, count=len(chains_all))
        flat = np.fromiter(chain.from_iterable(chains_all), dtype=np.int64, count=int(depths.sum()))
        tok = {k: np.concatenate([np.asarray(p.tokens[k]) for p in payloads]) for k in payloads[0].tokens}
        loff, lids = ids_csr([ids for p in payloads for ids in p.legal_ids])
        marks = [(g.arena, g.arena.length, len(g.arena.pages)) for g in games]
        t0 = time.perf_counter()
        try:
            plan, starts = wave_plan_flat([g.prefix for g in games], [g.prefix_len for g in games],
                                          [g.arena for g in games], counts, depths, flat,
                                          piece_ids_from_tokens(tok), side_ids_from_tokens(tok), (loff, lids))
            v, ll, logits = _step(model, pool, plan, buffers, full_logits)
        except BaseException:
            for arena, length, npages in reversed(marks):
                arena.truncate(length, npages)
            raise
        if stats is not None:
            stats.search_gpu += time.perf_counter() - t0
            stats.search_eval_calls += 1
            stats.search_eval_items += int(counts.sum())
        out = []
        r0 = 0
        for p, n, s in zip(payloads, counts.tolist(), starts.tolist()):
            entry = {
                "value_stm": v[r0 : r0 + n],
                "legal_logits": LegalLogits(ll, loff[r0 : r0 + n + 1]),
                "arena_rows": list(range(s, s + n)),
            }
            if logits is not None:
                entry["logits"] = logits[r0 : r0 + n]
            out.append(entry)
            r0 += n
        return out

    return executor
