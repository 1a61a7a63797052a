"""Step plans for the two request kinds of the search-inference path.

* ``root_plan``: append tokens to one or more pool sequences (a full game
  prefill, or an incremental extension of a persisted game prefix); each new
  token attends causally to everything before it in its own sequence
  (src/imba_chess/model/hstu_model.py:337-374; the incremental loop of
  src/imba_chess/eval/actor_server.py:749-781 as one batched step).
* ``wave_plan``: a grouped decode wave; every row reads its group's prefix
  (a sequence snapshot of ``prefix_len`` tokens), its parent chain in the
  turn arena and itself (hstu_attention.py:259-424; actor_server.py:806-914).

Both return a ``StepPlan`` (integer arrays only).  Sequences grow here:
``root_plan`` reserves the new tokens' slots, ``wave_plan`` reserves one arena
row per decode row, numbered consecutively like ``_KVArena.append``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .kvpool import KVSequence
from .plan import StepPlan
from .synth import TOKEN_FIELDS


def ids_csr(id_lists) -> tuple[np.ndarray, np.ndarray]:
    """List of per-row id lists -> (int32 offsets [R+1], int32 flat ids)."""
    lengths = np.fromiter((len(x) for x in id_lists), dtype=np.int64, count=len(id_lists))
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    flat = np.fromiter((int(v) for ids in id_lists for v in ids), dtype=np.int64, count=int(off[-1]))
    return off, flat.astype(np.int32)


def _token_arrays(tokens: list[dict]) -> tuple[np.ndarray, np.ndarray]:
    piece = np.concatenate([np.asarray(t["piece_ids"], dtype=np.int64).reshape(-1, 64) for t in tokens])
    if piece.size and (piece.min() < 0 or piece.max() > 12):
        raise ValueError("piece_ids values must be in [0, 12]")
    side = np.stack(
        [np.concatenate([np.asarray(t[k], dtype=np.int64).reshape(-1) for t in tokens]) for k in TOKEN_FIELDS[1:]],
        axis=1,
    )
    return piece.astype(np.uint8), side.clip(-(2**31), 2**31 - 1).astype(np.int32)


def root_plan(seqs: list[KVSequence], tokens: list[dict], legal_last: list | None = None) -> tuple[StepPlan, np.ndarray]:
    """Append ``tokens[g]`` to ``seqs[g]``.  Legal ids (when given) are
    attached to each sequence's last new token.  Returns the plan and the row
    index of each sequence's last token."""
    counts = np.asarray([len(t["piece_ids"]) for t in tokens], dtype=np.int64)
    G = len(seqs)
    starts = np.asarray([s.length for s in seqs], dtype=np.int64)
    row_group = np.repeat(np.arange(G), counts)
    local = np.arange(int(counts.sum())) - np.repeat(np.cumsum(counts) - counts, counts)
    positions = starts[row_group] + local
    dst = np.concatenate([s.reserve(int(n)) for s, n in zip(seqs, counts)]) if G else np.zeros(0, np.int64)
    pages = [s.page_array() for s in seqs]
    gpo = np.concatenate([[0], np.cumsum([len(p) for p in pages])]).astype(np.int32)
    piece, side = _token_arrays(tokens)
    R = int(counts.sum())
    last = (np.cumsum(counts) - 1).astype(np.int64)
    loff = lids = None
    if legal_last is not None:
        per_row = [()] * R
        for g, ids in enumerate(legal_last):
            per_row[last[g]] = ids
        loff, lids = ids_csr(per_row)
    plan = StepPlan(
        piece_ids=piece,
        side_ids=side,
        positions=positions.astype(np.int32),
        row_group=row_group.astype(np.int32),
        row_vis=(positions + 1).astype(np.int32),
        row_extra_off=np.zeros(R + 1, np.int32),
        extra_slot=np.zeros(0, np.int32),
        extra_pos=np.zeros(0, np.int32),
        row_dst_slot=dst.astype(np.int32),
        group_page_off=gpo,
        group_pages=np.concatenate(pages).astype(np.int32) if pages else np.zeros(0, np.int32),
        legal_off=loff,
        legal_ids=lids,
    )
    return plan, last


@dataclass
class WaveGroup:
    """One request of a wave: its prefix snapshot, its turn arena and, per
    row, the parent chain (arena row ids, root -> parent)."""

    prefix: KVSequence
    prefix_len: int
    arena: KVSequence
    chains: list[list[int]]


def wave_plan(groups: list[WaveGroup], piece: np.ndarray, side: np.ndarray, legal_ids: list) -> tuple[StepPlan, list[list[int]]]:
    """Grouped decode of every group's rows (rows ordered group by group).
    Returns the plan and, per group, the arena rows minted for its rows."""
    counts = [len(g.chains) for g in groups]
    own_rows: list[list[int]] = []
    dst_parts, es_parts, ep_parts, elen, positions, pages, gpo = [], [], [], [], [], [], [0]
    for g in groups:
        n = len(g.chains)
        start = g.arena.length
        dst = g.arena.reserve(n)
        own_rows.append(list(range(start, start + n)))
        P = g.prefix_len
        depths = np.fromiter((len(c) for c in g.chains), dtype=np.int64, count=n)
        flat = np.fromiter((x for c in g.chains for x in c), dtype=np.int64, count=int(depths.sum()))
        chain_slots = g.arena.slots_of(flat) if flat.size else np.zeros(0, np.int64)
        chain_pos = P + (np.arange(flat.size) - np.repeat(np.cumsum(depths) - depths, depths))
        ins = np.cumsum(depths)
        es_parts.append(np.insert(chain_slots, ins, dst))
        ep_parts.append(np.insert(chain_pos, ins, P + depths))
        elen.append(depths + 1)
        positions.append(P + depths)
        dst_parts.append(dst)
        pg = g.prefix.page_array(P)
        pages.append(pg)
        gpo.append(gpo[-1] + len(pg))
    loff, lids = ids_csr(legal_ids)
    elen_a = np.concatenate(elen) if elen else np.zeros(0, np.int64)
    plan = StepPlan(
        piece_ids=piece,
        side_ids=side,
        positions=np.concatenate(positions).astype(np.int32) if positions else np.zeros(0, np.int32),
        row_group=np.repeat(np.arange(len(groups)), counts).astype(np.int32),
        row_vis=np.repeat([g.prefix_len for g in groups], counts).astype(np.int32),
        row_extra_off=np.concatenate([[0], np.cumsum(elen_a)]).astype(np.int32),
        extra_slot=np.concatenate(es_parts).astype(np.int32) if es_parts else np.zeros(0, np.int32),
        extra_pos=np.concatenate(ep_parts).astype(np.int32) if ep_parts else np.zeros(0, np.int32),
        row_dst_slot=np.concatenate(dst_parts).astype(np.int32) if dst_parts else np.zeros(0, np.int32),
        group_page_off=np.asarray(gpo, dtype=np.int32),
        group_pages=np.concatenate(pages).astype(np.int32) if pages else np.zeros(0, np.int32),
        legal_off=loff,
        legal_ids=lids,
    )
    return plan, own_rows
