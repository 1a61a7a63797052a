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
from itertools import chain

import numpy as np

from . import _hostpath
from .kvpool import PAGE, KVSequence
from .plan import StepPlan
from .synth import TOKEN_FIELDS


def ids_csr(id_lists) -> tuple[np.ndarray, np.ndarray]:
    """List of per-row id lists -> (int32 offsets [R+1], int32 flat ids),
    built by the C++ host path (no per-element Python code)."""
    off_b, ids_b = _hostpath.ids_csr(id_lists)
    return np.frombuffer(off_b, dtype=np.int32), np.frombuffer(ids_b, dtype=np.int32)


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


def wave_plan(groups: list[WaveGroup], piece: np.ndarray, side: np.ndarray, legal_ids: list | None,
              legal_csr: tuple[np.ndarray, np.ndarray] | None = None) -> tuple[StepPlan, list[list[int]]]:
    """Grouped decode of every group's rows (rows ordered group by group).
    Legal ids come as per-row lists or, already packed, as ``legal_csr`` =
    (int32 offsets [R+1], int32 ids).  Returns the plan and, per group, the
    arena rows minted for its rows."""
    counts = np.fromiter((len(g.chains) for g in groups), dtype=np.int64, count=len(groups))
    all_chains = [c for g in groups for c in g.chains]
    depths = np.fromiter(map(len, all_chains), dtype=np.int64, count=len(all_chains))
    flat = np.fromiter(chain.from_iterable(all_chains), dtype=np.int64, count=int(depths.sum()))
    plan, starts = wave_plan_flat([g.prefix for g in groups], [g.prefix_len for g in groups],
                                  [g.arena for g in groups], counts, depths, flat, piece, side,
                                  legal_csr if legal_csr is not None else ids_csr(legal_ids))
    own_rows = [list(range(int(s), int(s) + int(n))) for s, n in zip(starts, counts)]
    return plan, own_rows


def wave_plan_flat(prefixes: list[KVSequence], prefix_lens, arenas: list[KVSequence], counts: np.ndarray,
                   depths: np.ndarray, chain_rows: np.ndarray, piece: np.ndarray, side: np.ndarray,
                   legal_csr: tuple[np.ndarray, np.ndarray]) -> tuple[StepPlan, np.ndarray]:
    """``wave_plan`` on flat arrays: group g has ``counts[g]`` rows; row r's
    parent chain (arena row ids of its group's arena, root -> parent) is
    ``chain_rows[sum(depths[:r]) : sum(depths[:r + 1])]``.  Reserves one
    arena row per decode row, numbered consecutively per arena in wave order
    like ``_KVArena.append`` (actor_server.py:246-255; an arena listed twice
    continues where its previous group stopped).  Returns the plan and, per
    group, the arena row id of its first new row."""
    G = len(prefixes)
    counts = np.asarray(counts, dtype=np.int64).reshape(G)
    R = int(counts.sum())
    starts = np.empty(G, dtype=np.int64)
    seen: dict[int, int] = {}
    for i, (a, n) in enumerate(zip(arenas, counts.tolist())):
        s0 = seen.get(id(a), a.length)
        starts[i] = s0
        seen[id(a)] = s0 + n
    dst = KVSequence.reserve_many(arenas, counts)
    plen = np.asarray(prefix_lens, dtype=np.int64).reshape(G)
    npre = [min(-(-int(n) // PAGE), len(p.pages)) for p, n in zip(prefixes, plen)]  # as page_array slices
    pages_cat = np.fromiter(chain.from_iterable(p.pages[:k] for p, k in zip(prefixes, npre)), dtype=np.int64,
                            count=sum(npre))
    row_group = np.repeat(np.arange(G), counts)
    prow = plen[row_group]
    depths = np.asarray(depths, dtype=np.int64).reshape(R)
    positions = prow + depths
    # Extras of row r: its chain (positions P + j), then itself (position P + depth).
    per_row = depths + 1
    eoff = np.zeros(R + 1, dtype=np.int64)
    np.cumsum(per_row, out=eoff[1:])
    E = int(eoff[-1])
    extra_slot = np.empty(E, dtype=np.int64)
    extra_pos = np.empty(E, dtype=np.int64)
    own_idx = eoff[1:] - 1
    extra_slot[own_idx] = dst
    extra_pos[own_idx] = positions
    if E > R:
        is_chain = np.ones(E, dtype=bool)
        is_chain[own_idx] = False
        # arena row -> slot through each row's arena page list (after the reservation)
        apages = [a.pages for a in arenas]
        anp = np.fromiter(map(len, apages), dtype=np.int64, count=G)
        abase = np.zeros(G, dtype=np.int64)
        np.cumsum(anp[:-1], out=abase[1:])
        acat = np.fromiter(chain.from_iterable(apages), dtype=np.int64, count=int(anp.sum()))
        rows = np.asarray(chain_rows, dtype=np.int64)
        grp = np.repeat(row_group, depths)
        if rows.size and (rows.min() < 0 or (rows // PAGE >= anp[grp]).any()):
            raise KeyError("a parent chain names an arena row its turn does not hold")
        extra_slot[is_chain] = acat[abase[grp] + rows // PAGE] * PAGE + rows % PAGE
        j = np.arange(E) - np.repeat(eoff[:-1], per_row)  # index within the row's extras
        extra_pos[is_chain] = (np.repeat(prow, per_row) + j)[is_chain]
    gpo = np.zeros(G + 1, dtype=np.int64)
    np.cumsum(npre, out=gpo[1:])
    loff, lids = legal_csr
    plan = StepPlan(
        piece_ids=piece,
        side_ids=side,
        positions=positions.astype(np.int32),
        row_group=row_group.astype(np.int32),
        row_vis=prow.astype(np.int32),
        row_extra_off=eoff.astype(np.int32),
        extra_slot=extra_slot.astype(np.int32),
        extra_pos=extra_pos.astype(np.int32),
        row_dst_slot=dst.astype(np.int32),
        group_page_off=gpo.astype(np.int32),
        group_pages=pages_cat.astype(np.int32),
        legal_off=loff,
        legal_ids=lids,
    )
    return plan, starts
