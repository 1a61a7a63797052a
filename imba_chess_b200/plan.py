"""Host-side planning of one jagged step (integer bookkeeping only).

A ``StepPlan`` holds every integer input of ``imba_step`` as numpy arrays.
``pack()`` lays them out in ONE int32 buffer so a step costs a single
host-to-device copy; ``DeviceStep`` points a ``StepDesc`` into the device
copy.  All arrays are built with vectorised numpy: no per-row Python loops.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import _native
from .synth import TOKEN_FIELDS

CHUNK = _native.CHUNK_ROWS

# Order of the int32 sections in the packed buffer.
_SECTIONS = (
    "side_ids",
    "positions",
    "row_vis",
    "row_extra_off",
    "extra_slot",
    "extra_pos",
    "row_dst_slot",
    "group_page_off",
    "group_pages",
    "chunk_group",
    "chunk_row_off",
    "chunk_nrows",
    "row_perm",
    "legal_off",
    "legal_ids",
)


def side_ids_from_tokens(tok: dict) -> np.ndarray:
    """[R, 7] int32: seq, turn, castle, ep, halfmove, fullmove, prev_move."""
    cols = [np.asarray(tok[k], dtype=np.int64).reshape(-1) for k in TOKEN_FIELDS[1:]]
    return np.stack(cols, axis=1).clip(-(2**31), 2**31 - 1).astype(np.int32)


def piece_ids_from_tokens(tok: dict) -> np.ndarray:
    p = np.asarray(tok["piece_ids"], dtype=np.int64).reshape(-1, 64)
    if p.size and (p.min() < 0 or p.max() > 12):
        raise ValueError("piece_ids values must be in [0, 12]")
    return p.astype(np.uint8)


def build_chunks(row_group: np.ndarray, num_groups: int, max_rows: int = 32, row_vis: np.ndarray | None = None):
    """Rows ordered by group (stable), split into chunks of <= ``max_rows``
    rows (the C ABI allows up to 64; 32 is one attention work item).  A group
    with more rows is split into equal-size chunks.  With ``row_vis`` the
    chunks are listed longest visible prefix first, so the attention kernel's
    dynamic work queue starts the longest items first."""
    if not 1 <= max_rows <= CHUNK:
        raise ValueError(f"max_rows must be in [1, {CHUNK}]")
    row_group = np.asarray(row_group, dtype=np.int64)
    order = np.argsort(row_group, kind="stable").astype(np.int32)
    counts = np.bincount(row_group, minlength=num_groups).astype(np.int64)
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int64)
    nch = (counts + max_rows - 1) // max_rows
    chunk_group = np.repeat(np.arange(num_groups, dtype=np.int64), nch)
    first = np.repeat(np.cumsum(nch) - nch, nch)
    cidx = np.arange(int(nch.sum()), dtype=np.int64) - first
    # balanced split: chunk i of a group with n rows and k chunks covers
    # [i*n//k, (i+1)*n//k)
    n_g = counts[chunk_group]
    k_g = nch[chunk_group]
    lo = cidx * n_g // k_g
    hi = (cidx + 1) * n_g // k_g
    chunk_row_off = starts[chunk_group] + lo
    chunk_nrows = hi - lo
    if row_vis is not None and chunk_group.size:
        vis_sorted = np.asarray(row_vis, dtype=np.int64)[order]
        # longest visible prefix of each chunk (rows of a chunk are contiguous in `order`)
        cost = np.maximum.reduceat(vis_sorted, chunk_row_off) if vis_sorted.size else np.zeros(0, np.int64)
        by_cost = np.argsort(-cost, kind="stable")
        chunk_group, chunk_row_off, chunk_nrows = chunk_group[by_cost], chunk_row_off[by_cost], chunk_nrows[by_cost]
    return (
        order,
        chunk_group.astype(np.int32),
        chunk_row_off.astype(np.int32),
        chunk_nrows.astype(np.int32),
    )


@dataclass
class StepPlan:
    piece_ids: np.ndarray          # uint8 [R, 64]
    side_ids: np.ndarray           # int32 [R, 7]
    positions: np.ndarray          # int32 [R]
    row_group: np.ndarray          # int32 [R]
    row_vis: np.ndarray            # int32 [R]
    row_extra_off: np.ndarray      # int32 [R + 1]
    extra_slot: np.ndarray         # int32 [E]
    extra_pos: np.ndarray          # int32 [E]
    row_dst_slot: np.ndarray       # int32 [R]
    group_page_off: np.ndarray     # int32 [G + 1]
    group_pages: np.ndarray        # int32 [NP]
    legal_off: np.ndarray | None = None  # int32 [R + 1]
    legal_ids: np.ndarray | None = None  # int32 [NL]
    chunks: tuple = field(default=None, repr=False)

    @property
    def num_rows(self) -> int:
        return int(self.positions.shape[0])

    @property
    def num_groups(self) -> int:
        return int(self.group_page_off.shape[0]) - 1

    def finalize(self) -> "StepPlan":
        if self.chunks is None:
            # Steps without extra keys (prefills) take 64-row chunks: the
            # prefill attention stacks a chunk's rows for two heads in one
            # 128-row tensor-core tile.
            rows = CHUNK if self.extra_slot.shape[0] == 0 else 32
            self.chunks = build_chunks(self.row_group, self.num_groups, max_rows=rows, row_vis=self.row_vis)
        return self

    def arrays(self) -> dict[str, np.ndarray]:
        self.finalize()
        row_perm, cg, co, cn = self.chunks
        R = self.num_rows
        out = {
            "side_ids": self.side_ids.reshape(-1),
            "positions": self.positions,
            "row_vis": self.row_vis,
            "row_extra_off": self.row_extra_off,
            "extra_slot": self.extra_slot,
            "extra_pos": self.extra_pos,
            "row_dst_slot": self.row_dst_slot,
            "group_page_off": self.group_page_off,
            "group_pages": self.group_pages,
            "chunk_group": cg,
            "chunk_row_off": co,
            "chunk_nrows": cn,
            "row_perm": row_perm,
            "legal_off": self.legal_off if self.legal_off is not None else np.zeros(R + 1, np.int32),
            "legal_ids": self.legal_ids if self.legal_ids is not None else np.zeros(0, np.int32),
        }
        return {k: np.ascontiguousarray(v, dtype=np.int32).reshape(-1) for k, v in out.items()}

    def layout(self) -> tuple[int, dict[str, tuple[int, int]], dict[str, np.ndarray]]:
        """(int32 words, {name: (offset in int32 elements, length)}, arrays)
        of the packed buffer: piece bytes (padded to 16 B), then each section
        padded to a multiple of 4 elements."""
        arrs = self.arrays()
        R = self.num_rows
        piece_words = -(-(R * 64) // 16) * 4
        layout: dict[str, tuple[int, int]] = {"piece_ids": (0, R * 64)}
        off = piece_words
        for name in _SECTIONS:
            n = int(arrs[name].shape[0])
            layout[name] = (off, n)
            off += -(-max(n, 1) // 4) * 4
        return off, layout, arrs

    def pack_into(self, buf: np.ndarray, words: int, layout, arrs) -> None:
        """Write the packed plan into ``buf`` (int32, at least ``words`` long)."""
        R = self.num_rows
        buf[:words] = 0
        buf.view(np.uint8)[: R * 64] = self.piece_ids.reshape(-1)
        for name in _SECTIONS:
            o, n = layout[name]
            buf[o : o + n] = arrs[name]

    def pack(self) -> tuple[np.ndarray, dict[str, tuple[int, int]]]:
        """One int32 buffer holding every integer input of the step (see
        ``layout``).  Returns (buffer, {name: (offset in int32 elements,
        length)})."""
        words, layout, arrs = self.layout()
        buf = np.zeros(words, dtype=np.int32)
        self.pack_into(buf, words, layout, arrs)
        return buf, layout

    def counts(self) -> dict[str, int]:
        self.finalize()
        return {
            "num_rows": self.num_rows,
            "num_groups": self.num_groups,
            "num_chunks": int(self.chunks[1].shape[0]),
            "num_legal": 0 if self.legal_ids is None else int(self.legal_ids.shape[0]),
            "num_extra": int(self.extra_slot.shape[0]),
            "num_group_pages": int(self.group_pages.shape[0]),
        }


class StepBuffers:
    """Pinned host and device buffers reused by consecutive steps on one
    device: the packed plan (written on the host, copied once per step) and
    the step's float32 results.  One step may be in flight at a time: the
    caller synchronises before staging the next one."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self._host: torch.Tensor | None = None
        self._dev: torch.Tensor | None = None
        self._out_host: torch.Tensor | None = None
        self._out_dev: torch.Tensor | None = None

    @staticmethod
    def _grow(n: int) -> int:
        return max(1024, int(n * 1.25))

    def stage(self, plan: "StepPlan", stream: torch.cuda.Stream | None = None) -> "DeviceStep":
        """Pack ``plan`` into the pinned buffer and enqueue its copy to the
        device on ``stream`` (default: the current stream)."""
        words, layout, arrs = plan.layout()
        if self._host is None or self._host.numel() < words:
            self._host = torch.empty(self._grow(words), dtype=torch.int32, pin_memory=True)
            self._dev = torch.empty(self._host.numel(), dtype=torch.int32, device=self.device)
        plan.pack_into(self._host.numpy(), words, layout, arrs)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        with torch.cuda.stream(s):
            self._dev[:words].copy_(self._host[:words], non_blocking=True)
        return DeviceStep.over(plan, self._dev, layout, words)

    def outputs(self, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(device float32 [n], pinned host float32 [n]) result buffers."""
        if self._out_host is None or self._out_host.numel() < n:
            size = self._grow(n)
            self._out_host = torch.empty(size, dtype=torch.float32, pin_memory=True)
            self._out_dev = torch.empty(size, dtype=torch.float32, device=self.device)
        return self._out_dev[:n], self._out_host[:n]


class DeviceStep:
    """A packed plan resident on the device, with a ``StepDesc`` pointing
    into it.  Output pointers are filled by the caller."""

    def __init__(self, plan: StepPlan, device: torch.device, *, pinned: bool = False,
                 stream: torch.cuda.Stream | None = None) -> None:
        buf, layout = plan.pack()
        host = torch.from_numpy(buf)
        if pinned:
            host = host.pin_memory()
        self.host = host
        self.buf = torch.empty_like(host, device=device)
        self.buf.copy_(host, non_blocking=pinned)
        self.layout = layout
        self.has_legal = plan.legal_off is not None
        self.desc = _native.StepDesc()
        for k, v in plan.counts().items():
            setattr(self.desc, k, v)
        base = self.buf.data_ptr()
        for name, (off, _n) in layout.items():
            setattr(self.desc, name, base + 4 * off)
        if not self.has_legal:
            self.desc.legal_off = None
            self.desc.legal_ids = None

    @classmethod
    def over(cls, plan: "StepPlan", dev: torch.Tensor, layout, words: int) -> "DeviceStep":
        """A step whose packed plan already sits at the start of ``dev``."""
        self = cls.__new__(cls)
        self.host = None
        self.buf = dev[:words]
        self.layout = layout
        self.has_legal = plan.legal_off is not None
        self.desc = _native.StepDesc()
        for k, v in plan.counts().items():
            setattr(self.desc, k, v)
        base = dev.data_ptr()
        for name, (off, _n) in layout.items():
            setattr(self.desc, name, base + 4 * off)
        if not self.has_legal:
            self.desc.legal_off = None
            self.desc.legal_ids = None
        return self

    @property
    def h2d_bytes(self) -> int:
        return int(self.buf.numel() * 4)
