"""Paged, device-resident KV pool and the token sequences that live in it.

One pool per model per device: a ``[num_pages, page_elems]`` tensor in the
model dtype whose page layout is ``[layer][K: H x 16 x d_qk | V: H x 16 x
d_v]`` (include/imba_b200.h).  A ``KVSequence`` is an append-only list of
pages plus a token count; token ``t`` lives at physical slot
``pages[t // 16] * 16 + t % 16``.

The reference keeps two kinds of KV stores (src/imba_chess/eval/
actor_server.py:206-344):

* a game's growing root prefix (``_GameState``), re-built by ``torch.cat``
  on every incremental extension, and
* a turn's decode-node arena (``_KVArena``), a ``[L, H, capacity, d]`` tensor
  grown by doubling, whose rows are minted consecutively in wave order.

Both map onto ``KVSequence``: appending never moves existing tokens, so a
turn's snapshot of a game prefix (a sequence plus the length it had) stays
valid while the game grows, and arena row ``r`` of a turn is token ``r`` of
that turn's arena sequence - the same row ids the reference mints.
Sequences are reference-counted; pages return to the pool when the last
holder releases them.
"""

from __future__ import annotations

from itertools import chain

import numpy as np
import torch

from . import _native

PAGE = _native.PAGE_TOKENS


class KVPoolExhausted(RuntimeError):
    """The pool has fewer free pages than a request needs."""


class KVPool:
    def __init__(self, *, num_layers: int, num_heads: int, attention_dim: int, linear_dim: int,
                 num_pages: int, dtype: torch.dtype, device: torch.device) -> None:
        if num_pages <= 0:
            raise ValueError("num_pages must be positive")
        self.page_elems = num_layers * num_heads * PAGE * (attention_dim + linear_dim)
        self.num_pages = int(num_pages)
        self.dtype = dtype
        self.device = device
        self.data = torch.zeros((self.num_pages, self.page_elems), dtype=dtype, device=device)
        self._free = np.arange(self.num_pages - 1, -1, -1, dtype=np.int64).tolist()
        self.desc = _native.PoolDesc(self.data.data_ptr(), self.num_pages)

    @property
    def free_pages(self) -> int:
        return len(self._free)

    @property
    def page_bytes(self) -> int:
        return self.page_elems * self.data.element_size()

    def alloc(self, n: int) -> list[int]:
        if n > len(self._free):
            raise KVPoolExhausted(
                f"KV pool exhausted: need {n} pages, {len(self._free)} of {self.num_pages} free"
            )
        if n <= 0:
            return []
        out = self._free[-n:]
        del self._free[-n:]
        out.reverse()
        return out

    def release_pages(self, pages: list[int]) -> None:
        self._free.extend(reversed(pages))


class KVSequence:
    """Append-only token sequence in a ``KVPool`` (reference-counted)."""

    __slots__ = ("pool", "pages", "length", "refs")

    def __init__(self, pool: KVPool) -> None:
        self.pool = pool
        self.pages: list[int] = []
        self.length = 0
        self.refs = 1

    def retain(self) -> "KVSequence":
        if self.refs <= 0:
            raise RuntimeError("retain() on a released KV sequence")
        self.refs += 1
        return self

    def release(self) -> None:
        if self.refs <= 0:
            return
        self.refs -= 1
        if self.refs == 0:
            self.pool.release_pages(self.pages)
            self.pages = []
            self.length = 0

    def reserve(self, n: int) -> np.ndarray:
        """Append ``n`` token slots; returns their physical slots (int64)."""
        start = self.length
        need_pages = -(-(start + n) // PAGE) - len(self.pages)
        if need_pages > 0:
            self.pages.extend(self.pool.alloc(need_pages))
        self.length = start + n
        return self.slots(start, start + n)

    @staticmethod
    def reserve_many(seqs: "list[KVSequence]", counts) -> np.ndarray:
        """``seqs[i].reserve(counts[i])`` for every i, in order; returns all
        the new slots concatenated (int64), computed in one pass over the
        sequences' page lists instead of one small array per sequence."""
        n = len(seqs)
        starts = np.empty(n, dtype=np.int64)
        for i, (s, c) in enumerate(zip(seqs, counts)):
            start = s.length
            need = -(-(start + int(c)) // PAGE) - len(s.pages)
            if need > 0:
                s.pages.extend(s.pool.alloc(need))
            s.length = start + int(c)
            starts[i] = start
        cnt = np.asarray(counts, dtype=np.int64).reshape(n)
        total = int(cnt.sum())
        if total == 0:
            return np.zeros(0, dtype=np.int64)
        npg = np.fromiter((len(s.pages) for s in seqs), dtype=np.int64, count=n)
        pbase = np.zeros(n, dtype=np.int64)
        np.cumsum(npg[:-1], out=pbase[1:])
        cat = np.fromiter(chain.from_iterable(s.pages for s in seqs), dtype=np.int64, count=int(npg.sum()))
        rbase = np.zeros(n, dtype=np.int64)
        np.cumsum(cnt[:-1], out=rbase[1:])
        t = np.repeat(starts, cnt) + np.arange(total, dtype=np.int64) - np.repeat(rbase, cnt)
        return cat[np.repeat(pbase, cnt) + t // PAGE] * PAGE + t % PAGE

    def truncate(self, length: int, num_pages: int) -> None:
        """Undo reservations: back to ``length`` tokens on the first
        ``num_pages`` pages (values recorded before the reservations); the
        pages past them return to the pool."""
        if num_pages < len(self.pages):
            self.pool.release_pages(self.pages[num_pages:])
            del self.pages[num_pages:]
        self.length = min(self.length, int(length))

    def slots(self, start: int, stop: int) -> np.ndarray:
        t = np.arange(start, stop, dtype=np.int64)
        pages = np.asarray(self.pages, dtype=np.int64)
        return pages[t // PAGE] * PAGE + t % PAGE

    def slots_of(self, tokens) -> np.ndarray:
        t = np.asarray(tokens, dtype=np.int64)
        pages = np.asarray(self.pages, dtype=np.int64)
        return pages[t // PAGE] * PAGE + t % PAGE

    def page_array(self, length: int | None = None) -> np.ndarray:
        n = self.length if length is None else length
        return np.asarray(self.pages[: -(-n // PAGE)], dtype=np.int32)
