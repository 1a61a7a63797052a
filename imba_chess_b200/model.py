"""``B200HSTUChessModel``: the HSTU chess model's inference API on the B200
library.

Drop-in for the inference surface of the reference ``HSTUChessModel``
(src/imba_chess/model/hstu_model.py:337-374, :600-649, :651-752):

* ``forward(batch, *, block_mask=None, return_loss=False, return_kv=True)``
* ``forward_decode(*, new_token_batch, positions, prefix_kv, suffix_kv=None,
  suffix_positions=None, suffix_mask=None)``
* ``forward_decode_grouped(*, new_token_batch, positions, group_index,
  prefix_kv_grouped, prefix_lens, prefix_lens_list, suffix_kv=None,
  suffix_positions=None, suffix_mask=None)``

with the same argument meaning, output dicts and ``ValueError`` guards.
These dense-tensor entry points stage their KV into a scratch paged pool and
run one jagged step; the actor server (``imba_chess_b200.server``) skips the
staging and keeps every prefix and node resident in a persistent pool.

Every call runs the CUDA library; there is no CPU path.  Output logits and
value logits are fp32; returned k/v are in the model dtype.
"""

from __future__ import annotations

import ctypes
from types import SimpleNamespace
from typing import Any, Mapping

import numpy as np
import torch

from . import _native
from .kvpool import PAGE, KVPool
from .plan import DeviceStep, StepBuffers, StepPlan, piece_ids_from_tokens, side_ids_from_tokens
from .weights import PackedWeights

_TOKEN_KEYS = (
    "piece_ids",
    "seq_token_id",
    "turn_id",
    "castle_id",
    "ep_file_id",
    "halfmove_bucket_id",
    "fullmove_bucket_id",
    "prev_move_id",
)


def _np(x, dtype=None) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu().numpy()
    a = np.asarray(x)
    return a.astype(dtype) if dtype is not None else a


def _tokens(batch: Mapping[str, Any]) -> dict[str, np.ndarray]:
    return {k: _np(batch[k], np.int64) for k in _TOKEN_KEYS}


class _ValueHeadMarker:
    """Stands in for ``model.value_head`` (the server only checks it is not None)."""

    def __repr__(self) -> str:
        return "B200ValueHead()"


class B200HSTUChessModel:
    """Inference-only HSTU chess model running on the imba_b200 library."""

    training = False

    def __init__(self, state_dict: Mapping[str, Any], *, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str = "cuda", simt: tuple[str, ...] = ()) -> None:
        """``simt`` is a test hook for bf16 models: component names ("gemm",
        "attn", "board") whose fp32-accumulating SIMT kernels replace the
        tensor-core ones, so tests can compare the two on identical inputs."""
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("B200HSTUChessModel runs on a CUDA device only (no CPU fallback)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        with torch.cuda.device(self.device):
            self.weights = PackedWeights(state_dict, dtype=dtype, device=self.device)
        d = self.weights.dims
        self.dims = d
        self.config = SimpleNamespace(
            model_dim=d.model_dim,
            num_layers=d.num_layers,
            num_heads=d.num_heads,
            attention_dim=d.attention_dim,
            linear_hidden_dim=d.linear_dim,
            move_vocab_size=d.vocab,
            max_position_embeddings=d.max_pos,
            halfmove_vocab_size=d.halfmove_vocab,
            fullmove_vocab_size=d.fullmove_vocab,
            enable_value_head=d.value_head,
        )
        self.position_embedding = SimpleNamespace(max_seq_len=d.max_pos)
        self.value_head = _ValueHeadMarker() if d.value_head else None
        self._lib = _native.load()
        flags = 0
        for name in simt:
            if name not in _native.SIMT_FLAGS:
                raise ValueError(f"unknown SIMT component {name!r}: use {sorted(_native.SIMT_FLAGS)}")
            flags |= _native.SIMT_FLAGS[name]
        self.weights.desc.flags = flags
        handle = ctypes.c_void_p()
        _native.check(self._lib.imba_model_create(ctypes.byref(self.weights.desc), ctypes.byref(handle)),
                      "imba_model_create")
        self._handle = handle
        self._workspace: torch.Tensor | None = None
        self._status = torch.zeros(1, dtype=torch.int32, device=self.device)

    # ------------------------------------------------------------------
    @classmethod
    def from_reference(cls, model, *, dtype: torch.dtype | None = None, device=None) -> "B200HSTUChessModel":
        """Build from a reference ``HSTUChessModel`` instance (its state_dict)."""
        sd = model.state_dict()
        dev = device if device is not None else "cuda"
        return cls(sd, dtype=dtype or torch.bfloat16, device=dev)

    @classmethod
    def from_checkpoint(cls, path, *, dtype: torch.dtype = torch.bfloat16, device=None,
                        require_value_head: bool = False) -> "B200HSTUChessModel":
        """Load a reference checkpoint file (plain or Ignite state dict) with
        the reference loader's key normalisation, value-head guard and strict
        key check (``weights.load_checkpoint_state_dict``)."""
        from .weights import load_checkpoint_state_dict

        sd = load_checkpoint_state_dict(path, require_value_head=require_value_head)
        return cls(sd, dtype=dtype, device=device if device is not None else "cuda")

    def eval(self) -> "B200HSTUChessModel":
        return self

    def __del__(self) -> None:
        h = getattr(self, "_handle", None)
        if h is not None and h.value:
            try:
                self._lib.imba_model_destroy(h)
            except Exception:
                pass

    # ------------------------------------------------------------------
    def new_pool(self, num_pages: int) -> KVPool:
        d = self.dims
        return KVPool(num_layers=d.num_layers, num_heads=d.num_heads, attention_dim=d.attention_dim,
                      linear_dim=d.linear_dim, num_pages=num_pages, dtype=self.dtype, device=self.device)

    def workspace(self, rows: int) -> torch.Tensor:
        need = int(self._lib.imba_step_workspace_bytes(self._handle, int(rows)))
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=self.device)
        return self._workspace

    def run(self, dstep: DeviceStep, pool: KVPool, *, logits=None, value_logits=None, value_stm=None,
            legal_logits=None, legal_logprob=None, hidden=None, status: torch.Tensor | None = None,
            stream: torch.cuda.Stream | None = None) -> None:
        """Enqueue one step on ``stream`` (default: torch's current stream)."""
        desc = dstep.desc
        rows = desc.num_rows

        def ptr(t):
            return None if t is None else t.data_ptr()

        desc.logits = ptr(logits)
        desc.value_logits = ptr(value_logits)
        desc.value_stm = ptr(value_stm)
        desc.legal_logits = ptr(legal_logits)
        desc.legal_logprob = ptr(legal_logprob)
        desc.hidden = ptr(hidden)
        desc.status = ptr(status if status is not None else self._status)
        ws = self.workspace(rows)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            code = self._lib.imba_step(self._handle, ctypes.byref(desc), ctypes.byref(pool.desc), ws.data_ptr(),
                                       ws.numel(), s.cuda_stream)
        _native.check(code, "imba_step")

    def check_status(self, status: torch.Tensor | None = None) -> None:
        st = status if status is not None else self._status
        code = int(st.item())
        if code != _native.IMBA_OK:
            st.zero_()
            raise _native.ImbaError(code, "device-side check")

    def kv_scatter(self, pool: KVPool, layer: int, slots: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        n = int(slots.numel())
        s = torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            code = self._lib.imba_kv_scatter(self._handle, ctypes.byref(pool.desc), layer, n, slots.data_ptr(),
                                             k.data_ptr(), v.data_ptr(), self._status.data_ptr(), s.cuda_stream)
        _native.check(code, "imba_kv_scatter")

    def kv_gather(self, pool: KVPool, layer: int, slots: torch.Tensor):
        n = int(slots.numel())
        d = self.dims
        k = torch.empty((n, d.num_heads, d.attention_dim), dtype=self.dtype, device=self.device)
        v = torch.empty((n, d.num_heads, d.linear_dim), dtype=self.dtype, device=self.device)
        s = torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            code = self._lib.imba_kv_gather(self._handle, ctypes.byref(pool.desc), layer, n, slots.data_ptr(),
                                            k.data_ptr(), v.data_ptr(), self._status.data_ptr(), s.cuda_stream)
        _native.check(code, "imba_kv_gather")
        return k, v

    # ------------------------------------------------------------------
    # Reference API: prefill
    # ------------------------------------------------------------------
    def forward(self, batch: Mapping[str, Any], *, block_mask=None, return_loss: bool = True,
                return_kv: bool = False) -> dict[str, Any]:
        """Jagged prefill (hstu_model.py:337-374): per-document causal
        attention over ``seq_offsets``; ``block_mask`` is accepted and ignored
        (documents are read from ``seq_offsets``).  Inference only."""
        if return_loss:
            raise ValueError("B200HSTUChessModel is inference-only: call forward(..., return_loss=False)")
        tok = _tokens(batch)
        offsets = _np(batch["seq_offsets"], np.int64)
        S = int(offsets[-1])
        lengths = offsets[1:] - offsets[:-1]
        ndocs = len(lengths)
        doc_pages = -(-lengths // PAGE)
        page_off = np.concatenate([[0], np.cumsum(doc_pages)]).astype(np.int64)
        total_pages = max(int(page_off[-1]), 1)
        pool = self._scratch_pool(total_pages)
        row_doc = np.repeat(np.arange(ndocs), lengths)
        local = np.arange(S) - np.repeat(offsets[:-1], lengths)
        slots = (page_off[row_doc] + local // PAGE) * PAGE + local % PAGE
        plan = StepPlan(
            piece_ids=piece_ids_from_tokens(tok),
            side_ids=side_ids_from_tokens(tok),
            positions=local.astype(np.int32),
            row_group=row_doc.astype(np.int32),
            row_vis=(local + 1).astype(np.int32),
            row_extra_off=np.zeros(S + 1, np.int32),
            extra_slot=np.zeros(0, np.int32),
            extra_pos=np.zeros(0, np.int32),
            row_dst_slot=slots.astype(np.int32),
            group_page_off=page_off.astype(np.int32),
            group_pages=np.arange(int(page_off[-1]), dtype=np.int32),
        )
        out = self._run_dense(plan, pool)
        result: dict[str, Any] = {"logits": out["logits"], "policy_logits": out["logits"]}
        if self.value_head is not None:
            result["value_logits"] = out["value_logits"]
        if return_kv:
            slot_t = torch.from_numpy(slots.astype(np.int32)).to(self.device)
            kv = []
            for l in range(self.dims.num_layers):
                k, v = self.kv_gather(pool, l, slot_t)
                kv.append((k.transpose(0, 1).contiguous(), v.transpose(0, 1).contiguous()))
            result["kv_caches"] = kv
        self.check_status()
        return result

    # ------------------------------------------------------------------
    # Reference API: decode
    # ------------------------------------------------------------------
    def forward_decode(self, *, new_token_batch, positions, prefix_kv, suffix_kv=None, suffix_positions=None,
                       suffix_mask=None) -> dict[str, Any]:
        """Single shared prefix (hstu_model.py:600-649)."""
        n = int(_np(positions).reshape(-1).shape[0])
        T = int(prefix_kv[0][0].shape[1]) if prefix_kv else 0
        grouped = [(k.unsqueeze(0), v.unsqueeze(0)) for k, v in prefix_kv]
        return self.forward_decode_grouped(
            new_token_batch=new_token_batch,
            positions=positions,
            group_index=np.zeros(n, np.int64),
            prefix_kv_grouped=grouped,
            prefix_lens=np.array([T], np.int64),
            prefix_lens_list=[T],
            suffix_kv=suffix_kv,
            suffix_positions=suffix_positions,
            suffix_mask=suffix_mask,
        )

    def forward_decode_grouped(self, *, new_token_batch, positions, group_index, prefix_kv_grouped, prefix_lens,
                               prefix_lens_list, suffix_kv=None, suffix_positions=None,
                               suffix_mask=None) -> dict[str, Any]:
        """Grouped decode (hstu_model.py:651-752, hstu_attention.py:259-424):
        row r reads only group ``group_index[r]``'s real prefix slice, its
        masked suffix and itself."""
        if (suffix_kv is None) != (suffix_positions is None) or (suffix_kv is None) != (suffix_mask is None):
            raise AssertionError("suffix tensors must be provided together")
        tok = _tokens(new_token_batch)
        pos = _np(positions, np.int64).reshape(-1)
        gidx = _np(group_index, np.int64).reshape(-1)
        B = int(tok["piece_ids"].shape[0])
        lens_t = _np(prefix_lens, np.int64).reshape(-1)
        G = int(lens_t.shape[0])
        if len(prefix_lens_list) != G:
            raise ValueError(
                "prefix_lens_list must have length num_groups "
                f"(== prefix_lens.numel() == {G}), got {len(prefix_lens_list)}"
            )
        if int(gidx.shape[0]) != B:
            raise ValueError("group_index must have shape [B] matching new_token_batch")
        if gidx.size and ((gidx < 0) | (gidx >= G)).any():
            raise ValueError("group_index values must be in [0, num_groups)")
        L = self.dims.num_layers
        max_p = int(prefix_kv_grouped[0][0].shape[2]) if G else 0
        lens = [int(x) for x in prefix_lens_list]
        present = np.zeros(G, dtype=bool)
        present[gidx] = True
        for g in range(G):
            if present[g] and not 0 <= lens[g] <= max_p:
                raise ValueError(f"prefix_lens[{g}]={lens[g]} out of range for padded prefix length {max_p}")
        has_suffix = suffix_kv is not None and int(suffix_kv[0][0].shape[2]) > 0
        if has_suffix:
            smask = _np(suffix_mask, bool).reshape(B, -1)
            spos = _np(suffix_positions, np.int64).reshape(B, -1)
            s_max = int(smask.shape[1])
        else:
            smask = np.zeros((B, 0), bool)
            spos = np.zeros((B, 0), np.int64)
            s_max = 0
        lens_arr = np.asarray([min(max(x, 0), max_p) for x in lens], dtype=np.int64)
        # Page layout of the scratch pool: every group's prefix, then one
        # region holding each row's valid suffix tokens followed by itself.
        gp = -(-lens_arr // PAGE)
        gpage_off = np.concatenate([[0], np.cumsum(gp)]).astype(np.int64)
        n_valid = int(smask.sum())
        extra_tokens = n_valid + B
        region0 = int(gpage_off[-1])
        total_pages = max(region0 + -(-extra_tokens // PAGE), 1)
        pool = self._scratch_pool(total_pages)
        # extras: row r's valid suffix entries (in order), then its own slot
        per_row = smask.sum(axis=1).astype(np.int64) + 1
        extra_off = np.concatenate([[0], np.cumsum(per_row)]).astype(np.int64)
        tok_idx = np.arange(extra_tokens, dtype=np.int64)
        extra_slot = region0 * PAGE + tok_idx
        own_idx = extra_off[1:] - 1
        rr, cc = np.nonzero(smask)
        suffix_dst = np.setdiff1d(tok_idx, own_idx, assume_unique=True)  # in row-major order of (rr, cc)
        extra_pos = np.empty(extra_tokens, np.int64)
        extra_pos[own_idx] = pos
        extra_pos[suffix_dst] = spos[rr, cc]
        plan = StepPlan(
            piece_ids=piece_ids_from_tokens(tok),
            side_ids=side_ids_from_tokens(tok),
            positions=pos.astype(np.int32),
            row_group=gidx.astype(np.int32),
            row_vis=lens_arr[gidx].astype(np.int32) if B else np.zeros(0, np.int32),
            row_extra_off=extra_off.astype(np.int32),
            extra_slot=extra_slot.astype(np.int32),
            extra_pos=extra_pos.astype(np.int32),
            row_dst_slot=extra_slot[own_idx].astype(np.int32),
            group_page_off=gpage_off.astype(np.int32),
            group_pages=np.arange(region0, dtype=np.int32),
        )
        # Stage the caller's dense prefix stack and suffix tensors straight
        # into the scratch pool (one strided scatter per layer and tensor; the
        # index arrays go to the device in one copy).
        g_tok = np.concatenate([np.arange(n) for n in lens_arr]) if G else np.zeros(0, np.int64)
        g_of = np.repeat(np.arange(G), lens_arr)
        prefix_slots = (gpage_off[g_of] + g_tok // PAGE) * PAGE + g_tok % PAGE
        suffix_slots = region0 * PAGE + suffix_dst
        np_, ns_ = int(prefix_slots.size), int(suffix_slots.size) if has_suffix else 0
        idx = np.concatenate([prefix_slots, g_of, g_tok, suffix_slots[:ns_], rr[:ns_], cc[:ns_],
                              plan.row_dst_slot]).astype(np.int32)
        idx_d = torch.from_numpy(idx).to(self.device, non_blocking=True)
        o = 0
        p_slots, p_a, p_b = idx_d[o:o + np_], idx_d[o + np_:o + 2 * np_], idx_d[o + 2 * np_:o + 3 * np_]
        o += 3 * np_
        s_slots, s_a, s_b = idx_d[o:o + ns_], idx_d[o + ns_:o + 2 * ns_], idx_d[o + 2 * ns_:o + 3 * ns_]
        o += 3 * ns_
        own_t = idx_d[o:o + B]
        for l in range(L):
            if np_:
                pk, pv = prefix_kv_grouped[l]
                self._scatter_dense(pool, l, np_, p_slots, p_a, p_b, pk, pv)
            if ns_:
                sk, sv = suffix_kv[l]
                self._scatter_dense(pool, l, ns_, s_slots, s_a, s_b, sk, sv)
        out = self._run_dense(plan, pool)
        new_kv = []
        for l in range(L):
            k, v = self.kv_gather(pool, l, own_t)
            new_kv.append((k.unsqueeze(2), v.unsqueeze(2)))
        result: dict[str, Any] = {"logits": out["logits"], "kv": new_kv}
        if self.value_head is not None:
            result["value_logits"] = out["value_logits"]
        self.check_status()
        return result

    def _scratch_pool(self, num_pages: int) -> KVPool:
        """The dense-API entry points' scratch pool, reused across calls and
        grown (by a quarter more than asked) when a call needs more pages."""
        pool = getattr(self, "_scratch", None)
        if pool is None or pool.num_pages < num_pages:
            pool = self._scratch = self.new_pool(max(num_pages, int(num_pages * 1.25), 64))
        return pool

    def _scatter_dense(self, pool: KVPool, layer: int, n: int, slots, ia, ib, k: torch.Tensor,
                       v: torch.Tensor) -> None:
        """Rows (ia[r], :, ib[r], :) of dense [A, H, B, d] K / V tensors into
        ``slots`` of ``pool`` (imba_kv_scatter_indexed)."""
        if k.device != self.device or k.dtype != self.dtype:
            k = k.to(device=self.device, dtype=self.dtype)
        if v.device != self.device or v.dtype != self.dtype:
            v = v.to(device=self.device, dtype=self.dtype)
        # [A, H, B, d] tensors: strides in the order (a, b, head, dim)
        sk = (ctypes.c_int64 * 4)(k.stride(0), k.stride(2), k.stride(1), k.stride(3))
        sv = (ctypes.c_int64 * 4)(v.stride(0), v.stride(2), v.stride(1), v.stride(3))
        s = torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            code = self._lib.imba_kv_scatter_indexed(self._handle, ctypes.byref(pool.desc), layer, n,
                                                     slots.data_ptr(), ia.data_ptr(), ib.data_ptr(), k.data_ptr(),
                                                     v.data_ptr(), sk, sv, self._status.data_ptr(), s.cuda_stream)
        _native.check(code, "imba_kv_scatter_indexed")

    def _run_dense(self, plan: StepPlan, pool: KVPool) -> dict[str, torch.Tensor]:
        R = plan.num_rows
        logits = torch.empty((R, self.dims.vocab), dtype=torch.float32, device=self.device)
        value_logits = torch.empty((R, 3), dtype=torch.float32, device=self.device)
        if R:
            if getattr(self, "_buffers", None) is None:
                self._buffers = StepBuffers(self.device)
            dstep = self._buffers.stage(plan)  # reused pinned buffers: every dense call ends synchronised
            self.run(dstep, pool, logits=logits, value_logits=value_logits)
        return {"logits": logits, "value_logits": value_logits}
