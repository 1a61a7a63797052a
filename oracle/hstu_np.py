"""CPU oracle: a numpy (float32) restatement of the reference HSTU chess
model's inference paths.

TEST INFRASTRUCTURE ONLY.  This module is the oracle the CUDA path is tested
against: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may import it.  The product (``imba_chess_b200``) never
does.

Pinned against the reference itself: ``tests/golden/make_golden.py`` imports
the reference package, runs it on seeded weights and inputs, and stores its
outputs in ``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this
module against every stored case.

Every function follows one reference function, cited by file:line of the
reference tree (src/imba_chess/...).  All arithmetic is float32, as in the
reference's fp32 CPU path.
"""

from __future__ import annotations

import math
from typing import Any

import numpy as np

F32 = np.float32
BOARD_DIM = 64
BOARD_HEADS = 4
BOARD_LAYERS = 2


def layer_norm(x: np.ndarray, eps: float, weight=None, bias=None) -> np.ndarray:
    """``F.layer_norm`` over the last dim (biased variance)."""
    x = x.astype(F32, copy=False)
    mu = x.mean(axis=-1, keepdims=True, dtype=F32)
    xc = x - mu
    var = (xc * xc).mean(axis=-1, keepdims=True, dtype=F32)
    y = xc / np.sqrt(var + F32(eps))
    if weight is not None:
        y = y * weight + bias
    return y.astype(F32, copy=False)


def silu(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (x / (F32(1.0) + np.exp(-x))).astype(F32, copy=False)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    m = np.max(x, axis=axis, keepdims=True)
    m = np.where(np.isfinite(m), m, F32(0.0))
    e = np.exp(x - m)
    return (e / e.sum(axis=axis, keepdims=True)).astype(F32, copy=False)


def log_softmax_f32(raw: np.ndarray) -> np.ndarray:
    """Legal-move log-priors: float64 max-shift + log-sum-exp, rounded to
    float32 at the end (src/imba_chess/eval/actor_worker.py:267-291)."""
    raw = np.asarray(raw, dtype=np.float64)
    if raw.size == 0:
        return raw.astype(F32)
    shifted = raw - raw.max()
    return (shifted - np.log(np.exp(shifted).sum())).astype(F32)


def value_stm(value_logits: np.ndarray) -> np.ndarray:
    """``v = softmax(value_logits)[2] - softmax(value_logits)[0]`` in float32
    (src/imba_chess/eval/actor_server.py:168-173; class 0 = loss, 2 = win)."""
    p = softmax(np.asarray(value_logits, dtype=F32), axis=-1)
    return (p[:, 2] - p[:, 0]).astype(F32)


def gather_legal(logits: np.ndarray, legal_ids: list) -> list[np.ndarray]:
    """Raw logits at each row's legal ids, in the given order
    (src/imba_chess/eval/actor_server.py:176-203)."""
    return [logits[r, np.asarray(ids, dtype=np.int64)] for r, ids in enumerate(legal_ids)]


class OracleModel:
    """Inference-only restatement of ``HSTUChessModel``
    (src/imba_chess/model/hstu_model.py:182-752) over a float32 state dict
    with the reference's key names."""

    def __init__(self, state_dict: dict[str, np.ndarray], dims: Any) -> None:
        self.sd = {k: np.asarray(v, dtype=F32) for k, v in state_dict.items()}
        self.dims = dims
        self.d = int(dims.model_dim)
        self.L = int(dims.num_layers)
        self.H = int(dims.num_heads)
        self.dqk = int(dims.attention_dim)
        self.dv = int(dims.linear_dim)
        self.max_pos = int(dims.max_pos)
        self.has_value = bool(dims.value_head)

    # ------------------------------------------------------------------
    # Content embedding (hstu_model.py:113-179, :275-335)
    # ------------------------------------------------------------------
    def board_encoder(self, piece_ids: np.ndarray, chunk: int = 256) -> np.ndarray:
        """``BoardSquareEncoder`` over the joint (piece, square) table:
        ``pair = piece*64 + square`` (hstu_model.py:275-278), two pre-LN
        square-attention blocks (:118-144), final LN, mean over squares,
        ``out_proj`` (:170-179)."""
        n = piece_ids.shape[0]
        out = np.empty((n, self.d), dtype=F32)
        for s in range(0, n, chunk):
            out[s : s + chunk] = self._board_chunk(piece_ids[s : s + chunk])
        return out

    def _board_chunk(self, piece_ids: np.ndarray) -> np.ndarray:
        sd = self.sd
        n = piece_ids.shape[0]
        pair = piece_ids.astype(np.int64) * 64 + np.arange(64)
        x = sd["piece_square_embedding.weight"][pair]  # [n, 64, 64]
        hd = BOARD_DIM // BOARD_HEADS
        for b in range(BOARD_LAYERS):
            p = f"board_encoder.blocks.{b}."
            h = layer_norm(x, 1e-5, sd[p + "attn_norm.weight"], sd[p + "attn_norm.bias"])
            qkv = h @ sd[p + "qkv.weight"].T  # [n, 64, 192]
            qkv = qkv.reshape(n, 64, 3, BOARD_HEADS, hd).transpose(2, 0, 3, 1, 4)
            q, k, v = qkv[0], qkv[1], qkv[2]  # [n, 4, 64, 16]
            s = (q @ k.transpose(0, 1, 3, 2)) * F32(1.0 / math.sqrt(hd))
            a = softmax(s) @ v
            a = a.transpose(0, 2, 1, 3).reshape(n, 64, BOARD_DIM)
            x = x + a @ sd[p + "attn_out.weight"].T
            h = layer_norm(x, 1e-5, sd[p + "mlp_norm.weight"], sd[p + "mlp_norm.bias"])
            m = silu(h @ sd[p + "mlp.0.weight"].T + sd[p + "mlp.0.bias"])
            x = x + (m @ sd[p + "mlp.2.weight"].T + sd[p + "mlp.2.bias"])
        h = layer_norm(x, 1e-5, sd["board_encoder.final_norm.weight"], sd["board_encoder.final_norm.bias"])
        pooled = h.mean(axis=1, dtype=F32)
        return pooled @ sd["board_encoder.out_proj.weight"].T + sd["board_encoder.out_proj.bias"]

    def content(self, tok: dict[str, np.ndarray]) -> np.ndarray:
        """``_build_content``: board vector plus seven clamped side-feature
        embeddings, summed left to right (hstu_model.py:283-335)."""
        sd = self.sd

        def emb(name: str, ids) -> np.ndarray:
            table = sd[name]
            return table[np.clip(np.asarray(ids, dtype=np.int64), 0, table.shape[0] - 1)]

        x = self.board_encoder(np.asarray(tok["piece_ids"]))
        x = x + emb("seq_token_embedding.weight", tok["seq_token_id"])
        x = x + emb("turn_embedding.weight", tok["turn_id"])
        x = x + emb("castle_embedding.weight", tok["castle_id"])
        x = x + emb("ep_embedding.weight", tok["ep_file_id"])
        x = x + emb("halfmove_embedding.weight", tok["halfmove_bucket_id"])
        x = x + emb("fullmove_embedding.weight", tok["fullmove_bucket_id"])
        x = x + emb("prev_move_embedding.weight", tok["prev_move_id"])
        return x.astype(F32, copy=False)

    def at_positions(self, content: np.ndarray, positions) -> np.ndarray:
        """``content * sqrt(d) + pos_emb[min(pos, max-1)]``
        (src/imba_chess/model/position_embedding.py:52-62, :34-50)."""
        pos = np.minimum(np.asarray(positions, dtype=np.int64), self.max_pos - 1)
        scale = F32(self.d ** 0.5)
        return (content * scale + self.sd["position_embedding.embedding.weight"][pos]).astype(F32)

    # ------------------------------------------------------------------
    # STU layer pieces (src/imba_chess/model/hstu_attention.py)
    # ------------------------------------------------------------------
    def uvqk(self, layer: int, x: np.ndarray):
        """LN (no affine, eps 1e-6) -> ``_uvqk`` -> SiLU -> split u, v, q, k
        (hstu_attention.py:307-325)."""
        n = x.shape[0]
        h = layer_norm(x, 1e-6)
        y = silu(h @ self.sd[f"layers.{layer}._uvqk.weight"].T)
        H, dv, dqk = self.H, self.dv, self.dqk
        u = y[:, : H * dv]
        v = y[:, H * dv : 2 * H * dv].reshape(n, H, dv)
        q = y[:, 2 * H * dv : 2 * H * dv + H * dqk].reshape(n, H, dqk)
        k = y[:, 2 * H * dv + H * dqk :].reshape(n, H, dqk)
        return u, v, q, k

    def out_proj(self, layer: int, x: np.ndarray, attn: np.ndarray, u: np.ndarray) -> np.ndarray:
        """LN(attn) (no affine, eps 1e-6) gated by u -> ``_o`` + bias ->
        + residual (hstu_attention.py:415-424)."""
        a = layer_norm(attn, 1e-6)
        o = (u * a) @ self.sd[f"layers.{layer}._o.weight"].T + self.sd[f"layers.{layer}._o.bias"]
        return (o + x).astype(F32)

    def rel_bias(self, layer: int, k_pos: np.ndarray, q_pos) -> np.ndarray:
        """Per-head bias ``ps_w[h, clamp(k - q + max - 1, 0, 2max - 2)]``
        (hstu_attention.py:64-76, :134-148).  Returns ``[H, ...]``."""
        idx = np.clip(
            np.asarray(k_pos, dtype=np.int64) - np.asarray(q_pos, dtype=np.int64) + (self.max_pos - 1),
            0,
            2 * self.max_pos - 2,
        )
        return self.sd[f"layers.{layer}._ps_w"][:, idx]

    def heads(self, x: np.ndarray):
        """final LN (affine, eps 1e-5) -> tied policy head; value MLP
        (hstu_model.py:367-378, :745-751)."""
        sd = self.sd
        xf = layer_norm(x, 1e-5, sd["final_norm.weight"], sd["final_norm.bias"])
        logits = xf @ sd["prediction_head.weight"].T
        value = None
        if self.has_value:
            h = silu(xf @ sd["value_head.0.weight"].T + sd["value_head.0.bias"])
            value = (h @ sd["value_head.2.weight"].T + sd["value_head.2.bias"]).astype(F32)
        return logits.astype(F32), value

    # ------------------------------------------------------------------
    # Prefill: forward(return_kv=True) (hstu_model.py:337-374,
    # hstu_attention.py:81-132): per-document causal softmax attention.
    # ------------------------------------------------------------------
    def forward(self, tok: dict[str, np.ndarray], seq_offsets) -> dict[str, Any]:
        offsets = np.asarray(seq_offsets, dtype=np.int64)
        S = int(offsets[-1])
        lengths = offsets[1:] - offsets[:-1]
        starts = np.repeat(offsets[:-1], lengths)
        positions = np.arange(S) - starts
        x = self.at_positions(self.content(tok), positions)
        scale = F32(self.dqk ** -0.5)
        kv_caches = []
        for l in range(self.L):
            u, v, q, k = self.uvqk(l, x)
            attn = np.zeros((S, self.H, self.dv), dtype=F32)
            for di in range(len(lengths)):
                a, b = int(offsets[di]), int(offsets[di + 1])
                if b == a:
                    continue
                T = b - a
                qi = np.arange(T)
                bias = self.rel_bias(l, qi[None, :], qi[:, None])  # [H, T(q), T(k)]
                causal = qi[None, :] <= qi[:, None]
                for h in range(self.H):
                    s = (q[a:b, h] @ k[a:b, h].T) * scale + bias[h]
                    s = np.where(causal, s, F32(-np.inf))
                    attn[a:b, h] = softmax(s) @ v[a:b, h]
            x = self.out_proj(l, x, attn.reshape(S, -1), u)
            kv_caches.append((k.transpose(1, 0, 2).copy(), v.transpose(1, 0, 2).copy()))
        logits, value = self.heads(x)
        out = {"logits": logits, "policy_logits": logits, "kv_caches": kv_caches}
        if value is not None:
            out["value_logits"] = value
        return out

    # ------------------------------------------------------------------
    # Decode against cached K/V.
    # ------------------------------------------------------------------
    def _attend_rows(self, layer, q, k_new, v_new, q_pos, pk, pv, plen, sk, sv, spos, smask):
        """One group's rows: scores over [prefix | masked suffix | self],
        float32 softmax, weighted sum (hstu_attention.py:358-411)."""
        n = q.shape[0]
        scale = F32(self.dqk ** -0.5)
        out = np.zeros((n, self.H, self.dv), dtype=F32)
        for r in range(n):
            kpos = np.arange(plen)
            parts_bias = [self.rel_bias(layer, kpos, q_pos[r])]  # [H, P]
            for h in range(self.H):
                scores = [(pk[h, :plen] @ q[r, h]) * scale + parts_bias[0][h]]
                vals = [pv[h, :plen]]
                if sk is not None and sk.shape[2] > 0:
                    sb = self.rel_bias(layer, spos[r], q_pos[r])[h]
                    ss = (sk[r, h] @ q[r, h]) * scale + sb
                    ss = np.where(smask[r], ss, F32(-np.inf))
                    scores.append(ss)
                    vals.append(sv[r, h])
                self_s = F32(np.dot(q[r, h], k_new[r, h])) * scale + self.sd[f"layers.{layer}._ps_w"][h, self.max_pos - 1]
                scores.append(np.array([self_s], dtype=F32))
                vals.append(v_new[r, h][None, :])
                w = softmax(np.concatenate(scores).astype(F32))
                out[r, h] = w @ np.concatenate(vals, axis=0)
        return out

    def forward_decode_grouped(
        self,
        *,
        new_token_batch: dict[str, np.ndarray],
        positions,
        group_index,
        prefix_kv_grouped: list,
        prefix_lens_list: list[int],
        suffix_kv: list | None = None,
        suffix_positions=None,
        suffix_mask=None,
    ) -> dict[str, Any]:
        """``HSTUChessModel.forward_decode_grouped`` (hstu_model.py:651-752)
        with ``SequentialTransductionUnitJagged.forward_decode_grouped``
        (hstu_attention.py:259-424) per layer: rows read only their own
        group's real (unpadded) prefix slice."""
        positions = np.asarray(positions, dtype=np.int64)
        group_index = np.asarray(group_index, dtype=np.int64)
        G = len(prefix_lens_list)
        if group_index.shape[0] and ((group_index < 0) | (group_index >= G)).any():
            raise ValueError("group_index values must be in [0, num_groups)")
        x = self.at_positions(self.content(new_token_batch), positions)
        n = x.shape[0]
        new_kv = []
        for l in range(self.L):
            u, v_new, q, k_new = self.uvqk(l, x)
            pk, pv = prefix_kv_grouped[l]
            sk, sv = (suffix_kv[l] if suffix_kv is not None else (None, None))
            attn = np.zeros((n, self.H, self.dv), dtype=F32)
            for g in range(G):
                rows = np.nonzero(group_index == g)[0]
                if rows.size == 0:
                    continue
                plen = int(prefix_lens_list[g])
                if not 0 <= plen <= pk.shape[2]:
                    raise ValueError(f"prefix_lens[{g}]={plen} out of range for padded prefix length {pk.shape[2]}")
                attn[rows] = self._attend_rows(
                    l, q[rows], k_new[rows], v_new[rows], positions[rows], pk[g], pv[g], plen,
                    None if sk is None else sk[rows], None if sv is None else sv[rows],
                    None if suffix_positions is None else np.asarray(suffix_positions)[rows],
                    None if suffix_mask is None else np.asarray(suffix_mask)[rows],
                )
            x = self.out_proj(l, x, attn.reshape(n, -1), u)
            new_kv.append((k_new[:, :, None, :].copy(), v_new[:, :, None, :].copy()))
        logits, value = self.heads(x)
        out = {"logits": logits, "kv": new_kv}
        if value is not None:
            out["value_logits"] = value
        return out

    def forward_decode(
        self,
        *,
        new_token_batch: dict[str, np.ndarray],
        positions,
        prefix_kv: list,
        suffix_kv: list | None = None,
        suffix_positions=None,
        suffix_mask=None,
    ) -> dict[str, Any]:
        """``HSTUChessModel.forward_decode`` (hstu_model.py:600-649): one
        shared prefix ``[H, T, d]`` per layer for every row."""
        n = int(np.asarray(positions).shape[0])
        grouped = [(k[None], v[None]) for k, v in prefix_kv]
        T = int(prefix_kv[0][0].shape[1]) if prefix_kv else 0
        return self.forward_decode_grouped(
            new_token_batch=new_token_batch,
            positions=positions,
            group_index=np.zeros(n, dtype=np.int64),
            prefix_kv_grouped=grouped,
            prefix_lens_list=[T],
            suffix_kv=suffix_kv,
            suffix_positions=suffix_positions,
            suffix_mask=suffix_mask,
        )


class KVArenaOracle:
    """Logical row numbering of the reference's per-turn decode arena
    (``_KVArena``, src/imba_chess/eval/actor_server.py:206-280): rows are
    minted consecutively in wave order by ``append``; capacity starts at
    ``max(n, 16)`` and doubles until it fits; ``gather_suffix`` reads rows by
    index.  Payload is ``[L, H, capacity, d]`` for k and v."""

    def __init__(self, k_rows: np.ndarray, v_rows: np.ndarray) -> None:
        cap = max(int(k_rows.shape[2]), 16)
        self.k = np.zeros(k_rows.shape[:2] + (cap,) + k_rows.shape[3:], dtype=k_rows.dtype)
        self.v = np.zeros(v_rows.shape[:2] + (cap,) + v_rows.shape[3:], dtype=v_rows.dtype)
        self.size = 0

    def _ensure_capacity(self, extra: int) -> None:
        needed = self.size + extra
        cap = self.k.shape[2]
        if needed <= cap:
            return
        new_cap = max(cap, 1)
        while new_cap < needed:
            new_cap *= 2
        for name in ("k", "v"):
            old = getattr(self, name)
            new = np.zeros(old.shape[:2] + (new_cap,) + old.shape[3:], dtype=old.dtype)
            new[:, :, : self.size] = old[:, :, : self.size]
            setattr(self, name, new)

    def append(self, k_rows: np.ndarray, v_rows: np.ndarray) -> list[int]:
        n = int(k_rows.shape[2])
        self._ensure_capacity(n)
        start = self.size
        self.k[:, :, start : start + n] = k_rows
        self.v[:, :, start : start + n] = v_rows
        self.size += n
        return list(range(start, start + n))

    def gather_suffix(self, idx: np.ndarray):
        """``[B, S]`` row ids -> per-layer ``([B, H, S, d], [B, H, S, d])``."""
        gk = self.k[:, :, idx, :].transpose(0, 2, 1, 3, 4)
        gv = self.v[:, :, idx, :].transpose(0, 2, 1, 3, 4)
        return [(gk[l], gv[l]) for l in range(gk.shape[0])]


def wave_suffix_index(parent_chains: list[list[int]]):
    """Suffix index/mask matrices a wave builds from its rows' parent chains:
    row r holds ``chain_r`` left-aligned, padded with row 0 and mask False
    (src/imba_chess/eval/actor_server.py:827-856)."""
    b = len(parent_chains)
    s = max((len(c) for c in parent_chains), default=0)
    idx = np.zeros((b, s), dtype=np.int64)
    mask = np.zeros((b, s), dtype=bool)
    for r, chain in enumerate(parent_chains):
        idx[r, : len(chain)] = chain
        mask[r, : len(chain)] = True
    return idx, mask
