"""Pack a reference-layout state dict into device tensors and the C-ABI
``imba_model_desc``.

Accepts the reference's parameter names (``HSTUChessModel.state_dict()``,
src/imba_chess/model/hstu_model.py:185-273) with the ``module.`` /
``_orig_mod.`` prefixes that ``load_hstu_checkpoint`` strips
(src/imba_chess/eval/position_evaluator.py:136-145).  Architecture sizes are
read off the tensor shapes.  All tables stay fp32; the GEMM weights are
stored in the model dtype, and for bf16 the tied policy matrix is split into
a bf16 high part and a bf16 residual, laid out [hi | hi | lo] along K, so the
policy GEMM against [x_hi | x_lo | x_hi] keeps ~16 mantissa bits.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Mapping

import numpy as np
import torch

from . import _native

BOARD_BLOCK_KEYS = (
    "attn_norm.weight",
    "attn_norm.bias",
    "qkv.weight",
    "attn_out.weight",
    "mlp_norm.weight",
    "mlp_norm.bias",
    "mlp.0.weight",
    "mlp.0.bias",
    "mlp.2.weight",
    "mlp.2.bias",
)


@dataclass(frozen=True)
class Dims:
    model_dim: int
    num_layers: int
    num_heads: int
    attention_dim: int
    linear_dim: int
    vocab: int
    max_pos: int
    halfmove_vocab: int
    fullmove_vocab: int
    value_head: bool


def normalize_state_dict(state_dict: Mapping[str, Any]) -> dict[str, torch.Tensor]:
    out: dict[str, torch.Tensor] = {}
    for key, value in state_dict.items():
        if not isinstance(key, str):
            raise TypeError("state_dict keys must be strings")
        k = key
        if k.startswith("module."):
            k = k[len("module.") :]
        if k.startswith("_orig_mod."):
            k = k[len("_orig_mod.") :]
        t = value if isinstance(value, torch.Tensor) else torch.from_numpy(np.asarray(value))
        out[k] = t.detach()
    return out


def load_checkpoint_state_dict(path, *, require_value_head: bool = False) -> dict[str, torch.Tensor]:
    """A checkpoint file's normalised state dict, read like the reference's
    ``load_hstu_checkpoint`` (src/imba_chess/eval/position_evaluator.py:118-167):
    a plain state dict or an Ignite checkpoint holding it under ``"model"``
    (``TypeError`` otherwise), ``module.`` / ``_orig_mod.`` prefixes stripped,
    ``ValueError`` when a value head is required but absent, and a strict
    key / shape check against the architecture the tensors describe
    (``RuntimeError`` listing missing, unexpected and mis-shaped keys, as
    ``load_state_dict(strict=True)`` would)."""
    checkpoint = torch.load(path, map_location="cpu")
    state_dict = checkpoint["model"] if isinstance(checkpoint, dict) and "model" in checkpoint else checkpoint
    if not isinstance(state_dict, dict):
        raise TypeError("Checkpoint must be a model state_dict or Ignite checkpoint containing key 'model'.")
    for key in state_dict:
        if not isinstance(key, str):
            raise TypeError("Checkpoint state_dict keys must be strings")
    sd = normalize_state_dict(state_dict)
    has_value = any(k.startswith("value_head.") for k in sd)
    if require_value_head and not has_value:
        raise ValueError(
            "model_move_policy in {value_rerank,value_search_d2} requires a checkpoint with value_head "
            "parameters, but checkpoint contains no 'value_head.*' keys."
        )
    check_state_dict(sd)
    return sd


def check_state_dict(sd: Mapping[str, torch.Tensor]) -> None:
    """Strict key and shape check of a normalised state dict against the
    reference architecture its tensors describe."""
    from .synth import ModelDims, state_dict_shapes

    dims = infer_dims(sd)
    expected = state_dict_shapes(ModelDims(
        model_dim=dims.model_dim, num_layers=dims.num_layers, num_heads=dims.num_heads,
        attention_dim=dims.attention_dim, linear_dim=dims.linear_dim, vocab=dims.vocab, max_pos=dims.max_pos,
        halfmove_vocab=dims.halfmove_vocab, fullmove_vocab=dims.fullmove_vocab, value_head=dims.value_head))
    missing = [k for k in expected if k not in sd]
    unexpected = [k for k in sd if k not in expected]
    shapes = [f"{k}: {tuple(sd[k].shape)} vs {v}" for k, v in expected.items() if k in sd and tuple(sd[k].shape) != v]
    if missing or unexpected or shapes:
        parts = []
        if missing:
            parts.append("Missing key(s): " + ", ".join(missing))
        if unexpected:
            parts.append("Unexpected key(s): " + ", ".join(unexpected))
        if shapes:
            parts.append("Size mismatch: " + "; ".join(shapes))
        raise RuntimeError("Error(s) in loading state_dict for HSTUChessModel: " + " | ".join(parts))


def infer_dims(sd: Mapping[str, torch.Tensor]) -> Dims:
    d = int(sd["final_norm.weight"].shape[0])
    L = 0
    while f"layers.{L}._uvqk.weight" in sd:
        L += 1
    if L == 0:
        raise ValueError("state dict has no STU layers")
    H = int(sd["layers.0._ps_w"].shape[0])
    max_pos = (int(sd["layers.0._ps_w"].shape[1]) + 1) // 2
    dv = int(sd["layers.0._o.weight"].shape[1]) // H
    uvqk_rows = int(sd["layers.0._uvqk.weight"].shape[0])
    dqk = uvqk_rows // (2 * H) - dv
    vocab_key = "prediction_head.weight" if "prediction_head.weight" in sd else "prev_move_embedding.weight"
    return Dims(
        model_dim=d,
        num_layers=L,
        num_heads=H,
        attention_dim=dqk,
        linear_dim=dv,
        vocab=int(sd[vocab_key].shape[0]),
        max_pos=max_pos,
        halfmove_vocab=int(sd["halfmove_embedding.weight"].shape[0]),
        fullmove_vocab=int(sd["fullmove_embedding.weight"].shape[0]),
        value_head="value_head.0.weight" in sd,
    )


class PackedWeights:
    """Device copies of every weight plus the filled ``ModelDesc``.  Owns the
    tensors the descriptor points into; keep it alive as long as the native
    handle."""

    def __init__(self, state_dict: Mapping[str, Any], *, dtype: torch.dtype, device: torch.device) -> None:
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError(f"unsupported dtype {dtype}: use torch.float32 or torch.bfloat16")
        sd = normalize_state_dict(state_dict)
        self.dims = infer_dims(sd)
        self.dtype = dtype
        self.device = device
        dims = self.dims
        self._keep: list[torch.Tensor] = []

        def f32(name: str) -> torch.Tensor:
            t = sd[name].to(device=device, dtype=torch.float32).contiguous()
            self._keep.append(t)
            return t

        def wdt(t: torch.Tensor) -> torch.Tensor:
            t = t.to(device=device, dtype=torch.float32).to(dtype).contiguous()
            self._keep.append(t)
            return t

        board = []
        for b in range(2):
            for k in BOARD_BLOCK_KEYS:
                board.append(sd[f"board_encoder.blocks.{b}.{k}"].to(torch.float32).reshape(-1))
        board.append(sd["board_encoder.final_norm.weight"].to(torch.float32).reshape(-1))
        board.append(sd["board_encoder.final_norm.bias"].to(torch.float32).reshape(-1))
        board_params = torch.cat(board).to(device).contiguous()
        if board_params.numel() != _native.BOARD_PARAM_FLOATS:
            raise ValueError("board encoder parameters have unexpected shapes")
        self._keep.append(board_params)

        desc = _native.ModelDesc()
        desc.model_dim = dims.model_dim
        desc.num_layers = dims.num_layers
        desc.num_heads = dims.num_heads
        desc.attention_dim = dims.attention_dim
        desc.linear_dim = dims.linear_dim
        desc.vocab = dims.vocab
        desc.max_pos = dims.max_pos
        desc.halfmove_vocab = dims.halfmove_vocab
        desc.fullmove_vocab = dims.fullmove_vocab
        desc.has_value_head = int(dims.value_head)
        desc.dtype = _native.DTYPE_BF16 if dtype == torch.bfloat16 else _native.DTYPE_F32
        desc.piece_square = f32("piece_square_embedding.weight").data_ptr()
        desc.board_params = board_params.data_ptr()
        desc.board_out_w = f32("board_encoder.out_proj.weight").data_ptr()
        desc.board_out_b = f32("board_encoder.out_proj.bias").data_ptr()
        desc.emb_seq = f32("seq_token_embedding.weight").data_ptr()
        desc.emb_turn = f32("turn_embedding.weight").data_ptr()
        desc.emb_castle = f32("castle_embedding.weight").data_ptr()
        desc.emb_ep = f32("ep_embedding.weight").data_ptr()
        desc.emb_halfmove = f32("halfmove_embedding.weight").data_ptr()
        desc.emb_fullmove = f32("fullmove_embedding.weight").data_ptr()
        prev = f32("prev_move_embedding.weight")
        desc.emb_prev_move = prev.data_ptr()
        desc.emb_pos = f32("position_embedding.embedding.weight").data_ptr()
        if dims.num_layers > _native.MAX_LAYERS:
            raise ValueError(f"at most {_native.MAX_LAYERS} layers are supported")
        for l in range(dims.num_layers):
            desc.uvqk_w[l] = wdt(sd[f"layers.{l}._uvqk.weight"]).data_ptr()
            desc.o_w[l] = wdt(sd[f"layers.{l}._o.weight"]).data_ptr()
            desc.o_b[l] = f32(f"layers.{l}._o.bias").data_ptr()
            desc.ps_w[l] = f32(f"layers.{l}._ps_w").data_ptr()
        desc.final_norm_w = f32("final_norm.weight").data_ptr()
        desc.final_norm_b = f32("final_norm.bias").data_ptr()
        policy = sd.get("prediction_head.weight", sd["prev_move_embedding.weight"]).to(device=device, dtype=torch.float32)
        policy = policy.contiguous()
        self._keep.append(policy)
        desc.policy_w32 = policy.data_ptr()
        if dtype == torch.bfloat16:
            hi = policy.to(torch.bfloat16)
            lo = (policy - hi.float()).to(torch.bfloat16)
            split = torch.cat([hi, hi, lo], dim=1).contiguous()  # [vocab, 3d]
            self._keep.append(split)
            desc.policy_w = split.data_ptr()
        else:
            desc.policy_w = policy.data_ptr()
        if dims.value_head:
            desc.value0_w = wdt(sd["value_head.0.weight"]).data_ptr()
            desc.value0_b = f32("value_head.0.bias").data_ptr()
            desc.value2_w = f32("value_head.2.weight").data_ptr()
            desc.value2_b = f32("value_head.2.bias").data_ptr()
        self.desc = desc
