"""CPU: reading reference checkpoint files like ``load_hstu_checkpoint``
(src/imba_chess/eval/position_evaluator.py:118-167)."""

from __future__ import annotations

import pytest
import torch

from imba_chess_b200 import synth
from imba_chess_b200.weights import infer_dims, load_checkpoint_state_dict


def _sd(value_head=True):
    dims = synth.ModelDims(128, 2, 2, max_pos=48, value_head=value_head)
    return dims, {k: torch.from_numpy(v) for k, v in synth.make_state_dict(dims, 4, profile="reference").items()}


def test_ignite_checkpoint_with_prefixes(tmp_path):
    dims, sd = _sd()
    path = tmp_path / "ckpt.pt"
    torch.save({"model": {"module._orig_mod." + k: v for k, v in sd.items()}, "optimizer": {}}, path)
    out = load_checkpoint_state_dict(path, require_value_head=True)
    assert set(out) == set(sd)
    assert all(torch.equal(out[k], sd[k]) for k in sd)
    d = infer_dims(out)
    assert (d.model_dim, d.num_layers, d.num_heads, d.max_pos, d.value_head) == (128, 2, 2, 48, True)


def test_plain_state_dict_and_guards(tmp_path):
    dims, sd = _sd(value_head=False)
    path = tmp_path / "plain.pt"
    torch.save(sd, path)
    assert set(load_checkpoint_state_dict(path)) == set(sd)
    with pytest.raises(ValueError, match="value_head"):
        load_checkpoint_state_dict(path, require_value_head=True)
    bad = tmp_path / "bad.pt"
    torch.save([1, 2, 3], bad)
    with pytest.raises(TypeError, match="Ignite"):
        load_checkpoint_state_dict(bad)


def test_strict_key_and_shape_check(tmp_path):
    dims, sd = _sd()
    extra = dict(sd, **{"stray.weight": torch.zeros(3)})
    torch.save(extra, tmp_path / "extra.pt")
    with pytest.raises(RuntimeError, match="Unexpected key"):
        load_checkpoint_state_dict(tmp_path / "extra.pt")
    missing = {k: v for k, v in sd.items() if not k.startswith("moves_left_head.")}
    torch.save(missing, tmp_path / "missing.pt")
    with pytest.raises(RuntimeError, match="Missing key"):
        load_checkpoint_state_dict(tmp_path / "missing.pt")
    wrong = dict(sd)
    wrong["final_norm.bias"] = torch.zeros(7)
    torch.save(wrong, tmp_path / "wrong.pt")
    with pytest.raises(RuntimeError, match="Size mismatch"):
        load_checkpoint_state_dict(tmp_path / "wrong.pt")
