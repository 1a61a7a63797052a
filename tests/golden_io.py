"""Loaders for the committed golden fixtures (tests/golden/)."""

from __future__ import annotations

import json
import os

import numpy as np

from imba_chess_b200 import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TINY_SEED = 7
SMALL_SEED = 11


def load(name: str) -> dict[str, np.ndarray]:
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


def load_session() -> dict:
    with open(os.path.join(GOLDEN, "server_session.json")) as f:
        return json.load(f)


def tokens(g: dict, tag: str) -> dict[str, np.ndarray]:
    return {k: g[f"{tag}/tok/{k}"] for k in synth.TOKEN_FIELDS}


def kv_list(g: dict, tag: str, kind: str, layers: int):
    return [(g[f"{tag}/{kind}/{l}/k"], g[f"{tag}/{kind}/{l}/v"]) for l in range(layers)]


def grouped_inputs(g: dict, tag: str, layers: int) -> dict:
    has_suffix = f"{tag}/suffix_positions" in g
    return dict(
        new_token_batch=tokens(g, tag),
        positions=g[f"{tag}/positions"],
        group_index=g[f"{tag}/group_index"],
        prefix_kv_grouped=kv_list(g, tag, "prefix", layers),
        prefix_lens_list=[int(x) for x in g[f"{tag}/prefix_lens"]],
        suffix_kv=kv_list(g, tag, "suffix", layers) if has_suffix else None,
        suffix_positions=g.get(f"{tag}/suffix_positions"),
        suffix_mask=g.get(f"{tag}/suffix_mask"),
    )


def tiny_weights():
    return synth.TINY, synth.make_state_dict(synth.TINY, TINY_SEED, profile="sharp")


def small_weights():
    return synth.SMALL, synth.make_state_dict(synth.SMALL, SMALL_SEED, profile="sharp")
