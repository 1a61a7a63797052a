"""Import shims that let the reference imba-chess package load without its
optional dependencies.  TEST INFRASTRUCTURE ONLY: used by
``tests/golden/make_golden.py`` (fixture generation) and by ``bench.py``'s
reference arm (the reference's own decode path, timed as the baseline),
never by the product.

Three stand-ins, each written from the documented semantics of the missing
package rather than from its source:

* ``attn_gym.masks`` (attn_gym 0.0.4, pinned in the reference's uv.lock):
  the reference imports ``generate_prefix_lm_mask`` and
  ``generate_doc_mask_mod`` (src/imba_chess/model/hstu_model.py:9, :99-100).
  A prefix-LM mask with prefix length ``p`` lets query ``q`` see key ``k``
  when ``k <= q`` or ``k < p``; the document mask keeps a pair only when both
  indices fall in the same jagged document (``offsets``) and then applies the
  inner mask to document-local indices.
* ``chess`` / ``cozy_chess``: the decode and root paths of the reference's
  actor server never call chess code; permissive module stubs whose attributes
  are inert objects satisfy the module-level imports.
* ``TORCHDYNAMO_DISABLE=1``: the reference wraps ``create_block_mask`` in
  ``torch.compile``; with dynamo disabled it runs eagerly.

``install(reference_path)`` takes the directory that holds the reference's
``imba_chess`` package (its source tree's ``src`` or a pip ``--target``
install) and puts it first on ``sys.path``.
"""

from __future__ import annotations

import os
import sys
import types

class _Inert:
    """Object whose every attribute, call, index and iteration is inert."""

    def __init__(self, *a, **k):
        pass

    def __getattr__(self, name):
        if name.startswith("__") and name.endswith("__"):
            raise AttributeError(name)
        return _Inert()

    def __call__(self, *a, **k):
        return _Inert()

    def __getitem__(self, k):
        return _Inert()

    def __iter__(self):
        return iter(())

    def __or__(self, other):
        return self

    __ror__ = __and__ = __rand__ = __or__

    def __mro_entries__(self, bases):
        return (object,)


class _StubModule(types.ModuleType):
    def __getattr__(self, name):
        if name.startswith("__") and name.endswith("__"):
            raise AttributeError(name)
        return _Inert()


def _make_attn_gym():
    import torch

    def generate_prefix_lm_mask(prefix_length: int):
        def prefix_lm(b, h, q_idx, kv_idx):
            return (kv_idx <= q_idx) | (kv_idx < prefix_length)

        return prefix_lm

    def generate_doc_mask_mod(mask_mod, offsets):
        offsets = offsets.to(torch.long)
        total = int(offsets[-1].item())
        lengths = offsets[1:] - offsets[:-1]
        doc_of = torch.repeat_interleave(
            torch.arange(lengths.numel(), device=offsets.device), lengths
        )
        if doc_of.numel() < total:  # defensive: never for well-formed offsets
            doc_of = torch.nn.functional.pad(doc_of, (0, total - doc_of.numel()))

        def doc_mask(b, h, q_idx, kv_idx):
            same = doc_of[q_idx] == doc_of[kv_idx]
            q_local = q_idx - offsets[doc_of[q_idx]]
            kv_local = kv_idx - offsets[doc_of[kv_idx]]
            return same & mask_mod(b, h, q_local, kv_local)

        return doc_mask

    pkg = types.ModuleType("attn_gym")
    masks = types.ModuleType("attn_gym.masks")
    masks.generate_prefix_lm_mask = generate_prefix_lm_mask
    masks.generate_doc_mask_mod = generate_doc_mask_mod
    pkg.masks = masks
    return pkg, masks


def install(reference_path: str) -> None:
    """Install the shims and put ``reference_path`` (the directory holding
    the reference's ``imba_chess`` package) first on ``sys.path``."""
    if not os.path.isdir(os.path.join(reference_path, "imba_chess")):
        raise FileNotFoundError(f"no imba_chess package under {reference_path}")
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    if "attn_gym" not in sys.modules:
        pkg, masks = _make_attn_gym()
        sys.modules["attn_gym"] = pkg
        sys.modules["attn_gym.masks"] = masks
    for name in ("chess", "cozy_chess"):
        if name not in sys.modules:
            mod = _StubModule(name)
            mod.__path__ = []  # a package, so ``import chess.engine`` resolves below
            sys.modules[name] = mod
    for sub in ("engine", "pgn", "svg", "polyglot"):
        full = f"chess.{sub}"
        if full not in sys.modules:
            sys.modules[full] = _StubModule(full)
            setattr(sys.modules["chess"], sub, sys.modules[full])
    if reference_path not in sys.path:
        sys.path.insert(0, reference_path)
