"""B200-native (sm_100a) batched search-inference path of the imba-chess HSTU
model: jagged prefix prefill and grouped one-token decode against a paged
device KV pool, behind the reference's model decode API and actor-server
``service()`` contract.

The compute runs in the in-tree C-ABI library ``libimba_b200.so``
(include/imba_b200.h); this package is the host side.
"""

from .synth import ModelDims  # noqa: F401

__all__ = ["ModelDims", "B200HSTUChessModel", "ActorInferenceServer", "build"]


def __getattr__(name):
    if name == "B200HSTUChessModel":
        from .model import B200HSTUChessModel

        return B200HSTUChessModel
    if name == "ActorInferenceServer":
        from .server import ActorInferenceServer

        return ActorInferenceServer
    if name == "build":
        from .build import build

        return build
    raise AttributeError(name)
