"""B200-native CUDA carrier for StrideWeave: contraction and reduction on
sm_100a kernels behind the reference's Carrier / Operation plugin API.

    from strideweave_b200 import CUDA, mx
    t = sw.Tensor(CUDA.from_numpy(x), 0, layout)      # HBM-resident tensor
    sw.reduce_max(t, "a b -> a")                       # dispatches to the GPU
    q = mx.quantize(t, "MXFP8_E4M3")                   # MX multi-sub-tensor
    c = mx.matmul(q, q)                                # tcgen05 block-scaled

Submodules are imported lazily so that the build recipe
(``strideweave_b200.build``) needs neither the library nor the framework.
"""

from __future__ import annotations

import importlib
from typing import Any

__all__ = ["BFloat16", "CUDA", "dlpack", "einsum", "kernels", "move", "mx", "nn", "ops", "sharding"]


def __getattr__(name: str) -> Any:
    if name == "CUDA":
        return importlib.import_module(".carrier", __name__).CUDA
    if name == "BFloat16":
        return importlib.import_module("._host", __name__).BFloat16
    if name in ("kernels", "mx", "ops", "sharding", "carrier", "layout_plan", "nn", "dlpack", "einsum", "move"):
        return importlib.import_module("." + name, __name__)
    raise AttributeError(name)
