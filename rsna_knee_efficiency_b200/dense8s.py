"""The reference module's surface (`knee.dense8s`, src/knee/dense8s.py): what a pack-building or
inference script imports from it, backed by this repository's implementation.

`emulate` (the reference's float64 model of the arithmetic) is not part of the product: its
restatement lives in oracle/ as test infrastructure.
"""
from __future__ import annotations

from .encoder import Dense8SEncoder
from .pack import (KIND, PACK_FORMAT, f16_layers as f16_layers_meta, is_pack, kernels_sha, load_pack,
                   make_pack, pack_meta, pack_params, save_pack)
from .quant import (BOTTLENECK, GROUP, GROWTH, QS, QU, SBlock, SLayer, SPlan, _abh, _abh_ab, _affine,
                    _chunked, _wq, calibrate, head_params, kernel_params, make_plan, stem_weights8,
                    stem_weights16)

__all__ = ["Dense8SEncoder", "KIND", "PACK_FORMAT", "f16_layers_meta", "is_pack", "kernels_sha",
           "load_pack", "make_pack", "pack_meta", "pack_params", "save_pack", "BOTTLENECK", "GROUP",
           "GROWTH", "QS", "QU", "SBlock", "SLayer", "SPlan", "_abh", "_abh_ab", "_affine", "_chunked",
           "_wq", "calibrate", "head_params", "kernel_params", "make_plan", "stem_weights8",
           "stem_weights16"]
