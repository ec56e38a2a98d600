"""Quantisation configs.

Parity: sglang_neuron/quant.py:14-61 registers inert QuantizationConfig objects for `mxfp4` and `quark`: the
model loads its quantised weights itself. Same here: `mxfp4` (GPT-OSS checkpoints ship e2m1 blocks + e8m0
scales per 32 values, consumed as-is by the block-scaled tcgen05 grouped GEMM) and `fp8` (bf16 expert weights
quantised at load to MXFP8: e4m3 values with one e8m0 scale per 32).
"""
from __future__ import annotations

import dataclasses
from typing import Optional


@dataclasses.dataclass(frozen=True)
class QuantConfig:
    name: str
    weight_format: str          # "e2m1" | "e4m3"
    block_size: int = 32        # values per shared scale
    scale_format: str = "e8m0"
    applies_to: str = "experts"

    def get_name(self) -> str:
        return self.name

    def is_passthrough(self) -> bool:
        """The model loader consumes the format itself (no generic linear method)."""
        return True


_CONFIGS = {
    "mxfp4": QuantConfig("mxfp4", "e2m1"),
    "fp8": QuantConfig("fp8", "e4m3"),
    "mxfp8": QuantConfig("mxfp8", "e4m3"),
}


def get_quant_config(name: Optional[str]) -> Optional[QuantConfig]:
    if name is None:
        return None
    if name not in _CONFIGS:
        raise ValueError(f"quantization {name!r} is not served; served: {sorted(_CONFIGS)}")
    return _CONFIGS[name]
