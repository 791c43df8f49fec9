"""MoE configuration fields read by ``moe_swiglu_ffn``.

kappa passes its frozen ``Qwen3Config`` (kappa/qwen3/architecture.py:19-51)
to ``moe_swiglu_ffn``; the drop-in reads only the fields below, by name, so
kappa's own config object works unchanged.  ``MoEConfig`` carries the same
fields, with kappa's defaults (architecture.py:43-51), for callers without
kappa installed.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

MoEImpl = Literal["gather_einsum", "fixed_capacity", "ragged_jax", "ragged_tokamax"]
QuantMode = Literal["none", "w8"]


@dataclass(frozen=True, slots=True)
class MoEConfig:
    use_moe: bool
    num_experts: int
    num_experts_per_tok: int
    moe_impl: MoEImpl = "gather_einsum"
    moe_capacity_factor: float = 1.25
    moe_fixed_capacity_slots: int | None = None
    moe_ragged_decode_token_threshold: int = 64
    quantization: QuantMode = "w8"


def qwen3_30b_a3b_moe() -> MoEConfig:
    """MoE fields of kappa's ``qwen3-30b-a3b`` preset (architecture.py:94-112)."""
    return MoEConfig(use_moe=True, num_experts=128, num_experts_per_tok=8)
