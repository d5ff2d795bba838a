"""Gated activation enum and dispatcher (int8_hybrid_moe/activation.py:1-41 of
the reference); only SiLU has a kernel, as in the reference."""

from enum import Enum

import torch

from . import ops


class MoEActivation(Enum):
    SILU = "silu"
    GELU = "gelu"
    SILU_NO_MUL = "silu_no_mul"
    GELU_NO_MUL = "gelu_no_mul"

    @property
    def is_gated(self) -> bool:
        return not self.value.endswith("_no_mul")


def apply_moe_activation(activation: MoEActivation, output: torch.Tensor,
                         input: torch.Tensor) -> torch.Tensor:
    assert input.dim() == 2
    assert output.dim() == 2
    if activation != MoEActivation.SILU:
        raise ValueError(f"Unsupported activation: {activation}")
    ops.silu_and_mul(output, input)
    return output
