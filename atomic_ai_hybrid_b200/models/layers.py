"""Basic parameter-holding layers with the reference's flax parameter names.

Every ``Dense`` stores ``kernel`` with the flax layout ``(in, out)`` and an
optional ``bias`` ``(out,)``; ``RMSNorm`` stores ``scale``.  Parameters are fp32
master copies; the forward pass computes in the module's compute dtype (bf16 on
the GPU, fp32 in CPU parity tests), like flax ``dtype=bf16`` modules.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from .. import ops


def lecun_normal_(t: torch.Tensor, fan_in: int) -> torch.Tensor:
    """Flax ``lecun_normal``: truncated normal (2 sigma) with variance 1/fan_in."""
    std = math.sqrt(1.0 / fan_in) / 0.87962566103423978
    with torch.no_grad():
        return nn.init.trunc_normal_(t, 0.0, std, -2 * std, 2 * std)


class Dense(nn.Module):
    def __init__(self, d_in: int, d_out: int, bias: bool = False, dtype=torch.float32):
        super().__init__()
        self.d_in, self.d_out = d_in, d_out
        self.kernel = nn.Parameter(torch.empty(d_in, d_out, dtype=dtype))
        self.bias = nn.Parameter(torch.zeros(d_out, dtype=torch.float32)) if bias else None
        lecun_normal_(self.kernel.data, d_in)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if ops.use_cuda(x) and x.dtype == torch.bfloat16:
            from ..ops import kernels as K
            return K.linear_multi(x, [(self.kernel, self.bias)])[0]
        return ops.linear(x, self.kernel, self.bias)


class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(d, dtype=torch.float32))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rmsnorm(x, self.scale, self.eps)


def compute_dtype_of(module: nn.Module) -> torch.dtype:
    return getattr(module, "_compute_dtype", torch.float32)
