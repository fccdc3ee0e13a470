"""The config-5 stack: x <- x + SPARCMixer(RMSNorm(x)) per layer.

There is no reference counterpart (the reference ships only the mixer); this is the model the
multi-GPU workload trains. RMSNorm has a float32 weight initialised to ones and eps 1e-6. Each
block runs as one fused call of the mixer kernels (`sparc_block`: the norm is applied to the
tiles as they are read and the residual added as the output is written), so no separate norm or
residual pass touches HBM. `RMSNorm` stays available as a module for unfused use.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .mixer import SPARCMixer, sparc_block


class RMSNorm(nn.Module):
    def __init__(self, width: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(width))

    def forward(self, x):
        return F.rms_norm(x, (x.shape[-1],), self.weight.to(x.dtype), self.eps)


class SPARCBlock(nn.Module):
    """x + SPARCMixer(RMSNorm(x)) in one fused call (parameters: norm.weight, mixer.*)."""

    def __init__(self, width: int, eps: float = 1e-6):
        super().__init__()
        self.norm = RMSNorm(width, eps)
        self.mixer = SPARCMixer(width)

    def forward(self, x, fused: bool = True):
        if not fused:
            y, _ = self.mixer(self.norm(x))
            return x + y
        out, _ = sparc_block(x, self.mixer._params(), self.norm.weight, self.norm.eps, max_spin=self.mixer.max_spin)
        return out


class SPARCStack(nn.Module):
    """`layers` blocks; the state dict keeps the layout norms.<i>.weight, mixers.<i>.*."""

    def __init__(self, width: int, layers: int = 4, eps: float = 1e-6, fused: bool = True):
        super().__init__()
        self.fused = fused
        self.norms = nn.ModuleList(RMSNorm(width, eps) for _ in range(layers))
        self.mixers = nn.ModuleList(SPARCMixer(width) for _ in range(layers))

    def forward(self, x):
        for norm, mixer in zip(self.norms, self.mixers):
            if self.fused:
                x, _ = sparc_block(x, mixer._params(), norm.weight, norm.eps, max_spin=mixer.max_spin)
            else:
                y, _ = mixer(norm(x))
                x = x + y
        return x
