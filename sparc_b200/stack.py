"""The 4-layer benchmark stack: x <- x + SPARCMixer(RMSNorm(x)) per layer.

There is no reference counterpart (the reference ships only the mixer); this is the model the
multi-GPU workload trains. RMSNorm has a float32 weight initialised to ones and eps 1e-6; it is
applied in the activation dtype by torch's fused rms_norm.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .mixer import SPARCMixer


class RMSNorm(nn.Module):
    def __init__(self, width: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(width))

    def forward(self, x):
        return F.rms_norm(x, (x.shape[-1],), self.weight.to(x.dtype), self.eps)


class SPARCStack(nn.Module):
    def __init__(self, width: int, layers: int = 4, eps: float = 1e-6):
        super().__init__()
        self.norms = nn.ModuleList(RMSNorm(width, eps) for _ in range(layers))
        self.mixers = nn.ModuleList(SPARCMixer(width) for _ in range(layers))

    def forward(self, x):
        for norm, mixer in zip(self.norms, self.mixers):
            y, _ = mixer(norm(x))
            x = x + y
        return x
