"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): float64 CPU restatement of the gated RMSNorm on the rule's
output, the reference's one-pass gnorm kernels (src/macai/layer/_gated_norm.py:1-16 formulas, :28-104 kernels,
:154-197 autograd) without their rounding points (the float64 truth its tests compare against,
tests/test_layer.py:176-177 `ref_gated`):

    r     = rsqrt(mean(x^2) + eps),  n = x r
    o     = w n silu(z)
    dz    = do w n sig (1 + z (1 - sig)),            sig = sigmoid(z)
    dn    = do silu(z) w
    dx    = r (dn - n <n, dn> / D)
    dw    = sum over rows of do silu(z) n

x, z: [..., D]; w: [D]. Everything here runs in float64.
"""
from __future__ import annotations

import torch

EPS = 1e-6


def forward(x, z, w, eps=EPS):
    """o in float64 (_gated_norm.py:28-53)."""
    x, z, w = x.double(), z.double(), w.double()
    r = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return w * (x * r) * (z * torch.sigmoid(z))


def backward(x, z, w, do, eps=EPS):
    """(dx, dz, dw) in float64 (_gated_norm.py:55-104, :127-137)."""
    x, z, w, do = x.double(), z.double(), w.double(), do.double()
    D = x.shape[-1]
    r = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    n = x * r
    sig = torch.sigmoid(z)
    s = z * sig
    dz = do * w * n * sig * (1.0 + z * (1.0 - sig))
    dn = do * s * w
    dx = r * (dn - n * (n * dn).sum(-1, keepdim=True) / D)
    dw = (do * s * n).reshape(-1, D).sum(0)
    return dx, dz, dw
