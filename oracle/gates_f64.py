"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): float64 CPU restatement of the linear-attention layer's gates,
the reference's one-pass gates kernels (src/macai/layer/_gates.py:1-13 formulas, :20-48 kernels, :82-121 autograd):

    beta = sigmoid(b)
    g    = -exp(A_log) * softplus(a + dt_bias)         softplus(x) = x above 20 (PyTorch's threshold), else log1p(exp(x))
    db   = dbeta * beta * (1 - beta)
    da   = dg * (-exp(A_log)) * (1 if x > 20 else sigmoid(x)),  x = a + dt_bias
    dA_log  = sum over tokens of dg * g               (per head: the reduction of _gates.py:112-114)
    ddt_bias = sum over tokens of da (before its cast)  (_gates.py:109-111, :115-116)

Inputs b, a: [..., H] (any float dtype, read as their values); A_log, dt_bias: [H]. Everything here runs in float64.
"""
from __future__ import annotations

import torch

THRESHOLD = 20.0


def forward(b, a, A_log, dt_bias):
    """(beta, g) in float64 (_gates.py:28-35)."""
    b, a = b.double(), a.double()
    al, dtb = A_log.double(), dt_bias.double()
    beta = torch.sigmoid(b)
    x = a + dtb
    sp = torch.where(x > THRESHOLD, x, torch.log1p(torch.exp(torch.clamp(x, max=THRESHOLD))))
    g = -torch.exp(al) * sp
    return beta, g


def backward(b, a, A_log, dt_bias, dbeta, dg):
    """(db, da, dA_log, ddt_bias) in float64 (_gates.py:38-48, :104-121)."""
    b, a = b.double(), a.double()
    al, dtb = A_log.double(), dt_bias.double()
    dbeta, dg = dbeta.double(), dg.double()
    sb = torch.sigmoid(b)
    db = dbeta * sb * (1.0 - sb)
    x = a + dtb
    sx = torch.where(x > THRESHOLD, torch.ones_like(x), torch.sigmoid(x))
    da = dg * (-torch.exp(al)) * sx
    H = al.shape[0]
    _, g = forward(b, a, A_log, dt_bias)
    dA = (dg * g).reshape(-1, H).sum(0)
    ddt = da.reshape(-1, H).sum(0)
    return db, da, dA, ddt
