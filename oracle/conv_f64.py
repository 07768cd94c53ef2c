"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): float64 CPU restatement of the linear-attention layer's
convolution path, the reference's one-pass conv kernels (src/macai/layer/_conv.py:1-21 formulas, :52-137 kernels,
:188-237 autograd), without their rounding points:

    u[t, c]  = sum_j w[c, j] x[t - 3 + j, c]            (x = 0 before the sequence start)
    y        = u sigmoid(u)
    q, k, v  = y split [kd, kd, vd] along the channels, as [B, T, heads, width]; q and k repeated `rep` times per key
               head (repeat_interleave over the value heads)
    du       = dy sigmoid(u) (1 + u (1 - sigmoid(u)))    (dy of q and k summed over each key head's rep copies)
    dx[t, c] = sum_j w[c, j] du[t + 3 - j, c]            (du = 0 past the sequence end)
    dw[c, j] = sum_{b, t} du[t, c] x[t - 3 + j, c]

x: [B, T, C]; w: [C, 4] (or the layer's [C, 1, 4]). Everything here runs in float64.
"""
from __future__ import annotations

import torch

K = 4


def _u(x, w):
    B, T, C = x.shape
    xp = torch.cat([x.new_zeros(B, K - 1, C), x], dim=1)  # x[t - 3 .. t] at xp[t .. t + 3]
    return sum(w[:, j] * xp[:, j:j + T] for j in range(K))


def forward(x, w, kd, dk, rep, dv):
    """(q, k, v) in float64 (_conv.py:52-83)."""
    x = x.double()
    w = w.double().reshape(x.shape[-1], K)
    B, T, C = x.shape
    u = _u(x, w)
    y = u * torch.sigmoid(u)
    q, k, v = torch.split(y, [kd, kd, C - 2 * kd], dim=-1)
    q = q.reshape(B, T, -1, dk).repeat_interleave(rep, dim=2)
    k = k.reshape(B, T, -1, dk).repeat_interleave(rep, dim=2)
    return q, k, v.reshape(B, T, -1, dv)


def backward(x, w, dq, dk_, dv_, kd, dk, rep, dv):
    """(dx, dw [C, 4]) in float64 (_conv.py:84-137, :158-167); a None cotangent is zero."""
    x = x.double()
    w = w.double().reshape(x.shape[-1], K)
    B, T, C = x.shape
    vd = C - 2 * kd

    def fold(g, width):  # [B, T, hv, width] summed over each key head's rep copies -> [B, T, kd]
        if g is None:
            return x.new_zeros(B, T, width)
        g = g.double()
        return g.reshape(B, T, -1, rep, g.shape[-1]).sum(3).reshape(B, T, -1)
    gq, gk = fold(dq, kd), fold(dk_, kd)
    gv = x.new_zeros(B, T, vd) if dv_ is None else dv_.double().reshape(B, T, vd)
    g = torch.cat([gq, gk, gv], dim=-1)
    u = _u(x, w)
    s = torch.sigmoid(u)
    du = g * s * (1.0 + u * (1.0 - s))
    dup = torch.cat([du, du.new_zeros(B, K - 1, C)], dim=1)  # du[t .. t + 3] at dup[t .. t + 3]
    dx = sum(w[:, j] * dup[:, K - 1 - j:K - 1 - j + T] for j in range(K))
    xp = torch.cat([x.new_zeros(B, K - 1, C), x], dim=1)
    dw = torch.stack([(du * xp[:, j:j + T]).sum((0, 1)) for j in range(K)], dim=-1)
    return dx, dw
