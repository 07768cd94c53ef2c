"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): float64 CPU restatement of the gated delta rule.

Every function cites the reference file:line it restates. All tensors are torch float64 on the CPU; layouts follow the
reference's drop-in: q, k [B, T, H, DK]; v [B, T, H, DV]; g, beta [B, T, H]; states [B, H, DK, DV].
"""
from __future__ import annotations

import torch

F64 = torch.float64
EPS = 1e-6


def l2norm(x: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    """x * rsqrt(sum(x^2) + eps) over the last dim. Reference: src/macai/gated_delta/op.py:260-261 and the fused
    prologue's equation src/macai/gated_delta/_norm.py:1-9 (transformers' l2norm, TF modeling_qwen3_5.py:228-231)."""
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def l2norm_scale_backward(x: torch.Tensor, dy: torch.Tensor, scale: float, eps: float = EPS) -> torch.Tensor:
    """dx of y = l2norm(x) * scale: dx = scale r (dy - x_hat (x_hat . dy)), r = rsqrt(sum x^2 + eps), x_hat = x r.
    Reference: src/macai/gated_delta/_norm.py:6-9 (equation) and :44-56 (l2n_bwd kernel)."""
    r = torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)
    xh = x * r
    return scale * r * (dy - xh * (xh * dy).sum(-1, keepdim=True))


def recurrence(q, k, v, g, beta, s0):
    """The token-serial gated delta rule. Reference: src/macai/gated_delta/op.py:301-314 (recurrent_reference).

    q already normalised and scaled, k normalised. Returns (o [B,T,H,DV], S_T [B,H,DK,DV])."""
    T = q.shape[1]
    s = s0.clone()
    outs = []
    for t in range(T):
        a = g[:, t].exp()[..., None, None]
        st = s * a
        u = (st * k[:, t, :, :, None]).sum(-2)
        d = beta[:, t, :, None] * (v[:, t] - u)
        s = st + k[:, t, :, :, None] * d[:, :, None, :]
        outs.append((s * q[:, t, :, :, None]).sum(-2))
    return torch.stack(outs, 1), s


def recurrence_grads(q, k, v, g, beta, s0, do, dsT):
    """(o, S_T, dq, dk, dv, dg, dbeta, ds0) by float64 autograd through `recurrence`, the ground truth of the
    reference's harness (tests/test_harness.py:34-57)."""
    xs = [t.detach().to(F64).clone().requires_grad_(True) for t in (q, k, v, g, beta, s0)]
    o, sT = recurrence(*xs)
    ((o * do.to(F64)).sum() + (sT * dsT.to(F64)).sum()).backward()
    return (o.detach(), sT.detach(), *(x.grad for x in xs))


def _bh(x):
    """[B, T, H, ...] -> [B, H, T, ...]."""
    return x.transpose(1, 2)


def chunked(q, k, v, g, beta, s0, do=None, dsT=None, C: int = 64):
    """The chunked (WY/UT) forward F1-F5 and hand-derived backward B1-B6, restated from
    tools/check_chunk_equations.py:22-79 (equations also at src/macai/gated_delta/_chunked.py:1-35), vectorised over
    (batch, head). A tail chunk of n < C rows is handled by slicing, as the reference's checker does (:25-27).

    Returns (o, S_T) or, with do given, (o, S_T, dq, dk, dv, dg, dbeta, ds0), all float64 in the drop-in layouts."""
    q, k, v, g, beta = (_bh(t).to(F64) for t in (q, k, v, g, beta))
    B, H, T, DK = q.shape
    DV = v.shape[-1]
    S = s0.to(F64).clone()
    O = torch.zeros(B, H, T, DV, dtype=F64)
    tr = lambda x: x.transpose(-1, -2)
    saved = []
    NT = (T + C - 1) // C
    for c in range(NT):                                              # check_chunk_equations.py:26
        sl = slice(c * C, min((c + 1) * C, T))
        Q, K, V, gc, bc = q[:, :, sl], k[:, :, sl], v[:, :, sl], g[:, :, sl], beta[:, :, sl]
        n = Q.shape[2]
        G = torch.cumsum(gc, -1)                                     # F1 (:30)
        gam = torch.exp(G)
        e = torch.exp(G[..., -1:] - G)
        diff = G[..., :, None] - G[..., None, :]
        low = torch.tril(torch.ones(n, n, dtype=torch.bool), -1)
        lowi = torch.tril(torch.ones(n, n, dtype=torch.bool), 0)
        Gam = torch.where(lowi, torch.exp(torch.where(lowi, diff, torch.zeros_like(diff))), torch.zeros_like(diff))
        Kg = K @ tr(K)                                               # F2 (:37)
        L = torch.where(low, bc[..., None] * Kg * Gam, torch.zeros_like(Kg))
        A = torch.linalg.inv(torch.eye(n, dtype=F64) + L)
        W = A @ ((bc * gam)[..., None] * K)                          # F3 (:40)
        U = A @ (bc[..., None] * V)
        Vn = U - W @ S                                               # F4 (:42)
        M = Gam * (Q @ tr(K))                                        # F5 (:43)
        O[:, :, sl] = gam[..., None] * (Q @ S) + M @ Vn
        saved.append((sl, Q, K, V, bc, gam, e, Gam, low, Kg, L, A, W, Vn, M, S.clone()))
        S = gam[..., -1:, None] * S + tr(K) @ (e[..., None] * Vn)
    if do is None:
        return _bh(O), S
    do = _bh(do).to(F64)
    dq, dk, dv = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
    dg, db = torch.zeros_like(g), torch.zeros_like(beta)
    dSn = (torch.zeros_like(S) if dsT is None else dsT.to(F64)).clone()
    for (sl, Q, K, V, bc, gam, e, Gam, low, Kg, L, A, W, Vn, M, Sc) in reversed(saved):   # (:49)
        dOc = do[:, :, sl]
        dVn = tr(M) @ dOc + e[..., None] * (K @ dSn)                                       # B1 (:51)
        dSc = gam[..., -1:, None] * dSn + tr(gam[..., None] * Q) @ dOc - tr(W) @ dVn       # B2 (:52)
        dM = Gam * (dOc @ tr(Vn))                                                           # B3 (:53)
        dQ = gam[..., None] * (dOc @ tr(Sc)) + dM @ K
        dKs = e[..., None] * (Vn @ tr(dSn))
        dK = tr(dM) @ Q + dKs
        dW = -dVn @ tr(Sc)
        dU = dVn
        X, Y = tr(A) @ dW, tr(A) @ dU                                                       # B5 (:63)
        dK = dK + (bc * gam)[..., None] * X
        dbc = gam * (K * X).sum(-1) + (V * Y).sum(-1)
        dV = bc[..., None] * Y
        dA = torch.where(low, dW @ tr((bc * gam)[..., None] * K) + dU @ tr(bc[..., None] * V), torch.zeros_like(Kg))
        dL = torch.where(low, -tr(A) @ dA @ tr(A), torch.zeros_like(Kg))
        P = dL * Gam
        dK = dK + bc[..., None] * (P @ K) + tr(P) @ (bc[..., None] * K)
        dbc = dbc + (P * Kg).sum(-1)
        dgc = _dg_chunk(Q, K, Sc, dSn, dOc, gam, e, bc, X, dM, M, dL, L, dKs, low)          # B4 + B6
        dq[:, :, sl], dk[:, :, sl], dv[:, :, sl], dg[:, :, sl], db[:, :, sl] = dQ, dK, dV, dgc, dbc
        dSn = dSc
    return (_bh(O), S, _bh(dq), _bh(dk), _bh(dv), _bh(dg), _bh(db), dSn)


def _exclusive_cumsum(x):
    """sum_{j < t} x_j along the last dim, without forming the inclusive sum (no x_t - x_t cancellation)."""
    z = torch.zeros_like(x[..., :1])
    return torch.cat([z, torch.cumsum(x[..., :-1], -1)], -1)


def _dg_chunk(Q, K, Sc, dSn, dOc, gam, e, bc, X, dM, M, dL, L, dKs, low):
    """dg of one chunk without cancellation (B4 + B6 of tools/check_chunk_equations.py:61-76, regrouped the way the
    reference's kernel does for strong decay, src/macai/gated_delta/_chunked.py:1138-1142).

    With dG_r = dLoss/dG_r and dg_t = sum_{s >= t} dG_s (B6), every term is summed where it does not cancel:
      a_s = gamma_s q_s . (dO_s S_c^T)        and  w_s = beta_s gamma_s k_s . X_s   enter dG_s       -> suffix sums;
      gamma_last <S_c, dS_{c+1}>              enters dG_last                                        -> every t;
      E_r = e_r k_r . (Vn_r dS_{c+1}^T)       enters dG_last (+) and dG_r (-)                        -> sum_{r < t};
      R_ij = dM_ij (QK^T)_ij + dL_ij L_ij, i > j, enters dG_i (+) and dG_j (-)                      -> sum_{i >= t > j}.
    The literal B4 (row sums minus column sums, then the reverse cumsum) loses ~1e-7 relative in float64 at g = -20."""
    tr = lambda x: x.transpose(-1, -2)
    a = gam * (Q * (dOc @ tr(Sc))).sum(-1)
    w = bc * gam * (K * X).sum(-1)
    suffix = torch.flip(torch.cumsum(torch.flip(a + w, [-1]), -1), [-1])
    s_last = gam[..., -1] * (Sc * dSn).sum((-1, -2))
    E = (K * dKs).sum(-1)
    prefix_excl = _exclusive_cumsum(E)
    QKt = Q @ tr(K)
    R = torch.where(low, dM * QKt + dL * L, torch.zeros_like(L))
    # rect_t = sum_{i >= t} sum_{j < t} R_ij
    rowpre = _exclusive_cumsum(R)                         # [.., i, t] = sum_{j < t} R_ij
    rect = torch.flip(torch.cumsum(torch.flip(rowpre, [-2]), -2), [-2]).diagonal(dim1=-2, dim2=-1)
    return suffix + s_last[..., None] + prefix_excl + rect


def dropin(query, key, value, g, beta, initial_state=None, do=None, dsT=None, use_qk_l2norm_in_kernel=True,
           chunk: int | None = 64):
    """Float64 truth of the drop-in chunk_gated_delta_rule (src/macai/gated_delta/op.py:264-298): the l2 prologue with
    query scale DK^-1/2 (:276-283), the rule, and with `do` the gradients of every raw input through the prologue.

    GQA: when value has more heads than query/key, each key head serves H_v / H_k consecutive value heads (the
    repeat_interleave the Qwen3.5 layer applies before calling the rule, TF modeling_qwen3_5.py:494-496); the key-side
    gradients are summed over the value heads a key head serves.

    `chunk` None runs the token recurrence (autograd); an int runs the chunked equations (same values to ~1e-13, faster).
    Returns (o, S_T) or (o, S_T, dquery, dkey, dvalue, dg, dbeta, ds0), float64."""
    qr, kr = query.to(F64), key.to(F64)
    vv, gg, bb = value.to(F64), g.to(F64), beta.to(F64)
    B, T, Hk, DK = qr.shape
    Hv, DV = vv.shape[2], vv.shape[3]
    rep = Hv // Hk
    s0 = torch.zeros(B, Hv, DK, DV, dtype=F64) if initial_state is None else initial_state.to(F64)
    scale = DK ** -0.5
    if use_qk_l2norm_in_kernel:
        qn, kn = l2norm(qr) * scale, l2norm(kr)
    else:
        qn, kn = qr * scale, kr
    qv = qn.repeat_interleave(rep, dim=2) if rep > 1 else qn
    kv = kn.repeat_interleave(rep, dim=2) if rep > 1 else kn
    if do is None:
        if chunk is None:
            return recurrence(qv, kv, vv, gg, bb, s0)
        return chunked(qv, kv, vv, gg, bb, s0, C=chunk)
    dsT = torch.zeros_like(s0) if dsT is None else dsT.to(F64)
    if chunk is None:
        o, sT, dqn, dkn, dv, dg_, db_, ds0 = recurrence_grads(qv, kv, vv, gg, bb, s0, do, dsT)
    else:
        o, sT, dqn, dkn, dv, dg_, db_, ds0 = chunked(qv, kv, vv, gg, bb, s0, do, dsT, C=chunk)
    if rep > 1:
        dqn = dqn.view(B, T, Hk, rep, DK).sum(3)
        dkn = dkn.view(B, T, Hk, rep, DK).sum(3)
    if use_qk_l2norm_in_kernel:
        dquery = l2norm_scale_backward(qr, dqn, scale)
        dkey = l2norm_scale_backward(kr, dkn, 1.0)
    else:
        dquery, dkey = dqn * scale, dkn
    return o, sT, dquery, dkey, dv, dg_, db_, ds0


def dropin_packed(query, key, value, g, beta, cu_seqlens, initial_state=None, do=None, dsT=None,
                  use_qk_l2norm_in_kernel=True, chunk: int | None = 64):
    """Float64 truth of the drop-in over packed rows (cu_seqlens): batch size 1, sequence n at rows
    cu_seqlens[n] .. cu_seqlens[n + 1] - 1, each run as its own row by `dropin` (its own initial state
    initial_state[n], its own final state), the outputs and gradients concatenated back along the tokens and the
    states stacked [N, H, DK, DV]. A sequence without tokens passes its state (and the state's gradient) through.
    The reference refuses cu_seqlens (src/macai/gated_delta/op.py:270-273); these are the packed-sequence semantics of
    fla's kernels, which transformers' Qwen3.5 layer calls with cu_seqlens (layer/_qwen3_5.py:163-165)."""
    cu = [int(x) for x in cu_seqlens]
    N = len(cu) - 1
    Hv, DK, DV = value.shape[2], query.shape[3], value.shape[3]
    s0 = torch.zeros(N, Hv, DK, DV, dtype=F64) if initial_state is None else initial_state.to(F64)
    outs = []
    for n in range(N):
        a, b = cu[n], cu[n + 1]
        if b == a:
            empty = [torch.zeros(1, 0, *x.shape[2:], dtype=F64) for x in (query, key, value)]
            e3 = torch.zeros(1, 0, Hv, dtype=F64)
            if do is None:
                outs.append((empty[2], s0[n:n + 1]))
            else:
                d = torch.zeros_like(s0[n:n + 1]) if dsT is None else dsT[n:n + 1].to(F64)
                outs.append((empty[2], s0[n:n + 1], empty[0], empty[1], empty[2], e3, e3, d))
            continue
        sl = slice(a, b)
        r = dropin(query[:, sl], key[:, sl], value[:, sl], g[:, sl], beta[:, sl], s0[n:n + 1],
                   None if do is None else do[:, sl], None if dsT is None else dsT[n:n + 1],
                   use_qk_l2norm_in_kernel, chunk)
        outs.append(r)
    cat = lambda i: torch.cat([o[i] for o in outs], dim=1)
    stack = lambda i: torch.cat([o[i] for o in outs], dim=0)
    if do is None:
        return cat(0), stack(1)
    return cat(0), stack(1), cat(2), cat(3), cat(4), cat(5), cat(6), stack(7)


def recurrence_packed(q, k, v, g, beta, s0, cu_seqlens):
    """The token recurrence over a packed stream [1, T, H, D] (q, k already normalised and scaled, GQA expanded) with
    the state set to s0[n] at each sequence's first token and recorded after its last: an independent restatement of
    the packed semantics, against which `dropin_packed` is pinned. Returns (o [1, T, H, DV], S_T [N, H, DK, DV])."""
    cu = [int(x) for x in cu_seqlens]
    N = len(cu) - 1
    H, DK, DV = q.shape[2], q.shape[3], v.shape[3]
    o = torch.zeros(1, q.shape[1], H, DV, dtype=F64)
    sT = torch.zeros(N, H, DK, DV, dtype=F64)
    for n in range(N):
        S = s0[n].to(F64).clone()
        for t in range(cu[n], cu[n + 1]):
            S = S * torch.exp(g[0, t].to(F64))[:, None, None]
            kt, vt = k[0, t].to(F64), v[0, t].to(F64)
            pred = torch.einsum("hk,hkv->hv", kt, S)
            S = S + torch.einsum("hk,hv->hkv", kt, beta[0, t].to(F64)[:, None] * (vt - pred))
            o[0, t] = torch.einsum("hk,hkv->hv", q[0, t].to(F64), S)
        sT[n] = S
    return o, sT
