"""Plain-torch oracle for the Mamba3 SISO layer (chunked SSD and recurrence).

Same mathematics as the reference's XLA path
(``src/base_model/models/mamba3_jax.py:62-419``) and recurrent step
(``src/base_model/models/mamba3.py:466-578``), restated in batched torch:

* RoPE on the first ``2*R`` state dims of the biased B (key) and C (query),
  with angles ``theta_t = sum_{i<=t} tanh(a_i) * pi * dt_i`` reduced mod 2*pi;
* trapezoidal weights ``gamma_t = dt_t * sigmoid(trap_t)``,
  ``scale_t = gamma_t + dt_{t+1} * (1 - sigmoid(trap_{t+1}))``;
* strictly lower-triangular intra-chunk attention with decay
  ``exp(cum_l - cum_s)``, the cross-chunk state recurrence, and the diagonal
  ``(D + (C.B) * gamma) * x`` term; output gated by ``silu(z)``.

All tensors carry a leading batch dim.  Layouts: ``Q, K`` (Bt, L, H, N);
``V, Z`` (Bt, L, H, P); ``ADT, DT, Trap`` (Bt, H, L); ``angles`` (Bt, L, R)
(shared by all heads, as in the fused path of the reference, ngroups = 1).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

TWO_PI = 2.0 * math.pi


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs ``(x[2i], x[2i+1])`` for ``i < cos.shape[-1]``."""
    d = x.shape[-1]
    r = cos.shape[-1]
    xp = x.reshape(*x.shape[:-1], d // 2, 2)
    x0, x1 = xp[..., 0], xp[..., 1]
    if r < d // 2:
        pad = d // 2 - r
        cos = F.pad(cos, (0, pad), value=1.0)
        sin = F.pad(sin, (0, pad), value=0.0)
    o0 = x0 * cos - x1 * sin
    o1 = x0 * sin + x1 * cos
    return torch.stack([o0, o1], dim=-1).reshape(x.shape)


def angle_cumsum(angles: torch.Tensor, DT: torch.Tensor, offset=None) -> torch.Tensor:
    """angles (Bt, L, R), DT (Bt, H, L) -> cumulative angles (Bt, L, H, R) mod 2*pi,
    starting from ``offset`` (Bt, H, R) when given (a sequence continued from a carry)."""
    rate = torch.tanh(angles)[:, :, None, :] * math.pi * DT.transpose(1, 2)[..., None]
    cs = torch.cumsum(rate, dim=1)
    if offset is not None:
        cs = cs + offset[:, None]
    return cs - TWO_PI * torch.floor(cs / TWO_PI)


def trapezoid_gamma_scale(DT: torch.Tensor, Trap: torch.Tensor):
    sig = torch.sigmoid(Trap)
    gamma = DT * sig
    shifted = F.pad(DT[..., 1:] * (1.0 - sig[..., 1:]), (0, 1))
    return gamma, gamma + shifted


def segsum(x: torch.Tensor) -> torch.Tensor:
    """(..., T) -> (..., T, T): cs[l] - cs[s] on and below the diagonal, -inf above."""
    T = x.shape[-1]
    cs = torch.cumsum(x, dim=-1)
    d = cs[..., :, None] - cs[..., None, :]
    mask = torch.tril(torch.ones(T, T, dtype=torch.bool, device=x.device))
    return d.masked_fill(~mask, float("-inf"))


def mamba3_ssd_chunked(Q, K, V, ADT, DT, Trap, angles, Q_bias, K_bias, D, Z, chunk_size=64,
                       return_final_state=False, initial_state=None, angle_offset=None):
    """Chunked SSD forward; returns y (Bt, L, H, P) (and the final state (Bt, H, P, N)).

    ``initial_state`` (Bt, H, P, N) and ``angle_offset`` (Bt, H, R) continue a sequence
    from a carry (context parallelism); the last token's trapezoid term that the next
    segment's first token would add is left out, as at the end of a sequence."""
    Bt, L, H, N = Q.shape
    P = V.shape[-1]
    CS = chunk_size
    ang = angle_cumsum(angles, DT, angle_offset)            # (Bt, L, H, R)
    cos, sin = torch.cos(ang), torch.sin(ang)
    gamma, scale = trapezoid_gamma_scale(DT, Trap)          # (Bt, H, L)
    Qb = Q + Q_bias
    Kb = K + K_bias
    qk = (Qb * Kb).sum(-1) * gamma.transpose(1, 2)          # (Bt, L, H)
    Qr = apply_rope(Qb, cos, sin)
    Kr = apply_rope(Kb, cos, sin) * scale.transpose(1, 2)[..., None]

    pad = (CS - L % CS) % CS
    if pad:
        Qr = F.pad(Qr, (0, 0, 0, 0, 0, pad))
        Kr = F.pad(Kr, (0, 0, 0, 0, 0, pad))
        V_ = F.pad(V, (0, 0, 0, 0, 0, pad))
        Z_ = F.pad(Z, (0, 0, 0, 0, 0, pad))
        qk = F.pad(qk, (0, 0, 0, pad))
        ADT_ = F.pad(ADT, (0, pad))
    else:
        V_, Z_, ADT_ = V, Z, ADT
    Lp = L + pad
    nc = Lp // CS
    Qc = Qr.reshape(Bt, nc, CS, H, N)
    Kc = Kr.reshape(Bt, nc, CS, H, N)
    Vc = V_.reshape(Bt, nc, CS, H, P)
    Zc = Z_.reshape(Bt, nc, CS, H, P)
    qkc = qk.reshape(Bt, nc, CS, H)
    Ac = ADT_.reshape(Bt, H, nc, CS)
    cum = torch.cumsum(Ac, dim=-1)                          # (Bt, H, nc, CS)

    Lmat = torch.exp(segsum(Ac))                            # (Bt, H, nc, CS, CS)
    strict = torch.tril(torch.ones(CS, CS, dtype=torch.bool, device=Q.device), -1)
    Lmat = Lmat * strict
    S = torch.einsum("bclhn,bcshn->bhcls", Qc, Kc) * Lmat
    Y = torch.einsum("bhcls,bcshp->bclhp", S, Vc)

    decay_states = torch.exp(cum[..., -1:] - cum)          # (Bt, H, nc, CS)
    states = torch.einsum("bcshp,bhcs,bcshn->bchpn", Vc, decay_states, Kc)
    st = torch.zeros(Bt, H, P, N, dtype=states.dtype, device=Q.device) if initial_state is None \
        else initial_state.to(states.dtype)
    A_end = cum[..., -1]                                    # (Bt, H, nc)
    ins = []
    for c in range(nc):
        ins.append(st)
        st = torch.exp(A_end[:, :, c])[..., None, None] * st + states[:, c]
    S_in = torch.stack(ins, dim=1)                          # (Bt, nc, H, P, N)
    Y = Y + torch.einsum("bclhn,bchpn,bhcl->bclhp", Qc, S_in, torch.exp(cum))
    Y = Y + (D[None, None, None, :, None] + qkc[..., None]) * Vc
    Y = Y * F.silu(Zc)
    Y = Y.reshape(Bt, Lp, H, P)[:, :L]
    if return_final_state == "all":
        return Y, st, ang, Kr_unscaled_last(Kb, cos, sin), cum
    if return_final_state:
        return Y, st
    return Y


def Kr_unscaled_last(Kb, cos, sin):
    """The last token's rotated (unscaled) key: the decode state's k_prev."""
    return apply_rope(Kb[:, -1:], cos[:, -1:], sin[:, -1:])[:, 0]


def mamba3_recurrent(Q, K, V, ADT, DT, Trap, angles, Q_bias, K_bias, D, Z, state=None):
    """Token-by-token recurrence (the decode path); same signature as the chunked op.

    ``state`` is ``(angle (Bt,H,R), ssm (Bt,H,P,N), k_prev (Bt,H,N), v_prev (Bt,H,P))``.
    Returns ``(y (Bt,L,H,P), new_state)``.
    """
    Bt, L, H, N = Q.shape
    P = V.shape[-1]
    R = angles.shape[-1]
    if state is None:
        z = lambda *s: torch.zeros(*s, dtype=torch.float32, device=Q.device)
        state = (z(Bt, H, R), z(Bt, H, P, N), z(Bt, H, N), z(Bt, H, P))
    ang, ssm, k_prev, v_prev = state
    sig = torch.sigmoid(Trap)
    ys = []
    for t in range(L):
        dt = DT[:, :, t]
        ang = ang + torch.tanh(angles[:, t])[:, None, :] * math.pi * dt[..., None]
        ang = ang - TWO_PI * torch.floor(ang / TWO_PI)
        c, s = torch.cos(ang), torch.sin(ang)
        Kr = apply_rope(K[:, t] + K_bias, c, s)
        Qr = apply_rope(Q[:, t] + Q_bias, c, s)
        decay = torch.exp(ADT[:, :, t])[..., None, None]
        tr = sig[:, :, t][..., None, None]
        dtx = dt[..., None, None]
        ssm = decay * ssm + (1 - tr) * dtx * decay * (v_prev[..., :, None] * k_prev[..., None, :])
        ssm = ssm + tr * dtx * (V[:, t][..., :, None] * Kr[..., None, :])
        y = torch.einsum("bhn,bhpn->bhp", Qr, ssm) + D[None, :, None] * V[:, t]
        y = y * F.silu(Z[:, t])
        ys.append(y)
        k_prev, v_prev = Kr, V[:, t]
    return torch.stack(ys, dim=1), (ang, ssm, k_prev, v_prev)
