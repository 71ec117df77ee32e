"""CUDA execution of Mamba3 layers.

Two autograd functions:

* :func:`mamba3_sequence_layer` -- the whole pre-norm ``half_glu1`` residual
  block (LayerNorm -> in_proj -> Mamba3 SSD -> out_norm -> out_proj -> GELU ->
  out2 gate -> residual) as ONE autograd node.  It owns its saved tensors
  (the fp32 layer input, the bf16 projection, the pre-norm SSD output and the
  two GLU pre-activations) and recomputes the cheap ones in backward (the
  LayerNorm output, out_norm output and GELU).
* :func:`mamba3_mixer` -- the mixer alone (in_proj ... out_proj), used where the
  residual wrapper is not fused (e.g. the book pre-layer at width 503).

GEMMs run on the package's tcgen05 kernel (``ops/gemm.py``): bf16 operands, fp32
accumulation; weight gradients are reduce-added in fp32 straight into the flat gradient
buffer.  The SSD, its pre/post-processing and all row/elementwise work are the sm_100a
kernels of ``csrc/`` too.  The projection buffer's row stride is padded to a
multiple of 8 elements so every kernel can use 16-byte accesses.
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from ._ext import ext
from . import gemm as G
from . import weights as W

EPS = 1e-6
# keep the forward's passed SSD chunk states for the backward instead of recomputing
# them (S0_RECOMPUTE_SSD_STATES=1 trades ~1 ms per layer-step for ~0.7 GB per layer)
SAVE_STATES = os.environ.get("S0_RECOMPUTE_SSD_STATES", "0") in ("0", "", "false")
# keep the fused layer's LayerNorm output and GELU output (bf16, 2 x T x d_model) for the
# backward instead of recomputing them (S0_SAVE_LAYER_ACTS=0 recomputes: memory for time)
SAVE_ACTS = os.environ.get("S0_SAVE_LAYER_ACTS", "1") not in ("0", "", "false")


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


def _check_dims(m) -> None:
    d = m.dims
    if (d.d_state, d.headdim, d.chunk_size, d.R) != (128, 64, 64, 32):
        raise NotImplementedError(
            f"the CUDA Mamba3 kernels are built for d_state=128, headdim=64, chunk=64, 32 rope angles; "
            f"got {d}; use impl='torch' for other geometries")


class _Mamba3Core:
    """Forward/backward of in_proj -> SSD -> out_norm -> out_proj on flat rows."""

    @staticmethod
    def forward(xn, B, L, m, want_gelu: bool = False):
        """``want_gelu``: also return gelu(o) from the out_proj GEMM's epilogue."""
        C = ext()
        d = m.dims
        ldp = _pad8(d.d_in_proj)
        H = xn.shape[1]
        Hp = _pad8(H)
        w_in = W.bf16_padded(m.in_proj.kernel, ldp)
        if Hp != H:   # odd widths (the 503-wide book layers): pad K so the GEMM rows are 16-byte aligned
            xn = F.pad(xn, (0, Hp - H))
            w_in = F.pad(w_in, (0, 0, 0, Hp - H))
        ag = getattr(m.in_proj.kernel, "_s0_ag", None)      # FSDP: in_proj gathered inside its GEMM
        proj = ag(xn) if (ag is not None and Hp == H and ldp == d.d_in_proj) else G.proj(xn, w_in)   # [T, ldp]
        out = C.m3_fwd(proj, B, L, d.n_heads, m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias,
                       m.C_bias, m.D, m.A_floor, m.B_norm.eps, return_prep=SAVE_STATES)
        y, states = out[0], out[1]
        prep = tuple(out[4:]) if SAVE_STATES else ()
        y2 = y.view(-1, d.d_inner)
        yn, yr = C.rms_fwd(y2, m.out_norm.scale, m.out_norm.eps)
        g = None
        if want_gelu and Hp == H:
            o, g = G.proj_gelu(yn, W.bf16_padded(m.out_proj.kernel, Hp))
        else:
            o = G.proj(yn, W.bf16_padded(m.out_proj.kernel, Hp))      # [T, Hp]
        if Hp != H:
            o = o[:, :H]
        if want_gelu:
            return o, g, proj, y2, yr, ((states,) + prep if SAVE_STATES else None)
        # the passed chunk states (bf16, B*nh*nc*P*N) and the per-token prep (BCNorm'd B/C,
        # dt, decay, gate, angle rates, chunk carries: ~1/8 of the states' size) are kept for
        # the backward unless the model is set to recompute them (memory for time)
        return o, proj, y2, yr, ((states,) + prep if SAVE_STATES else None)

    @staticmethod
    def backward(do, xn, proj, y2, yr, B, L, m, states=None):
        """``states``: None, or the forward's saved (states, *prep) tuple."""
        """Returns (dxn bf16, grads dict keyed by parameter)."""
        C = ext()
        d = m.dims
        ldp = proj.shape[1]
        H = xn.shape[1]
        Hp = _pad8(H)
        w_out = W.bf16_padded(m.out_proj.kernel, Hp)
        w_in = W.bf16_padded(m.in_proj.kernel, ldp)
        if Hp != H:
            do = F.pad(do, (0, Hp - H))
            xn = F.pad(xn, (0, Hp - H))
            w_in = F.pad(w_in, (0, 0, 0, Hp - H))
        yn, _ = C.rms_fwd(y2, m.out_norm.scale, m.out_norm.eps)
        g_out_proj = G.wgrad(m.out_proj.kernel, yn, do)
        dyn = G.proj_dx(do, w_out)
        dy, g_out_norm = C.rms_bwd(dyn.contiguous(), y2, m.out_norm.scale, yr)
        saved_states = states[0] if states else None
        saved_prep = list(states[1:]) if states and len(states) in (7, 8) else None
        dproj, dwB, dwC, ddtb, dD, dCb, dBb = C.m3_bwd(
            proj, dy, m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D, B, L,
            d.n_heads, m.A_floor, m.B_norm.eps, saved_states=saved_states, saved_prep=saved_prep)
        g_in = G.wgrad(m.in_proj.kernel, xn, dproj)
        dxn = G.proj_dx(dproj, w_in)[:, :H]
        grads = {m.out_proj.kernel: g_out_proj, m.out_norm.scale: g_out_norm, m.in_proj.kernel: g_in,
                 m.B_norm.scale: dwB, m.C_norm.scale: dwC, m.dt_bias: ddtb, m.D: dD,
                 m.C_bias: dCb, m.B_bias: dBb}
        return dxn, grads


def _mixer_params(m):
    return [m.in_proj.kernel, m.dt_bias, m.B_bias, m.C_bias, m.B_norm.scale, m.C_norm.scale, m.D,
            m.out_norm.scale, m.out_proj.kernel]


class _MixerFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, module, *params):
        B, L, H = u.shape
        xn = u.reshape(-1, H).to(torch.bfloat16).contiguous()
        o, proj, y2, yr, st = _Mamba3Core.forward(xn, B, L, module)
        ctx.module, ctx.shape, ctx.in_dtype = module, (B, L, H), u.dtype
        ctx.n_st = 0 if st is None else len(st)
        ctx.save_for_backward(xn, proj, y2, yr, *(st or ()))
        return o.view(B, L, H)

    @staticmethod
    def backward(ctx, do):
        xn, proj, y2, yr, *st = ctx.saved_tensors
        st = tuple(st) if ctx.n_st else None
        B, L, H = ctx.shape
        m = ctx.module
        do = do.reshape(-1, H).to(torch.bfloat16).contiguous()
        dxn, grads = _Mamba3Core.backward(do, xn, proj, y2, yr, B, L, m, st)
        du = dxn.view(B, L, H).to(ctx.in_dtype)
        return (du, None) + tuple(grads[p] for p in _mixer_params(m))


def mamba3_mixer(u: torch.Tensor, module) -> torch.Tensor:
    _check_dims(module)
    return _MixerFn.apply(u, module, *_mixer_params(module))


class _LayerFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, layer, *params):
        C = ext()
        m = layer.seq
        B, L, H = x.shape
        xf = x.reshape(-1, H)
        if xf.dtype != torch.float32 or not xf.is_contiguous():
            xf = xf.float().contiguous()
        fs = getattr(layer, "_s0_fsdp", None)
        if fs is not None:                # sharded kernels: gather this layer's (parallel/fsdp.py)
            fs.before_forward(layer)
        xn, mu, rs = C.ln_fwd(xf, layer.norm.scale, layer.norm.bias, layer.norm.eps)
        o, g, proj, y2, yr, st = _Mamba3Core.forward(xn, B, L, m, want_gelu=True)
        if g is None:
            g = C.gelu_fwd(o)
        h = G.proj(g, W.bf16(layer.out2.kernel))
        out = C.glu_res_fwd(xf, g, h, layer.out2.bias)
        ctx.layer, ctx.shape = layer, (B, L, H)
        ctx.n_st = 0 if st is None else len(st)
        ctx.saved_acts = SAVE_ACTS
        acts = (xn, g) if SAVE_ACTS else ()
        ctx.save_for_backward(xf, mu, rs, proj, y2, yr, o, h, *acts, *(st or ()))
        return out.view(B, L, H)

    @staticmethod
    def backward(ctx, dout):
        C = ext()
        xf, mu, rs, proj, y2, yr, o, h, *rest = ctx.saved_tensors
        if ctx.saved_acts:
            xn_s, g_s, *rest = rest
        st = tuple(rest) if ctx.n_st else None
        layer = ctx.layer
        m = layer.seq
        B, L, H = ctx.shape
        fs = getattr(layer, "_s0_fsdp", None)
        if fs is not None:                # gather the kernels again, point their grads at the layer buffer
            fs.before_backward(layer)
        dout = dout.reshape(-1, H)
        if dout.dtype != torch.float32 or not dout.is_contiguous():
            dout = dout.float().contiguous()
        g = g_s if ctx.saved_acts else C.gelu_fwd(o)
        dh, dgp, db2 = C.glu_res_bwd(dout, g, h, layer.out2.bias)
        g_out2 = G.wgrad(layer.out2.kernel, g, dh)
        dgm = G.proj_dx(dh, W.bf16(layer.out2.kernel))
        do = C.gelu_bwd(o, dgp, dgm.contiguous())
        xn = xn_s if ctx.saved_acts else C.ln_fwd(xf, layer.norm.scale, layer.norm.bias, layer.norm.eps)[0]
        dxn, grads = _Mamba3Core.backward(do, xn, proj, y2, yr, B, L, m, st)
        dx, dlw, dlb = C.ln_bwd(dxn.contiguous(), xf, mu, rs, layer.norm.scale, dout)
        grads[layer.norm.scale] = dlw
        grads[layer.norm.bias] = dlb
        grads[layer.out2.kernel] = g_out2
        grads[layer.out2.bias] = db2
        if fs is not None:                # reduce-scatter the layer's kernel gradients (side stream)
            fs.after_backward(layer)
        return (dx.view(B, L, H), None) + tuple(grads[p] for p in _layer_params(layer))


@torch.no_grad()
def mamba3_layer_prefill(x: torch.Tensor, layer):
    """(decode state, output) of the fused half_glu1 Mamba3 layer over a context: the same
    kernels as the training forward (LayerNorm, chunked SSD with its final state, RMSNorm,
    GELU, gate + residual), so generation conditions on exactly the training function."""
    C = ext()
    B, L, H = x.shape
    xf = x.reshape(-1, H)
    if xf.dtype != torch.float32 or not xf.is_contiguous():
        xf = xf.float().contiguous()
    xn, _, _ = C.ln_fwd(xf, layer.norm.scale, layer.norm.bias, layer.norm.eps)
    st, o = layer.seq.prefill(xn.view(B, L, H))
    g = C.gelu_fwd(o.reshape(-1, H).to(torch.bfloat16).contiguous())
    h = g @ W.bf16(layer.out2.kernel)
    out = C.glu_res_fwd(xf, g, h, layer.out2.bias)
    return st, out.view(B, L, H)


@torch.no_grad()
def mamba3_layer_step(state, x: torch.Tensor, layer):
    """Recurrent step (1..8 known tokens) of the fused half_glu1 Mamba3 layer with the
    training forward's row kernels (4 launches + 3 GEMMs + the decode kernel per layer
    instead of a chain of elementwise ops)."""
    C = ext()
    B, L, H = x.shape
    xf = x.reshape(-1, H)
    if xf.dtype != torch.float32 or not xf.is_contiguous():
        xf = xf.float().contiguous()
    xn, _, _ = C.ln_fwd(xf, layer.norm.scale, layer.norm.bias, layer.norm.eps)
    state, o = layer.seq.step(state, xn.view(B, L, H))
    g = C.gelu_fwd(o.reshape(-1, H).to(torch.bfloat16).contiguous())
    h = g @ W.bf16(layer.out2.kernel)
    out = C.glu_res_fwd(xf, g, h, layer.out2.bias)
    return state, out.view(B, L, H)


def _layer_params(layer):
    return [layer.norm.scale, layer.norm.bias] + _mixer_params(layer.seq) + [layer.out2.kernel, layer.out2.bias]


def mamba3_sequence_layer(x: torch.Tensor, layer) -> torch.Tensor:
    _check_dims(layer.seq)
    if x.shape[-1] % 8:
        raise NotImplementedError("the fused layer path needs d_model % 8 == 0")
    return _LayerFn.apply(x, layer, *_layer_params(layer))


class _SSDCarryFn(torch.autograd.Function):
    """The SSD on a projection buffer, continued from a carried state and angle (context
    parallelism): ``(proj, init_state, init_angle, params) -> (y, final_state)``, with the
    gradients of both inputs from the reverse walker (the gradient of the final state enters
    as its initial carry)."""

    @staticmethod
    def forward(ctx, proj, s0, th0, m, B, L, wB, wC, dt_bias, Bb, Cb, D):
        C = ext()
        d = m.dims
        out = C.m3_fwd(proj, B, L, d.n_heads, wB, wC, dt_bias, Bb, Cb, D, m.A_floor, m.B_norm.eps,
                       want_final=True, return_prep=True, init_state=s0,
                       init_angle=th0 if th0 is not None else torch.zeros(B, d.n_heads, d.R, device=proj.device))
        y, states, fin = out[0], out[1], out[2]
        ctx.m, ctx.B, ctx.L = m, B, L
        ctx.has_s0, ctx.has_th0 = s0 is not None, th0 is not None
        ctx.save_for_backward(proj, states, fin, wB, wC, dt_bias, Bb, Cb, D, *out[4:])
        return y, fin

    @staticmethod
    def backward(ctx, dy, dfin):
        C = ext()
        proj, states, fin, wB, wC, dt_bias, Bb, Cb, D, *prep = ctx.saved_tensors
        m, B, L = ctx.m, ctx.B, ctx.L
        d = m.dims
        if dy is None:
            dy = torch.zeros(B, L, d.d_inner, dtype=torch.bfloat16, device=proj.device)
        res = C.m3_bwd(proj, dy.to(torch.bfloat16).contiguous(), wB, wC, dt_bias, Bb, Cb, D, B, L, d.n_heads,
                       m.A_floor, m.B_norm.eps, saved_states=states, saved_prep=list(prep),
                       d_final=dfin.float().contiguous() if dfin is not None else None, want_d_init=True,
                       final_state=fin)
        dproj, dwB, dwC, ddtb, dD, dCb, dBb, ds0, dth0 = res
        return (dproj, ds0 if ctx.has_s0 else None, dth0 if ctx.has_th0 else None, None, None, None,
                dwB, dwC, ddtb, dBb, dCb, dD)


def mamba3_ssd_carry(proj, m, B, L, init_state=None, init_angle=None):
    """SSD of ``proj`` ([B*L, ldp] bf16, the module's projection layout) continued from
    ``init_state`` ([B, nh, P, N] fp32) and ``init_angle`` ([B, nh, R]); returns
    ``(y [B, L, d_inner] bf16, final_state [B, nh, P, N] fp32)``, differentiable in all."""
    _check_dims(m)
    return _SSDCarryFn.apply(proj, init_state, init_angle, m, B, L, m.B_norm.scale, m.C_norm.scale, m.dt_bias,
                             m.B_bias, m.C_bias, m.D)
