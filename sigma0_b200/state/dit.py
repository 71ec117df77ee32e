"""FrameDiT: a diffusion transformer that denoises a window of book frames, one token per frame.

Compatibility contract with the reference (``src/state/dit.py:165-235``): the parameter
tree (module names and shapes) and the function it computes are the same, so state
dicts and trained checkpoints move between the two code bases.  The computation:

* ``h = input_proj([x_t | cond | gen])`` -- the noisy frames, the clean context
  (zeros where a frame is generated) and a 0/1 "generate this frame" channel;
  ``C`` input columns only for an unconditional model;
* flow-time conditioning: a sinusoidal code of ``1000 t`` (cosines then sines,
  float32) through ``time_embedding`` (Linear, SiLU, Linear) and ``time_projection``
  (SiLU, Linear to 6 x H); each block adds its own learned (1, 6, H) table and splits
  the sum into shift / scale / gate for the attention and the MLP branch;
* each block: ``h += gate_a * attn(LN(h) * (1 + scale_a) + shift_a)`` and
  ``h += gate_m * mlp(LN(h) * (1 + scale_m) + shift_m)``, LayerNorms without affine;
  attention is bidirectional over the frames with per-head RMSNorm on queries and keys
  followed by rotary position phases on consecutive pairs of channels;
* output: affine LayerNorm, then ``velocity_head``.

At construction the velocity head is zero (the model starts at v = 0) and the input
columns of the context and mask channels are zero, so a conditional model initialised
from an unconditional checkpoint starts out computing the same function.

This module's own choices: rotary phases as complex multiplication computed per call
in float32 (no cached table), the sinusoid from a frequency vector held as a plain
tensor, ``torch.nn.RMSNorm`` for the query / key norms, and the conditioning binders
as small callable objects.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

_TIME_SCALE = 1000.0        # flow time t in [0, 1] is embedded as the position 1000 t
_ROPE_BASE = 10000.0
_NORM_EPS = 1e-6


@dataclass
class FrameDiTConfig:
    channels: int = 41            # chart channels per frame
    hidden: int = 128
    depth: int = 4
    heads: int = 4
    mlp_ratio: float = 4.0
    max_seq_len: int = 4096       # longest frame window the model accepts
    freq_dim: int = 256           # width of the sinusoidal time code
    conditional: bool = True      # input carries context + mask channels

    def __post_init__(self):
        if self.hidden % self.heads or (self.hidden // self.heads) % 2:
            raise ValueError(f"hidden={self.hidden} must split into {self.heads} heads of even width")

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def input_dim(self) -> int:
        return self.channels * (2 if self.conditional else 1) + int(self.conditional)


def timestep_embedding(t: torch.Tensor, dim: int) -> torch.Tensor:
    """Sinusoidal code of the flow time: [cos(1000 t f_k), sin(1000 t f_k)] with the
    geometric frequencies f_k = 10000^(-k / (dim/2)), k < dim/2 (computed in float32)."""
    freqs = torch.exp(torch.arange(dim // 2, device=t.device, dtype=torch.float32)
                      * (-math.log(_ROPE_BASE) / (dim // 2)))
    phase = torch.outer(t.float() * _TIME_SCALE, freqs)
    return torch.cat((torch.cos(phase), torch.sin(phase)), dim=-1).to(t.dtype)


def _rotate_pairs(x: torch.Tensor, max_len: int) -> torch.Tensor:
    """Rotary position phases on consecutive channel pairs (2i, 2i+1) of ``x`` (B, heads, L, d):
    pair i of frame p turns by the angle p * 10000^(-2i/d), in float32."""
    L, d = x.shape[-2], x.shape[-1]
    if L > max_len:
        raise ValueError(f"sequence of {L} frames exceeds max_seq_len={max_len}")
    inv = _ROPE_BASE ** (-torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d)
    phase = torch.polar(torch.ones(L, d // 2, device=x.device),
                        torch.arange(L, device=x.device, dtype=torch.float32)[:, None] * inv)
    z = torch.view_as_complex(x.float().reshape(*x.shape[:-1], d // 2, 2).contiguous())
    return torch.view_as_real(z * phase).flatten(-2).to(x.dtype)


class FrameSelfAttention(nn.Module):
    """Bidirectional multi-head attention over frames (parameter names q, k, v, o,
    q_norm, k_norm as in the reference tree)."""

    def __init__(self, hidden: int, heads: int, max_seq_len: int):
        super().__init__()
        self.heads, self.max_seq_len = heads, max_seq_len
        self.q = nn.Linear(hidden, hidden)
        self.k = nn.Linear(hidden, hidden)
        self.v = nn.Linear(hidden, hidden)
        self.o = nn.Linear(hidden, hidden)
        d = hidden // heads
        self.q_norm = nn.RMSNorm(d, eps=_NORM_EPS)
        self.k_norm = nn.RMSNorm(d, eps=_NORM_EPS)

    def _heads(self, y: torch.Tensor) -> torch.Tensor:
        B, L, _ = y.shape
        return y.unflatten(-1, (self.heads, -1)).permute(0, 2, 1, 3)      # (B, heads, L, d)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        q = _rotate_pairs(self.q_norm(self._heads(self.q(x))), self.max_seq_len)
        k = _rotate_pairs(self.k_norm(self._heads(self.k(x))), self.max_seq_len)
        y = F.scaled_dot_product_attention(q, k, self._heads(self.v(x)))
        return self.o(y.permute(0, 2, 1, 3).flatten(-2))


class FrameBlock(nn.Module):
    """One transformer block with a shift / scale / gate modulation per branch."""

    def __init__(self, cfg: FrameDiTConfig):
        super().__init__()
        H = cfg.hidden
        self.norm1 = nn.LayerNorm(H, elementwise_affine=False)
        self.attn = FrameSelfAttention(H, cfg.heads, cfg.max_seq_len)
        self.norm2 = nn.LayerNorm(H, elementwise_affine=False)
        inner = int(H * cfg.mlp_ratio)
        self.ffn = nn.Sequential(nn.Linear(H, inner), nn.GELU(approximate="tanh"), nn.Linear(inner, H))
        self.modulation = nn.Parameter(torch.randn(1, 6, H) * H ** -0.5)

    def forward(self, h: torch.Tensor, tmod: torch.Tensor) -> torch.Tensor:
        m = (self.modulation + tmod)[:, :, None, :]                 # (B, 6, 1, H)
        shift_a, scale_a, gate_a, shift_m, scale_m, gate_m = m.unbind(1)
        h = h + gate_a * self.attn(torch.addcmul(shift_a, self.norm1(h), 1 + scale_a))
        return h + gate_m * self.ffn(torch.addcmul(shift_m, self.norm2(h), 1 + scale_m))


class FrameDiT(nn.Module):
    """``forward(x (B, L, input_dim), t (B,)) -> velocity (B, L, channels)``."""

    def __init__(self, cfg: FrameDiTConfig):
        super().__init__()
        self.cfg = cfg
        H = cfg.hidden
        self.input_proj = nn.Linear(cfg.input_dim, H)
        self.time_embedding = nn.Sequential(nn.Linear(cfg.freq_dim, H), nn.SiLU(), nn.Linear(H, H))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(H, 6 * H))
        self.blocks = nn.ModuleList(FrameBlock(cfg) for _ in range(cfg.depth))
        self.final_norm = nn.LayerNorm(H)
        self.velocity_head = nn.Linear(H, cfg.channels)
        self._zero_init()

    @torch.no_grad()
    def _zero_init(self) -> None:
        nn.init.zeros_(self.velocity_head.weight)
        nn.init.zeros_(self.velocity_head.bias)
        if self.cfg.conditional:                      # context and mask columns start silent
            self.input_proj.weight[:, self.cfg.channels:] = 0.0

    def forward(self, x: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        tcode = self.time_embedding(timestep_embedding(t, self.cfg.freq_dim))
        tmod = self.time_projection(tcode).unflatten(-1, (6, self.cfg.hidden))
        h = self.input_proj(x)
        for block in self.blocks:
            h = block(h, tmod)
        return self.velocity_head(self.final_norm(h))


class _Conditioned:
    """A ``flow.ModelFn`` of a conditional FrameDiT with fixed context / mask channels."""

    def __init__(self, model: FrameDiT, cond: torch.Tensor, gen: torch.Tensor):
        self.model, self.cond, self.gen = model, cond, gen

    def __call__(self, x_t: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        cond = self.cond if self.cond is not None else torch.zeros_like(x_t)
        gen = self.gen if self.gen is not None else torch.ones_like(x_t[..., :1])
        return self.model(torch.cat((x_t, cond, gen), dim=-1), t)


def bind_condition(model: FrameDiT, context: torch.Tensor, obs_mask: torch.Tensor):
    """ModelFn that conditions on the clean ``context`` (B, L, C) wherever ``obs_mask``
    (B, L) is 1; the mask channel the model reads is its complement (1 = generate)."""
    if not model.cfg.conditional:
        raise ValueError("the model was built unconditional")
    given = obs_mask.to(context.dtype).unsqueeze(-1)
    return _Conditioned(model, context * given, 1.0 - given)


def bind_unconditional(model: FrameDiT):
    """ModelFn with no frame given (every frame generated)."""
    return _Conditioned(model, None, None) if model.cfg.conditional else model
