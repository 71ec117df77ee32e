"""SequenceLayer and StackedEncoder: the residual wrapper around every mixer.

Same structure as the reference (``src/base_model/models/layers.py:21-170``,
``seq_model.py:7-180``): pre-LayerNorm -> mixer -> GELU (tanh form) -> GLU
variant -> residual, or the post-norm ordering when ``prenorm`` is False.
Attention mixers (``is_transformer``) carry their own norm and residual and are
passed straight through.  Hybrid stacks place a second mixer factory at
``attn_layers`` positions.

On CUDA the Mamba3 pre-norm ``half_glu1`` layer -- the production
configuration -- runs as one fused autograd function
(:func:`sigma0_b200.ops.mamba3_layer.mamba3_sequence_layer`).
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch
import torch.nn as nn
import torch.utils.checkpoint
import torch.nn.functional as F

from .common import Dense, Embed, LayerNorm, gelu_tanh


class SequenceLayer(nn.Module):
    def __init__(self, mixer: nn.Module, d_model: int, activation: str = "half_glu1",
                 prenorm: bool = True, dropout: float = 0.0):
        super().__init__()
        self.seq = mixer
        self.d_model = d_model
        self.activation = activation
        self.prenorm = prenorm
        self.dropout = dropout
        self.is_transformer = bool(getattr(mixer, "is_transformer", False))
        if not self.is_transformer:
            if activation == "full_glu":
                self.out1 = Dense(d_model, d_model)
                self.out2 = Dense(d_model, d_model)
            elif activation in ("half_glu1", "half_glu2"):
                self.out2 = Dense(d_model, d_model)
            elif activation != "gelu":
                raise NotImplementedError(f"Activation: {activation} not implemented")
            self.norm = LayerNorm(d_model)

    def _fused_ok(self, x) -> bool:
        from .mamba3 import Mamba3
        return (x.is_cuda and isinstance(self.seq, Mamba3) and self.seq.impl == "cuda"
                and type(self.norm) is LayerNorm and self.prenorm and self.activation == "half_glu1" and self.dropout == 0.0
                and self.d_model % 8 == 0)

    def _act(self, x):
        cd = getattr(self.seq, "compute_dtype", torch.float32)
        if self.activation == "full_glu":
            g = gelu_tanh(x)
            return self.out1(g, dtype=cd).float() * torch.sigmoid(self.out2(g, dtype=cd).float())
        if self.activation == "half_glu1":
            g = gelu_tanh(x)
            return g.float() * torch.sigmoid(self.out2(g, dtype=cd).float())
        if self.activation == "half_glu2":
            g = gelu_tanh(x)
            return x.float() * torch.sigmoid(self.out2(g, dtype=cd).float())
        return gelu_tanh(x).float()

    def forward(self, x):
        if self.is_transformer:
            return self.seq(x)
        if self._fused_ok(x):
            from ..ops.mamba3_layer import mamba3_sequence_layer
            return mamba3_sequence_layer(x, self)
        skip = x
        if self.prenorm:
            x = self.norm(x)
        x = self.seq(x)
        x = F.dropout(self._act(x), self.dropout, self.training)
        x = skip + x
        if not self.prenorm:
            x = self.norm(x)
        return x

    # -- decode ---------------------------------------------------------------------
    def initial_state(self, batch, device=None, **kw):
        return self.seq.initial_state(batch, device=device, **kw)

    def step(self, state, x):
        if self.is_transformer:
            return self.seq.step(state, x)
        if self._fused_ok(x) and x.shape[1] <= 8:
            from ..ops.mamba3_layer import mamba3_layer_step
            return mamba3_layer_step(state, x, self)
        skip = x
        if self.prenorm:
            x = self.norm(x)
        state, x = self.seq.step(state, x)
        x = skip + self._act(x)
        if not self.prenorm:
            x = self.norm(x)
        return state, x

    @torch.no_grad()
    def prefill(self, x, max_cache_len=None):
        """Training-identical forward that also returns the decode state."""
        if self.is_transformer:
            return self.seq.prefill(x, max_cache_len)
        if self._fused_ok(x):
            from ..ops.mamba3_layer import mamba3_layer_prefill
            return mamba3_layer_prefill(x, self)
        skip = x
        h = self.norm(x) if self.prenorm else x
        if hasattr(self.seq, "prefill"):
            state, h = self.seq.prefill(h)
        else:
            state, h = self.seq.step(self.seq.initial_state(x.shape[0], x.device), h)
        x = skip + self._act(h)
        if not self.prenorm:
            x = self.norm(x)
        return state, x


class StackedEncoder(nn.Module):
    """Encoder (Embed or Dense) followed by ``n_layers`` SequenceLayers (``layers_i``)."""

    def __init__(self, factory: Callable[[], nn.Module], d_model: int, n_layers: int,
                 d_input: Optional[int] = None, use_embed_layer: bool = False,
                 vocab_size: int = -1, activation: str = "half_glu1", prenorm: bool = True,
                 dropout: float = 0.0, attn_factory: Optional[Callable[[], nn.Module]] = None,
                 attn_layers: Sequence[int] = ()):
        super().__init__()
        self.encoder = Embed(vocab_size, d_model) if use_embed_layer else Dense(d_input, d_model)
        # dtype of the input Dense's GEMM on CUDA (bf16 tensor cores when the model computes
        # in bf16; fp32 would run a SIMT GEMM); the embedding lookup ignores it
        self.compute_dtype = torch.float32
        attn_at = frozenset(attn_layers) if attn_factory is not None else frozenset()
        if attn_at and max(attn_at) >= n_layers:
            raise ValueError(f"attn_layers={tuple(sorted(attn_at))} out of range for n_layers={n_layers}")
        self.n_layers = n_layers
        self.remat = False            # recompute each layer's activations in the backward pass
        for i in range(n_layers):
            mixer = attn_factory() if i in attn_at else factory()
            self.add_module(f"layers_{i}", SequenceLayer(mixer, d_model, activation, prenorm, dropout))

    @property
    def layers(self):
        return [getattr(self, f"layers_{i}") for i in range(self.n_layers)]

    def _encode(self, x):
        if isinstance(self.encoder, Dense) and x.is_cuda and self.compute_dtype != torch.float32:
            return self.encoder(x, dtype=self.compute_dtype)
        return self.encoder(x)

    def forward(self, x):
        x = self._encode(x)
        remat = self.remat and self.training and torch.is_grad_enabled()
        for layer in self.layers:
            x = torch.utils.checkpoint.checkpoint(layer, x, use_reentrant=False) if remat else layer(x)
        return x

    def initial_state(self, batch, device=None):
        return [l.initial_state(batch, device) for l in self.layers]

    @torch.no_grad()
    def prefill(self, x, max_cache_len=None):
        x = self._encode(x)
        states = []
        for layer in self.layers:
            st, x = layer.prefill(x, max_cache_len)
            states.append(st)
        return states, x

    def step(self, states, x):
        x = self._encode(x)
        new = []
        for s, layer in zip(states, self.layers):
            s, x = layer.step(s, x)
            new.append(s)
        return new, x
