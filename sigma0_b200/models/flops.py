"""Training FLOPs and model FLOPs utilisation for the LOB models.

The reference estimates FLOPs as ``correction(d_model) * 6 * N * D`` with an
empirically measured correction (``src/base_model/models/flops.py:1-120``).
Here the count is analytical and per component, for the kernels this
framework runs: every dense projection costs 2*in*out FLOPs per token forward
and twice that backward; the Mamba3 SSD adds its chunked contractions
(intra-chunk Q.K^T and (.)V, chunk states K^T.V, state readout Q.S) with the
backward counted as twice the forward plus the state recompute.  MFU is
reported against the measured bf16 peak of the GPU (``MEASURED_PEAKS.json``)
or a stated fallback.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

from .mamba3 import mamba3_dims


@dataclass
class FlopBreakdown:
    dense_fwd: float      # per token
    ssd_fwd: float        # per token
    decoder_fwd: float    # per token

    @property
    def fwd(self) -> float:
        return self.dense_fwd + self.ssd_fwd + self.decoder_fwd

    @property
    def train(self) -> float:
        """Forward + backward (2x forward for the projections; the SSD backward
        recomputes the chunk states: 2x forward plus one chunk-state pass)."""
        return 3 * (self.dense_fwd + self.decoder_fwd) + 3 * self.ssd_fwd + self.ssd_state_fwd

    ssd_state_fwd: float = 0.0


def mamba3_layer_flops(d_model: int, d_state=128, expand=2, headdim=64, chunk=64, rope_fraction=0.5):
    d = mamba3_dims(d_model, d_state, expand, headdim, chunk, rope_fraction)
    dense = 2 * d_model * d.d_in_proj + 2 * d.d_inner * d_model
    glu = 2 * d_model * d_model          # half-GLU output projection of the SequenceLayer
    nh, P, N, C = d.n_heads, d.headdim, d.d_state, d.chunk_size
    # per token, per head: QK^T row (C*N), scores x V (C*P), chunk state K^T V (N*P), readout Q S (N*P)
    intra = 2 * nh * (C * N + C * P) / 2          # causal: half the chunk on average
    states = 2 * nh * N * P
    readout = 2 * nh * N * P
    return dense + glu, intra + states + readout, states


def lob_model_flops(args) -> FlopBreakdown:
    """Per-token FLOPs of the outer LOB model for a preset/argparse namespace."""
    H = args.d_model
    kw = dict(d_state=args.mamba3_d_state, expand=args.mamba3_expand, headdim=args.mamba3_headdim,
              chunk=args.mamba3_chunk_size, rope_fraction=args.mamba3_rope_fraction)
    dense = ssd = st = 0.0
    for width, n in ((H, args.n_message_layers + args.n_layers + args.n_book_post_layers),
                     (args.d_book, args.n_book_pre_layers)):
        if n:
            a, b, c = mamba3_layer_flops(width, **kw)
            dense, ssd, st = dense + n * a, ssd + n * b, st + n * c
    if args.use_book_data:
        dense += 2 * args.d_book * H
        dense += 2 * (2 * H) * H      # fused encoder input projection from the concatenated streams
    dec = 2 * H * args.vocab_size
    return FlopBreakdown(dense, ssd, dec, st)


def measured_bf16_peak(default_tflops: float = 1590.0, sustained: bool = True) -> float:
    """bf16 dense peak in FLOP/s: MEASURED_PEAKS.json next to the package if present."""
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    p = os.path.join(here, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        key = "bf16_tflops_sustained" if sustained and "bf16_tflops_sustained" in d else "bf16_tflops"
        return float(d[key]) * 1e12
    except (OSError, KeyError, ValueError):
        return default_tflops * 1e12


def mfu(args, tokens_per_s: float, n_gpus: int = 1, peak_flops: float = None) -> float:
    peak = peak_flops or measured_bf16_peak()
    return lob_model_flops(args).train * tokens_per_s / (peak * n_gpus)
