"""Autoregressive generation: syntax masks, sampling, the engine-in-the-loop generator."""
from .validation import syntax_validation_matrix, sample
from .generate import Generator, GenOutput, apply_message_cpu, gen_layout, safe_mid_price

__all__ = ["syntax_validation_matrix", "sample", "Generator", "GenOutput", "apply_message_cpu", "gen_layout",
           "safe_mid_price"]
