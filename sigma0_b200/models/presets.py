"""Named model/workload presets (the benchmark configurations).

* ``smoke``: the CPU smoke configuration -- d_model 128, two Mamba3 layers
  (one message, one fused), d_state 16, headdim 32, expand 2, 22-token
  messages, batch 2 x 20 messages.
* ``350m``: the flagship training configuration -- Mamba3, d_model 1024,
  48 Mamba3 layers in total (2 message + 1 book pre + 1 book post + 44 fused),
  d_state 128, headdim 64, expand 2, 22-token messages with the vocabulary
  padded to 12,288, 500 messages (11,000 tokens) per sequence, 8 sequences per
  GPU (global batch 64 on 8 GPUs), bf16 compute with float32 master weights.
* ``75m``: the reference's published recipe model (``docs/training.md:108-111``):
  d_model 1024, 2 message + 6 fused layers, 1 book pre + 1 book post layer.
* ``hybrid1b`` / ``nsa1b``: the long-context configuration -- d_model 2048, 24 layers
  (2 message + 1 book pre + 1 book post + 20 fused), 3,000 messages (66,000 tokens) per
  sequence, 8 sequences per optimizer step (4 accumulated micro-batches of 2: the
  activations of 8 whole sequences do not fit in 180 GB), meant to run context-parallel
  over 8 GPUs.  ``hybrid1b`` is
  hybrid_mamba3 with one attention block (16 heads of dim 128) after every four Mamba3
  layers of the trunk; ``nsa1b`` is the NSA transformer with compression block 32,
  selection block 64, top-16 selected blocks and a 512-token sliding window.
"""
from __future__ import annotations

from types import SimpleNamespace

PRESETS = {
    "smoke": dict(architecture="mamba3", d_model=128, mamba3_d_state=16, mamba3_headdim=32,
                  mamba3_expand=2, n_message_layers=1, n_layers=1, n_book_pre_layers=0,
                  n_book_post_layers=0, token_mode="22tok", vocab_size=12012, msg_len=22,
                  n_messages=20, micro_bsz=2, dtype="float32", d_book=503),
    "350m": dict(architecture="mamba3", d_model=1024, mamba3_d_state=128, mamba3_headdim=64,
                 mamba3_expand=2, n_message_layers=2, n_layers=44, n_book_pre_layers=1,
                 n_book_post_layers=1, token_mode="22tok", vocab_size=12288, msg_len=22,
                 n_messages=500, micro_bsz=8, dtype="bfloat16", d_book=503),
    # GDN backbone ~1B, d_model 2048, 24 layers (2 message + 1 book pre + 1 book
    # post + 20 fused), 16 heads of dim 128 (value dim 256), chunk 64; 1,000 messages x 22 tokens;
    # run with tensor parallelism (--tp 4 on 8 GPUs: TP4 x DP2)
    "gdn1b": dict(architecture="gdn", d_model=2048, gdn_head_dim=128, gdn_num_heads=16, gdn_expand_v=2,
                  gdn_chunk_size=64, n_message_layers=2, n_layers=20, n_book_pre_layers=1,
                  n_book_post_layers=1, token_mode="22tok", vocab_size=12288, msg_len=22,
                  n_messages=1000, micro_bsz=4, dtype="float32", d_book=503),
    "75m": dict(architecture="mamba3", d_model=1024, mamba3_d_state=128, mamba3_headdim=64,
                mamba3_expand=2, n_message_layers=2, n_layers=6, n_book_pre_layers=1,
                n_book_post_layers=1, token_mode="26tok", vocab_size=2112, msg_len=26,
                n_messages=500, micro_bsz=1, dtype="bfloat16", d_book=503),
    "hybrid1b": dict(architecture="hybrid_mamba3", d_model=2048, mamba3_d_state=128, mamba3_headdim=64,
                     mamba3_expand=2, n_message_layers=2, n_layers=20, n_book_pre_layers=1,
                     n_book_post_layers=1, hybrid_attn_layers="4,9,14,19", hybrid_attn_heads=16,
                     token_mode="22tok", vocab_size=12288, msg_len=22, n_messages=3000, micro_bsz=2,
                     accum_steps=4,
                     dtype="bfloat16", d_book=503),
    "nsa1b": dict(architecture="nsa", d_model=2048, n_heads=16, nsa_strict_block=False, block_size=32,
                  nsa_select_block=64, block_counts=16, window_size=512, n_message_layers=2, n_layers=20,
                  n_book_pre_layers=1, n_book_post_layers=1, token_mode="22tok", vocab_size=12288,
                  msg_len=22, n_messages=3000, micro_bsz=2, accum_steps=4, dtype="bfloat16", d_book=503),
}

_DEFAULTS = dict(activation_fn="half_glu1", prenorm=True, p_dropout=0.0, use_book_data=True,
                 mamba3_chunk_size=64, mamba3_rope_fraction=0.5, tp_size=1, impl="torch",
                 ssm_lr_base=1e-3, lr_factor=1.0, weight_decay=0.05, max_grad_norm=1.0,
                 warmup_end=0.01, ignore_times=False)


def preset_args(name: str, **overrides) -> SimpleNamespace:
    if name not in PRESETS:
        raise ValueError(f"unknown preset {name!r}; choose one of {sorted(PRESETS)}")
    d = dict(_DEFAULTS)
    d.update(PRESETS[name])
    d.update(overrides)
    return SimpleNamespace(**d)
