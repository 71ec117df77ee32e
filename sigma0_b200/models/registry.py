"""Backbone registry: the one place where an architecture name becomes layer factories.

Behaviour kept compatible with the reference (``src/base_model/models/registry.py``):

* the seven architectures and their properties (who owns the residual wrapper, prefill,
  attention, whether ``--dtype`` is honoured) -- ``:63-76``;
* strict selection from ``--architecture`` plus the legacy ``ssm_type`` / ``model_type``
  metadata of old checkpoints, refusing any disagreement -- ``:136-187``;
* the Nemotron-H attention placement of ``hybrid_mamba3`` -- ``:79-100``;
* the recurrent-carry and attention-cache geometry of a layer rebuilt at another width
  (the book layers run at ``d_book``) -- ``:198-262``.

Here the architectures are rows of one table (:data:`ARCHITECTURES`); each row names
the builder that turns the run arguments into layer factories.  The selector tables
(every accepted and refused combination) and the placement indices are pinned by
``tests/test_registry.py`` against a golden file.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Dict, Mapping, Optional, Tuple

import torch

DEFAULT_ARCHITECTURE = "mamba3"


@dataclass(frozen=True)
class ArchSpec:
    """One architecture.  ``residual``: "wrapped" when the SequenceLayer adds the norm,
    GLU and residual around the mixer, "own" when the block carries them itself
    (attention blocks)."""
    name: str
    residual: str
    prefill: bool
    attention: bool
    reads_dtype: bool
    builder: str
    stepwise: bool = True

    @property
    def wrapper_policy(self) -> str:       # the reference's field name
        return "internal" if self.residual == "own" else "external"

    @property
    def supports_prefill(self) -> bool:
        return self.prefill

    @property
    def supports_stepwise_inference(self) -> bool:
        return self.stepwise

    @property
    def has_attention(self) -> bool:
        return self.attention


BackboneDefinition = ArchSpec   # the reference's name for the same record

#: architecture name -> properties; the order is the CLI order (the default first)
ARCHITECTURES: Dict[str, ArchSpec] = {s.name: s for s in (
    ArchSpec("mamba3", "wrapped", prefill=False, attention=False, reads_dtype=True, builder="mamba3"),
    ArchSpec("s5", "wrapped", prefill=False, attention=False, reads_dtype=False, builder="s5"),
    ArchSpec("gdn", "wrapped", prefill=False, attention=False, reads_dtype=False, builder="delta"),
    ArchSpec("kda", "wrapped", prefill=False, attention=False, reads_dtype=False, builder="delta"),
    ArchSpec("transformer", "own", prefill=True, attention=True, reads_dtype=True, builder="attention"),
    ArchSpec("nsa", "own", prefill=True, attention=True, reads_dtype=True, builder="attention"),
    ArchSpec("hybrid_mamba3", "wrapped", prefill=False, attention=True, reads_dtype=True, builder="mamba3"),
)}

#: names that used to exist and are refused with a pointer to their replacement
RETIRED = {"mamba2": "architecture 'mamba2' is intentionally not part of this model zoo; "
                     "use 'mamba3' for new experiments"}

DTYPE_AWARE_ARCHITECTURES = frozenset(n for n, s in ARCHITECTURES.items() if s.reads_dtype)


@dataclass(frozen=True)
class BackboneBuild:
    definition: ArchSpec
    factory_at: Callable[[int], Any]               # width -> mixer module
    carry_kwargs: Mapping[str, Any]
    attention_config: Optional[Mapping[str, Any]] = None
    attn_factory_at: Optional[Callable[[int], Any]] = None
    attn_layers: Tuple[int, ...] = ()

    @property
    def is_attention(self) -> bool:
        return self.definition.residual == "own"

    @property
    def is_hybrid(self) -> bool:
        return self.attn_factory_at is not None


# ---------------------------------------------------------------------------------------------
# names and selection
# ---------------------------------------------------------------------------------------------
def available_architectures() -> Tuple[str, ...]:
    return tuple(ARCHITECTURES)


def get_definition(name: str) -> ArchSpec:
    spec = ARCHITECTURES.get(name)
    if spec is not None:
        return spec
    if name in RETIRED:
        raise ValueError(RETIRED[name])
    raise ValueError(f"unknown architecture {name!r}; choose one of: {', '.join(ARCHITECTURES)}")


def architecture_has_attention(name: Optional[str]) -> bool:
    """Whether the architecture builds attention layers (so needs a KV cache and an
    attention config); read from the table, never from a list of names."""
    spec = ARCHITECTURES.get(name or "")
    return bool(spec and spec.attention)


def _lower(v: Optional[str]) -> Optional[str]:
    return v.lower() if v else None


# model_type values that name an attention architecture: old attention checkpoints stored
# one of these next to the argument parser's default ssm_type 's5'
_ATTENTION_MODEL_TYPES = frozenset(n for n, s in ARCHITECTURES.items() if s.residual == "own")


def _legacy_vote(ssm_type: Optional[str], model_type: Optional[str]) -> Optional[str]:
    """The architecture implied by the legacy pair, or None when it implies nothing."""
    if model_type in _ATTENTION_MODEL_TYPES:
        if ssm_type is not None and ssm_type not in ("s5", model_type):
            raise ValueError(f"conflicting legacy selectors: model_type={model_type!r}, ssm_type={ssm_type!r}")
        return model_type
    if ssm_type:                       # the real selector of recurrent checkpoints
        return ssm_type
    return model_type if model_type in ARCHITECTURES else None


def resolve_architecture(architecture: Optional[str] = None, *, ssm_type: Optional[str] = None,
                         model_type: Optional[str] = None) -> str:
    """The one canonical architecture name for a set of selectors.

    ``model_type`` must be empty, ``"ssm"`` or a known architecture (an unknown value never
    silently falls back to the default).  The explicit selector and the one implied by the
    legacy pair must agree; with neither, the default is used."""
    arch, ssm, mt = _lower(architecture), _lower(ssm_type), _lower(model_type)
    if mt is not None and mt != "ssm" and mt not in ARCHITECTURES:
        get_definition(mt)
    votes = [(k, v) for k, v in (("architecture", arch), ("legacy selector", _legacy_vote(ssm, mt))) if v]
    if not votes:
        return DEFAULT_ARCHITECTURE
    if len({v for _, v in votes}) > 1:
        raise ValueError("conflicting architecture selectors: " + ", ".join(f"{k}={v!r}" for k, v in votes))
    return get_definition(votes[0][1]).name


def architecture_from_args(args: Any) -> str:
    return resolve_architecture(getattr(args, "architecture", None), ssm_type=getattr(args, "ssm_type", None),
                                model_type=getattr(args, "model_type", None))


def stamp_architecture(args: Any, architecture: str) -> None:
    """Write the canonical name into every selector field (new checkpoints carry all three)."""
    args.architecture = architecture
    args.ssm_type = architecture
    args.model_type = architecture if architecture in _ATTENTION_MODEL_TYPES else "ssm"


# ---------------------------------------------------------------------------------------------
# hybrid placement
# ---------------------------------------------------------------------------------------------
# Nemotron-H interleaves 4 attention layers among its 31 sequence-mixing layers at relative
# depths between about a quarter and seven tenths; a stack of L layers gets the same share
# of attention layers spread evenly over that band, never in the first two layers or the last.
NEMOTRON_ATTENTION_FRACTION = 4 / 31
NEMOTRON_DEPTH_BAND = (0.26, 0.71)
_SINGLE_LAYER_DEPTH = 0.48            # one attention layer: the band's centre of mass


def nemotron_attention_indices(n_layers: int) -> Tuple[int, ...]:
    count = max(1, round(n_layers * NEMOTRON_ATTENTION_FRACTION))
    lo, hi = NEMOTRON_DEPTH_BAND
    rel = ([_SINGLE_LAYER_DEPTH] if count == 1 else
           [lo + (hi - lo) * j / (count - 1) for j in range(count)])
    first, last = 2, n_layers - 2
    return tuple(sorted({min(max(round(r * n_layers), first), last) for r in rel}))


# ---------------------------------------------------------------------------------------------
# geometry of layers rebuilt at another width
# ---------------------------------------------------------------------------------------------
def recurrent_carry_for_width(carry_kwargs: Mapping[str, Any], width: int) -> dict:
    """The recurrent-state geometry a mixer has at ``width`` (it shrinks heads the same way)."""
    c = dict(carry_kwargs)
    width = int(width)
    kind = c.get("ssm_type")
    if kind == "mamba3":
        inner = int(c["expand"]) * width
        hd = min(int(c.get("requested_headdim", c["headdim"])), inner)
        heads = max(1, inner // hd)
        tp = int(c.get("tp_size", 1))
        c.update(headdim=hd, n_heads=heads // (tp if heads % tp == 0 else 1))
    elif kind in ("gdn", "kda"):
        want_dim = int(c.get("requested_head_dim", c["head_dim"]))
        want_heads = int(c.get("requested_num_heads", c["num_heads"]))
        hd = min(want_dim, width)
        c.update(num_heads=min(want_heads, max(1, width // want_dim)), head_dim=hd,
                 head_v_dim=hd * int(c["expand_v"]))
    return c


def attention_config_for_width(backbone: BackboneBuild, width: int, *, max_cache_len=None) -> dict:
    """Attention-cache geometry at ``width``: the largest head count <= the configured one
    that divides the width."""
    if backbone.attention_config is None:
        raise ValueError(f"architecture {backbone.definition.name!r} does not use an attention cache")
    cfg = dict(backbone.attention_config)
    heads = _largest_divisor_heads(width, int(cfg["n_heads"]))
    cfg.update(n_heads=heads, head_dim=width // heads)
    if max_cache_len is not None:
        cfg["max_cache_len"] = int(max_cache_len)
    return cfg


# ---------------------------------------------------------------------------------------------
# builders: run arguments -> layer factories
# ---------------------------------------------------------------------------------------------
def _compute_dtype(args):
    return torch.bfloat16 if str(getattr(args, "dtype", "float32")) == "bfloat16" else torch.float32


def _arg(args, key, default):
    v = getattr(args, key, None)
    return default if v is None else v


def _largest_divisor_heads(width: int, heads: int) -> int:
    while heads > 1 and width % heads:
        heads -= 1
    return heads


def _build_mamba3(spec: ArchSpec, args, width: int, dtype, impl: str) -> BackboneBuild:
    from .mamba3 import Mamba3
    d_state = int(_arg(args, "mamba3_d_state", 128))
    expand = int(_arg(args, "mamba3_expand", 2))
    headdim = int(_arg(args, "mamba3_headdim", 64))
    chunk = int(_arg(args, "mamba3_chunk_size", 64))
    rope = float(_arg(args, "mamba3_rope_fraction", 0.5))
    tp = int(_arg(args, "tp_size", 1))

    def factory_at(w):
        return Mamba3(w, d_state=d_state, expand=expand, headdim=headdim, chunk_size=chunk,
                      rope_fraction=rope, tp_size=tp, dtype=dtype, impl=impl)

    carry = recurrent_carry_for_width({"ssm_type": "mamba3", "n_heads": 0, "headdim": headdim,
                                       "d_state": d_state, "num_rope_angles": int(d_state * rope / 2),
                                       "expand": expand, "tp_size": tp, "requested_headdim": headdim}, width)
    if spec.name != "hybrid_mamba3":
        return BackboneBuild(spec, factory_at, carry)

    from .transformer import TransformerBlock
    n_layers = int(_arg(args, "n_layers", 6))
    given = getattr(args, "hybrid_attn_layers", None)
    layers = (tuple(int(v) for v in str(given).split(",") if v.strip()) if given
              else nemotron_attention_indices(n_layers))
    if any(not 0 <= i < n_layers for i in layers):
        raise ValueError(f"hybrid_attn_layers={layers} out of range for n_layers={n_layers}")
    args.hybrid_attn_layers = ",".join(map(str, layers))
    heads = _largest_divisor_heads(width, int(_arg(args, "hybrid_attn_heads", 10)))
    d_ff = int(_arg(args, "hybrid_attn_d_ff", 0)) or 4 * width
    cache = int(_arg(args, "attention_max_cache_len", 26000))
    use_pe = bool(_arg(args, "hybrid_attn_positional_encoding", False))

    def attn_at(w):
        return TransformerBlock(w, n_heads=heads, d_ff=d_ff, dtype=dtype, max_cache_len=cache,
                                use_positional_encoding=use_pe, impl=impl)

    cfg = {"model_type": "transformer", "n_heads": heads, "head_dim": width // heads, "max_cache_len": cache}
    return BackboneBuild(spec, factory_at, carry, attention_config=cfg, attn_factory_at=attn_at,
                         attn_layers=layers)


def _build_delta(spec: ArchSpec, args, width: int, dtype, impl: str) -> BackboneBuild:
    from .gdn import GDN
    head_dim = int(_arg(args, "gdn_head_dim", 128))
    heads = int(getattr(args, "gdn_num_heads", None) or max(1, width // head_dim))
    expand_v = int(_arg(args, "gdn_expand_v", 2))
    use_conv = bool(_arg(args, "gdn_use_conv", True))
    chunk = int(_arg(args, "gdn_chunk_size", 64))
    kda = spec.name == "kda"

    def factory_at(w):
        return GDN(w, num_heads=heads, head_dim=head_dim, expand_v=expand_v, chunk_size=chunk,
                   use_conv=use_conv, use_kda=kda, impl=impl)

    carry = recurrent_carry_for_width({"ssm_type": spec.name, "num_heads": heads, "head_dim": head_dim,
                                       "head_v_dim": head_dim * expand_v, "expand_v": expand_v,
                                       "use_conv": use_conv, "requested_num_heads": heads,
                                       "requested_head_dim": head_dim}, width)
    return BackboneBuild(spec, factory_at, carry)


def _build_s5(spec: ArchSpec, args, width: int, dtype, impl: str) -> BackboneBuild:
    from .s5 import make_s5_factory
    size = int(_arg(args, "ssm_size_base", 32))
    blocks = int(_arg(args, "blocks", 8))
    if size % blocks:
        raise ValueError("ssm_size_base must be divisible by blocks for S5")
    factory_at = make_s5_factory(size, blocks, conj_sym=bool(_arg(args, "conj_sym", True)),
                                 C_init=str(_arg(args, "C_init", "trunc_standard_normal")),
                                 discretization=str(_arg(args, "discretization", "zoh")),
                                 dt_min=float(_arg(args, "dt_min", 0.001)), dt_max=float(_arg(args, "dt_max", 0.1)),
                                 clip_eigs=bool(_arg(args, "clip_eigs", False)),
                                 bidirectional=bool(_arg(args, "bidirectional", False)))
    return BackboneBuild(spec, factory_at, {"ssm_type": spec.name})


def _build_attention(spec: ArchSpec, args, width: int, dtype, impl: str) -> BackboneBuild:
    heads = int(_arg(args, "n_heads", 16))
    if width % heads:
        raise ValueError(f"d_model={width} must be divisible by n_heads={heads}")
    d_ff = int(_arg(args, "d_ff", 0)) or 4 * width
    cache = int(_arg(args, "attention_max_cache_len", 26000))
    cfg = {"model_type": spec.name, "n_heads": heads, "head_dim": width // heads, "max_cache_len": cache,
           "dtype": dtype}
    if spec.name == "transformer":
        from .transformer import TransformerBlock

        def factory_at(w):
            return TransformerBlock(w, n_heads=heads, d_ff=d_ff, dtype=dtype, max_cache_len=cache, impl=impl)
    else:
        from .nsa import NSABlock
        from ..encoding import Message_Tokenizer
        msg_len = int(Message_Tokenizer.MSG_LEN)
        block = int(_arg(args, "block_size", msg_len))
        if bool(_arg(args, "nsa_strict_block", True)) and block != msg_len:
            raise ValueError(f"NSA block_size must equal the message length of the active encoding "
                             f"({msg_len}); got {block}")
        sel = int(_arg(args, "nsa_select_block", block))
        opts = dict(block_counts=int(_arg(args, "block_counts", 16)), window_size=int(_arg(args, "window_size", 512)),
                    full_causal_window=bool(_arg(args, "nsa_full_causal", True)),
                    pe_type=str(_arg(args, "pe_type", "rope")), rope_base=float(_arg(args, "rope_base", 10000.0)))

        def factory_at(w):
            return NSABlock(w, n_heads=heads, d_ff=d_ff, block_size=block, select_block=sel, dtype=dtype,
                            max_cache_len=cache, impl=impl, **opts)
        cfg["block_size"] = block
    carry = {"ssm_type": spec.name, "is_transformer": True, "transformer_config": cfg}
    return BackboneBuild(spec, factory_at, carry, cfg)


_BUILDERS = {"mamba3": _build_mamba3, "delta": _build_delta, "s5": _build_s5, "attention": _build_attention}


def build_backbone(args: Any, *, print_shapes: bool = False) -> BackboneBuild:
    spec = get_definition(architecture_from_args(args))
    dtype_name = str(getattr(args, "dtype", "float32"))
    if dtype_name != "float32" and not spec.reads_dtype:
        raise ValueError(f"--dtype={dtype_name} has no effect on architecture '{spec.name}': only "
                         f"{sorted(DTYPE_AWARE_ARCHITECTURES)} read it.")
    build = _BUILDERS[spec.builder](spec, args, int(args.d_model), _compute_dtype(args),
                                    str(_arg(args, "impl", "torch")))
    if print_shapes:
        print(f"[backbone] architecture={spec.name} wrapper={spec.wrapper_policy}")
        if build.attn_layers:
            print(f"[backbone] hybrid attention at trunk layers {build.attn_layers}")
    return build


def build_model(args: Any):
    """Build the outer LOB model for ``args`` (an argparse namespace or similar).  With
    ``remat`` every sequence layer recomputes its activations in the backward pass (the
    reference's ``--remat``, ``nn.remat`` of each layer); with ``batchnorm`` the sequence
    layers normalise with ``BatchNorm`` (momentum ``bn_momentum``) instead of ``LayerNorm``."""
    model = _build_model(args)
    if bool(_arg(args, "batchnorm", False)):
        from .common import BatchNorm
        from .layers import SequenceLayer
        mom = float(_arg(args, "bn_momentum", 0.9))
        for m in model.modules():
            if isinstance(m, SequenceLayer) and hasattr(m, "norm"):
                m.norm = BatchNorm(m.d_model, momentum=mom)
    if bool(_arg(args, "remat", False)):
        from .layers import StackedEncoder
        for m in model.modules():
            if isinstance(m, StackedEncoder):
                m.remat = True
    return model


def _build_model(args: Any):
    from .lob_model import LobModel
    from .legacy_norm import apply_legacy_norm, legacy_norm_enabled
    bb = build_backbone(args)
    if str(_arg(args, "token_mode", "")) == "1tok":      # the 1-token-per-message model family
        from .lob_model_1tok import OneTokenLobModel
        model = OneTokenLobModel(bb.factory_at, d_model=int(args.d_model), d_book=int(_arg(args, "d_book", 503)),
                                 n_fused_layers=int(_arg(args, "n_layers", 6)),
                                 n_book_pre_layers=int(_arg(args, "n_book_pre_layers", 1)),
                                 n_book_post_layers=int(_arg(args, "n_book_post_layers", 1)),
                                 activation=str(_arg(args, "activation_fn", "half_glu1")),
                                 prenorm=bool(_arg(args, "prenorm", True)), dropout=float(_arg(args, "p_dropout", 0.0)),
                                 use_book_data=bool(_arg(args, "use_book_data", True)),
                                 attn_factory_at=bb.attn_factory_at, attn_layers=bb.attn_layers)
        if str(_arg(args, "impl", "torch")) == "cuda" and hasattr(model, "book_encoder"):
            model.book_encoder.compute_dtype = _compute_dtype(args)
        return model
    model = LobModel(bb.factory_at, vocab_size=int(args.vocab_size), d_model=int(args.d_model),
                     d_book=int(_arg(args, "d_book", 503)),
                     n_message_layers=int(_arg(args, "n_message_layers", 2)),
                     n_fused_layers=int(_arg(args, "n_layers", 6)),
                     n_book_pre_layers=int(_arg(args, "n_book_pre_layers", 1)),
                     n_book_post_layers=int(_arg(args, "n_book_post_layers", 1)),
                     activation=str(_arg(args, "activation_fn", "half_glu1")),
                     prenorm=bool(_arg(args, "prenorm", True)),
                     dropout=float(_arg(args, "p_dropout", 0.0)),
                     msg_len=int(_arg(args, "msg_len", 22)),
                     use_book_data=bool(_arg(args, "use_book_data", True)),
                     attn_factory_at=bb.attn_factory_at, attn_layers=bb.attn_layers)
    if bool(_arg(args, "legacy_norm", False)) or legacy_norm_enabled():
        apply_legacy_norm(model)
    if str(_arg(args, "impl", "torch")) == "cuda":
        for enc in (getattr(model, "book_encoder", None), getattr(model, "message_encoder", None),
                    getattr(model, "fused_s5", None)):
            if enc is not None and hasattr(enc, "compute_dtype"):
                enc.compute_dtype = _compute_dtype(args)
    return model
