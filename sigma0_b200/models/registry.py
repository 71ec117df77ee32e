"""Strict backbone registry: the only place a name becomes a layer factory.

Same contract as the reference (``src/base_model/models/registry.py:63-530``):
the architecture set and per-architecture flags, the strict
``--architecture`` / legacy ``ssm_type`` / ``model_type`` resolution with its
conflict rules, the Nemotron-H attention placement for ``hybrid_mamba3``, the
``--dtype`` guard, and the carry geometry of layers rebuilt at another width.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from functools import partial
from typing import Any, Callable, Mapping, Optional, Tuple

import torch

DEFAULT_ARCHITECTURE = "mamba3"


@dataclass(frozen=True)
class BackboneDefinition:
    name: str
    wrapper_policy: str
    supports_prefill: bool
    supports_stepwise_inference: bool = True
    has_attention: bool = False


@dataclass(frozen=True)
class BackboneBuild:
    definition: BackboneDefinition
    factory_at: Callable[[int], Any]               # width -> mixer module
    carry_kwargs: Mapping[str, Any]
    attention_config: Optional[Mapping[str, Any]] = None
    attn_factory_at: Optional[Callable[[int], Any]] = None
    attn_layers: Tuple[int, ...] = ()

    @property
    def is_attention(self) -> bool:
        return self.definition.wrapper_policy == "internal"

    @property
    def is_hybrid(self) -> bool:
        return self.attn_factory_at is not None


_DEFINITIONS = {
    "mamba3": BackboneDefinition("mamba3", "external", False),
    "s5": BackboneDefinition("s5", "external", False),
    "gdn": BackboneDefinition("gdn", "external", False),
    "kda": BackboneDefinition("kda", "external", False),
    "transformer": BackboneDefinition("transformer", "internal", True, has_attention=True),
    "nsa": BackboneDefinition("nsa", "internal", True, has_attention=True),
    "hybrid_mamba3": BackboneDefinition("hybrid_mamba3", "external", False, has_attention=True),
}

# Nemotron-H placement: 4 attention layers among 31 mixing layers, relative depths
# spread over the band below; never the first two or the last layer.
NEMOTRON_ATTENTION_FRACTION = 4 / 31
NEMOTRON_DEPTH_BAND = (0.26, 0.71)


def nemotron_attention_indices(n_layers: int) -> Tuple[int, ...]:
    k = max(1, round(NEMOTRON_ATTENTION_FRACTION * n_layers))
    if k == 1:
        depths = [0.48]
    else:
        lo, hi = NEMOTRON_DEPTH_BAND
        depths = [lo + (hi - lo) * i / (k - 1) for i in range(k)]
    idx = {min(max(round(d * n_layers), 2), n_layers - 2) for d in depths}
    return tuple(sorted(idx))


def available_architectures() -> Tuple[str, ...]:
    return tuple(_DEFINITIONS)


def architecture_has_attention(name: Optional[str]) -> bool:
    d = _DEFINITIONS.get(name or "")
    return d is not None and d.has_attention


def get_definition(name: str) -> BackboneDefinition:
    try:
        return _DEFINITIONS[name]
    except KeyError as exc:
        if name == "mamba2":
            raise ValueError("architecture 'mamba2' is intentionally not part of this model zoo; "
                             "use 'mamba3' for new experiments") from exc
        raise ValueError(f"unknown architecture {name!r}; choose one of: "
                         f"{', '.join(available_architectures())}") from exc


def resolve_architecture(architecture: Optional[str] = None, *, ssm_type: Optional[str] = None,
                         model_type: Optional[str] = None) -> str:
    """Canonical selector; legacy ``ssm_type``/``model_type`` must agree with it."""
    architecture = architecture.lower() if architecture else None
    ssm_type = ssm_type.lower() if ssm_type else None
    model_type = model_type.lower() if model_type else None
    if model_type not in {None, "ssm", *_DEFINITIONS}:
        get_definition(model_type)
    if model_type in {"transformer", "nsa"}:
        if ssm_type not in {None, "s5", model_type}:
            raise ValueError(f"conflicting legacy selectors: model_type={model_type!r}, ssm_type={ssm_type!r}")
        legacy = model_type
    elif ssm_type:
        legacy = ssm_type
    elif model_type in _DEFINITIONS:
        legacy = model_type
    else:
        legacy = None
    cands = []
    if architecture:
        cands.append(("architecture", architecture))
    if legacy:
        cands.append(("legacy selector", legacy))
    if not cands:
        return DEFAULT_ARCHITECTURE
    if len({v for _, v in cands}) != 1:
        rendered = ", ".join(f"{k}={v!r}" for k, v in cands)
        raise ValueError(f"conflicting architecture selectors: {rendered}")
    get_definition(cands[0][1])
    return cands[0][1]


def architecture_from_args(args: Any) -> str:
    return resolve_architecture(getattr(args, "architecture", None),
                                ssm_type=getattr(args, "ssm_type", None),
                                model_type=getattr(args, "model_type", None))


def stamp_architecture(args: Any, architecture: str) -> None:
    args.architecture = architecture
    args.ssm_type = architecture
    args.model_type = architecture if architecture in {"transformer", "nsa"} else "ssm"


def recurrent_carry_for_width(carry_kwargs: Mapping[str, Any], width: int) -> dict:
    """Resize recurrent carry metadata the way the layer resizes itself."""
    c = dict(carry_kwargs)
    width = int(width)
    name = c.get("ssm_type")
    if name == "mamba3":
        expand = int(c["expand"])
        req = int(c.get("requested_headdim", c["headdim"]))
        target = expand * width
        hd = min(req, target)
        nh = max(1, target // hd)
        tp = int(c.get("tp_size", 1))
        eff = tp if nh % tp == 0 else 1
        c["headdim"] = hd
        c["n_heads"] = nh // eff
    elif name in {"gdn", "kda"}:
        rh = int(c.get("requested_num_heads", c["num_heads"]))
        rd = int(c.get("requested_head_dim", c["head_dim"]))
        hd = min(rd, width)
        c["num_heads"] = min(rh, max(1, width // rd))
        c["head_dim"] = hd
        c["head_v_dim"] = hd * int(c["expand_v"])
    return c


def attention_config_for_width(backbone: BackboneBuild, width: int, *, max_cache_len=None) -> dict:
    if backbone.attention_config is None:
        raise ValueError(f"architecture {backbone.definition.name!r} does not use an attention cache")
    cfg = dict(backbone.attention_config)
    nh = int(cfg["n_heads"])
    while nh > 1 and width % nh:
        nh -= 1
    cfg["n_heads"] = nh
    cfg["head_dim"] = width // nh
    if max_cache_len is not None:
        cfg["max_cache_len"] = int(max_cache_len)
    return cfg


DTYPE_AWARE_ARCHITECTURES = frozenset({"transformer", "nsa", "mamba3", "hybrid_mamba3"})


def _compute_dtype(args):
    return {"float32": torch.float32, "bfloat16": torch.bfloat16}.get(
        str(getattr(args, "dtype", "float32")), torch.float32)


def _g(args, k, default):
    v = getattr(args, k, None)
    return default if v is None else v


def build_backbone(args: Any, *, print_shapes: bool = False) -> BackboneBuild:
    name = architecture_from_args(args)
    definition = get_definition(name)
    H = int(args.d_model)
    req_dtype = str(getattr(args, "dtype", "float32"))
    if req_dtype != "float32" and name not in DTYPE_AWARE_ARCHITECTURES:
        raise ValueError(f"--dtype={req_dtype} has no effect on architecture '{name}': only "
                         f"{sorted(DTYPE_AWARE_ARCHITECTURES)} read it.")
    dtype = _compute_dtype(args)
    impl = str(_g(args, "impl", "torch"))
    attn_factory_at = None
    attn_layers: Tuple[int, ...] = ()
    attention_config = None

    if name in {"mamba3", "hybrid_mamba3"}:
        from .mamba3 import Mamba3
        d_state = int(_g(args, "mamba3_d_state", 128))
        expand = int(_g(args, "mamba3_expand", 2))
        headdim = int(_g(args, "mamba3_headdim", 64))
        chunk = int(_g(args, "mamba3_chunk_size", 64))
        rope = float(_g(args, "mamba3_rope_fraction", 0.5))
        tp = int(_g(args, "tp_size", 1))
        factory_at = lambda w: Mamba3(w, d_state=d_state, expand=expand, headdim=headdim,
                                      chunk_size=chunk, rope_fraction=rope, tp_size=tp,
                                      dtype=dtype, impl=impl)
        carry = recurrent_carry_for_width({
            "ssm_type": "mamba3", "n_heads": 0, "headdim": headdim, "d_state": d_state,
            "num_rope_angles": int(d_state * rope / 2), "expand": expand, "tp_size": tp,
            "requested_headdim": headdim}, H)
        if name == "hybrid_mamba3":
            from .transformer import TransformerBlock
            n_layers = int(_g(args, "n_layers", 6))
            override = getattr(args, "hybrid_attn_layers", None)
            attn_layers = (tuple(int(v) for v in str(override).split(",") if v.strip() != "")
                           if override else nemotron_attention_indices(n_layers))
            bad = [i for i in attn_layers if not 0 <= i < n_layers]
            if bad:
                raise ValueError(f"hybrid_attn_layers={attn_layers} out of range for n_layers={n_layers}")
            args.hybrid_attn_layers = ",".join(str(i) for i in attn_layers)
            n_heads = int(_g(args, "hybrid_attn_heads", 10))
            while n_heads > 1 and H % n_heads:
                n_heads -= 1
            head_dim = H // n_heads
            d_ff = int(_g(args, "hybrid_attn_d_ff", 0)) or 4 * H
            max_cache = int(_g(args, "attention_max_cache_len", 26000))
            use_pe = bool(_g(args, "hybrid_attn_positional_encoding", False))
            attn_factory_at = lambda w: TransformerBlock(w, n_heads=n_heads, d_ff=d_ff, dtype=dtype,
                                                         max_cache_len=max_cache,
                                                         use_positional_encoding=use_pe, impl=impl)
            attention_config = {"model_type": "transformer", "n_heads": n_heads,
                                "head_dim": head_dim, "max_cache_len": max_cache}
    elif name in {"gdn", "kda"}:
        from .gdn import GDN
        head_dim = int(_g(args, "gdn_head_dim", 128))
        num_heads = getattr(args, "gdn_num_heads", None) or max(1, H // head_dim)
        expand_v = int(_g(args, "gdn_expand_v", 2))
        use_conv = bool(_g(args, "gdn_use_conv", True))
        chunk = int(_g(args, "gdn_chunk_size", 64))
        factory_at = lambda w: GDN(w, num_heads=int(num_heads), head_dim=head_dim, expand_v=expand_v,
                                   chunk_size=chunk, use_conv=use_conv, use_kda=(name == "kda"),
                                   impl=impl)
        carry = recurrent_carry_for_width({
            "ssm_type": name, "num_heads": int(num_heads), "head_dim": head_dim,
            "head_v_dim": head_dim * expand_v, "expand_v": expand_v, "use_conv": use_conv,
            "requested_num_heads": int(num_heads), "requested_head_dim": head_dim}, H)
    elif name == "s5":
        from .s5 import make_s5_factory
        state_size = int(_g(args, "ssm_size_base", 32))
        blocks = int(_g(args, "blocks", 8))
        if state_size % blocks:
            raise ValueError("ssm_size_base must be divisible by blocks for S5")
        factory_at = make_s5_factory(state_size, blocks, conj_sym=bool(_g(args, "conj_sym", True)),
                                     C_init=str(_g(args, "C_init", "trunc_standard_normal")),
                                     discretization=str(_g(args, "discretization", "zoh")),
                                     dt_min=float(_g(args, "dt_min", 0.001)),
                                     dt_max=float(_g(args, "dt_max", 0.1)),
                                     clip_eigs=bool(_g(args, "clip_eigs", False)),
                                     bidirectional=bool(_g(args, "bidirectional", False)))
        carry = {"ssm_type": name}
    else:
        n_heads = int(_g(args, "n_heads", 16))
        if H % n_heads:
            raise ValueError(f"d_model={H} must be divisible by n_heads={n_heads}")
        d_ff = int(_g(args, "d_ff", 0)) or 4 * H
        max_cache = int(_g(args, "attention_max_cache_len", 26000))
        attention = {"model_type": name, "n_heads": n_heads, "head_dim": H // n_heads,
                     "max_cache_len": max_cache, "dtype": dtype}
        if name == "transformer":
            from .transformer import TransformerBlock
            factory_at = lambda w: TransformerBlock(w, n_heads=n_heads, d_ff=d_ff, dtype=dtype,
                                                    max_cache_len=max_cache, impl=impl)
        else:
            from .nsa import NSABlock
            from ..encoding import Message_Tokenizer
            msg_len = int(Message_Tokenizer.MSG_LEN)
            block_size = int(_g(args, "block_size", msg_len))
            strict = bool(_g(args, "nsa_strict_block", True))
            if strict and block_size != msg_len:
                raise ValueError(f"NSA block_size must equal the message length of the active "
                                 f"encoding ({msg_len}); got {block_size}")
            sel_block = int(_g(args, "nsa_select_block", block_size))
            factory_at = lambda w: NSABlock(w, n_heads=n_heads, d_ff=d_ff, block_size=block_size,
                                            select_block=sel_block,
                                            block_counts=int(_g(args, "block_counts", 16)),
                                            window_size=int(_g(args, "window_size", 512)),
                                            full_causal_window=bool(_g(args, "nsa_full_causal", True)),
                                            dtype=dtype, max_cache_len=max_cache,
                                            pe_type=str(_g(args, "pe_type", "rope")),
                                            rope_base=float(_g(args, "rope_base", 10000.0)), impl=impl)
            attention = {**attention, "block_size": block_size}
        carry = {"ssm_type": name, "is_transformer": True, "transformer_config": attention}
        return BackboneBuild(definition, factory_at, carry, attention)

    if print_shapes:
        print(f"[backbone] architecture={name} wrapper={definition.wrapper_policy}")
        if attn_layers:
            print(f"[backbone] hybrid attention at trunk layers {attn_layers}")
    return BackboneBuild(definition, factory_at, carry, attention_config=attention_config,
                         attn_factory_at=attn_factory_at, attn_layers=attn_layers)


def build_model(args: Any):
    """Build the outer LOB model for ``args`` (an argparse namespace or similar)."""
    from .lob_model import LobModel
    from .legacy_norm import apply_legacy_norm, legacy_norm_enabled
    bb = build_backbone(args)
    model = LobModel(bb.factory_at, vocab_size=int(args.vocab_size), d_model=int(args.d_model),
                    d_book=int(_g(args, "d_book", 503)),
                    n_message_layers=int(_g(args, "n_message_layers", 2)),
                    n_fused_layers=int(_g(args, "n_layers", 6)),
                    n_book_pre_layers=int(_g(args, "n_book_pre_layers", 1)),
                    n_book_post_layers=int(_g(args, "n_book_post_layers", 1)),
                    activation=str(_g(args, "activation_fn", "half_glu1")),
                    prenorm=bool(_g(args, "prenorm", True)),
                    dropout=float(_g(args, "p_dropout", 0.0)),
                    msg_len=int(_g(args, "msg_len", 22)),
                    use_book_data=bool(_g(args, "use_book_data", True)),
                    attn_factory_at=bb.attn_factory_at, attn_layers=bb.attn_layers)
    if bool(_g(args, "legacy_norm", False)) or legacy_norm_enabled():
        apply_legacy_norm(model)
    if str(_g(args, "impl", "torch")) == "cuda":
        for enc in (getattr(model, "book_encoder", None), getattr(model, "message_encoder", None),
                    getattr(model, "fused_s5", None)):
            if enc is not None and hasattr(enc, "compute_dtype"):
                enc.compute_dtype = _compute_dtype(args)
    return model
