"""Backbones, the outer LOB model and the registry."""
from .registry import (build_backbone, build_model, resolve_architecture, available_architectures,
                       nemotron_attention_indices, architecture_has_attention, get_definition)
from .presets import PRESETS, preset_args
