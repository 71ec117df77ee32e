"""The backbone registry against a golden table of the reference's selector behaviour.

``tests/data/registry_selectors.json`` enumerates every combination of
``--architecture`` / legacy ``ssm_type`` / ``model_type`` over the known names, a retired
name, an unknown one, ``ssm``, an upper-case spelling and the empty string, with the
reference's outcome (the canonical name, or the kind of refusal), plus the hybrid
attention placement for 1 to 64 layers (``src/base_model/models/registry.py:79-187``).
"""
import json
import os
from types import SimpleNamespace

import pytest

from sigma0_b200.models import registry as R

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "data", "registry_selectors.json")))
SEL = GOLD["selectors"]


def test_every_accepted_selector_combination():
    assert len(GOLD["accepted"]) > 300
    for a, s, m, want in GOLD["accepted"]:
        assert R.resolve_architecture(SEL[a], ssm_type=SEL[s], model_type=SEL[m]) == want, (SEL[a], SEL[s], SEL[m])


@pytest.mark.parametrize("kind,needle", [("conflict", "conflicting"), ("unknown", "unknown architecture"),
                                         ("mamba2", "intentionally not part")])
def test_every_refused_selector_combination(kind, needle):
    cases = [c for c in GOLD["rejected"] if c[3] == kind]
    assert cases
    for a, s, m, _ in cases:
        with pytest.raises(ValueError, match=needle):
            R.resolve_architecture(SEL[a], ssm_type=SEL[s], model_type=SEL[m])


def test_nemotron_placement_matches_for_4_to_64_layers():
    for L in range(4, 65):
        assert list(R.nemotron_attention_indices(L)) == GOLD["nemotron"][str(L)], L


def test_table_properties_and_stamp():
    assert R.available_architectures() == ("mamba3", "s5", "gdn", "kda", "transformer", "nsa", "hybrid_mamba3")
    assert [n for n in R.ARCHITECTURES if R.architecture_has_attention(n)] == ["transformer", "nsa", "hybrid_mamba3"]
    assert R.get_definition("nsa").wrapper_policy == "internal"
    assert R.get_definition("hybrid_mamba3").wrapper_policy == "external"
    assert R.DTYPE_AWARE_ARCHITECTURES == {"transformer", "nsa", "mamba3", "hybrid_mamba3"}
    args = SimpleNamespace()
    for name in R.available_architectures():
        R.stamp_architecture(args, name)
        assert R.architecture_from_args(args) == name


def test_dtype_guard_and_width_geometry():
    with pytest.raises(ValueError, match="has no effect"):
        R.build_backbone(SimpleNamespace(architecture="s5", d_model=64, dtype="bfloat16"))
    c = R.recurrent_carry_for_width({"ssm_type": "mamba3", "n_heads": 0, "headdim": 64, "expand": 2,
                                     "requested_headdim": 64, "tp_size": 1}, 503)
    assert (c["headdim"], c["n_heads"]) == (64, 15)
    c = R.recurrent_carry_for_width({"ssm_type": "gdn", "num_heads": 8, "head_dim": 128, "expand_v": 2}, 503)
    assert (c["num_heads"], c["head_dim"], c["head_v_dim"]) == (3, 128, 256)
    bb = R.build_backbone(SimpleNamespace(architecture="transformer", d_model=64, n_heads=8))
    cfg = R.attention_config_for_width(bb, 503)
    assert (cfg["n_heads"], cfg["head_dim"]) == (1, 503)
