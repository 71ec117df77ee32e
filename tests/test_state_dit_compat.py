"""FrameDiT against a state dict under the reference's parameter names
(``src/state/dit.py:165-235``): strict load, and the outputs of a fixed set of weights
and inputs, conditional and unconditional (golden values in tests/data)."""
import json
import os

import torch

from sigma0_b200.state.dit import FrameDiT, FrameDiTConfig, bind_condition, bind_unconditional

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "data", "framedit_golden.json")))


def _ref_tree(C, H, depth, heads, freq, ratio=4):
    """Parameter names and shapes of the reference module tree."""
    F_ = H * ratio
    tree = {"input_proj.weight": (H, 2 * C + 1), "input_proj.bias": (H,),
            "time_embedding.0.weight": (H, freq), "time_embedding.0.bias": (H,),
            "time_embedding.2.weight": (H, H), "time_embedding.2.bias": (H,),
            "time_projection.1.weight": (6 * H, H), "time_projection.1.bias": (6 * H,),
            "final_norm.weight": (H,), "final_norm.bias": (H,),
            "velocity_head.weight": (C, H), "velocity_head.bias": (C,)}
    for i in range(depth):
        p = f"blocks.{i}."
        tree[p + "modulation"] = (1, 6, H)
        for n in "qkvo":
            tree[p + f"attn.{n}.weight"] = (H, H)
            tree[p + f"attn.{n}.bias"] = (H,)
        tree[p + "attn.q_norm.weight"] = (H // heads,)
        tree[p + "attn.k_norm.weight"] = (H // heads,)
        tree[p + "ffn.0.weight"], tree[p + "ffn.0.bias"] = (F_, H), (F_,)
        tree[p + "ffn.2.weight"], tree[p + "ffn.2.bias"] = (H, F_), (H,)
    return tree


def test_parameter_tree_matches_reference_names_and_shapes():
    m = FrameDiT(FrameDiTConfig(channels=41, hidden=128, depth=4, heads=4))
    got = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    assert got == _ref_tree(41, 128, 4, 4, 256)
    sd = {k: torch.randn(s) for k, s in _ref_tree(41, 128, 4, 4, 256).items()}
    m.load_state_dict(sd, strict=True)


def test_outputs_of_a_reference_named_state_dict():
    cfg = FrameDiTConfig(**GOLD["cfg"])
    m = FrameDiT(cfg)
    m.load_state_dict({k: torch.tensor(v).view(s) for k, (s, v) in GOLD["state"].items()}, strict=True)
    x = torch.tensor(GOLD["x"]).view(2, 5, cfg.channels)
    ctx = torch.tensor(GOLD["ctx"]).view(2, 5, cfg.channels)
    obs = torch.tensor(GOLD["obs"]).view(2, 5)
    t = torch.tensor(GOLD["t"])
    with torch.no_grad():
        oc = bind_condition(m, ctx, obs)(x, t)
        ou = bind_unconditional(m)(x, t)
    torch.testing.assert_close(oc.flatten(), torch.tensor(GOLD["out_cond"]), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(ou.flatten(), torch.tensor(GOLD["out_uncond"]), rtol=1e-5, atol=1e-5)


def test_fresh_model_predicts_zero_velocity_and_ignores_context():
    m = FrameDiT(FrameDiTConfig(channels=4, hidden=16, depth=1, heads=2, max_seq_len=8))
    x, t = torch.randn(2, 6, 4), torch.rand(2)
    with torch.no_grad():
        assert m(torch.cat([x, torch.randn(2, 6, 4), torch.ones(2, 6, 1)], -1), t).abs().max() == 0
