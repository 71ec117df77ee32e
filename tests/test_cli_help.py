"""Every command-line entry point of the package parses ``--help`` and exits cleanly (the
reference's CLI smoke test, ``tests/smoke/test_cli_help.py``), without a GPU."""
import importlib
import inspect

import pytest

ENTRY_POINTS = [
    "sigma0_b200.cli.train", "sigma0_b200.cli.infer", "sigma0_b200.cli.launch", "sigma0_b200.cli.rl",
    "sigma0_b200.cli.plan", "sigma0_b200.pipeline.register", "sigma0_b200.pipeline.integrity", "sigma0_b200.pipeline.injection", "sigma0_b200.data.lobster", "sigma0_b200.ckpt.inspect", "sigma0_b200.eval.model_zoo_ce", "sigma0_b200.eval.trade_anchors", "sigma0_b200.pipeline.lobbench",
    "sigma0_b200.sim.divergence", "sigma0_b200.eval.return_bench", "sigma0_b200.eval.gen_metrics", "sigma0_b200.eval.ce_by_position", "sigma0_b200.eval.stylized",
    "sigma0_b200.eval.s5_bench", "sigma0_b200.eval.attn_bench", "sigma0_b200.eval.nsa_bench",
    "sigma0_b200.eval.gdn_bench", "sigma0_b200.eval.ag_gemm_bench", "sigma0_b200.eval.gemm_bench",
    "sigma0_b200.eval.ssd_bench", "sigma0_b200.parallel.tp_bench", "sigma0_b200.state.train",
    "sigma0_b200.utils.step_profile",
]


@pytest.mark.parametrize("mod", ENTRY_POINTS)
def test_help(mod, capsys):
    m = importlib.import_module(mod)
    main = getattr(m, "main")
    if not inspect.signature(main).parameters:
        pytest.skip(f"{mod}.main takes no argument list")
    with pytest.raises(SystemExit) as e:
        main(["--help"])
    assert e.value.code in (0, None)
    assert "usage" in capsys.readouterr().out.lower()
