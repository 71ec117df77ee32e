"""The kernel benchmark commands cited in profiles/ run end to end at tiny sizes and print
their JSON record (attention, gated delta, NSA, S5, single-rank fused TP)."""
import json

import pytest

pytestmark = pytest.mark.gpu


def _last_json(capsys):
    lines = [l for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert lines
    return json.loads(lines[-1])


def test_kernel_benches_run(capsys):
    from sigma0_b200.eval import attn_bench, gdn_bench, nsa_bench, s5_bench
    from sigma0_b200.parallel import tp_bench
    attn_bench.main(["--B", "1", "--L", "256", "--nh", "2", "--window", "64", "--iters", "1", "--warmup", "1"])
    r = _last_json(capsys)
    assert r["causal"]["rel_diff_fwd"] < 2e-2 and r["window64"]["ours"]["fwd_ms"] > 0
    gdn_bench.main(["--L", "256", "--nh", "2", "--hd", "64", "--hvd", "128", "--iters", "1", "--warmup", "1"])
    assert _last_json(capsys)["rel_diff"] < 2e-2
    nsa_bench.main(["--L", "512", "--H", "256", "--nh", "4", "--top", "4", "--iters", "1", "--warmup", "1"])
    assert _last_json(capsys)["rel_diff"] < 2e-2
    s5_bench.main(["--B", "1", "--L", "300", "--H", "64", "--state", "64", "--blocks", "2", "--iters", "1",
                   "--warmup", "1"])
    assert _last_json(capsys)["rel_diff"] < 1e-4
    tp_bench.main(["--tokens", "1024", "--k_total", "256", "--n_out", "256", "--iters", "2", "--warmup", "1"])
    r = _last_json(capsys)
    assert r["world"] == 1 and r["rel_err_vs_fp32"] < 1e-2
