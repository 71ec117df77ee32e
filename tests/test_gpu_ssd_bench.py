"""The SSD kernel bench (parity + timing records) on a small geometry."""
import pytest

pytestmark = pytest.mark.gpu


def test_ssd_bench_parity_and_speed():
    from sigma0_b200.eval import ssd_bench
    par = ssd_bench.parity(nh=8, L=300)
    assert par["y"] < 2e-2, par
    for k, v in par.items():
        assert v < 6e-2, (k, v)
    sp = ssd_bench.speed(nh=8, L=2048, warmup=1, iters=2, oracle=True)
    assert sp["cuda_fwd_ms"] > 0 and sp["cuda_fwd_bwd_ms"] >= sp["cuda_fwd_ms"] * 0.5
    assert sp["speedup_fwd_bwd"] > 1.0
