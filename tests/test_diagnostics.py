"""Analyse-only diagnostics: register rendering, sanity gate, stylized facts, TSTR, provenance."""
import json

import numpy as np
import pytest

from sigma0_b200.data.synthetic import generate_day
from sigma0_b200.eval import stylized as S
from sigma0_b200.pipeline import register as R


def test_register_render_splice_check(tmp_path):
    reg = {"classes": {"X": "Class X, Execution", "I": "Class I, Init"},
           "columns": ["id", "statement", "sites", "silent", "status"],
           "records": [{"id": "X1", "class": "X", "statement": "a | b", "sites": ["f.py:1", "g.py:2"],
                        "silent": True, "status": "FIXED"},
                       {"id": "I1", "class": "I", "statement": "line\nbreak", "sites": [], "silent": False,
                        "status": "OPEN"}]}
    body = R.render(reg)
    assert "### Class X, Execution" in body and "1 of 1 closed." in body and "0 of 1 closed." in body
    assert "a \\| b" in body and "`f.py:1`; `g.py:2`" in body and "**FIXED**" in body and "line break" in body
    rp, dp = tmp_path / "reg.json", tmp_path / "doc.md"
    rp.write_text(json.dumps(reg))
    dp.write_text(f"# Doc\nprose\n{R.BEGIN}\nstale\n{R.END}\ntail\n")
    assert R.main([str(rp), str(dp), "--check"]) == 1
    assert R.main([str(rp), str(dp)]) == 0
    assert R.main([str(rp), str(dp), "--check"]) == 0
    assert dp.read_text().startswith("# Doc\nprose\n") and dp.read_text().endswith("tail\n")


def _run(seed, n=600):
    d = generate_day(n, seed=seed)
    m = d.msgs
    msgs = np.stack([m[:, 8], m[:, 9], m[:, 1], m[:, 0], m[:, 5], m[:, 3], np.where(m[:, 2] == 1, 1, -1)], 1)
    return msgs.astype(np.float64), d.books[:, 3:].astype(np.float64)


def test_sanity_gate_stylized_facts_tstr_provenance(tmp_path):
    real = [_run(s) for s in range(6)]
    gen = [_run(100 + s) for s in range(6)]
    mr, br = [r[0] for r in real], [r[1] for r in real]
    mg, bg = [g[0] for g in gen], [g[1] for g in gen]
    origin = S.build_origin(str(tmp_path), experiment="synthetic", ticker="SYN", depth=br[0].shape[1] // 4)
    info = S.assert_generation_sane(br, bg, origin)
    assert info["bad_fraction"] <= 0.05
    corrupt = [b.copy() for b in bg]
    for b in corrupt:
        b[:, 0] = b[:, 2] + 1e9                               # absurd spreads
    with pytest.raises(S.GenerationCorrupt):
        S.assert_generation_sane(br, corrupt, origin)
    sf = S.stylized_facts(br, br)
    assert all(abs(v) < 1e-12 or np.isnan(v) for v in sf["diff"].values())
    sf2 = S.stylized_facts(br, bg)
    assert set(sf2["real"]) == {"ret_acf1", "absret_acf1", "absret_acf5", "absret_acf20", "hill_tail_index",
                                "leverage5"}
    t = S.tstr(mr, br, mg, bg)
    assert "n_test" in t and ("skipped" in t or 0.0 <= t["auc_trained_on_real"] <= 1.0)
    assert S.auc(np.array([0.1, 0.9, 0.8, 0.2]), np.array([0, 1, 1, 0])) == 1.0
    p = S.write_provenance(str(tmp_path / "out"), origin, {"windows": 6})
    assert json.load(open(p))["origin"]["ticker"] == "SYN"
    assert S.stamp({"x": 1}, origin)["origin"]["experiment"] == "synthetic"
    assert 0.5 < S.hill_index(np.random.default_rng(0).standard_t(3, 200000), 0.01) < 6
