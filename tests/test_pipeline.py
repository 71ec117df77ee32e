"""Pipeline: scoring a generation run, J4 injection gate, model store, packaging, evidence."""
import json
import os

import numpy as np
import pytest
import torch


@pytest.fixture(scope="module")
def run_dir(tmp_path_factory):
    from sigma0_b200.cli.infer import main
    out = tmp_path_factory.mktemp("run")
    assert main(["--preset", "smoke", "--impl", "torch", "--synthetic", "3", "--n_sequences", "3", "--batch_size", "3",
                 "--n_cond_msgs", "4", "--n_gen_msgs", "6", "--sample_top_n", "1", "--save_dir", str(out)]) == 0
    return str(out)


def test_lobbench_modes_and_merge(run_dir):
    from sigma0_b200.pipeline.lobbench import score_run, merge, load_run, shard
    assert len(load_run(run_dir)) == 3
    for mode in ("uncond", "cond", "context", "time_lagged"):
        r = score_run(run_dir, mode, n_boot=5)
        assert r["n_windows"] >= 2 and "order_size/wasserstein" in r["scores"]
    d = score_run(run_dir, "divergence", buckets=2)
    assert len(d["buckets"]) == 2
    parts = [score_run(run_dir, "cond", windows=shard([0, 1, 2], 2, k)) for k in range(2)]
    m = merge(parts)
    assert m["n_windows"] == 3


def test_injection_j4(tmp_path):
    from sigma0_b200.cli.infer import main
    from sigma0_b200.pipeline.injection import verify_injection
    out = tmp_path / "inj"
    assert main(["--preset", "smoke", "--impl", "torch", "--synthetic", "2", "--n_sequences", "2", "--batch_size", "2",
                 "--n_cond_msgs", "4", "--n_gen_msgs", "4", "--sample_top_n", "1", "--save_dir", str(out),
                 "--inject_step", "2", "--inject_event_type", "1", "--inject_side", "1", "--inject_qty", "37",
                 "--inject_price_offset_ticks", "-1"]) == 0
    r = verify_injection(str(out), step=2, side=1, qty=37, offset_ticks=-1)
    assert r["J4"], r
    bad = verify_injection(str(out), step=2, side=1, qty=38, offset_ticks=-1)
    assert not bad["J4"]


def test_model_store_and_packaging(tmp_path):
    from sigma0_b200.ckpt import CheckpointManager
    from sigma0_b200.models import preset_args
    from sigma0_b200.pipeline.model_store import pin, resolve, ModelStoreError
    from sigma0_b200.pipeline.package import pack, verify, unpack
    from sigma0_b200.pipeline.integrity import tree_sha256, record_evidence, check_evidence
    from sigma0_b200.train.trainer import Trainer
    tr = Trainer(preset_args("smoke"), device=torch.device("cpu"))
    ck = tmp_path / "ck"
    CheckpointManager(str(ck)).save(5, tr, blocking=True)
    store = str(tmp_path / "pins.json")
    pin(store, "smoke-5", str(ck), 5, architecture="mamba3")
    assert resolve(store, "smoke-5")["step"] == 5
    with open(ck / "5" / "metadata" / "metadata", "a") as f:
        f.write(" ")
    with pytest.raises(ModelStoreError):
        resolve(store, "smoke-5")
    arc = str(tmp_path / "run.tar")
    man = pack(str(ck), arc)
    assert man and verify(arc) == {"mismatch": [], "missing": [], "extra": []}
    unpack(arc, str(tmp_path / "restored"))
    os.remove(tmp_path / "restored" / "MANIFEST.sha256.json")
    assert tree_sha256(str(tmp_path / "restored")) == tree_sha256(str(ck))
    src = str(tmp_path / "src.txt")
    open(src, "w").write("x")
    ev = str(tmp_path / "ev.json")
    record_evidence(ev, [src], {"two": lambda: 1 + 1 == 2})
    assert check_evidence(ev) == {"changed": [], "missing": [], "failed": []}
    open(src, "w").write("y")
    assert check_evidence(ev)["changed"] == [src]


def test_guards_and_tools(tmp_path):
    from sigma0_b200.pipeline.guards import non_english_lines, forbidden_imports, perplexity_decomposition_ok
    import sigma0_b200
    root = os.path.dirname(sigma0_b200.__file__)
    assert non_english_lines([root]) == []
    assert forbidden_imports([root], ["triton", "jax", "flax"]) == []
    f = tmp_path / "x.py"
    f.write_text("import triton.language as tl\n# café\n")
    assert forbidden_imports([str(f)], ["triton"]) and non_english_lines([str(f)])
    rep = {"roles": {"main": 1.0, "absolute_time": 0.5, "reference": 0.25}, "full": {"nats_per_message": 1.75}}
    assert perplexity_decomposition_ok(rep)


def test_snapshots_and_ce_by_position():
    from sigma0_b200.data.synthetic import generate_day
    from sigma0_b200.data.lobster import make_snapshots
    from sigma0_b200.eval.ce_by_position import main
    d = generate_day(50, seed=2)
    t = d.books[:, 1].astype(np.int64) * 10**9 + d.books[:, 2].astype(np.int64)
    snap = make_snapshots(d.books, [t[5], t[5] + 1])
    assert np.array_equal(snap[0], d.books[6, 3:]) and np.array_equal(snap[1], d.books[6, 3:])
    assert main(["--preset", "smoke", "--impl", "torch", "--n_messages", "4", "--max_batches", "1"]) == 0


def test_evidence_declared_assertions_and_self_test(tmp_path, capsys):
    """Declarative assertions are re-evaluated from the record itself, and the self-test
    plants every kind of defect and sees each one go red."""
    from sigma0_b200.pipeline import integrity as I
    src = tmp_path / "s.py"
    src.write_text("a = 1\n")
    ev = str(tmp_path / "ev.json")
    I.record_evidence(ev, [str(src)], {}, metrics={"bench": {"ic": [0.8, 0.6]}},
                      declared=[{"name": "ic holds", "metric": "bench.ic.1", "op": ">=", "value": 0.5}])
    assert I.audit(ev) == {"changed": [], "missing": [], "failed": []}
    import json
    rec = json.load(open(ev))
    rec["metrics"]["bench"]["ic"][1] = 0.4                # a number edited after the fact
    json.dump(rec, open(ev, "w"))
    assert I.audit(ev)["failed"] and I.main([ev]) == 1
    assert I.self_test() == 0 and I.main(["--self-test"]) == 0
    assert "self-test passed" in capsys.readouterr().out


def test_injection_report_with_reference_arms(tmp_path):
    """Off, on and a repeated off run of the same generation: J4 gates, J0 / J1 / J2 / J5 hold
    for deterministic argmax sampling on the CPU, and the written report re-audits clean; a
    tampered verdict is caught."""
    from sigma0_b200.cli.infer import main
    from sigma0_b200.pipeline import injection as J
    base = ["--preset", "smoke", "--impl", "torch", "--synthetic", "2", "--n_sequences", "2", "--batch_size", "2",
            "--n_cond_msgs", "4", "--n_gen_msgs", "5", "--sample_top_n", "1"]
    inj = ["--inject_step", "2", "--inject_event_type", "1", "--inject_side", "1", "--inject_qty", "37",
           "--inject_price_offset_ticks", "-1"]
    runs = {}
    for name, extra in (("p", []), ("p2", []), ("o", []), ("i", inj)):
        runs[name] = str(tmp_path / name)
        assert main(base + ["--save_dir", runs[name]] + extra) == 0
    rep = J.verify_arms(runs["i"], 2, 1, 37, -1, dir_o=runs["o"], dir_p=runs["p"], dir_p2=runs["p2"])
    assert rep["overall_pass"] == 1 and rep["j4_book_injection"]["n_windows"] == 2
    assert rep["j0_determinism"]["pass"] == 1 and rep["j1_off_means_off"]["pass"] == 1
    assert rep["j2_prefix"]["pass"] == 1 and rep["j5_divergence"]["pass"] == 1
    path = str(tmp_path / "report.json")
    assert J.main(["--dir_i", runs["i"], "--dir_o", runs["o"], "--step", "2", "--side", "1", "--qty", "37",
                   "--offset_ticks", "-1", "--out", path]) == 0
    assert J.check_report(path) == []
    r = json.load(open(path))
    r["overall_pass"] = 0
    json.dump(r, open(path, "w"))
    assert J.check_report(path) and J.main(["--check", path]) == 1


def test_package_run_layout_and_index(run_dir, tmp_path):
    """A scored run becomes one archive with manifest, scores and predictions, verified by its
    SHA-256 manifest, plus a sidecar index listing it without opening the archive."""
    from sigma0_b200.pipeline.lobbench import score_run
    from sigma0_b200.pipeline.package import package_run, plan_package, unpack, verify
    scores = tmp_path / "scores.json"
    scores.write_text(json.dumps(score_run(run_dir, "uncond", n_boot=3)))
    with pytest.raises(FileNotFoundError):
        plan_package("r1", str(tmp_path / "nope"), str(scores), str(tmp_path / "pk"))
    idx = package_run("r1", run_dir, str(scores), str(tmp_path / "pk"))
    assert idx["archive"] == "r1.tar" and "manifest.json" in idx["members"] and "scores.json" in idx["members"]
    assert any(m.startswith("predictions/data_gen/") for m in idx["members"]) and idx["metric_names"]
    arc = str(tmp_path / "pk" / "r1.tar")
    assert verify(arc) == {"mismatch": [], "missing": [], "extra": []}
    unpack(arc, str(tmp_path / "out"))
    man = json.load(open(tmp_path / "out" / "manifest.json"))
    assert man["run_name"] == "r1" and man["n_files"] == len(man["files"])
    assert json.load(open(tmp_path / "pk" / "index_r1.json"))["sha256"]["scores.json"]


def test_packed_tree_overlay_resolve_cat_listing(tmp_path):
    """A packed tree is patched through its overlay (an override, a whiteout) without
    repacking; ``resolve`` yields the merged directory and cleans up; ``cat`` / ``listing``
    read the archive without unpacking; a directory resolves to itself."""
    from sigma0_b200.pipeline import package as pk
    tree = tmp_path / "run"
    (tree / "data_gen").mkdir(parents=True)
    (tree / "data_gen" / "a.csv").write_text("a")
    (tree / "data_gen" / "b.csv").write_text("b")
    (tree / "scores.json").write_text("{}")
    pk.pack(str(tree), pk.image_for(str(tree)))
    assert pk.listing(pk.image_for(str(tree))) == ["data_gen/a.csv", "data_gen/b.csv", "scores.json"]
    assert pk.cat(pk.image_for(str(tree)), "data_gen/b.csv") == b"b"
    with pk.resolve(str(tree)) as d:
        assert d == str(tree)                                  # a directory is used as it is
    import shutil
    shutil.rmtree(tree)
    pk.overlay_override(str(tree), "data_gen/a.csv", "A2")
    pk.overlay_exclude(str(tree), "data_gen/b.csv")
    pk.overlay_override(str(tree), "extra/new.txt", b"n")
    with pk.resolve(str(tree), tmp_root=str(tmp_path)) as d:
        got = sorted(os.path.relpath(os.path.join(r, f), d) for r, _, fs in os.walk(d) for f in fs)
        assert got == ["data_gen/a.csv", "extra/new.txt", "scores.json"]
        assert open(os.path.join(d, "data_gen", "a.csv")).read() == "A2"
        merged = d
    assert not os.path.exists(merged)
    pk.overlay_override(str(tree), "data_gen/b.csv", "B2")      # an override lifts the whiteout
    with pk.resolve(pk.image_for(str(tree))) as d:
        assert open(os.path.join(d, "data_gen", "b.csv")).read() == "B2"
    assert pk.verify(pk.image_for(str(tree))) == {"mismatch": [], "missing": [], "extra": []}
    with pytest.raises(FileNotFoundError):
        with pk.resolve(str(tmp_path / "nothing")):
            pass
    with pk.resolve(str(tmp_path / "nothing"), require=False) as d:
        assert d == str(tmp_path / "nothing")
