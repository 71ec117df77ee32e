"""CLIs (train/infer/plan) and evaluation metrics on CPU."""
import glob
import json
import os

import numpy as np
import pytest
import torch


def test_train_cli_runs_and_resumes(tmp_path, capsys):
    from sigma0_b200.cli.train import main
    base = ["--preset", "smoke", "--impl", "torch", "--synthetic", "2", "--n_messages", "4", "--micro_bsz", "2",
            "--log_every", "1", "--watchdog_timeout", "0", "--ckpt_dir", str(tmp_path / "ck")]
    assert main(base + ["--steps", "2", "--save_every", "1"]) == 0
    assert main(base + ["--steps", "3"]) == 0
    lines = [json.loads(l) for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert any(l.get("event") == "resumed" and l["trainer_step"] == 2 for l in lines)
    assert lines[-1]["event"] == "finished" and lines[-1]["steps"] == 3


def test_train_cli_context_parallel_matches_single_process():
    """``--context_parallel`` on two gloo ranks (torchrun) logs the single process's losses."""
    import socket
    import subprocess
    import sys
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    args = ["-m", "sigma0_b200.cli.train", "--preset", "smoke", "--impl", "torch", "--synthetic", "2",
            "--n_messages", "4", "--micro_bsz", "2", "--log_every", "1", "--watchdog_timeout", "0", "--steps", "2"]
    env = dict(os.environ, OMP_NUM_THREADS="1")

    def losses(cmd):
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
        assert out.returncode == 0, out.stderr[-2000:]
        return [json.loads(l)["loss"] for l in out.stdout.splitlines() if l.startswith('{"step"')]
    one = losses([sys.executable] + args)
    two = losses([sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
                  "--master-addr", "127.0.0.1", "--master-port", str(port)] + args + ["--context_parallel"])
    assert len(one) == len(two) == 2
    np.testing.assert_allclose(two, one, rtol=1e-5)


def test_train_cli_config_file(tmp_path):
    from sigma0_b200.cli.train import parse
    (tmp_path / "c.yaml").write_text("steps: 7\nlog_every: 3\nenv_S0_TEST_KNOB: 1\n")
    a = parse(["--config", str(tmp_path / "c.yaml"), "--log_every", "5"])
    assert a.steps == 7 and a.log_every == 5 and os.environ.get("S0_TEST_KNOB") == "1"


def test_infer_cli_writes_lobster_csvs(tmp_path):
    import pandas as pd
    from sigma0_b200.cli.infer import main
    out = tmp_path / "gen"
    assert main(["--preset", "smoke", "--impl", "torch", "--synthetic", "2", "--n_sequences", "2", "--batch_size",
                 "2", "--n_cond_msgs", "4", "--n_gen_msgs", "3", "--sample_top_n", "1", "--save_dir", str(out)]) == 0
    gen = sorted(glob.glob(str(out / "data_gen" / "*_message_real_id_*_gen_id_0.csv")))
    assert len(gen) == 2
    df = pd.read_csv(gen[0])
    assert list(df.columns) == ["time", "event_type", "order_id", "size", "price", "direction"] and len(df) == 3
    assert set(df.direction) <= {-1, 1}
    cond = pd.read_csv(glob.glob(str(out / "data_cond" / "*_orderbook_real_id_0.csv"))[0])
    assert len(cond) == 5                                   # N + 1 book rows
    assert os.path.exists(out / "sample_indices_rank0.json")


def test_plan_commands(tmp_path):
    from sigma0_b200.cli.plan import build_plan
    (tmp_path / "p.yaml").write_text("name: smoke\nsbatch_nodes: 1\nenv_MODEL_PRESET: 75m\n")
    p = build_plan(str(tmp_path / "p.yaml"))
    s = p.shell()
    assert "--nproc-per-node=8" in s and "MODEL_PRESET=75m" in s and "sigma0_b200.cli.train" in s
    (tmp_path / "m.yaml").write_text("include: p.yaml\nsbatch_nodes: 4\nsbatch_time: 02:00:00\n")
    s = build_plan(str(tmp_path / "m.yaml")).shell()
    assert s.startswith("env") and "sbatch" in s and "--nodes=4" in s and "srun" in s


def test_message_perplexity_decomposes():
    from sigma0_b200.data import make_sequences, LobWindowDataset, collate
    from sigma0_b200.encoding import get_tokenizer
    from sigma0_b200.eval.perplexity import message_perplexity
    from sigma0_b200.models import preset_args, build_model
    torch.manual_seed(0)
    m = build_model(preset_args("smoke")).eval()
    ds = LobWindowDataset.from_days(make_sequences(2, 5, seed=1), 4, token_mode="22tok")
    mp = message_perplexity(m, [collate([ds[0], ds[1]])], get_tokenizer("22tok"))
    d = mp.as_dict()
    assert mp.n_messages == 8
    assert abs(mp.full_nats - (mp.roles["main"] + mp.roles["absolute_time"] + mp.roles["reference"])) < 1e-9
    assert 0 < d["main"]["nats_per_message"] < d["full"]["nats_per_message"]


def test_lob_metrics_on_engine_replay():
    from sigma0_b200.data.synthetic import generate_day
    from sigma0_b200.eval.lob_metrics import validity_report, marginals, score, event_returns
    d1, d2 = generate_day(400, seed=1), generate_day(400, seed=2)

    def view(d):
        m = d.msgs
        msgs = np.stack([m[:, 8], m[:, 9], m[:, 1], m[:, 0], m[:, 5], m[:, 3], m[:, 2] * 2 - 1], 1)
        return msgs, d.books[:, 3:]
    m1, b1 = view(d1)
    rep = validity_report(m1)
    assert rep["non_monotone_time"] == 0 and rep["bad_event_type"] == 0
    s = score(marginals(*view(d1)), marginals(*view(d2)), n_boot=10)
    names = {x.metric for x in s}
    assert "spread_ticks/wasserstein" in names and all(x.ci_low <= x.ci_high for x in s)
    same = {x.metric: x.value for x in score(marginals(m1, b1), marginals(m1, b1), n_boot=2)}
    assert same["order_size/ks"] == 0.0
    r = event_returns(m1, b1, horizons_ms=(1, 10))
    assert r["anchors"][0] > 0 and set(r["event"]) == {1, 10}


def test_diagnostics_cli_writes_every_breakdown(tmp_path):
    """The analyse-only diagnostics CLI over an inference run whose generated windows are
    copies of the real continuations: sanity gate passes, every breakdown is written and
    stamped with its origin."""
    import shutil
    from sigma0_b200.cli.infer import main as infer
    from sigma0_b200.eval.stylized import main as diag
    run = tmp_path / "gen"
    assert infer(["--preset", "smoke", "--impl", "torch", "--synthetic", "2", "--n_sequences", "4", "--batch_size",
                  "4", "--n_cond_msgs", "4", "--n_gen_msgs", "8", "--sample_top_n", "1", "--save_dir", str(run)]) == 0
    for p in glob.glob(str(run / "data_gen" / "*.csv")):
        os.remove(p)
    for p in glob.glob(str(run / "data_real" / "*.csv")):
        shutil.copy(p, str(run / "data_gen" / os.path.basename(p).replace(".csv", "_gen_id_0.csv")))
    out = tmp_path / "diag"
    diag(["--run", str(run), "--out", str(out), "--experiment", "smoke", "--bin_width", "2", "--cond_msgs", "4"])
    for name in ("sanity", "stylized_facts", "tstr", "tail", "regime", "position", "joint", "otm", "baselines",
                 "repro", "_provenance"):
        assert (out / f"{name}.json").exists(), name
    pos = json.load(open(out / "position.json"))
    assert pos["origin"]["experiment"] == "smoke" and pos["c"] == 4
    assert all(v is None or abs(v) < 1e-9 for v in pos["ws_tau"])


def test_model_zoo_ce_scores_every_checkpoint_on_one_sample(tmp_path, capsys):
    """Every complete checkpoint step is scored on the same fixed held-out sample; the record
    carries CE, accuracy, the iso-CE selection; config drift and missing steps are errors."""
    from sigma0_b200.cli.train import main as train
    from sigma0_b200.eval import model_zoo_ce as zoo
    ck = tmp_path / "ck"
    assert train(["--preset", "smoke", "--impl", "torch", "--synthetic", "2", "--n_messages", "4", "--micro_bsz",
                  "2", "--log_every", "1", "--watchdog_timeout", "0", "--ckpt_dir", str(ck), "--steps", "2",
                  "--save_every", "1"]) == 0
    out = tmp_path / "zoo.json"
    base = ["--checkpoint_root", str(ck), "--synthetic", "2", "--batch_size", "2", "--max_batches", "2",
            "--device", "cpu", "--targets", "9.5,9.0"]
    assert zoo.main(base + ["--output", str(out), "--expected_architecture", "mamba3"]) == 0
    rec = json.loads(out.read_text())
    assert [r["step"] for r in rec["results"]] == [1, 2]
    assert all(np.isfinite(r["validation_ce"]) and 0 <= r["validation_accuracy"] <= 1 for r in rec["results"])
    assert rec["selection"]["best_validation"]["step"] in (1, 2) and set(rec["selection"]["iso_ce"]) == {"9.5", "9"}
    assert rec["validation"]["sequences"] == 4
    # the same sample every time: a second run of one step reproduces its CE exactly
    assert zoo.main(base + ["--output", str(tmp_path / "one.json"), "--steps", "2"]) == 0
    one = json.loads((tmp_path / "one.json").read_text())["results"][0]
    assert one["validation_ce"] == rec["results"][1]["validation_ce"]
    with pytest.raises(ValueError, match="missing"):
        zoo.main(base + ["--output", str(tmp_path / "x.json"), "--steps", "7"])
    with pytest.raises(ValueError, match="architecture mismatch"):
        zoo.main(base + ["--output", str(tmp_path / "x.json"), "--expected_architecture", "gdn"])
    meta = ck / "2" / "metadata" / "metadata"
    m = json.loads(meta.read_text())
    m["config"]["d_model"] = 64
    meta.write_text(json.dumps(m))
    with pytest.raises(ValueError, match="drift at step 2: d_model"):
        zoo.main(base + ["--output", str(tmp_path / "x.json")])


def test_trade_anchors_feed_inference(tmp_path):
    """Anchored windows end on a trade, balance the two directions, skip a day stored twice,
    and inference runs exactly those windows."""
    from sigma0_b200.cli.infer import main as infer
    from sigma0_b200.data.lobster import save_day
    from sigma0_b200.data.synthetic import make_sequences
    from sigma0_b200.eval import trade_anchors as ta
    days = make_sequences(3, 300, seed=4)
    data = tmp_path / "days"
    save_day(days[0], str(data), "GOOG", "2025-12-01")
    save_day(days[1], str(data), "GOOG", "2025-12-02")
    save_day(days[2], str(data), "GOOG", "2025-12-03")
    dup = days[1]                               # the same session again under another time range
    np.save(data / "GOOG_2025-12-02_24900000_57900000_message.npy", dup.msgs)
    np.save(data / "GOOG_2025-12-02_24900000_57900000_book.npy", dup.books)
    out = tmp_path / "anchors.json"
    assert ta.main(["--data_dir", str(data), "--out", str(out), "--n_cond_msgs", "6", "--n_gen_msgs", "4",
                    "--n_samples", "20", "--seed", "1"]) == 0
    rec = json.loads(out.read_text())
    files = rec["message_files"]
    assert len(files) == 4 and rec["distinct_days_drawn_from"] == 3 and len(rec["windows"]) == 20
    same_day = {i for i, f in enumerate(files) if "2025-12-02" in f}
    assert len(same_day) == 2 and len(same_day & {i for i, _ in rec["windows"]}) == 1   # one file per day
    for (i, s), d in zip(rec["windows"], rec["anchor_direction"]):
        m = np.load(files[i])
        assert m[s + 5, 1] == 4 and m[s + 5, 2] == d          # the last conditioning message is the trade
    assert abs(rec["anchor_direction"].count(0) - rec["anchor_direction"].count(1)) <= 2
    run = tmp_path / "gen"
    assert infer(["--preset", "smoke", "--impl", "torch", "--data_dir", str(data), "--window_starts_file", str(out),
                  "--batch_size", "10", "--n_cond_msgs", "6", "--n_gen_msgs", "4", "--sample_top_n", "1",
                  "--save_dir", str(run)]) == 0
    got = json.loads((run / "sample_indices_rank0.json").read_text())["windows"]
    assert got == rec["windows"]
    cond = sorted(glob.glob(str(run / "data_cond" / "*_message_real_id_*.csv")))
    assert len(cond) == 20
