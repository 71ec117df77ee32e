"""The 1-token-per-message model (``OneTokenPaddedLobPredModel``'s tree): Flax-compatible
parameter names, per-field local inputs from the dataset, a training step that lowers the
loss, the recurrent step against the full forward, and the CLI flag."""
import torch

from sigma0_b200.encoding import tok1


def _args(**kw):
    from sigma0_b200.models import preset_args
    return preset_args("smoke", token_mode="1tok", d_model=32, mamba3_d_state=16, mamba3_headdim=16, n_messages=6,
                       micro_bsz=2, n_layers=2, n_book_pre_layers=1, n_book_post_layers=1, warmup_end=0.0,
                       ssm_lr_base=3e-3, **kw)


def _batch(n=2, m=6):
    from sigma0_b200.data import make_sequences, LobWindowDataset, collate
    ds = LobWindowDataset.from_days(make_sequences(n, m + 1, seed=0), m, token_mode="1tok")
    return collate([ds[i] for i in range(n)])


def test_parameter_tree_and_shapes():
    from sigma0_b200.models import build_model
    m = build_model(_args())
    names = dict(m.named_parameters())
    for i, v in enumerate(tok1.FIELD_VOCAB_SIZES_WITH_SPECIAL):
        assert names[f"field_embedding.field_{i}.embedding"].shape == (v, 32)
        assert names[f"decoder.head_{i}.kernel"].shape == (32, v)
        assert names[f"decoder.head_{i}.bias"].shape == (v,)
    assert not any(n.startswith("message_encoder") for n in names)
    assert any(n.startswith("book_encoder.pre_layers_0") for n in names)


def test_dataset_gives_local_field_ids():
    x, y, book = _batch()
    assert x.shape == (2, 6, tok1.N_FIELDS) and y.shape == x.shape and book.shape[:2] == (2, 6)
    for i, v in enumerate(tok1.FIELD_VOCAB_SIZES_WITH_SPECIAL):
        assert int(y[..., i].max()) < v and int(y[..., i].min()) >= 0
    assert torch.equal(x[:, 1:], y[:, :-1])


def test_training_lowers_the_loss_and_step_matches_forward():
    from sigma0_b200.train.trainer import Trainer
    tr = Trainer(_args(), device=torch.device("cpu"), total_steps=50)
    batch = _batch()
    l0 = tr.train_step(batch)
    for _ in range(8):
        l = tr.train_step(batch)
    assert l < l0 - 0.3, (l0, l)
    m = tr.model.eval()
    x, _, book = batch
    with torch.no_grad():
        full = m(x, book)
        st = m.initial_state(2)
        outs = []
        for t in range(x.shape[1]):
            st, lp = m.step(st, x[:, t:t + 1], book[:, t:t + 1])
            outs.append(lp)
    for i in range(tok1.N_FIELDS):
        step_i = torch.cat([o[i] for o in outs], 1)
        assert (full[i] - step_i).abs().max().item() < 2e-3, i


def test_cli_trains_the_1tok_model(tmp_path):
    from sigma0_b200.cli.train import main
    rc = main(["--preset", "smoke", "--token_mode", "1tok", "--d_model", "32", "--n_layers", "1", "--steps", "2",
               "--log_every", "1", "--n_messages", "6", "--micro_bsz", "2", "--synthetic", "2", "--impl", "torch",
               "--watchdog_timeout", "0"])
    assert rc == 0
