"""The training CLI's host logic (bin/train.rs:40-98, 298-366): flags,
defaults, model selection, parameter count and the Rust number formats of
its log lines, and the host side of a data-parallel run (the microbatch
split over ranks, the loss mean over gloo ranks).  No GPU."""
import numpy as np
import pytest

from rustane_b200 import train
from rustane_b200.model import ModelConfig
from rustane_b200.rustfmt import display_f32, exp_f32, json_f32, json_f64


def test_defaults_and_auto_schedule():
    a = train.parse_args(["--data", "x.bin"])
    assert (a.model, a.total_steps, a.val_interval, a.val_steps, a.checkpoint_interval) == \
        ("gpt_karpathy", 72000, 500, 20, 1000)
    assert a.warmup_steps == 1440 and a.max_lr == pytest.approx(3e-4)  # 72000 / 50
    a = train.parse_args(["--data", "x.bin", "--steps", "1000"])
    assert a.warmup_steps == 100  # max(1000 / 50, 100)
    a = train.parse_args(["--data", "x.bin", "--warmup", "7", "--lr", "1e-3"])
    assert a.warmup_steps == 7 and a.max_lr == pytest.approx(1e-3)


def test_overrides_reach_train_config():
    a = train.parse_args(["--data", "d", "--accum", "4", "--loss-scale", "128", "--grad-clip", "0.5", "--beta2",
                          "0.99", "--eps", "1e-6", "--wd", "0", "--embed-lr", "2", "--min-lr-frac", "0",
                          "--matrix-lr", "0.1", "--softcap", "15"])
    tc = train.train_config(a)
    assert (tc.accum_steps, tc.loss_scale, tc.grad_clip) == (4, 128.0, 0.5)
    assert (tc.beta2, tc.eps, tc.weight_decay, tc.embed_lr_scale) == (0.99, 1e-6, 0.0, 2.0)
    assert (tc.min_lr_frac, tc.matrix_lr_scale, tc.softcap) == (0.0, 0.1, 15.0)
    tc = train.train_config(train.parse_args(["--data", "d"]))  # TrainConfig::default (full_model.rs:51-70)
    assert (tc.accum_steps, tc.loss_scale, tc.weight_decay, tc.embed_lr_scale, tc.matrix_lr_scale) == \
        (10, 256.0, 0.1, 5.0, 0.05)


@pytest.mark.parametrize("argv,msg", [(["--data", "d", "--bogus", "1"], "Unknown arg: --bogus"),
                                      (["--steps", "5"], "--data required"),
                                      (["--data"], "--data needs a value")])
def test_usage_errors(argv, msg):
    with pytest.raises(train.UsageError, match=msg):
        train.parse_args(argv)
    assert train.main(argv) == 1


def test_model_selection():
    cfg = train.model_config("custom:1024,2816,12,256")  # bin/train.rs:301-310
    assert (cfg.dim, cfg.hidden, cfg.heads, cfg.hd, cfg.nlayers, cfg.seq, cfg.vocab) == \
        (1024, 2816, 8, 128, 12, 256, 8192)
    assert train.model_config("mha_28l") == ModelConfig.mha_28l()
    assert train.model_config("target_600m") == ModelConfig.target_600m()
    for bad in ["gpt_3", "custom:1,2"]:
        with pytest.raises(train.UsageError, match="Unknown model"):
            train.model_config(bad)


def test_param_count_line():
    # bin/train.rs:320-322 for gpt_karpathy: 8192*768 + 6*(4*768^2 + 3*768*2048 + 2*768) + 768
    assert train.total_params(ModelConfig.gpt_karpathy()) == 48768768
    # 20*(4*1536^2 + 3*1536*4096 + 2*1536) + 8192*1536 + 1536
    assert f"{train.total_params(ModelConfig.target_600m()) / 1e6:.1f}M" == "578.9M"


def test_rust_number_formats():
    assert exp_f32(3e-4, 2) == "3.00e-4" and exp_f32(3e-4, 0) == "3e-4" and exp_f32(1e-8, 0) == "1e-8"
    assert exp_f32(2.5e-5, 2) == "2.50e-5" and exp_f32(1.0, 2) == "1.00e0"
    assert [display_f32(x) for x in (0.95, 256.0, 1.0, 0.05, 0.0, 1e-8)] == \
        ["0.95", "256", "1", "0.05", "0", "0.00000001"]
    assert [json_f32(x) for x in (961.0, 0.1, 533.3333, 1e-7, 1.5e30, 0.001234, 0.0)] == \
        ["961.0", "0.1", "533.3333", "1e-7", "1.5e30", "0.001234", "0.0"]
    assert json_f64(579.716608) == "579.716608" and json_f64(float("nan")) == "null"


def test_rank_micros_partition_the_accum_loop():
    for accum, world in ((8, 8), (8, 2), (6, 3), (4, 1)):
        blocks = [train.rank_micros(accum, world, r) for r in range(world)]
        assert [m for b in blocks for m in b] == list(range(accum))
        assert all(len(b) == accum // world for b in blocks)
    with pytest.raises(train.UsageError, match="not a multiple"):
        train.rank_micros(6, 4, 0)


def test_dist_info_from_torchrun_env():
    assert train.DistInfo.from_env({}) == train.DistInfo(1, 0, 0)
    assert train.DistInfo.from_env({"WORLD_SIZE": "1", "RANK": "0"}) == train.DistInfo(1, 0, 0)
    assert train.DistInfo.from_env({"WORLD_SIZE": "4", "RANK": "6", "LOCAL_RANK": "2"}) == train.DistInfo(4, 6, 2)


def test_main_rejects_accum_not_divisible_by_world(monkeypatch, capsys):
    monkeypatch.setenv("WORLD_SIZE", "4")
    monkeypatch.setenv("RANK", "0")
    assert train.main(["--data", "d", "--accum", "6"]) == 1
    assert "not a multiple" in capsys.readouterr().err


def _mean_rank(rank, port, out):
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    g = train._Group(train.DistInfo(2, rank, rank))
    try:
        m = g.mean([9.25, 8.75][rank])
        if rank == 0:
            np.save(out, np.array([m]))
    finally:
        g.close()


def test_group_mean_over_gloo_ranks(tmp_path):
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = str(tmp_path / "m.npy")
    mp.spawn(_mean_rank, args=(port, out), nprocs=2, join=True)
    assert np.load(out)[0] == np.float32(9.0)
