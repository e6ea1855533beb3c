"""The training CLI end to end on the GPU (bin/train.rs:298-446): token files
on disk, the reference's window positions, per-step losses against the CPU
oracle's train_step on the same windows from the same init, validation and
bits per byte, RSTK checkpoints, and a resume that continues the run."""
import numpy as np
import pytest

import pyoracle as po
from rustane_b200 import engine, train
from rustane_b200.data import TokenBytes, TokenData, compute_bpb, load_checkpoint
from rustane_b200.tensors import ModelOptState, ModelTensors

pytestmark = pytest.mark.gpu

MODEL = "custom:256,512,2,128"  # heads 2, hd 128, vocab 8192


@pytest.fixture
def files(tmp_path):
    rng = np.random.default_rng(5)
    # a learnable stream: runs of a short repeated phrase with noise
    phrase = rng.integers(0, 8192, size=37)
    train_tok = np.tile(phrase, 2000)[:60000].copy()
    noise = rng.random(train_tok.size) < 0.1
    train_tok[noise] = rng.integers(0, 8192, size=noise.sum())
    val_tok = np.tile(phrase, 300)[:9000]
    (tmp_path / "train.bin").write_bytes(train_tok.astype("<u2").tobytes())
    (tmp_path / "val.bin").write_bytes(val_tok.astype("<u2").tobytes())
    table = rng.integers(1, 6, size=8192).astype("<i4")
    table[:4] = 0
    (tmp_path / "token_bytes.bin").write_bytes(table.tobytes())
    return tmp_path


def args(files, *extra):
    return train.parse_args(["--model", MODEL, "--data", str(files / "train.bin"), "--val", str(files / "val.bin"),
                             "--token-bytes", str(files / "token_bytes.bin"), "--accum", "2", "--warmup", "2",
                             "--lr", "1e-3", "--val-steps", "3", *extra])


def test_cli_losses_follow_oracle(files):
    a = args(files, "--steps", "4", "--val-interval", "2")
    lines = []
    res = train.run(a, out=lines.append)
    assert len(res.losses) == 4 and all(np.isfinite(res.losses))
    assert abs(res.losses[0] - np.log(8192)) < 0.1

    cfg = train.model_config(MODEL)
    tc = train.train_config(a)
    otc = po.default_train_config(**{k: getattr(tc, k) for k in (
        "max_lr", "min_lr_frac", "warmup_steps", "total_steps", "beta1", "beta2", "eps", "weight_decay",
        "matrix_lr_scale", "embed_lr_scale", "loss_scale", "accum_steps", "grad_clip", "softcap")})
    o = po.Oracle(cfg, tc.accum_steps)
    w = engine.random_weights(cfg)
    g, opt = ModelTensors.zeros(cfg), ModelOptState.zeros(cfg)
    with TokenData.open(a.data_path) as td:
        for step in range(4):
            wins = [td.train_window(step, m, cfg.seq) for m in range(tc.accum_steps)]
            tok = np.concatenate([x[0] for x in wins])
            tgt = np.concatenate([x[1] for x in wins])
            loss_ref, _ = o.train_step(w, g, opt, tok, tgt, step, otc)
            assert abs(res.losses[step] - loss_ref) < 3e-3, (step, res.losses[step], loss_ref)
    assert res.losses[-1] < res.losses[0]

    # final validation against the oracle forward of the trained weights' windows
    o_val = po.Oracle(cfg, 1)
    tb = TokenBytes.load(a.token_bytes_path)
    losses, targets = [], []
    with TokenData.open(a.val_path) as vd:
        for vs in range(3):
            tok, tgt = vd.val_window(vs, cfg.seq)
            _, _, ptl = o_val.forward(w, tok, tgt, want_token_losses=True)
            losses.append(np.asarray(ptl, np.float32))
            targets.append(tgt)
    ref_loss = float(np.mean(np.concatenate(losses)))
    ref_bpb, _, _ = compute_bpb(np.concatenate(losses), np.concatenate(targets), tb)
    step_, vl, vb = res.val[-1]
    # the GPU weights trained in bf16 against the oracle's fp32: 2e-2 nats
    assert step_ == 4 and abs(vl - ref_loss) < 2e-2 and abs(vb - ref_bpb) < 3e-3 * ref_bpb
    assert any(line.startswith("step     3: loss = ") for line in lines)
    assert any(line.startswith("  >>> val_loss = ") for line in lines)
    assert lines[-1].startswith("  best val_bpb: ")


def test_cli_checkpoint_and_resume(files):
    ck = files / "ck"
    full = train.run(args(files, "--steps", "4", "--val-interval", "100", "--ckpt-interval", "2", "--ckpt-dir",
                          str(ck), "--ckpt-opt"), out=lambda s: None)
    assert [p.name for p in full.checkpoints] == ["ckpt_000002.bin", "ckpt_000004.bin"]
    cfg = train.model_config(MODEL)
    w, opt, step, version = load_checkpoint(ck / "ckpt_000002.bin", cfg)
    assert (step, version) == (2, 2) and opt is not None and np.abs(opt.v.embed).max() > 0
    resumed = train.run(args(files, "--steps", "4", "--val-interval", "100", "--resume",
                             str(ck / "ckpt_000002.bin")), out=lambda s: None)
    assert len(resumed.losses) == 2
    np.testing.assert_allclose(resumed.losses, full.losses[2:], rtol=1e-6)


def test_sweep_writes_bench_result(tmp_path):
    from rustane_b200 import bench_result as br
    from rustane_b200.sweep import run_sweep
    cfg = train.model_config(MODEL)
    res = run_sweep(cfg, "small", batch=2, out=lambda s: None)
    assert len(res.loss_trace) == 12 and all(np.isfinite(res.loss_trace))
    assert res.results.loss_start == res.loss_trace[0] and res.results.loss_end == res.loss_trace[-1]
    r = res.results
    assert 0 < r.ms_fwd + r.ms_bwd + r.ms_upd <= r.ms_per_step * 1.05 and r.tok_per_s > 0
    assert res.fingerprint == br.compute_fingerprint(res)
    p = br.write_result(res, tmp_path / "bench-result.json", out=lambda s: None)
    assert p.read_text() == br.to_json(res, pretty=True)


def _dp_rank(rank, port, root, ck):
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from pathlib import Path
    res = train.run(args(Path(root), "--steps", "3", "--val-interval", "100", "--ckpt-interval", "3", "--ckpt-dir",
                         ck, "--ckpt-opt"), out=lambda s: None, dist=train.DistInfo(2, rank, rank))
    if rank == 0:
        np.save(Path(root) / "dp_losses.npy", np.array([res.losses, res.gnorms]))


@pytest.mark.skipif(__import__("torch").cuda.device_count() < 2, reason="needs 2 GPUs")
def test_cli_data_parallel_matches_one_gpu(files):
    """torchrun-style data parallelism in the CLI: two ranks with one of the
    two microbatches each must give the losses, gradient norms and checkpoint
    of one GPU running both (the summation order differs, so to rounding)."""
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_dp_rank, args=(port, str(files), str(files / "ck_dp")), nprocs=2, join=True)
    losses, gnorms = np.load(files / "dp_losses.npy")
    one = train.run(args(files, "--steps", "3", "--val-interval", "100", "--ckpt-interval", "3", "--ckpt-dir",
                         str(files / "ck_one"), "--ckpt-opt"), out=lambda s: None)
    # step 0 starts from the same weights; later steps from weights that AdamW moved
    # a little differently (the gradients agree only to rounding)
    assert abs(losses[0] - one.losses[0]) < 2e-5 and abs(gnorms[0] - one.gnorms[0]) < 1e-3 * one.gnorms[0]
    np.testing.assert_allclose(losses, one.losses, rtol=0, atol=1e-3)
    np.testing.assert_allclose(gnorms, one.gnorms, rtol=2e-2)
    cfg = train.model_config(MODEL)
    w_dp, opt_dp, step_dp, _ = load_checkpoint(files / "ck_dp" / "ckpt_000003.bin", cfg)
    w_one, opt_one, step_one, _ = load_checkpoint(files / "ck_one" / "ckpt_000003.bin", cfg)
    assert step_dp == step_one == 3
    w0 = engine.random_weights(cfg)
    for (name, a), (_, b), (_, a0) in zip(w_one.tensors(), w_dp.tensors(), w0.tensors()):
        u1, u2 = a - a0, b - a0  # AdamW moves near-zero gradients by ~lr either way: compare whole updates
        assert np.linalg.norm(u1 - u2) <= 0.05 * np.linalg.norm(u1) + 1e-7, name
    for name, a in opt_one.m.tensors():
        b = dict(opt_dp.m.tensors())[name]
        assert np.linalg.norm(a - b) <= 0.05 * np.linalg.norm(a) + 1e-12, name
