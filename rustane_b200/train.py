"""Full-model training CLI on a B200 (the reference's `train` binary,
crates/engine/src/bin/train.rs): same flags, defaults, sampling positions,
schedule, validation and checkpoint files, with the step itself on the
device through librustane_cuda.so.

    python -m rustane_b200.train --data train.bin [--val val.bin] \\
        [--token-bytes token_bytes.bin] [--model gpt_karpathy] [--steps 72000] \\
        [--val-interval 500] [--val-steps 20] [--ckpt-dir DIR]

Flags of the reference (bin/train.rs:40-89): --model --data --val
--token-bytes --steps --warmup --lr --accum --loss-scale --grad-clip --beta2
--eps --wd --embed-lr --min-lr-frac --matrix-lr --val-interval --val-steps
--ckpt-interval --ckpt-dir.  Added here: --softcap F (TrainConfig.softcap),
--ckpt-opt (checkpoints carry the AdamW moments, RSTK version 2),
--resume PATH (continue from a checkpoint; version 2 restores the moments
too), --device N, and the presets target_600m / target_800m / target_1b /
target_1_5b besides gpt_karpathy / gpt_1024 / mha_28l / custom:dim,hidden,nlayers,seq.

Each optimizer step runs the accum microbatches as one device batch
(gradients summed over them, loss averaged): the same arithmetic as the
reference's microbatch loop (bin/train.rs:283-301), one launch sequence.

Data parallel (an addition; the reference trains on one device): launched by
torchrun with WORLD_SIZE > 1, rank r takes the contiguous block of accum/world
microbatches starting at r * accum/world on GPU LOCAL_RANK (--device is then
ignored), the library sums the gradients over the ranks inside the step
(rt_dist_init, data-parallel mode), and the printed loss is the mean of the
ranks' losses -- the same step as one GPU running all accum microbatches.
accum must be a multiple of the world size.  Every rank runs validation and
takes part in the checkpoint and grad-norm gathers; rank 0 alone prints and
writes files.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m rustane_b200.train \\
        --data train.bin --accum 8 ...
"""
from __future__ import annotations

import os
import sys
import time
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .data import TokenBytes, TokenData, load_checkpoint, save_checkpoint
from .engine import CompiledKernels, TrainConfig, learning_rate, random_weights
from .model import ModelConfig
from .rustfmt import display_f32, exp_f32

PRESETS = {
    "gpt_karpathy": ModelConfig.gpt_karpathy,
    "gpt_1024": ModelConfig.gpt_1024,
    "mha_28l": ModelConfig.mha_28l,
    "target_600m": ModelConfig.target_600m,
    "target_800m": ModelConfig.target_800m,
    "target_1b": ModelConfig.target_1b,
    "target_1_5b": ModelConfig.target_1_5b,
}


class UsageError(Exception):
    pass


@dataclass
class Args:
    """bin/train.rs:17-38 plus the flags added here."""
    model: str = "gpt_karpathy"
    data_path: Path | None = None
    val_path: Path | None = None
    token_bytes_path: Path | None = None
    total_steps: int = 72000
    warmup_steps: int = 0
    max_lr: float = 0.0
    accum_steps: int = 0
    loss_scale: float = 0.0
    grad_clip: float = 0.0
    beta2: float = 0.0
    eps: float = 0.0
    weight_decay: float = -1.0
    embed_lr_scale: float = -1.0
    min_lr_frac: float = -1.0
    matrix_lr_scale: float = -1.0
    val_interval: int = 500
    val_steps: int = 20
    checkpoint_interval: int = 1000
    checkpoint_dir: Path | None = None
    softcap: float = -1.0
    checkpoint_opt: bool = False
    resume: Path | None = None
    device: int = 0


_FLAGS = {
    "--model": ("model", str), "--data": ("data_path", Path), "--val": ("val_path", Path),
    "--token-bytes": ("token_bytes_path", Path), "--steps": ("total_steps", int), "--warmup": ("warmup_steps", int),
    "--lr": ("max_lr", float), "--accum": ("accum_steps", int), "--loss-scale": ("loss_scale", float),
    "--grad-clip": ("grad_clip", float), "--beta2": ("beta2", float), "--eps": ("eps", float),
    "--wd": ("weight_decay", float), "--embed-lr": ("embed_lr_scale", float),
    "--min-lr-frac": ("min_lr_frac", float), "--matrix-lr": ("matrix_lr_scale", float),
    "--val-interval": ("val_interval", int), "--val-steps": ("val_steps", int),
    "--ckpt-interval": ("checkpoint_interval", int), "--ckpt-dir": ("checkpoint_dir", Path),
    "--softcap": ("softcap", float), "--resume": ("resume", Path), "--device": ("device", int),
}


def parse_args(argv: list[str]) -> Args:
    """parse_args (bin/train.rs:40-98): flag/value pairs, auto warmup
    max(steps / 50, 100) and lr 3e-4 when left at 0."""
    a = Args()
    i = 0
    while i < len(argv):
        flag = argv[i]
        if flag == "--ckpt-opt":
            a.checkpoint_opt = True
            i += 1
            continue
        if flag not in _FLAGS:
            raise UsageError(f"Unknown arg: {flag}")
        if i + 1 >= len(argv):
            raise UsageError(f"{flag} needs a value")
        name, conv = _FLAGS[flag]
        try:
            setattr(a, name, conv(argv[i + 1]))
        except ValueError as e:
            raise UsageError(f"{flag}: {e}") from None
        i += 2
    if a.data_path is None:
        raise UsageError("--data required")
    if a.warmup_steps == 0:
        a.warmup_steps = max(a.total_steps // 50, 100)
    if a.max_lr == 0.0:
        a.max_lr = 3e-4
    return a


def model_config(name: str) -> ModelConfig:
    """bin/train.rs:300-318: a preset, or custom:dim,hidden,nlayers,seq with
    head_dim 128, heads = dim / 128 and vocab 8192."""
    if name.startswith("custom:"):
        try:
            dim, hidden, nl, seq = (int(x) for x in name[7:].split(","))
        except ValueError:
            raise UsageError(f"Unknown model: {name}") from None
        return ModelConfig.custom(dim, hidden, dim // 128, nl, seq=seq, vocab=8192)
    if name not in PRESETS:
        raise UsageError(f"Unknown model: {name}")
    return PRESETS[name]()


def total_params(cfg: ModelConfig) -> int:
    """bin/train.rs:320-322."""
    per_layer = (cfg.dim * cfg.q_dim + cfg.dim * cfg.kv_dim * 2 + cfg.q_dim * cfg.dim + cfg.dim * cfg.hidden * 3
                 + cfg.dim * 2)
    return cfg.vocab * cfg.dim + cfg.nlayers * per_layer + cfg.dim


def train_config(a: Args) -> TrainConfig:
    """TrainConfig::default overridden by the flags (bin/train.rs:352-366)."""
    tc = TrainConfig(total_steps=a.total_steps, warmup_steps=a.warmup_steps, max_lr=a.max_lr)
    if a.accum_steps > 0:
        tc.accum_steps = a.accum_steps
    if a.loss_scale > 0.0:
        tc.loss_scale = a.loss_scale
    if a.grad_clip > 0.0:
        tc.grad_clip = a.grad_clip
    if a.beta2 > 0.0:
        tc.beta2 = a.beta2
    if a.eps > 0.0:
        tc.eps = a.eps
    if a.weight_decay >= 0.0:
        tc.weight_decay = a.weight_decay
    if a.embed_lr_scale >= 0.0:
        tc.embed_lr_scale = a.embed_lr_scale
    if a.min_lr_frac >= 0.0:
        tc.min_lr_frac = a.min_lr_frac
    if a.matrix_lr_scale >= 0.0:
        tc.matrix_lr_scale = a.matrix_lr_scale
    if a.softcap >= 0.0:
        tc.softcap = a.softcap
    return tc


@dataclass
class DistInfo:
    """This process's place in a torchrun launch (one process per GPU)."""
    world: int = 1
    rank: int = 0
    local_rank: int = 0

    @classmethod
    def from_env(cls, env=os.environ) -> "DistInfo":
        world = int(env.get("WORLD_SIZE", "1"))
        if world <= 1:
            return cls()
        return cls(world, int(env["RANK"]), int(env.get("LOCAL_RANK", env["RANK"])))


def rank_micros(accum: int, world: int, rank: int) -> range:
    """The microbatch indices of the reference's accum loop (bin/train.rs:284)
    that `rank` runs: a contiguous block of accum / world."""
    if accum % world:
        raise UsageError(f"--accum {accum} is not a multiple of the {world} data-parallel ranks")
    per = accum // world
    return range(rank * per, (rank + 1) * per)


class _Group:
    """Host-side plumbing of a data-parallel CLI run over torch.distributed
    (gloo: only the communicator id and one loss per step cross it; the
    gradients move inside the library over NCCL)."""

    def __init__(self, d: DistInfo):
        import torch.distributed as tdist
        self.d, self.tdist = d, tdist
        self.owned = not tdist.is_initialized()
        if self.owned:  # a rank that fails ends the others' next host collective within the timeout
            import datetime
            tdist.init_process_group("gloo", rank=d.rank, world_size=d.world,
                                     timeout=datetime.timedelta(seconds=300))

    def join(self, kernels: CompiledKernels) -> None:
        uid = [CompiledKernels.nccl_unique_id() if self.d.rank == 0 else None]
        self.tdist.broadcast_object_list(uid, src=0)
        kernels.dist_init(self.d.world, self.d.rank, uid[0], timeout_ms=120000)

    def mean(self, x: float) -> float:
        import torch
        t = torch.tensor([x], dtype=torch.float64)
        self.tdist.all_reduce(t)
        return float(np.float32(t.item() / self.d.world))

    def close(self) -> None:
        if self.owned:
            self.tdist.destroy_process_group()


def f32sum(x: np.ndarray) -> np.float32:
    """Left-to-right f32 sum (Rust's Iterator::sum over f32)."""
    return np.cumsum(np.asarray(x, np.float32), dtype=np.float32)[-1] if len(x) else np.float32(0)


def validate(cfg: ModelConfig, kernels: CompiledKernels, val_data: TokenData, token_bytes: TokenBytes | None,
             steps: int, softcap: float) -> tuple[float, float]:
    """validate (bin/train.rs:116-162): mean per-token loss over `steps`
    windows at pos = vs * seq mod (n - seq - 1), bits per byte when the
    token_bytes table is given.  Windows go to the device in batches of up to
    the context's max_batch; the sums keep the reference's order."""
    from .data import compute_bpb
    total_loss = np.float32(0)
    all_losses, all_targets = [], []
    vs = 0
    while vs < steps:
        nb = min(kernels.max_batch, steps - vs)
        wins = [val_data.val_window(vs + j, cfg.seq) for j in range(nb)]
        tok = np.concatenate([w[0] for w in wins])
        tgt = np.concatenate([w[1] for w in wins])
        _, ptl = kernels.forward(tok, tgt, softcap, per_token=True)
        ptl = np.asarray(ptl, np.float32).reshape(nb, cfg.seq)
        for j in range(nb):
            total_loss = np.float32(total_loss + f32sum(ptl[j]))
        if token_bytes is not None:
            all_losses.append(ptl.reshape(-1))
            all_targets.append(tgt)
        vs += nb
    avg = float(np.float32(total_loss / np.float32(steps * cfg.seq))) if steps else float("nan")
    bpb = 0.0
    if token_bytes is not None and all_losses:
        bpb, _, _ = compute_bpb(np.concatenate(all_losses), np.concatenate(all_targets), token_bytes)
    return avg, bpb


@dataclass
class RunResult:
    losses: list = field(default_factory=list)
    gnorms: list = field(default_factory=list)
    lrs: list = field(default_factory=list)
    val: list = field(default_factory=list)  # (step, val_loss, val_bpb)
    checkpoints: list = field(default_factory=list)
    best_bpb: float = float("inf")
    seconds: float = 0.0


def run(a: Args, out=print, dist: DistInfo | None = None) -> RunResult:
    """main (bin/train.rs:298-446); data parallel over the ranks of `dist`
    (default: the torchrun environment)."""
    dist = dist if dist is not None else DistInfo.from_env()
    tc = train_config(a)
    micros = rank_micros(tc.accum_steps, dist.world, dist.rank)
    if dist.rank != 0:
        out = lambda s: None  # noqa: E731
    group = _Group(dist) if dist.world > 1 else None
    try:
        return _run(a, tc, micros, dist, group, out)
    finally:
        if group is not None:
            group.close()


def _run(a: Args, tc: TrainConfig, micros: range, dist: DistInfo, group, out) -> RunResult:
    cfg = model_config(a.model)
    out("=== Rustane Trainer ===")
    out(f"model: {a.model} ({cfg.nlayers}L, {cfg.dim}D, {cfg.vocab}V, {cfg.seq}S)")
    out(f"params: {total_params(cfg) / 1e6:.1f}M")

    out("\nLoading training data...")
    train_data = TokenData.open(a.data_path)
    out(f"  {len(train_data)} tokens ({len(train_data) * 2.0 / 1e6:.1f} MB)")
    val_data = None
    if a.val_path is not None:
        out("Loading validation data...")
        val_data = TokenData.open(a.val_path)
        out(f"  {len(val_data)} tokens ({len(val_data) * 2.0 / 1e6:.1f} MB)")
    token_bytes = None
    if a.token_bytes_path is not None:
        out("Loading token_bytes...")
        token_bytes = TokenBytes.load(a.token_bytes_path)

    out("\nCreating the B200 context...")
    t0 = time.perf_counter()
    max_batch = max(len(micros), min(max(a.val_steps, 1), 32))
    device = dist.local_rank if group is not None else a.device
    kernels = CompiledKernels.compile(cfg, max_batch=max_batch, device=device)
    try:
        return _train(a, cfg, tc, micros, dist, group, out, kernels, train_data, val_data, token_bytes, t0)
    finally:
        # a failing rank (non-finite loss, a communicator timeout) releases its
        # context and communicator at once instead of holding the other ranks
        kernels.close()
        train_data.close()
        if val_data is not None:
            val_data.close()


def _train(a: Args, cfg, tc: TrainConfig, micros: range, dist: DistInfo, group, out, kernels, train_data, val_data,
           token_bytes, t0: float) -> RunResult:
    if group is not None:
        group.join(kernels)
        out(f"  data parallel: {dist.world} ranks x {len(micros)} microbatches")
    out(f"  ready in {time.perf_counter() - t0:.1f}s ({kernels.device_bytes() / 2**30:.1f} GiB on the device)")

    first_step = 0
    if a.resume is not None:
        weights, opt, first_step, version = load_checkpoint(a.resume, cfg)
        kernels.upload_weights(weights)
        if opt is not None:
            kernels.upload_opt(opt)
        out(f"  resumed from {a.resume} at step {first_step} (version {version}"
            f"{', with optimizer state' if opt is not None else ''})")
    else:
        kernels.upload_weights(random_weights(cfg))  # ModelWeights::random

    out("\nTraining config:")
    out(f"  lr: {exp_f32(tc.max_lr, 0)} (warmup {tc.warmup_steps} → cosine, "
        f"min_lr_frac: {display_f32(tc.min_lr_frac)})")
    out(f"  accum: {tc.accum_steps} microbatches, loss_scale: {display_f32(tc.loss_scale)}")
    out(f"  beta1: {display_f32(tc.beta1)}, beta2: {display_f32(tc.beta2)}, eps: {exp_f32(tc.eps, 0)}")
    out(f"  weight_decay: {display_f32(tc.weight_decay)}, grad_clip: {display_f32(tc.grad_clip)}")
    out(f"  embed_lr_scale: {display_f32(tc.embed_lr_scale)}, matrix_lr_scale: {display_f32(tc.matrix_lr_scale)}")
    out(f"  softcap: {display_f32(tc.softcap)}")
    out(f"  total steps: {tc.total_steps}")
    out("")

    res = RunResult()
    if val_data is not None:
        vl, vb = validate(cfg, kernels, val_data, token_bytes, a.val_steps, tc.softcap)
        out(f"step {first_step}: val_loss = {vl:.4f}, val_bpb = {vb:.4f}")
        res.val.append((first_step, vl, vb))

    seq = cfg.seq
    accum = tc.accum_steps
    gsc = np.float32(1.0) / (np.float32(accum) * np.float32(tc.loss_scale))
    train_start = time.perf_counter()
    for step in range(first_step, tc.total_steps):
        step_t0 = time.perf_counter()
        wins = [train_data.train_window(step, micro, seq) for micro in micros]
        tok = np.concatenate([w[0] for w in wins])
        tgt = np.concatenate([w[1] for w in wins])
        avg_loss = kernels.train_step(tok, tgt, step, tc)
        if group is not None:
            avg_loss = group.mean(avg_loss)
        gnorm = float(np.float32(kernels.last_grad_norm()) * gsc)
        lr = learning_rate(step, tc)
        step_time = time.perf_counter() - step_t0
        elapsed = time.perf_counter() - train_start
        out(f"step {step:>5}: loss = {avg_loss:.4f}, lr = {exp_f32(lr, 2)}, gnorm = {gnorm:.2f}, "
            f"time = {step_time:.2f}s, elapsed = {elapsed:.0f}s")
        res.losses.append(avg_loss)
        res.gnorms.append(gnorm)
        res.lrs.append(lr)

        last = step + 1 == tc.total_steps
        if val_data is not None and ((step + 1) % a.val_interval == 0 or last):
            vl, vb = validate(cfg, kernels, val_data, token_bytes, a.val_steps, tc.softcap)
            best = vb < res.best_bpb
            if best:
                res.best_bpb = vb
            out(f"  >>> val_loss = {vl:.4f}, val_bpb = {vb:.4f}{' (best)' if best else ''}")
            res.val.append((step + 1, vl, vb))

        if a.checkpoint_dir is not None and ((step + 1) % a.checkpoint_interval == 0 or last):
            weights = kernels.download_weights()
            opt = kernels.download_opt() if a.checkpoint_opt else None
            if dist.rank == 0:
                path = save_checkpoint(cfg, weights, opt, step + 1, a.checkpoint_dir, with_opt=a.checkpoint_opt)
                out(f"  saved checkpoint: {path} ({path.stat().st_size / 1e6:.1f} MB)")
                res.checkpoints.append(path)

    res.seconds = time.perf_counter() - train_start
    out("\n=== Training complete ===")
    out(f"  steps: {tc.total_steps}")
    out(f"  time: {res.seconds:.1f}s ({res.seconds / 60.0:.1f} min)")
    if res.best_bpb < float("inf"):
        out(f"  best val_bpb: {res.best_bpb:.4f}")
    return res


def main(argv: list[str] | None = None) -> int:
    try:
        a = parse_args(sys.argv[1:] if argv is None else argv)
        model_config(a.model)
        d = DistInfo.from_env()
        rank_micros(train_config(a).accum_steps, d.world, d.rank)
    except UsageError as e:
        print(e, file=sys.stderr)
        return 1
    run(a, out=lambda s: print(s, flush=True))
    return 0


if __name__ == "__main__":
    sys.exit(main())
