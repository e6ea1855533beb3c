"""Parameter-sweep benchmark on a B200 (crates/engine/tests/bench_param_sweep.rs):
the reference's configurations and protocol, writing the leaderboard
bench-result file.

    python -m rustane_b200.sweep 600m-A [--batch 1] [--out target/bench-result.json]

Protocol (run_sweep, bench_param_sweep.rs:55-200): ModelWeights::random,
tokens (i*31 + 7) mod vocab, targets shifted by one; forward loss0; 10 train
steps with TrainConfig::default (learning_rate(step), AdamW t = step + 1, the
clip rule on 1/loss_scale); a final forward; then 5 timed steps, median.
A step here is one rt_train_step (zero grads, forward, backward, grad norm,
clip decision, AdamW) on `batch` copies of the sequence; ms_per_step is its
host wall time (the reference times its steps the same way), ms_fwd / ms_bwd
/ ms_upd the device time of each phase (CUDA events), tok_per_s =
batch * seq * 1000 / ms_per_step.  batch 1 is the reference's protocol.
"""
from __future__ import annotations

import argparse
import sys
import time

import numpy as np

from . import bench_result as br
from .engine import CompiledKernels, TrainConfig, random_weights
from .model import ModelConfig

# bench_param_sweep.rs:240-470 (dim, hidden, heads, nlayers, seq)
SWEEP = {
    "600m-A": (1536, 4096, 12, 20, 512), "600m-B": (1280, 3456, 10, 28, 512), "600m-C": (1792, 4864, 14, 14, 512),
    "600m-D": (1536, 6144, 12, 16, 512), "600m-E": (1536, 4096, 12, 20, 256),
    "1b-A": (2048, 5632, 16, 28, 512), "1b-B": (1792, 4864, 14, 36, 512), "1b-C": (2304, 6144, 18, 20, 512),
    "1b-D": (2048, 8192, 16, 20, 512), "1b-E": (2048, 5632, 16, 28, 256),
    "1.5b-A": (2304, 6144, 18, 32, 512), "1.5b-B": (2048, 5632, 16, 40, 512), "1.5b-C": (2560, 6912, 20, 24, 512),
    "1.5b-D": (2304, 9216, 18, 22, 512), "1.5b-E": (2304, 6144, 18, 32, 256),
    "3b-A": (2560, 6912, 20, 40, 512), "3b-B": (2304, 6144, 18, 48, 512), "3b-C": (3072, 8192, 24, 28, 512),
    "3b-D": (2560, 10240, 20, 28, 512), "3b-E": (2560, 6912, 20, 40, 256),
    "5b-A": (3072, 8192, 24, 44, 512), "5b-B": (2560, 6912, 20, 60, 512), "5b-C": (3584, 9600, 28, 32, 512),
    "5b-D": (3072, 12288, 24, 32, 512), "5b-E": (3072, 8192, 24, 44, 256),
    "7b": (4096, 11008, 32, 32, 512), "10b": (4096, 11008, 32, 48, 512),
}


def sweep_config(name: str) -> ModelConfig:
    """custom_config (bench_param_sweep.rs:17-29): MHA, hd 128, vocab 8192."""
    dim, hidden, heads, nl, seq = SWEEP[name]
    return ModelConfig.custom(dim, hidden, heads, nl, seq=seq, vocab=8192)


def sweep_tokens(cfg: ModelConfig, batch: int) -> tuple[np.ndarray, np.ndarray]:
    """bench_param_sweep.rs:75-76, repeated for each sequence of the batch."""
    i = np.arange(cfg.seq + 1, dtype=np.int64)
    ids = ((i * 31 + 7) % cfg.vocab).astype(np.uint32)
    return np.tile(ids[:-1], batch), np.tile(ids[1:], batch)


def run_sweep(cfg: ModelConfig, name: str, batch: int = 1, device: int = 0, out=print) -> br.BenchResult:
    params_m = cfg.param_count() / 1e6
    out("\n" + "=" * 60)
    out(f"  {name} — {cfg.dim}d/{cfg.hidden}h/{cfg.nlayers}L/seq{cfg.seq} — ~{params_m:.0f}M params — "
        f"h/d={cfg.hidden / cfg.dim:.2f}x")
    out("=" * 60)

    t0 = time.perf_counter()
    k = CompiledKernels.compile(cfg, max_batch=batch, device=device)
    out(f"  [1/4] Creating the B200 context... {time.perf_counter() - t0:.1f}s")

    tc = TrainConfig()
    k.upload_weights(random_weights(cfg))
    tok, tgt = sweep_tokens(cfg, batch)
    loss0 = k.forward(tok, tgt, tc.softcap)
    if not np.isfinite(loss0):
        raise RuntimeError(f"initial loss is not finite: {loss0}")
    out(f"  [2/4] Forward pass... loss={loss0:.4f}")

    losses = [loss0]
    for step in range(10):
        losses.append(k.train_step(tok, tgt, step, tc))
    final = k.forward(tok, tgt, tc.softcap)
    losses.append(final)
    delta = float(np.float32(final) - np.float32(loss0))
    out(f"  [3/4] Training 10 steps... {loss0:.4f} → {final:.4f} (delta={delta:+.4f})")

    step_ms, fwd_ms, bwd_ms, upd_ms = [], [], [], []
    for step in range(10, 15):
        t = time.perf_counter()
        k.train_step(tok, tgt, step, tc)
        step_ms.append((time.perf_counter() - t) * 1e3)
        tm = k.timings()
        fwd_ms.append(tm["fwd_ms"])
        bwd_ms.append(tm["bwd_ms"])
        upd_ms.append(tm["opt_ms"])
    med = [sorted(v)[2] for v in (step_ms, fwd_ms, bwd_ms, upd_ms)]
    med = [float(np.float32(x)) for x in med]  # f32 fields
    tok_per_s = float(np.float32(batch * cfg.seq) * np.float32(1000.0) / np.float32(med[0]))
    out(f"  [4/4] Timing 5 steps... {med[0]:.0f}ms/step (fwd={med[1]:.0f} bwd={med[2]:.0f} upd={med[3]:.0f}) "
        f"= {tok_per_s:.0f} tok/s")
    all_finite = all(np.isfinite(losses))
    if not all_finite:
        out("  WARNING: NaN/Inf detected!")
    k.close()

    res = br.BenchResult(
        schema_version=br.SCHEMA_VERSION, rustane_version=br.RUSTANE_VERSION, git_sha=br.git_sha(),
        benchmark="sweep_" + name.lower().replace("-", "_") + (f"_b{batch}" if batch != 1 else ""),
        config=br.ModelInfo(name=name, dim=cfg.dim, hidden=cfg.hidden, heads=cfg.heads, nlayers=cfg.nlayers,
                            seq=cfg.seq, params_m=params_m),
        results=br.TimingResults(ms_per_step=med[0], ms_fwd=med[1], ms_bwd=med[2], ms_upd=med[3],
                                 tok_per_s=tok_per_s, loss_start=loss0, loss_end=final, loss_delta=delta),
        loss_trace=[float(x) for x in losses], hardware=br.collect_hardware_info(),
        timestamp_utc=br.utc_timestamp())
    res.fingerprint = br.compute_fingerprint(res)
    return res


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("config", choices=sorted(SWEEP))
    ap.add_argument("--batch", type=int, default=1, help="sequences per step (1 = the reference's protocol)")
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--out", default="target/bench-result.json")
    a = ap.parse_args(argv)
    res = run_sweep(sweep_config(a.config), a.config, a.batch, a.device, out=lambda s: print(s, flush=True))
    br.write_result(res, a.out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
