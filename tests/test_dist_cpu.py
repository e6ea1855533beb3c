"""Data-parallel step semantics on CPU ranks (gloo, world size 2).

The library's data-parallel train step sums the gradients of all ranks with one
all-reduce before grad-norm and AdamW, and divides by world * batch * loss_scale
in the AdamW gradient scale (rt_train_step).  Here two gloo ranks run the oracle
on one sequence each, all-reduce their gradients, and apply that rule; the
result must equal one process doing the reference train_step over both
sequences (full_model.rs:661-714 with accum_steps = 2).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

CFG_ARGS = dict(dim=128, hidden=256, heads=1, nlayers=2, seq=32, vocab=96)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    rng = np.random.default_rng(77)
    n = 2 * CFG_ARGS["seq"]
    return rng.integers(0, CFG_ARGS["vocab"], n).astype(np.uint32), rng.integers(0, CFG_ARGS["vocab"], n).astype(np.uint32)


def _worker(rank: int, world: int, port: int, out_path: str) -> None:
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "oracle")]
    import pyoracle as po
    from rustane_b200.model import ModelConfig
    from rustane_b200.tensors import ModelOptState, ModelTensors

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ModelConfig.custom(CFG_ARGS["dim"], CFG_ARGS["hidden"], CFG_ARGS["heads"], CFG_ARGS["nlayers"],
                                 seq=CFG_ARGS["seq"], vocab=CFG_ARGS["vocab"])
        po.lib(threads=1)
        w = ModelTensors.normal(cfg, seed=5, std=0.05)
        tok, tgt = _data()
        S = cfg.seq
        mine = slice(rank * S, (rank + 1) * S)
        tc = po.default_train_config(warmup_steps=2, total_steps=10)
        o = po.Oracle(cfg, 1)
        loss, _, _ = o.forward(w, np.ascontiguousarray(tok[mine]), np.ascontiguousarray(tgt[mine]))
        g = ModelTensors.zeros(cfg)
        o.backward(w, np.ascontiguousarray(tok[mine]), g, loss_scale=tc.loss_scale)
        for _, a in g.tensors():  # the exchange step: one sum all-reduce of the gradients
            t = torch.from_numpy(a)
            dist.all_reduce(t)
        lt = torch.tensor([loss], dtype=torch.float64)
        dist.all_reduce(lt)
        gsc = 1.0 / (world * 1 * tc.loss_scale)
        raw = o.grad_norm(g)
        combined = tc.grad_clip / raw if raw * gsc > tc.grad_clip else gsc
        opt = ModelOptState.zeros(cfg)
        o.update_weights(w, g, opt, 1, po.learning_rate(0, tc), tc, combined)
        if rank == 0:
            np.savez(out_path, loss=lt.item() / world, **{n: a for n, a in w.tensors()})
    finally:
        dist.destroy_process_group()


def test_data_parallel_step_equals_single_process(tmp_path):
    import pyoracle as po
    from rustane_b200.model import ModelConfig
    from rustane_b200.tensors import ModelOptState, ModelTensors

    out = str(tmp_path / "rank0.npz")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    got = np.load(out)

    cfg = ModelConfig.custom(CFG_ARGS["dim"], CFG_ARGS["hidden"], CFG_ARGS["heads"], CFG_ARGS["nlayers"],
                             seq=CFG_ARGS["seq"], vocab=CFG_ARGS["vocab"])
    w = ModelTensors.normal(cfg, seed=5, std=0.05)
    tok, tgt = _data()
    tc = po.default_train_config(warmup_steps=2, total_steps=10)
    loss, _ = po.Oracle(cfg, 2).train_step(w, ModelTensors.zeros(cfg), ModelOptState.zeros(cfg), tok, tgt, 0, tc)
    assert abs(float(got["loss"]) - loss) < 1e-5
    for name, a in w.tensors():
        np.testing.assert_allclose(got[name], a, rtol=0, atol=1e-6, err_msg=name)
