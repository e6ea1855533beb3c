"""Data-parallel step semantics on CPU ranks (gloo, world size 2).

The library's data-parallel train step has two forms (rt_train_step):

* all-reduce: the gradients of all ranks are summed with one all-reduce before
  grad-norm and AdamW, and the AdamW gradient scale divides by
  world * batch * loss_scale;
* sharded optimizer (the default when every segment splits into 16-byte chunks):
  the gradient arena is cut into segments (the embedding, each layer's seven
  matrices, all gammas), each segment is reduce-scattered so that rank r holds
  the summed chunk r, the grad norm is the square root of the ranks' float64
  sums of squares of their chunks (all-reduced), every rank runs AdamW on its
  chunks only (its moments stay sharded) and all-gathers the updated weights.

Here two gloo ranks run the oracle on one sequence each and apply each protocol;
the result must equal one process doing the reference train_step over both
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


# ----------------------------------------------------------- sharded optimizer
STEPS = 2  # two steps: the second reads the sharded moments back (t = 2 bias correction)
CLIPS = (1e6, 1e-3)  # step 0 takes the plain scale, step 1 the clip branch (full_model.rs:696-704)


def _segments(t):
    """The runtime's data-parallel segments in arena order, each one AdamW group:
    (arrays, kind) with kind 0 = embedding, 2 = matrices, 1 = gammas (the
    oracle's for_each_tensor kinds)."""
    segs = [([t.embed], 0)]
    segs += [([L.wq, L.wk, L.wv, L.wo, L.w1, L.w3, L.w2], 2) for L in t.layers]
    segs.append(([a for L in t.layers for a in (L.gamma1, L.gamma2)] + [t.gamma_final], 1))
    return segs


def _scatter_back(flat, arrays):
    off = 0
    for a in arrays:
        a.reshape(-1)[...] = flat[off:off + a.size]
        off += a.size


def _sharded_worker(rank: int, world: int, port: int, out_path: str) -> None:
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "oracle")]
    import pyoracle as po
    from rustane_b200.model import ModelConfig
    from rustane_b200.tensors import ModelTensors

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ModelConfig.custom(CFG_ARGS["dim"], CFG_ARGS["hidden"], CFG_ARGS["heads"], CFG_ARGS["nlayers"],
                                 seq=CFG_ARGS["seq"], vocab=CFG_ARGS["vocab"])
        L = po.lib(threads=1)
        w = ModelTensors.normal(cfg, seed=5, std=0.05)
        tok, tgt = _sharded_data()
        S = cfg.seq
        o = po.Oracle(cfg, 1)
        nseg = len(_segments(w))
        lens = [sum(a.size for a in arrs) for arrs, _ in _segments(w)]
        assert all(n % (4 * world) == 0 for n in lens)  # the condition for the sharded form
        m_own = [np.zeros(n // world, np.float32) for n in lens]  # moments: this rank's chunks only
        v_own = [np.zeros(n // world, np.float32) for n in lens]
        losses = []
        for step in range(STEPS):
            tc = po.default_train_config(warmup_steps=2, total_steps=10, grad_clip=CLIPS[step])
            seq = step * world + rank
            mine = slice(seq * S, (seq + 1) * S)
            g = ModelTensors.zeros(cfg)
            loss, _, _ = o.forward(w, np.ascontiguousarray(tok[mine]), np.ascontiguousarray(tgt[mine]))
            o.backward(w, np.ascontiguousarray(tok[mine]), g, loss_scale=tc.loss_scale)
            lt = torch.tensor([loss], dtype=torch.float64)
            dist.all_reduce(lt)
            losses.append(lt.item() / world)
            # reduce-scatter each gradient segment: rank r keeps the summed chunk r
            g_own = []
            for arrs, _ in _segments(g):
                flat = torch.from_numpy(np.concatenate([a.reshape(-1) for a in arrs]))
                chunk = torch.empty(flat.numel() // world)
                dist.reduce_scatter_tensor(chunk, flat)
                g_own.append(chunk.numpy())
            # grad norm: float64 sums of squares of the own chunks, summed over the ranks
            ss = torch.tensor([sum(float(np.sum(c.astype(np.float64) ** 2)) for c in g_own)], dtype=torch.float64)
            dist.all_reduce(ss)
            raw = np.float32(np.sqrt(ss.item()))
            gsc = np.float32(1.0) / (np.float32(1) * np.float32(world) * np.float32(tc.loss_scale))
            combined = np.float32(tc.grad_clip) / raw if raw * gsc > np.float32(tc.grad_clip) else gsc
            lr = np.float32(po.learning_rate(step, tc))
            w_segs = _segments(w)
            for i in range(nseg):
                arrs, kind = w_segs[i]
                flat = np.concatenate([a.reshape(-1) for a in arrs])
                n = flat.size // world
                p_own = np.ascontiguousarray(flat[rank * n:(rank + 1) * n])
                tlr = lr * np.float32(tc.embed_lr_scale if kind == 0 else tc.matrix_lr_scale if kind == 2 else 1.0)
                wd = tc.weight_decay if kind == 2 else 0.0
                L.or_adam_step_fused(po.fp(p_own), po.fp(g_own[i]), po.fp(m_own[i]), po.fp(v_own[i]), n, step + 1,
                                     float(tlr), tc.beta1, tc.beta2, tc.eps, wd, float(combined))
                full = torch.empty(flat.size)
                dist.all_gather_into_tensor(full, torch.from_numpy(p_own))
                _scatter_back(full.numpy(), arrs)
        # gather the sharded moments for the comparison
        mv = {}
        for name, own in (("m", m_own), ("v", v_own)):
            for i, c in enumerate(own):
                full = torch.empty(c.size * world)
                dist.all_gather_into_tensor(full, torch.from_numpy(c))
                mv[f"{name}{i}"] = full.numpy()
        if rank == 0:
            np.savez(out_path, losses=np.array(losses), **{n: a for n, a in w.tensors()}, **mv)
    finally:
        dist.destroy_process_group()


def _sharded_data():
    rng = np.random.default_rng(78)
    n = STEPS * 2 * CFG_ARGS["seq"]
    return rng.integers(0, CFG_ARGS["vocab"], n).astype(np.uint32), rng.integers(0, CFG_ARGS["vocab"], n).astype(np.uint32)


def test_sharded_optimizer_step_equals_single_process(tmp_path):
    import pyoracle as po
    from rustane_b200.model import ModelConfig
    from rustane_b200.tensors import ModelOptState, ModelTensors

    out = str(tmp_path / "rank0.npz")
    mp.spawn(_sharded_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    got = np.load(out)

    cfg = ModelConfig.custom(CFG_ARGS["dim"], CFG_ARGS["hidden"], CFG_ARGS["heads"], CFG_ARGS["nlayers"],
                             seq=CFG_ARGS["seq"], vocab=CFG_ARGS["vocab"])
    w = ModelTensors.normal(cfg, seed=5, std=0.05)
    g, opt = ModelTensors.zeros(cfg), ModelOptState.zeros(cfg)
    tok, tgt = _sharded_data()
    S = cfg.seq
    o = po.Oracle(cfg, 2)
    clipped = []
    for step in range(STEPS):
        tc = po.default_train_config(warmup_steps=2, total_steps=10, grad_clip=CLIPS[step])
        part = slice(step * 2 * S, (step + 1) * 2 * S)
        loss, raw = o.train_step(w, g, opt, tok[part].copy(), tgt[part].copy(), step, tc)
        clipped.append(raw / (2 * tc.loss_scale) > tc.grad_clip)
        assert abs(float(got["losses"][step]) - loss) < 1e-5, step
    assert clipped == [False, True]  # both branches of the combined scale ran
    for name, a in w.tensors():
        np.testing.assert_allclose(got[name], a, rtol=0, atol=2e-6, err_msg=name)
    for name, st in (("m", opt.m), ("v", opt.v)):
        for i, (arrs, _) in enumerate(_segments(st)):
            ref = np.concatenate([x.reshape(-1) for x in arrs])
            np.testing.assert_allclose(got[f"{name}{i}"], ref, rtol=1e-4, atol=1e-12, err_msg=f"{name} segment {i}")
