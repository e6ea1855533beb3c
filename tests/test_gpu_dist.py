"""Data-parallel train step on 2 GPUs through the C ABI (rt_dist_init + NCCL
inside rt_train_step: gradients reduce-scattered, AdamW sharded, weights
all-gathered): two ranks with one sequence each must match one GPU stepping on
both sequences -- losses, gradients, weights and the AdamW moments (downloaded
whole, which gathers the shards).  Skipped on boxes with fewer than 2 GPUs.

The two runs sum the same per-token terms in a different order (each rank's
GEMMs see half the tokens, then the all-reduce adds the halves), so the
all-reduced gradients agree to rounding.  AdamW's first steps move every
weight by about lr * sign(g) whatever |g| is, so a gradient element that is
zero up to rounding can move a weight by up to 2 lr in opposite directions:
weights are therefore compared by their update as a whole (relative L2), and
the gradients element-wise."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

pytestmark = pytest.mark.gpu

CFG = dict(dim=256, hidden=512, heads=2, nlayers=2, seq=128, vocab=512)


def _cfg():
    from rustane_b200.model import ModelConfig
    return ModelConfig.custom(CFG["dim"], CFG["hidden"], CFG["heads"], CFG["nlayers"], seq=CFG["seq"],
                              vocab=CFG["vocab"])


def _data():
    rng = np.random.default_rng(31)
    n = 2 * CFG["seq"]
    return rng.integers(0, CFG["vocab"], n).astype(np.uint32), rng.integers(0, CFG["vocab"], n).astype(np.uint32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root)]
    from rustane_b200 import CompiledKernels, TrainConfig
    from rustane_b200.tensors import ModelTensors
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _cfg()
        k = CompiledKernels.compile(cfg, max_batch=1, device=rank)
        k.upload_weights(ModelTensors.normal(cfg, seed=3, std=0.02))
        uid = [CompiledKernels.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        k.dist_init(world, rank, uid[0], timeout_ms=60000)
        from rustane_b200 import RustaneError, _lib
        try:  # one communicator per context: a second join is refused before any NCCL call
            k.dist_init(world, rank, uid[0], timeout_ms=60000)
            raise AssertionError("a second rt_dist_init was accepted")
        except RustaneError as e:
            assert e.code == _lib.RT_ERR_STATE, e
        tok, tgt = _data()
        S = cfg.seq
        tc = TrainConfig(warmup_steps=2, total_steps=10)
        losses = [k.train_step(tok[rank * S:(rank + 1) * S], tgt[rank * S:(rank + 1) * S], 0, tc)]
        g = k.download_grads()  # all-reduced gradients of step 0
        losses.append(k.train_step(tok[rank * S:(rank + 1) * S], tgt[rank * S:(rank + 1) * S], 1, tc))
        w = k.download_weights()
        opt = k.download_opt()  # the sharded AdamW moments, gathered
        if rank == 0:
            np.savez(out, losses=np.array(losses), **{n: a for n, a in w.tensors()},
                     **{"grad_" + n: a for n, a in g.tensors()}, **{"m_" + n: a for n, a in opt.m.tensors()},
                     **{"v_" + n: a for n, a in opt.v.tensors()})
        else:
            np.save(out + ".rank1_losses.npy", np.array(losses))
        k.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dp2_matches_single_gpu(tmp_path):
    from rustane_b200 import CompiledKernels, TrainConfig
    from rustane_b200.tensors import ModelTensors
    out = str(tmp_path / "dp.npz")
    mp.spawn(_rank, args=(2, _free_port(), out), nprocs=2, join=True)
    got = np.load(out)
    cfg = _cfg()
    k = CompiledKernels.compile(cfg, max_batch=2, device=0)
    k.upload_weights(ModelTensors.normal(cfg, seed=3, std=0.02))
    tok, tgt = _data()
    tc = TrainConfig(warmup_steps=2, total_steps=10)
    losses = [k.train_step(tok, tgt, 0, tc)]
    g = k.download_grads()
    losses.append(k.train_step(tok, tgt, 1, tc))
    w = k.download_weights()
    opt = k.download_opt()
    # rt_train_step returns this rank's loss; their mean is the loss over both sequences
    both = 0.5 * (got["losses"] + np.load(out + ".rank1_losses.npy"))
    np.testing.assert_allclose(both, losses, rtol=1e-5, atol=1e-6)
    for name, a in g.tensors():
        b = got["grad_" + name]
        assert np.max(np.abs(a - b)) <= 1e-4 * max(np.max(np.abs(a)), 1e-6) + 1e-9, name
    w0 = ModelTensors.normal(cfg, seed=3, std=0.02)
    for (name, a), (_, a0) in zip(w.tensors(), w0.tensors()):
        u1, u2 = a - a0, got[name] - a0
        assert np.linalg.norm(u1 - u2) <= 0.05 * np.linalg.norm(u1) + 1e-7, name
    for pre, t in (("m_", opt.m), ("v_", opt.v)):  # moments of the scaled gradients: same bound
        for name, a in t.tensors():
            b = got[pre + name]
            assert np.linalg.norm(a - b) <= 0.05 * np.linalg.norm(a) + 1e-12, pre + name
