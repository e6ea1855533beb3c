"""A data-parallel rank that leaves: the survivor's next step fails cleanly.

Two ranks (child processes, one GPU each, NVLS off, no multicast anywhere in
the library) run one data-parallel rt_train_step together.  Both wait until
nothing is in flight (rt_join + rt_sync), meet at a host barrier, and rank 1
then destroys its context and exits -- between steps, with none of its kernels
or collectives running.  Rank 0's next rt_train_step reaches a reduce-scatter
that no peer will join; the library's bounded wait (timeout_ms) aborts the
communicator and the call returns RT_ERR_NCCL instead of hanging, after which
rt_ctx_destroy succeeds.  The reference has no multi-process path; its failures
panic through `.expect()` (layer.rs:243-259), which the Rust binding restores
from the status code.  Skipped with fewer than two GPUs.
"""
import ctypes
import os
import socket
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

TIMEOUT_MS = 3000


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from rustane_b200 import CompiledKernels, ModelConfig, RustaneError, TrainConfig, _lib
    from rustane_b200.tensors import ModelTensors
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ModelConfig.custom(256, 512, 2, 2, seq=128, vocab=512)
        k = CompiledKernels.compile(cfg, max_batch=1, device=rank)
        k.upload_weights(ModelTensors.normal(cfg, seed=3, std=0.02))
        uid = [CompiledKernels.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        k.dist_init(world, rank, uid[0], timeout_ms=TIMEOUT_MS)
        rng = np.random.default_rng(40 + rank)
        tok = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
        tgt = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
        tc = TrainConfig(warmup_steps=2, total_steps=10)
        k.train_step(tok, tgt, 0, tc)
        L = _lib.lib()
        k._check(L.rt_join(k.handle))  # the step's weight all-gathers too
        k._check(L.rt_sync(k.handle, None))
        dist.barrier()  # both ranks are between steps, nothing in flight
        if rank == 1:
            k.close()
            return
        time.sleep(1.0)  # rank 1 is gone
        t0 = time.perf_counter()
        code = None
        try:
            k.train_step(tok, tgt, 1, tc)
        except RustaneError as e:
            code = e.code
        elapsed = time.perf_counter() - t0
        rc_destroy = L.rt_ctx_destroy(k._h)
        k._h = None
        np.savez(out, code=code if code is not None else 0, elapsed=elapsed, rc_destroy=rc_destroy)
    finally:
        if rank == 0:
            dist.destroy_process_group()


def test_survivor_gets_nccl_error_and_tears_down(tmp_path):
    from rustane_b200 import _lib
    out = str(tmp_path / "rank0.npz")
    mp.spawn(_rank, args=(2, _free_port(), out), nprocs=2, join=True)
    got = np.load(out)
    assert int(got["code"]) == _lib.RT_ERR_NCCL
    assert float(got["elapsed"]) < TIMEOUT_MS / 1000 + 30
    assert int(got["rc_destroy"]) == _lib.RT_OK
    assert ctypes.c_int(int(got["rc_destroy"])).value == 0
