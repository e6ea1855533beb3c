"""One process, two devices: a context on each GPU runs a train step.

Kernels with more than 48 KB of dynamic shared memory need their limit raised
on every device that launches them (the attribute belongs to the device that
is current when it is set).  This test creates contexts on devices 0 and 1 in
the same process, runs the train step on both (the first launch of every
GEMM, attention and RMSNorm kernel happens on device 0, then on device 1) and
checks that both give the same loss and gradients bit for bit.  Skipped with
fewer than two GPUs.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from rustane_b200 import CompiledKernels, ModelConfig, TrainConfig  # noqa: E402
from rustane_b200.tensors import ModelTensors  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def test_contexts_on_two_devices_in_one_process():
    cfg = ModelConfig.custom(1536, 4096, 12, 1, seq=512, vocab=8192)  # >48 KB kernels at the 600M widths
    w = ModelTensors.normal(cfg, seed=31, std=0.02)
    rng = np.random.default_rng(32)
    tok = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    results = []
    for dev in (0, 1):
        k = CompiledKernels.compile(cfg, max_batch=2, device=dev)
        k.upload_weights(w)
        loss = k.train_step(tok, tgt, 0, TrainConfig())
        results.append((loss, k.download_grads()))
        k.close()
    assert results[0][0] == results[1][0]
    for (n, a), (_, b) in zip(results[0][1].tensors(), results[1][1].tensors()):
        assert np.array_equal(a, b), n
