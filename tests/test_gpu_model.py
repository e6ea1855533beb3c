"""Model-level parity: librustane_cuda.so (bf16 compute, fp32 accumulate / master
weights) against the CPU fp32 oracle of the reference engine, through the
engine API mirror (C ABI underneath).

Tolerances: loss within 2e-3 absolute; logits and
gradients within 2e-2 max relative error, measured normwise per tensor as
max|gpu - oracle| / max|oracle|; token / index handling bit-exact.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pyoracle as po  # noqa: E402
from rustane_b200 import CompiledKernels, ModelConfig, TrainConfig, full_model  # noqa: E402
from rustane_b200._lib import RT_ERR_TOKEN, RustaneError  # noqa: E402
from rustane_b200.tensors import ModelOptState, ModelTensors  # noqa: E402

pytestmark = pytest.mark.gpu

LOSS_TOL = 2e-3
REL_TOL = 2e-2
SMALL = ModelConfig.custom(256, 512, 2, 2, seq=128, vocab=512)


def nrel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def seeded(cfg, batch, seed=1000):
    rng = np.random.default_rng(seed)
    n = batch * cfg.seq
    return rng.integers(0, cfg.vocab, n).astype(np.uint32), rng.integers(0, cfg.vocab, n).astype(np.uint32)


def grads_close(g_gpu: ModelTensors, g_ref: ModelTensors, tol=REL_TOL):
    worst = {}
    for (name, a), (_, b) in zip(g_gpu.tensors(), g_ref.tensors()):
        if np.max(np.abs(b)) == 0:
            assert np.max(np.abs(a)) == 0, name
            continue
        worst[name] = nrel(a, b)
    bad = {k: v for k, v in worst.items() if v > tol}
    assert not bad, bad
    return worst


@pytest.mark.parametrize("cfg,batch", [(SMALL, 2), (ModelConfig.gpt_karpathy(), 1)], ids=["small-b2", "tiny-b1"])
def test_forward_backward_parity(cfg, batch):
    w = ModelTensors.normal(cfg, seed=1234, std=0.02)
    tok, tgt = seeded(cfg, batch)
    o = po.Oracle(cfg, batch)
    loss_ref, logits_ref, tl_ref = o.forward(w, tok, tgt, want_logits=True, want_token_losses=True)
    g_ref = ModelTensors.zeros(cfg)
    o.backward(w, tok, g_ref, loss_scale=256.0)

    k = CompiledKernels.compile(cfg, max_batch=batch)
    loss = full_model.forward(cfg, k, w, tok, tgt, 0.0)
    assert abs(loss - loss_ref) < LOSS_TOL
    assert nrel(k.logits(), logits_ref) < REL_TOL
    ptl = full_model.forward_losses(cfg, k, w, tok, tgt, 0.0)
    assert np.max(np.abs(ptl - tl_ref)) < 2e-2
    k.grads_zero()
    g = ModelTensors.zeros(cfg)
    full_model.backward(cfg, k, w, tok, 0.0, 256.0, g)
    grads_close(g, g_ref)


def test_softcap_parity():
    cfg = SMALL
    w = ModelTensors.normal(cfg, seed=7, std=0.05)
    tok, tgt = seeded(cfg, 1, seed=3)
    o = po.Oracle(cfg, 1)
    loss_ref, logits_ref, _ = o.forward(w, tok, tgt, softcap=2.0, want_logits=True)
    g_ref = ModelTensors.zeros(cfg)
    o.backward(w, tok, g_ref, softcap=2.0, loss_scale=1.0)
    k = CompiledKernels.compile(cfg, max_batch=1)
    loss = full_model.forward(cfg, k, w, tok, tgt, 2.0)
    assert abs(loss - loss_ref) < LOSS_TOL
    assert nrel(k.logits(), logits_ref) < REL_TOL
    g = ModelTensors.zeros(cfg)
    full_model.backward(cfg, k, w, tok, 2.0, 1.0, g)
    grads_close(g, g_ref)


def test_train_step_parity_and_trajectory():
    """train_step (full_model.rs:661-714) for 4 steps: per-step loss and the cumulative update.

    AdamW moves each weight by lr * m_hat / sqrt(v_hat): every entry is divided by
    its own gradient RMS, so entries whose gradient is near zero carry a relative
    error far above the tensor-level 2e-2 gradient bound (they can even step the
    other way).  The cumulative update is therefore compared in L2 per tensor:
    ||dW_gpu - dW_ref|| / ||dW_ref|| < 0.15, with the gradients themselves held
    to the 2e-2 bound."""
    cfg = SMALL
    batch = 2
    w0 = ModelTensors.normal(cfg, seed=11, std=0.02)
    w_ref = w0.copy()
    tc = TrainConfig(warmup_steps=2, total_steps=10)
    otc = po.default_train_config(warmup_steps=2, total_steps=10)
    o = po.Oracle(cfg, batch)
    g_ref, opt_ref = ModelTensors.zeros(cfg), ModelOptState.zeros(cfg)
    k = CompiledKernels.compile(cfg, max_batch=batch)
    k.upload_weights(w0.copy())
    for step in range(4):
        tok, tgt = seeded(cfg, batch, seed=50 + step)
        loss_ref, _ = o.train_step(w_ref, g_ref, opt_ref, tok, tgt, step, otc)
        loss = k.train_step(tok, tgt, step, tc)
        assert abs(loss - loss_ref) < LOSS_TOL, (step, loss, loss_ref)
    w_gpu = k.download_weights()
    for (name, a), (_, b), (_, a0) in zip(w_gpu.tensors(), w_ref.tensors(), w0.tensors()):
        d_gpu, d_ref = a.astype(np.float64) - a0, b.astype(np.float64) - a0
        assert np.linalg.norm(d_gpu - d_ref) <= 0.15 * np.linalg.norm(d_ref), name
    grads_close(k.download_grads(), g_ref)


def test_update_weights_matches_oracle():
    """update_weights (full_model.rs:490-593) on identical uploaded gradients: lr groups and wd."""
    cfg = SMALL
    w = ModelTensors.normal(cfg, seed=2, std=0.02)
    g = ModelTensors.normal(cfg, seed=3, std=1.0)
    opt = ModelOptState(ModelTensors.normal(cfg, seed=4, std=0.01), ModelTensors.normal(cfg, seed=5, std=0.01))
    for _, a in opt.v.tensors():
        np.abs(a, out=a)
    tc = TrainConfig()
    k = CompiledKernels.compile(cfg, max_batch=1)
    k.upload_weights(w)
    k.upload_grads(g)
    k.upload_opt(opt)
    w_ref, opt_ref = w.copy(), ModelOptState(opt.m.copy(), opt.v.copy())
    po.Oracle(cfg, 1).update_weights(w_ref, g, opt_ref, 7, 3e-4, po.default_train_config(), 0.125)
    full_model.update_weights(cfg, k, None, None, None, 7, 3e-4, tc, 0.125)
    w_out, opt_out = k.download_weights(), k.download_opt()
    for (n, a), (_, b) in zip(w_out.tensors(), w_ref.tensors()):
        assert nrel(a, b) < 1e-5, n
    for (n, a), (_, b) in zip(opt_out.m.tensors(), opt_ref.m.tensors()):
        assert nrel(a, b) < 1e-5, n
    for (n, a), (_, b) in zip(opt_out.v.tensors(), opt_ref.v.tensors()):
        assert nrel(a, b) < 1e-5, n


def test_grad_norm_and_clip():
    cfg = SMALL
    w = ModelTensors.normal(cfg, seed=8, std=0.02)
    tok, tgt = seeded(cfg, 1, seed=9)
    o = po.Oracle(cfg, 1)
    o.forward(w, tok, tgt)
    g_ref = ModelTensors.zeros(cfg)
    o.backward(w, tok, g_ref, loss_scale=256.0)
    k = CompiledKernels.compile(cfg, max_batch=1)
    full_model.forward(cfg, k, w, tok, tgt)
    k.grads_zero()
    k.backward(0.0, 256.0)
    n_ref = o.grad_norm(g_ref)
    n = full_model.grad_norm(k)
    assert abs(n - n_ref) / n_ref < REL_TOL
    full_model.clip_grads(k, 0.5 * n)
    assert abs(full_model.grad_norm(k) - 0.5 * n) / n < 1e-5


def test_published_init_loss_600m_full_depth():
    """600m-A, the reference init and tokens: 9.0108 (README.md:58)."""
    cfg = ModelConfig.target_600m()
    w = full_model.random_weights(cfg)
    tok, tgt = po.pattern_tokens(cfg)
    k = CompiledKernels.compile(cfg, max_batch=1)
    loss = full_model.forward(cfg, k, w, tok, tgt)
    assert abs(loss - 9.0108) < LOSS_TOL


@pytest.mark.parametrize("forward_only", [False, True], ids=["train-ctx", "forward-only-ctx"])
def test_published_init_loss_7b_width(forward_only):
    """7B forward, the reference init and tokens: 9.3228 (README.md:70).  Wo = W2 = 0 make
    every layer an identity map at this init, so one layer at the 7B width gives the
    32-layer loss; the forward-only context is the one the 7B bench line runs (bf16 weights)."""
    cfg = ModelConfig.custom(4096, 11008, 32, 1)
    w = full_model.random_weights(cfg)
    tok, tgt = po.pattern_tokens(cfg)
    k = CompiledKernels.compile(cfg, max_batch=1, forward_only=forward_only)
    try:
        loss = full_model.forward(cfg, k, w, tok, tgt)
    finally:
        k.close()
    assert abs(loss - 9.3228) < LOSS_TOL, loss


def test_exact_zero_grads_at_reference_init():
    """phase4_pretraining_checks.rs:30-76 on the GPU path (gpt_karpathy)."""
    cfg = ModelConfig.gpt_karpathy()
    w = full_model.random_weights(cfg)
    i = np.arange(cfg.seq + 1)
    tok, tgt = (i[:-1] % cfg.vocab).astype(np.uint32), (i[1:] % cfg.vocab).astype(np.uint32)
    k = CompiledKernels.compile(cfg, max_batch=1)
    full_model.forward(cfg, k, w, tok, tgt)
    k.grads_zero()
    g = ModelTensors.zeros(cfg)
    full_model.backward(cfg, k, None, tok, 0.0, 1.0, g)
    assert np.abs(g.embed).sum() > 0 and np.abs(g.gamma_final).sum() > 0
    for Lg in g.layers:
        for f in ("wq", "wk", "wv", "w1", "w3", "gamma1", "gamma2"):
            assert not np.any(getattr(Lg, f)), f
        assert np.abs(Lg.wo).sum() > 0 and np.abs(Lg.w2).sum() > 0


def test_deterministic_bitwise():
    cfg = SMALL
    w = ModelTensors.normal(cfg, seed=12, std=0.02)
    tok, tgt = seeded(cfg, 2, seed=13)
    k = CompiledKernels.compile(cfg, max_batch=2)
    outs = []
    for _ in range(2):
        loss = full_model.forward(cfg, k, w, tok, tgt)
        k.grads_zero()
        k.backward(0.0, 256.0)
        outs.append((loss, k.download_grads()))
    assert outs[0][0] == outs[1][0]
    for (n, a), (_, b) in zip(outs[0][1].tensors(), outs[1][1].tensors()):
        assert np.array_equal(a, b), n


def test_batch_equals_accumulated_microbatches():
    """One pass over B sequences == B accumulated single-sequence passes (full_model.rs:680-694)."""
    cfg = SMALL
    w = ModelTensors.normal(cfg, seed=14, std=0.02)
    tok, tgt = seeded(cfg, 2, seed=15)
    k = CompiledKernels.compile(cfg, max_batch=2)
    k.upload_weights(w)
    lb = k.forward(tok, tgt)
    k.grads_zero()
    k.backward(0.0, 1.0)
    gb = k.download_grads()
    k.grads_zero()
    ls = []
    for b in range(2):
        sl = slice(b * cfg.seq, (b + 1) * cfg.seq)
        ls.append(k.forward(tok[sl], tgt[sl]))
        k.backward(0.0, 1.0)
    ga = k.download_grads()
    assert abs(lb - np.mean(ls)) < 1e-5
    grads_close(ga, gb, tol=1e-4)


def test_bad_token_is_rejected():
    cfg = SMALL
    k = CompiledKernels.compile(cfg, max_batch=1)
    k.upload_weights(ModelTensors.normal(cfg, seed=1))
    tok, tgt = seeded(cfg, 1)
    tok[7] = cfg.vocab
    with pytest.raises(RustaneError) as e:
        k.forward(tok, tgt)
    assert e.value.code == RT_ERR_TOKEN


def test_backward_before_forward_is_state_error():
    cfg = SMALL
    k = CompiledKernels.compile(cfg, max_batch=1)
    with pytest.raises(RustaneError):
        k.backward(0.0, 1.0)


def test_timings_query_leaves_no_cuda_error():
    """rt_get_timings on a single-GPU context must not leave a CUDA error behind
    (the all-reduce phase events are never recorded there)."""
    cfg = SMALL
    k = CompiledKernels.compile(cfg, max_batch=1)
    k.upload_weights(ModelTensors.normal(cfg, seed=1))
    tok, tgt = seeded(cfg, 1)
    k.train_step(tok, tgt, 0, TrainConfig())
    t = k.timings()
    assert t["fwd_ms"] > 0 and t["bwd_ms"] > 0 and t["comm_ms"] == 0
    k.train_step(tok, tgt, 1, TrainConfig())  # the next launch must still succeed


def test_forward_only_context_matches_training_context():
    """RT_CTX_FORWARD_ONLY (bf16 weights, reused activations) gives the same loss bits as a
    training context, for host-uploaded and for seeded device-initialised weights."""
    cfg = SMALL
    w = ModelTensors.normal(cfg, seed=21, std=0.02)
    tok, tgt = seeded(cfg, 2, seed=22)
    kt = CompiledKernels.compile(cfg, max_batch=2)
    kf = CompiledKernels.compile(cfg, max_batch=2, forward_only=True)
    assert kf.device_bytes() < kt.device_bytes()
    assert full_model.forward(cfg, kt, w, tok, tgt) == full_model.forward(cfg, kf, w, tok, tgt)
    kt.init_normal(seed=5, std=0.02)
    kf.init_normal(seed=5, std=0.02)
    a, pa = kt.forward(tok, tgt, per_token=True)
    b, pb = kf.forward(tok, tgt, per_token=True)
    assert a == b and np.array_equal(pa, pb)
