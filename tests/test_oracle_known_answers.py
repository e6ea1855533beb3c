"""Pin the CPU oracle to the reference's own known answers (no GPU).

Sources: the reference's CPU unit tests (crates/engine/src/cpu/*.rs #[cfg(test)]),
its pre-training checks (crates/engine/tests/phase4_pretraining_checks.rs:30-76)
and its published initial losses (tests/golden/published_losses.json, extracted
from results/2026-03-18_1830_param-sweep.md and README.md by
tests/golden/extract_published.py).
"""
import json
from pathlib import Path

import numpy as np
import pytest

import pyoracle as po
from rustane_b200.model import ModelConfig
from rustane_b200.tensors import ModelTensors

GOLDEN = Path(__file__).resolve().parent / "golden"
L = po.lib()


def f32(*v):
    return np.array(v, dtype=np.float32)


# ---------------------------------------------------------------- RMSNorm
def test_rmsnorm_forward_unit_gamma():  # cpu/rmsnorm.rs:245-257
    x, g, out = f32(3, 4), f32(1, 1), np.zeros(2, np.float32)
    ri = L.or_rmsnorm_forward(po.fp(x), po.fp(g), po.fp(out), 2)
    r = np.sqrt(np.float32(12.5) + np.float32(1e-5))
    assert abs(ri - 1 / r) < 1e-5
    assert abs(out[0] - 3 / r) < 1e-5 and abs(out[1] - 4 / r) < 1e-5


def test_rmsnorm_forward_with_gamma():  # cpu/rmsnorm.rs:259-273
    x, g, out = f32(1, 2, 3, 4), f32(.5, .5, .5, .5), np.zeros(4, np.float32)
    ri = L.or_rmsnorm_forward(po.fp(x), po.fp(g), po.fp(out), 4)
    e = 1 / np.sqrt(7.5 + 1e-5)
    assert abs(ri - e) < 1e-5
    assert np.all(np.abs(out - x * e * 0.5) < 1e-5)


def test_rmsnorm_backward_numerical_gradient():  # cpu/rmsnorm.rs:275-314
    x, g, dy = f32(1, -2, 3, -0.5), f32(1, .5, 2, 1.5), f32(1, 1, 1, 1)
    out = np.zeros(4, np.float32)
    ri = L.or_rmsnorm_forward(po.fp(x), po.fp(g), po.fp(out), 4)
    dx, dg = np.zeros(4, np.float32), np.zeros(4, np.float32)
    L.or_rmsnorm_backward(po.fp(dy), po.fp(x), po.fp(g), ri, po.fp(dx), po.fp(dg), 4)
    eps = 1e-4
    for i in range(4):
        xp, xm = x.copy(), x.copy()
        xp[i] += eps
        xm[i] -= eps
        op, om = np.zeros(4, np.float32), np.zeros(4, np.float32)
        L.or_rmsnorm_forward(po.fp(xp), po.fp(g), po.fp(op), 4)
        L.or_rmsnorm_forward(po.fp(xm), po.fp(g), po.fp(om), 4)
        num = (op.sum() - om.sum()) / (2 * eps)
        assert abs(dx[i] - num) < 1e-2


def test_rmsnorm_channel_first_matches_per_position():  # cpu/rmsnorm.rs:316-407
    dim, seq = 4, 3
    g = f32(1.5, .5, 2, .8)
    rng = np.random.default_rng(0)
    x_cf = rng.standard_normal((dim, seq)).astype(np.float32)
    out_cf, ri = np.zeros_like(x_cf), np.zeros(seq, np.float32)
    L.or_rmsnorm_forward_cf(po.fp(x_cf), po.fp(g), po.fp(out_cf), po.fp(ri), dim, seq)
    dy = rng.standard_normal((dim, seq)).astype(np.float32)
    dx_cf, dg_cf = np.zeros_like(x_cf), np.zeros(dim, np.float32)
    L.or_rmsnorm_backward_cf(po.fp(dy), po.fp(x_cf), po.fp(g), po.fp(ri), po.fp(dx_cf), po.fp(dg_cf), dim, seq)
    dg_ref = np.zeros(dim, np.float32)
    for s in range(seq):
        xs = np.ascontiguousarray(x_cf[:, s])
        o = np.zeros(dim, np.float32)
        r = L.or_rmsnorm_forward(po.fp(xs), po.fp(g), po.fp(o), dim)
        assert abs(r - ri[s]) < 1e-6
        assert np.allclose(o, out_cf[:, s], atol=1e-5)
        dys = np.ascontiguousarray(dy[:, s])
        dxs = np.zeros(dim, np.float32)
        L.or_rmsnorm_backward(po.fp(dys), po.fp(xs), po.fp(g), r, po.fp(dxs), po.fp(dg_ref), dim)
        assert np.allclose(dxs, dx_cf[:, s], atol=1e-5)
    assert np.allclose(dg_ref, dg_cf, atol=1e-5)


# ---------------------------------------------------------- cross-entropy
def _ce(logits, t):
    ls = np.zeros_like(logits)
    return L.or_ce_forward(po.fp(logits), logits.size, t, po.fp(ls)), ls


def test_ce_loss_positive_and_confidence():  # cpu/cross_entropy.rs:103-121
    loss, _ = _ce(f32(1, 2, 3, 4), 3)
    assert 0 < loss < 2
    lo, _ = _ce(f32(1, 1, 1, 1), 3)
    hi, _ = _ce(f32(0, 0, 0, 10), 3)
    assert hi < lo


def test_ce_gradients_sum_to_zero():  # cpu/cross_entropy.rs:123-131
    _, ls = _ce(f32(1, 2, 3), 1)
    d = np.zeros(3, np.float32)
    L.or_ce_backward(po.fp(ls), 3, 1, po.fp(d))
    assert abs(d.sum()) < 1e-5


def test_ce_numerical_gradient():  # cpu/cross_entropy.rs:133-153
    logits, t = f32(2, -1, .5, 1.5), 2
    _, ls = _ce(logits, t)
    d = np.zeros(4, np.float32)
    L.or_ce_backward(po.fp(ls), 4, t, po.fp(d))
    for i in range(4):
        p, m = logits.copy(), logits.copy()
        p[i] += 1e-4
        m[i] -= 1e-4
        num = (_ce(p, t)[0] - _ce(m, t)[0]) / 2e-4
        assert abs(d[i] - num) < 5e-3


def test_ce_batch_matches_single():  # cpu/cross_entropy.rs:58-96
    rng = np.random.default_rng(1)
    S, V = 5, 37
    logits = rng.standard_normal((S, V)).astype(np.float32)
    tg = rng.integers(0, V, S).astype(np.uint32)
    dl = np.zeros_like(logits)
    tot = L.or_ce_forward_backward_batch(po.fp(logits), po.up(tg), S, V, po.fp(dl), 1.0 / S)
    ref = 0.0
    for s in range(S):
        row = np.ascontiguousarray(logits[s])
        l, ls = _ce(row, int(tg[s]))
        ref += l
        d = np.zeros(V, np.float32)
        L.or_ce_backward(po.fp(ls), V, int(tg[s]), po.fp(d))
        assert np.allclose(dl[s], d / S, atol=1e-6)
    assert abs(tot - ref) < 1e-4


# ------------------------------------------------------------------- Adam
def test_adam_momentum_accumulates():  # cpu/adam.rs:170-182
    p, g, m, v = f32(0, 0), f32(1, 1), f32(0, 0), f32(0, 0)
    L.or_adam_step(po.fp(p), po.fp(g), po.fp(m), po.fp(v), 2, 1, 1e-3, 0.9, 0.999, 1e-8, 0.0)
    assert abs(m[0] - 0.1) < 1e-6 and abs(v[0] - 0.001) < 1e-6


def test_adam_moves_toward_minimum_and_decay():  # cpu/adam.rs:139-168
    p, g, m, v = f32(5, 5, 5, 5), f32(1, 1, 1, 1), np.zeros(4, np.float32), np.zeros(4, np.float32)
    s0 = p.sum()
    for t in range(1, 11):
        L.or_adam_step(po.fp(p), po.fp(g), po.fp(m), po.fp(v), 4, t, 1e-3, 0.9, 0.999, 1e-8, 0.01)
    assert p.sum() < s0
    p, g, m, v = f32(1, 1), f32(0, 0), f32(0, 0), f32(0, 0)
    L.or_adam_step(po.fp(p), po.fp(g), po.fp(m), po.fp(v), 2, 1, 1e-3, 0.9, 0.999, 1e-8, 0.1)
    assert p[0] < 1.0


def test_adam_fused_matches_unfused():  # tests/auto_cpu_fused_adam.rs:34-122 (1e-5)
    rng = np.random.default_rng(2)
    n = 4099
    p0 = rng.standard_normal(n).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    a = [p0.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)]
    b = [p0.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)]
    for t in range(1, 6):
        L.or_adam_step(po.fp(a[0]), po.fp(g), po.fp(a[1]), po.fp(a[2]), n, t, 3e-4, 0.9, 0.95, 1e-8, 0.1)
        L.or_adam_step_fused(po.fp(b[0]), po.fp(g), po.fp(b[1]), po.fp(b[2]), n, t, 3e-4, 0.9, 0.95, 1e-8, 0.1,
                             1.0)
    for x, y in zip(a, b):
        assert np.max(np.abs(x - y)) < 1e-5


# -------------------------------------------------------------- embedding
def test_embedding_lookup_and_scatter():  # cpu/embedding.rs:51-94
    table = f32(1, 2, 3, 4, 5, 6)
    ids = np.array([2, 0, 1], np.uint32)
    out = np.zeros(6, np.float32)
    L.or_embedding_forward(po.fp(table), 2, po.up(ids), 3, po.fp(out))
    assert out.tolist() == [5, 6, 1, 2, 3, 4]
    d_out = f32(.1, .2, .3, .4, .5, .6)
    ids = np.array([1, 1, 2], np.uint32)
    dt = np.zeros(6, np.float32)
    L.or_embedding_backward(po.fp(d_out), 2, po.up(ids), 3, po.fp(dt))
    assert dt[0] == 0 and dt[1] == 0
    assert abs(dt[2] - .4) < 1e-6 and abs(dt[3] - .6) < 1e-6
    assert abs(dt[4] - .5) < 1e-6 and abs(dt[5] - .6) < 1e-6
    # channel-first scatter equals the row-major one on the transposed input
    d_cf = np.ascontiguousarray(d_out.reshape(3, 2).T)
    dt2 = np.zeros(6, np.float32)
    L.or_embedding_backward_cf(po.fp(d_cf), 2, po.up(ids), 3, po.fp(dt2))
    assert np.array_equal(dt, dt2)


# ------------------------------------------------------------------- SiLU
def test_silu_zero_and_numerical_gradient():  # cpu/silu.rs:53-94
    x = f32(0.0)
    o = np.zeros(1, np.float32)
    L.or_silu_forward(po.fp(x), po.fp(o), 1)
    assert abs(o[0]) < 1e-6
    x = f32(-2, -0.5, 0, 0.5, 2)
    dy = np.ones(5, np.float32)
    dx = np.zeros(5, np.float32)
    L.or_silu_backward(po.fp(dy), po.fp(x), po.fp(dx), 5)
    for i in range(5):
        p, m = x.copy(), x.copy()
        p[i] += 1e-3
        m[i] -= 1e-3
        op, om = np.zeros(5, np.float32), np.zeros(5, np.float32)
        L.or_silu_forward(po.fp(p), po.fp(op), 5)
        L.or_silu_forward(po.fp(m), po.fp(om), 5)
        assert abs(dx[i] - (op[i] - om[i]) / 2e-3) < 1e-3


# --------------------------------------------------------- learning rate
def test_learning_rate_schedule():  # full_model.rs:334-342
    tc = po.default_train_config()
    assert abs(po.learning_rate(0, tc) - 3e-6) < 1e-9
    assert abs(po.learning_rate(99, tc) - 3e-4) < 1e-9
    assert abs(po.learning_rate(100, tc) - 3e-4) < 1e-9
    assert abs(po.learning_rate(10000, tc) - 3e-5) < 1e-9
    mid = 100 + (10000 - 100) // 2
    assert abs(po.learning_rate(mid, tc) - (3e-5 + 0.5 * (3e-4 - 3e-5))) < 1e-7


# ----------------------------------------------------------- LCG init
def test_lcg_random_vec_first_values():  # layer.rs:404-413
    v = po.random_vec(4, 1.0)
    seed = 42 + 4
    exp = []
    for _ in range(4):
        seed = (seed * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        exp.append(np.float32(np.float32(seed >> 32) / np.float32(4294967295.0)) * np.float32(2) - np.float32(1))
    assert np.array_equal(v, np.array(exp, np.float32))


# ------------------------------------------------ published init losses
def _published():
    rows = json.loads((GOLDEN / "published_losses.json").read_text())
    seen, out = set(), []
    for r in rows:
        key = (r["dim"], r["seq"], r["decimals"])
        if key not in seen:
            seen.add(key)
            out.append(r)
    return out


@pytest.mark.parametrize("row", _published(), ids=lambda r: f"{r['name']}-d{r['dim']}-s{r['seq']}")
def test_published_init_loss(row):
    """Reference init (wo = w2 = 0 makes every layer an identity map, so one layer suffices)."""
    cfg = ModelConfig.custom(row["dim"], row["hidden"], row["heads"], 1, seq=row["seq"])
    w = po.reference_init(cfg)
    tok, tgt = po.pattern_tokens(cfg)
    loss, _, _ = po.Oracle(cfg, 1).forward(w, tok, tgt)
    assert abs(round(loss, row["decimals"]) - row["loss0"]) < 0.6 * 10 ** -row["decimals"], (loss, row)


def test_layers_are_identity_at_reference_init():
    base = ModelConfig.custom(256, 512, 2, 1, seq=64, vocab=512)
    losses = []
    for nl in (1, 3):
        cfg = base.with_(nlayers=nl)
        tok, tgt = po.pattern_tokens(cfg)
        losses.append(po.Oracle(cfg, 1).forward(po.reference_init(cfg), tok, tgt)[0])
    assert losses[0] == losses[1]


def test_published_600m_full_depth():
    """600m-A at all 20 layers: 9.0108 (README.md:58)."""
    cfg = ModelConfig.target_600m()
    tok, tgt = po.pattern_tokens(cfg)
    loss, _, _ = po.Oracle(cfg, 1).forward(po.reference_init(cfg), tok, tgt)
    assert abs(loss - 9.0108) < 6e-5


# ----------------------------------------------- pre-training checks
def test_exact_zero_grads_at_reference_init():
    """phase4_pretraining_checks.rs:30-76: with wo = w2 = 0, dWq/dWk/dWv/dW1/dW3 are exactly 0;
    dWo, dW2, dembed and dgamma_final are non-zero.  (dgamma1/dgamma2 are also exactly 0
    in exact arithmetic: their upstream gradients pass through wo / w2 = 0.)"""
    cfg = ModelConfig.gpt_karpathy()
    w = po.reference_init(cfg)
    i = np.arange(cfg.seq + 1)
    tok = (i[:-1] % cfg.vocab).astype(np.uint32)
    tgt = (i[1:] % cfg.vocab).astype(np.uint32)
    o = po.Oracle(cfg, 1)
    o.forward(w, tok, tgt)
    g = ModelTensors.zeros(cfg)
    o.backward(w, tok, g, loss_scale=1.0)
    assert np.abs(g.embed).sum() > 0 and np.abs(g.gamma_final).sum() > 0
    for Lg in g.layers:
        for f in ("wq", "wk", "wv", "w1", "w3", "gamma1", "gamma2"):
            assert not np.any(getattr(Lg, f)), f
        assert np.abs(Lg.wo).sum() > 0 and np.abs(Lg.w2).sum() > 0


def test_loss_scale_linearity():
    """phase4_pretraining_checks.rs:142-210: gradients scale linearly with loss_scale."""
    cfg = ModelConfig.custom(128, 256, 1, 2, seq=32, vocab=96)
    w = ModelTensors.normal(cfg, seed=5, std=0.05)
    rng = np.random.default_rng(3)
    tok = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
    o = po.Oracle(cfg, 1)
    o.forward(w, tok, tgt)
    g1, g256 = ModelTensors.zeros(cfg), ModelTensors.zeros(cfg)
    o.backward(w, tok, g1, loss_scale=1.0)
    o.backward(w, tok, g256, loss_scale=256.0)
    for (_, a), (_, b) in zip(g1.tensors(), g256.tensors()):
        assert np.allclose(a * 256.0, b, rtol=1e-4, atol=1e-9)
