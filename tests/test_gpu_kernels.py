"""Kernel-level parity on the GPU through the C ABI (rt_kernel_*).

Memory-bound kernels are checked against the CPU oracle (oracle/oracle.cpp);
index work (embedding gather / scatter) must be bit-exact; the attention
kernels are checked against a plain torch fp32 causal attention of the same
bf16 values (the oracle's attention is exercised by the model-level tests).
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pyoracle as po  # noqa: E402
from rustane_b200 import _lib  # noqa: E402

pytestmark = pytest.mark.gpu
L = _lib.lib()


def stream():
    return torch.cuda.current_stream().cuda_stream


def rel(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def ok(rc):
    torch.cuda.synchronize()
    assert rc == 0, rc


# -------------------------------------------------------------- embedding
def test_embed_gather_bit_exact_and_bad_token():
    V, D, M = 512, 256, 300
    g = torch.Generator().manual_seed(0)
    E = torch.randn(V, D, generator=g).cuda()
    tok = torch.randint(0, V, (M,), generator=g, dtype=torch.int64).to(torch.int32).cuda()
    x = torch.empty(M, D, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ok(L.rt_kernel_embed_gather(E.data_ptr(), tok.data_ptr(), x.data_ptr(), M, D, V, err.data_ptr(), stream()))
    assert err.item() == 0
    assert torch.equal(x, E[tok.long()])
    tok[5] = V + 3
    ok(L.rt_kernel_embed_gather(E.data_ptr(), tok.data_ptr(), x.data_ptr(), M, D, V, err.data_ptr(), stream()))
    assert err.item() == 4  # bad-token device code; row zeroed
    assert torch.count_nonzero(x[5]).item() == 0


def _segments(tok: np.ndarray):
    order = np.argsort(tok, kind="stable").astype(np.int32)
    uniq, starts = np.unique(tok[order], return_index=True)
    seg_start = np.append(starts, tok.size).astype(np.int32)
    return order, seg_start, uniq.astype(np.uint32)


def test_embed_scatter_bit_exact():  # cpu/embedding.rs:34-44 order: ascending positions
    V, D, M = 300, 128, 512
    rng = np.random.default_rng(1)
    tok = rng.integers(0, 40, M).astype(np.uint32)  # many repeats
    dx = rng.standard_normal((M, D)).astype(np.float32)
    dE0 = rng.standard_normal((V, D)).astype(np.float32)
    perm, seg_start, seg_tok = _segments(tok)
    exp = dE0.copy()
    for s in range(M):
        exp[tok[s]] = exp[tok[s]] + dx[s]
    t = {k: torch.from_numpy(v).cuda() for k, v in dict(dx=dx, dE=dE0.copy(), perm=perm, ss=seg_start,
                                                         st=seg_tok.view(np.int32)).items()}
    ok(L.rt_kernel_embed_scatter(t["dx"].data_ptr(), t["perm"].data_ptr(), t["ss"].data_ptr(), t["st"].data_ptr(),
                                 seg_tok.size, t["dE"].data_ptr(), D, stream()))
    assert np.array_equal(t["dE"].cpu().numpy(), exp)


# --------------------------------------------------------------- RMSNorm
# Backward: D a multiple of 256 up to 2048 takes the pipelined kernel (dgamma partials
# in the same pass), other widths the row + column-partial kernels.  Forward: D a
# multiple of 128 from 768 to 2560 keeps the row in registers, other widths re-read
# it (256, 1000).  M = 101 leaves a partial last block of rows.
@pytest.mark.parametrize("M", [96, 101])
@pytest.mark.parametrize("D", [256, 768, 1000, 1280, 1536, 2048, 2560])
def test_rmsnorm_fwd_bwd_vs_oracle(D, M):
    rng = np.random.default_rng(D)
    x = rng.standard_normal((M, D)).astype(np.float32)
    g = (1 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    dy = rng.standard_normal((M, D)).astype(np.float32)
    resid = rng.standard_normal((M, D)).astype(np.float32)
    # oracle, channel-first (cpu/rmsnorm.rs:149-238)
    xc = np.ascontiguousarray(x.T)
    oc, ri = np.zeros_like(xc), np.zeros(M, np.float32)
    po.lib().or_rmsnorm_forward_cf(po.fp(xc), po.fp(g), po.fp(oc), po.fp(ri), D, M)
    dyc = np.ascontiguousarray(dy.T)
    dxc, dgo = np.zeros_like(xc), np.ones(D, np.float32)
    po.lib().or_rmsnorm_backward_cf(po.fp(dyc), po.fp(xc), po.fp(g), po.fp(ri), po.fp(dxc), po.fp(dgo), D, M)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    tx, tg, tdy, tres = T(x), T(g), T(dy), T(resid)
    out = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    rms = torch.empty(M, device="cuda")
    ok(L.rt_kernel_rmsnorm_fwd(tx.data_ptr(), tg.data_ptr(), out.data_ptr(), rms.data_ptr(), M, D, stream()))
    assert rel(rms, ri) < 1e-6
    assert rel(out.float(), oc.T) < 8e-3
    dx = torch.empty(M, D, device="cuda")
    dxb = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    dgam = torch.ones(D, device="cuda")
    part = torch.empty(L.rt_kernel_rmsnorm_bwd_partials(M) * D, device="cuda")
    ok(L.rt_kernel_rmsnorm_bwd(tdy.data_ptr(), tx.data_ptr(), tg.data_ptr(), rms.data_ptr(), tres.data_ptr(),
                               dx.data_ptr(), dxb.data_ptr(), ctypes.c_float(0.5), dgam.data_ptr(), 1,
                               part.data_ptr(), M, D, stream()))
    assert rel(dx, dxc.T + resid) < 1e-5
    assert rel(dxb.float(), 0.5 * (dxc.T + resid)) < 8e-3
    assert rel(dgam, dgo) < 1e-5


# --------------------------------------------------------- cross-entropy
@pytest.mark.parametrize("softcap", [0.0, 15.0])
def test_cross_entropy_vs_oracle(softcap):
    M, V = 64, 8192
    rng = np.random.default_rng(3)
    logits = (3 * rng.standard_normal((M, V))).astype(np.float32)
    tgt = rng.integers(0, V, M).astype(np.uint32)
    z = logits if softcap == 0 else (softcap * np.tanh(logits / softcap)).astype(np.float32)
    dl_ref = np.zeros_like(z)
    tot = po.lib().or_ce_forward_backward_batch(po.fp(np.ascontiguousarray(z)), po.up(tgt), M, V, po.fp(dl_ref),
                                                1.0 / 512)
    tl = torch.from_numpy(logits).cuda()
    tt = torch.from_numpy(tgt.view(np.int32)).cuda()
    loss = torch.empty(M, device="cuda")
    lse = torch.empty(M, device="cuda")
    ok(L.rt_kernel_ce_fwd(tl.data_ptr(), tt.data_ptr(), loss.data_ptr(), lse.data_ptr(), M, V,
                          ctypes.c_float(softcap), stream()))
    assert abs(loss.sum().item() - tot) < 1e-4 * M
    dl = torch.empty(M, V, device="cuda", dtype=torch.bfloat16)
    scale = 256.0 / 512
    ok(L.rt_kernel_ce_bwd(tl.data_ptr(), lse.data_ptr(), tt.data_ptr(), dl.data_ptr(), M, V, ctypes.c_float(softcap),
                          ctypes.c_float(scale), stream()))
    exp = dl_ref * 256.0
    if softcap:
        exp = exp * (1 - np.tanh(logits / softcap) ** 2)
    assert rel(dl.float(), exp) < 8e-3


# ------------------------------------------------------------------ Adam
def test_adam_vs_oracle_step_fused():  # cpu/adam.rs:95-132
    n = 1 << 16
    rng = np.random.default_rng(4)
    p = rng.standard_normal(n).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    m = (0.1 * rng.standard_normal(n)).astype(np.float32)
    v = np.abs(0.01 * rng.standard_normal(n)).astype(np.float32)
    ref = [p.copy(), m.copy(), v.copy()]
    po.lib().or_adam_step_fused(po.fp(ref[0]), po.fp(g), po.fp(ref[1]), po.fp(ref[2]), n, 3, 1.5e-5, 0.9, 0.95,
                                1e-8, 0.1, 0.25)
    T = [torch.from_numpy(a.copy()).cuda() for a in (p, g, m, v)]
    pb = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    ok(L.rt_kernel_adam(T[0].data_ptr(), T[1].data_ptr(), T[2].data_ptr(), T[3].data_ptr(), pb.data_ptr(), n, 3,
                        ctypes.c_float(1.5e-5), ctypes.c_float(0.9), ctypes.c_float(0.95), ctypes.c_float(1e-8),
                        ctypes.c_float(0.1), ctypes.c_float(0.25), stream()))
    assert rel(T[0], ref[0]) < 1e-6
    assert rel(T[2], ref[1]) < 1e-6
    assert rel(T[3], ref[2]) < 1e-6
    assert torch.equal(pb, T[0].bfloat16())


def test_l2norm_deterministic():
    n = 10_000_003
    x = torch.randn(n, device="cuda")
    part = torch.empty(1024, device="cuda")
    out = torch.empty(2, device="cuda")
    ok(L.rt_kernel_l2norm(x.data_ptr(), n, part.data_ptr(), out.data_ptr(), stream()))
    first = out[0].item()
    ok(L.rt_kernel_l2norm(x.data_ptr(), n, part.data_ptr(), out[1:].data_ptr(), stream()))
    assert out[1].item() == first
    assert abs(first - x.double().norm().item()) / first < 1e-6


# ------------------------------------------------------------- attention
def _attn_ref(qkv, B, S, H):
    D = H * 128
    x = qkv.float().view(B, S, 3, H, 128)
    q, k, v = (x[:, :, i].permute(0, 2, 1, 3) for i in range(3))  # [B, H, S, 128]
    s = q @ k.transpose(-1, -2) / np.sqrt(128.0)
    mask = torch.ones(S, S, device=s.device, dtype=torch.bool).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    o = torch.softmax(s, -1) @ v
    lse = torch.logsumexp(s, -1)
    return o.permute(0, 2, 1, 3).reshape(B * S, D), lse


# amp = 6 makes the row max grow by more than 2^8 between key blocks, which the
# tcgen05 forward handles by rescaling the TMEM accumulator
@pytest.mark.parametrize("amp", [1.0, 6.0])
@pytest.mark.parametrize("B,S,H", [(2, 256, 2), (1, 512, 3), (3, 384, 1)])
def test_attention_forward(B, S, H, amp):
    D = H * 128
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = (amp * torch.randn(B * S, 3 * D, generator=g, device="cuda")).bfloat16()
    out = torch.empty(B * S, D, device="cuda", dtype=torch.bfloat16)
    lse2 = torch.empty(B, H, S, device="cuda")
    ok(L.rt_kernel_attention_fwd(qkv.data_ptr(), out.data_ptr(), lse2.data_ptr(), B, S, H, stream()))
    o_ref, lse = _attn_ref(qkv, B, S, H)
    assert rel(out.float(), o_ref) < 1e-2
    assert (lse2 - lse / np.log(2.0)).abs().max().item() < 2e-3


def _attn_bwd(impl, qkv, out, lse2, dout, tcb, tsb, B, S, H):
    D = H * 128
    dvec = torch.empty(B, H, S, device="cuda")
    dqkv = torch.full((B * S, 3 * D), float("nan"), device="cuda", dtype=torch.bfloat16)
    if impl == "tc":
        nbytes = L.rt_kernel_attention_bwd_scratch_bytes(B, S, H)
        assert nbytes == B * H * S * S * 2
        ds = torch.empty(nbytes // 2, device="cuda", dtype=torch.bfloat16)
        ok(L.rt_kernel_attention_bwd_tc(qkv.data_ptr(), out.data_ptr(), lse2.data_ptr(), dout.data_ptr(),
                                        dvec.data_ptr(), ds.data_ptr(), dqkv.data_ptr(), tcb.data_ptr(),
                                        tsb.data_ptr(), B, S, H, stream()))
    else:
        ok(L.rt_kernel_attention_bwd(qkv.data_ptr(), out.data_ptr(), lse2.data_ptr(), dout.data_ptr(),
                                     dvec.data_ptr(), dqkv.data_ptr(), tcb.data_ptr(), tsb.data_ptr(), B, S, H,
                                     stream()))
    torch.cuda.synchronize()
    return dqkv


# "tc": tcgen05 / TMEM kernels (the model step's path); "mma": the mma.sync kernels (noalloc entry).
# S = 128 is one key block (diagonal sub-blocks only); 384 and 1024 make ragged causal work per CTA;
# amp = 2 gives larger logits (sharper P).
@pytest.mark.parametrize("impl", ["tc", "mma"])
@pytest.mark.parametrize("B,S,H,amp", [(2, 256, 2, 1.0), (1, 512, 3, 1.0), (1, 128, 2, 1.0), (3, 384, 1, 1.0),
                                       (1, 1024, 2, 1.0), (1, 512, 2, 2.0)])
def test_attention_backward_with_rope(impl, B, S, H, amp):
    from rustane_b200.model import ModelConfig
    D = H * 128
    cfg = ModelConfig.custom(D, 256, H, 1, seq=S, vocab=256)
    _, _, cb, sb = po.Oracle(cfg, 1).rope_tables()
    g = torch.Generator(device="cuda").manual_seed(6)
    qkv = (amp * torch.randn(B * S, 3 * D, generator=g, device="cuda")).bfloat16()
    dout = torch.randn(B * S, D, generator=g, device="cuda").bfloat16()
    out = torch.empty(B * S, D, device="cuda", dtype=torch.bfloat16)
    lse2 = torch.empty(B, H, S, device="cuda")
    ok(L.rt_kernel_attention_fwd(qkv.data_ptr(), out.data_ptr(), lse2.data_ptr(), B, S, H, stream()))
    tcb, tsb = torch.from_numpy(cb).cuda(), torch.from_numpy(sb).cuda()
    dqkv = _attn_bwd(impl, qkv, out, lse2, dout, tcb, tsb, B, S, H)
    if impl == "tc":  # fixed summation order: bitwise repeatable
        assert torch.equal(_attn_bwd(impl, qkv, out, lse2, dout, tcb, tsb, B, S, H), dqkv)
    x = qkv.float().requires_grad_(True)
    o_ref, _ = _attn_ref(x, B, S, H)
    o_ref.backward(dout.float())
    gr = x.grad.view(B, S, 3, H, 128)
    pos = torch.arange(S, device="cuda")
    c = tcb.t()[pos].view(1, S, 1, 64)  # [S, 64] pair tables
    s = tsb.t()[pos].view(1, S, 1, 64)
    exp = gr.clone()
    for i in (0, 1):  # RoPE backward on dQ, dK (layer.rs:1880-1897)
        d0, d1 = gr[:, :, i, :, 0::2], gr[:, :, i, :, 1::2]
        exp[:, :, i, :, 0::2] = c * d0 + s * d1
        exp[:, :, i, :, 1::2] = -s * d0 + c * d1
    got = dqkv.float().view(B, S, 3, H, 128)
    for i, name in enumerate(("dq", "dk", "dv")):
        assert rel(got[:, :, i], exp[:, :, i]) < 2e-2, name
