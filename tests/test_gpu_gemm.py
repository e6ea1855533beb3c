"""tcgen05 GEMM parity on the GPU against a plain torch fp32 matmul.

Covers every operand-major combination (K-major / MN-major for A and B), the
single-CTA kernel at each tile width and the CTA-pair kernel (force_bn -256 /
-128: two SMs of a cluster own a 256-row tile), ring wrap-around (K > stages * 64), persistent CTAs with more tiles
than SMs (TMEM double buffer), ragged M/N edges, and each fused epilogue the LM
step uses.  Inputs are bf16; the reference multiplies the same bf16 values in
fp32, so only accumulation order differs (tolerance 1e-4 normwise).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from rustane_b200 import _lib  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30)).item()


def rope_tables(seq, hd=128):
    # crates/engine/src/kernels/sdpa_fwd.rs:18-33, f32 arithmetic
    p = np.arange(seq, dtype=np.float32)[:, None]
    i = np.arange(hd // 2, dtype=np.float32)[None, :]
    theta = p / np.power(np.float32(10000.0), np.float32(2.0) * i / np.float32(hd))
    return np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)


def gemm(A, a_mn, B, b_mn, M, N, K, epi, out, out2=None, aux=None, alpha=1.0, beta=0, rope=None, seq=0,
         rope_cols=0, n_half=0, force_bn=0):
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    cos_p = rope[0].data_ptr() if rope is not None else None
    sin_p = rope[1].data_ptr() if rope is not None else None
    rc = _lib.lib().rt_kernel_gemm(
        A.data_ptr(), A.stride(0), int(a_mn), B.data_ptr(), B.stride(0), int(b_mn), M, N, K, epi,
        out.data_ptr(), out.stride(0), out2.data_ptr() if out2 is not None else None,
        out2.stride(0) if out2 is not None else 0, aux.data_ptr() if aux is not None else None,
        aux.stride(0) if aux is not None else 0, alpha, beta, cos_p, sin_p, seq, rope_cols, n_half, force_bn,
        err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, rc
    assert err.item() == 0, err.item()


def operands(M, N, K, a_mn, b_mn, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn((K, M) if a_mn else (M, K), generator=g, device="cuda").bfloat16()
    B = torch.randn((K, N) if b_mn else (N, K), generator=g, device="cuda").bfloat16()
    A_log = A.t() if a_mn else A
    B_log = B.t() if b_mn else B
    ref = A_log.float() @ B_log.float().t()
    return A, B, ref


@pytest.fixture(autouse=True)
def _no_tf32():
    torch.backends.cuda.matmul.allow_tf32 = False


PAIR = [-256, -128]
PAIR192 = -192  # 96 B rows per CTA: K-major B only


def _skip_pair192(bn, b_mn):
    if bn == PAIR192 and b_mn:
        pytest.skip("the 192-wide CTA pair takes K-major B only")


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("bn", [128, 192, 256] + PAIR + [PAIR192])
def test_gemm_majors_f32(a_mn, b_mn, bn):
    _skip_pair192(bn, b_mn)
    M, N, K = 256, 576, 640  # K > stages x stage depth: the shared-memory ring wraps; N ragged for 192 / 256
    A, B, ref = operands(M, N, K, a_mn, b_mn)
    out = torch.empty(M, N, device="cuda")
    gemm(A, a_mn, B, b_mn, M, N, K, _lib.EPI_F32, out, force_bn=bn)
    assert _rel(out, ref) < TOL


@pytest.mark.parametrize("bn", [128, 256] + PAIR)
def test_gemm_persistent_many_tiles(bn):
    # more tiles than SMs: every CTA cycles both TMEM accumulators several times
    M, N, K = 2048, 4096, 256
    A, B, ref = operands(M, N, K, False, True, seed=1)
    out = torch.empty(M, N, device="cuda")
    gemm(A, False, B, True, M, N, K, _lib.EPI_F32, out, force_bn=bn)
    assert _rel(out, ref) < TOL


@pytest.mark.parametrize("bn", [0] + PAIR + [PAIR192])
@pytest.mark.parametrize("M", [200, 328])
def test_gemm_ragged_edges(bn, M):
    # M not a multiple of the tile height and N not a multiple of the tile width;
    # rows past M must stay untouched
    N, K = 352, 256
    A, B, ref = operands(M, N, K, False, False, seed=2)
    out = torch.full((M + 8, N), 7.0, device="cuda")
    gemm(A, False, B, False, M, N, K, _lib.EPI_F32, out, force_bn=bn)
    assert _rel(out[:M], ref) < TOL
    assert bool((out[M:] == 7.0).all())


@pytest.mark.parametrize("bn", [0] + PAIR)
def test_gemm_bf16_out(bn):
    M, N, K = 384, 768, 512
    A, B, ref = operands(M, N, K, False, True, seed=3)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    gemm(A, False, B, True, M, N, K, _lib.EPI_BF16, out, force_bn=bn)
    assert _rel(out, ref) < 8e-3


@pytest.mark.parametrize("bn", [0] + PAIR)
@pytest.mark.parametrize("beta", [0, 1])
def test_gemm_f32_accumulate(beta, bn):
    M, N, K = 256, 384, 1024
    A, B, ref = operands(M, N, K, True, True, seed=4)
    out = torch.randn(M, N, device="cuda")
    base = out.clone()
    gemm(A, True, B, True, M, N, K, _lib.EPI_F32_ACC, out, beta=beta, force_bn=bn)
    expect = ref + base if beta else ref
    assert _rel(out, expect) < TOL


@pytest.mark.parametrize("bn", [0] + PAIR + [PAIR192])
@pytest.mark.parametrize("b_mn", [True, False])
def test_gemm_residual(b_mn, bn):
    _skip_pair192(bn, b_mn)
    M, N, K = 512, 768, 768
    A, B, ref = operands(M, N, K, False, b_mn, seed=5)
    resid = torch.randn(M, N, device="cuda")
    out = torch.empty(M, N, device="cuda")
    alpha = 0.1581
    gemm(A, False, B, b_mn, M, N, K, _lib.EPI_RESIDUAL, out, aux=resid, alpha=alpha, force_bn=bn)
    assert _rel(out, resid + alpha * ref) < TOL


@pytest.mark.parametrize("bn", [0] + PAIR)
def test_gemm_rope_qkv(bn):
    seq, D, B = 256, 256, 2
    M, N, K = B * seq, 3 * D, 256
    A, Bw, ref = operands(M, N, K, False, True, seed=6)
    cos, sin = rope_tables(seq)
    rope = (torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda())
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    gemm(A, False, Bw, True, M, N, K, _lib.EPI_ROPE, out, rope=rope, seq=seq, rope_cols=2 * D, force_bn=bn)
    exp = ref.clone()
    pos = torch.arange(M, device="cuda") % seq
    c = rope[0][pos].repeat(1, 2 * D // 128)  # [M, D] pairs
    s = rope[1][pos].repeat(1, 2 * D // 128)
    x0 = ref[:, 0:2 * D:2]
    x1 = ref[:, 1:2 * D:2]
    exp[:, 0:2 * D:2] = x0 * c - x1 * s
    exp[:, 1:2 * D:2] = x1 * c + x0 * s
    assert _rel(out, exp) < 8e-3


@pytest.mark.parametrize("bn", [128, 256] + PAIR)
def test_gemm_swiglu(bn):
    M, D, H = 512, 256, 640
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(M, D, generator=g, device="cuda").bfloat16()
    w13 = (0.1 * torch.randn(D, 2 * H, generator=g, device="cuda")).bfloat16()  # [D, w1 | w3]
    h13 = torch.empty(M, 2 * H, device="cuda", dtype=torch.bfloat16)
    gate = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    gemm(x, False, w13, True, M, H, D, _lib.EPI_SWIGLU, h13, out2=gate, n_half=H, force_bn=bn)
    h = x.float() @ w13.float()
    h1, h3 = h[:, :H], h[:, H:]
    assert _rel(h13[:, :H], h1) < 8e-3
    assert _rel(h13[:, H:], h3) < 8e-3
    assert _rel(gate, torch.nn.functional.silu(h1) * h3) < 8e-3


@pytest.mark.parametrize("bn", [0] + PAIR)
def test_gemm_swiglu_bwd(bn):
    M, D, H = 256, 256, 384
    g = torch.Generator(device="cuda").manual_seed(8)
    dffn = torch.randn(M, D, generator=g, device="cuda").bfloat16()
    w2 = (0.1 * torch.randn(D, H, generator=g, device="cuda")).bfloat16()  # reference layout [D, H]
    h13 = torch.randn(M, 2 * H, generator=g, device="cuda").bfloat16()
    dh13 = torch.empty(M, 2 * H, device="cuda", dtype=torch.bfloat16)
    gemm(dffn, False, w2, True, M, H, D, _lib.EPI_SWIGLU_BWD, dh13, aux=h13, n_half=H, force_bn=bn)
    dg = dffn.float() @ w2.float()
    h1, h3 = h13[:, :H].float(), h13[:, H:].float()
    sig = torch.sigmoid(h1)
    dh3 = dg * h1 * sig
    dh1 = dg * h3 * sig * (1 + h1 * (1 - sig))
    assert _rel(dh13[:, :H], dh1) < 8e-3
    assert _rel(dh13[:, H:], dh3) < 8e-3


def test_gemm_odd_kblock_count():
    # stages hold two 64-deep k-blocks; an odd count ends with a half stage
    M, N, K = 512, 1024, 448
    A, B, ref = operands(M, N, K, False, True, seed=9)
    for bn in (128, 192, 256, -256, -128):
        out = torch.empty(M, N, device="cuda")
        gemm(A, False, B, True, M, N, K, _lib.EPI_F32, out, force_bn=bn)
        assert _rel(out, ref) < TOL, bn
    A2, B2, ref2 = operands(M, N, K, True, False, seed=10)
    out = torch.empty(M, N, device="cuda")
    gemm(A2, True, B2, False, M, N, K, _lib.EPI_F32, out, force_bn=-192)
    assert _rel(out, ref2) < TOL


@pytest.mark.parametrize("epi", [_lib.EPI_BF16, _lib.EPI_F32])
def test_gemm_pair192_many_tiles(epi):
    # the backward data-gradient shape (N = D = 1536, K-major weights) on 192-wide pair tiles
    M, N, K = 4096, 1536, 1536
    A, B, ref = operands(M, N, K, False, False, seed=16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16 if epi == _lib.EPI_BF16 else torch.float32)
    gemm(A, False, B, False, M, N, K, epi, out, force_bn=PAIR192)
    assert _rel(out, ref) < (8e-3 if epi == _lib.EPI_BF16 else TOL)
    At, Bt, reft = operands(M, N, K, True, False, seed=17)
    acc = torch.randn(M, N, device="cuda")
    base = acc.clone()
    gemm(At, True, Bt, False, M, N, K, _lib.EPI_F32_ACC, acc, beta=1, force_bn=PAIR192)
    assert _rel(acc, reft + base) < TOL


def _rowdot_ref(out, O, seq):
    M, N = out.shape
    prod = (out.float() * O.float()).view(M // seq, seq, N // 128, 128).sum(-1)
    return prod.permute(0, 2, 1).contiguous()  # [batch][head][pos]


@pytest.mark.parametrize("bn", [0, 256, -256])
@pytest.mark.parametrize("shape", [(576, 640, 384, 192), (4096, 1536, 1536, 512)])
def test_gemm_bf16_rowdot(bn, shape):
    # dO = dx2s Wo^T with the attention backward's rowsum(dO * O) per head in the
    # epilogue: ragged M against 256-row tiles, an odd head count (the last tile's
    # second half is outside N), and the 600M shape
    M, N, K, seq = shape
    A, B, ref = operands(M, N, K, False, False, seed=21)
    g = torch.Generator(device="cuda").manual_seed(22)
    O = torch.randn(M, N, generator=g, device="cuda").bfloat16()
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    dvec = torch.full((M // seq, N // 128, seq), float("nan"), device="cuda")
    gemm(A, False, B, False, M, N, K, _lib.EPI_BF16_ROWDOT, out, out2=dvec, aux=O, seq=seq, force_bn=bn)
    assert _rel(out, ref) < 8e-3
    if bn != 0:  # the same tile kernel without the row dot writes the same bits
        plain = torch.empty_like(out)
        gemm(A, False, B, False, M, N, K, _lib.EPI_BF16, plain, force_bn=bn)
        assert torch.equal(plain, out)
    want = _rowdot_ref(out, O, seq)
    assert torch.isfinite(dvec).all()
    assert ((dvec - want).norm() / want.norm()).item() < 1e-5


def test_gemm_bf16_rowdot_rejects():
    M, N, K, seq = 512, 384, 128, 256
    A, B, _ = operands(M, N, K, False, False, seed=23)
    O = torch.zeros(M, N, device="cuda").bfloat16()
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    dvec = torch.empty(M // seq * (N // 128), seq, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    L = _lib.lib()

    def call(n, bn, seq_, b_mn=0):
        return L.rt_kernel_gemm(A.data_ptr(), A.stride(0), 0, B.data_ptr(), B.stride(0), b_mn, M, n, K,
                                _lib.EPI_BF16_ROWDOT, out.data_ptr(), out.stride(0), dvec.data_ptr(), 0,
                                O.data_ptr(), O.stride(0), 1.0, 0, None, None, seq_, 0, 0, bn, err.data_ptr(), st)

    assert call(N, 128, seq) != 0     # tiles narrower than two heads
    assert call(N, -128, seq) != 0
    assert call(N - 32, 0, seq) != 0  # N not a whole number of heads
    assert call(N, 0, 0) != 0         # no sequence length
    assert call(N, 0, 384) != 0       # M not a whole number of sequences
    assert call(N, 0, seq, b_mn=1) != 0
    torch.cuda.synchronize()
    assert err.item() == 0
