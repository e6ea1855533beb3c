"""Single-kernel timing of the LM-step kernels at a chosen shape (CUDA events).

    python -m rustane_b200.kernel_bench gemm --m 4096 --n 4096 --k 1536 --b-mn --epi swiglu [--bn -256 | --cublas]
    python -m rustane_b200.kernel_bench attention --batch 8 --seq 512 --heads 12 [--bwd [--impl tc|mma]]
    python -m rustane_b200.kernel_bench rmsnorm_bwd --m 4096 --d 1536   (or rmsnorm_fwd)

Prints one JSON line (mean us per launch, TFLOP/s or GB/s).  Buffers come from
torch; the kernels run through librustane_cuda.so's rt_kernel_* entry points.
Inputs are larger than L2 for the default 600M shapes.
"""
from __future__ import annotations

import argparse
import json

from . import _lib

EPIS = {"bf16": _lib.EPI_BF16, "f32": _lib.EPI_F32, "f32acc": _lib.EPI_F32_ACC, "residual": _lib.EPI_RESIDUAL,
        "rope": _lib.EPI_ROPE, "swiglu": _lib.EPI_SWIGLU, "swiglu_bwd": _lib.EPI_SWIGLU_BWD,
        "rowdot": _lib.EPI_BF16_ROWDOT}


def _time(fn, iters, warmup=3):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / iters  # us


def bench_gemm(args):
    import torch
    L = _lib.lib()
    M, N, K = args.m, args.n, args.k
    epi = EPIS[args.epi]
    ncols = 2 * N if epi == _lib.EPI_SWIGLU else N
    A = torch.randn((K, M) if args.a_mn else (M, K), device="cuda").bfloat16()
    B = torch.randn((K, ncols) if args.b_mn else (ncols, K), device="cuda").bfloat16()
    out_dtype = torch.float32 if epi in (_lib.EPI_F32, _lib.EPI_F32_ACC, _lib.EPI_RESIDUAL) else torch.bfloat16
    out_cols = 2 * N if epi in (_lib.EPI_SWIGLU, _lib.EPI_SWIGLU_BWD) else N
    out = torch.zeros(M, out_cols, device="cuda", dtype=out_dtype)
    out2 = torch.empty(M, N, device="cuda", dtype=torch.bfloat16) if epi == _lib.EPI_SWIGLU else None
    if epi == _lib.EPI_BF16_ROWDOT:
        out2 = torch.empty(M // args.seq * (N // 128), args.seq, device="cuda")
    aux = None
    if epi == _lib.EPI_RESIDUAL:
        aux = torch.randn(M, N, device="cuda")
    elif epi == _lib.EPI_SWIGLU_BWD:
        aux = torch.randn(M, 2 * N, device="cuda").bfloat16()
    elif epi == _lib.EPI_BF16_ROWDOT:
        aux = torch.randn(M, N, device="cuda").bfloat16()
    rope = None
    if epi == _lib.EPI_ROPE:
        rope = (torch.rand(args.seq, 64, device="cuda"), torch.rand(args.seq, 64, device="cuda"))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream

    def run():
        rc = L.rt_kernel_gemm(A.data_ptr(), A.stride(0), int(args.a_mn), B.data_ptr(), B.stride(0), int(args.b_mn),
                              M, N, K, epi, out.data_ptr(), out.stride(0),
                              out2.data_ptr() if out2 is not None else None, out2.stride(0) if out2 is not None else 0,
                              aux.data_ptr() if aux is not None else None, aux.stride(0) if aux is not None else 0,
                              0.5, int(args.beta), rope[0].data_ptr() if rope else None,
                              rope[1].data_ptr() if rope else None, args.seq, 2 * N // 3 // 128 * 128 if rope else 0,
                              N if epi in (_lib.EPI_SWIGLU, _lib.EPI_SWIGLU_BWD) else 0, args.bn, err.data_ptr(), st)
        assert rc == 0, rc

    flops = 2.0 * M * ncols * K
    if args.cublas:
        # the same operands through torch.matmul (cuBLAS), bf16 output: a library
        # reference point for the mainloop, without our fused epilogue
        A_log = A.t() if args.a_mn else A
        B_log = B if args.b_mn else B.t()
        C = torch.empty(M, ncols, device="cuda", dtype=torch.bfloat16)
        us = _time(lambda: torch.matmul(A_log, B_log, out=C), args.iters)
        return {"kernel": "cublas_bf16", "M": M, "N": ncols, "K": K, "us": us, "tflops": flops / us / 1e6}
    us = _time(run, args.iters)
    assert err.item() == 0
    return {"kernel": "gemm", "M": M, "N": N, "K": K, "epi": args.epi, "a_mn": args.a_mn, "b_mn": args.b_mn,
            "bn": args.bn, "us": us, "tflops": flops / us / 1e6}


def bench_attention(args):
    import torch
    L = _lib.lib()
    B, S, H = args.batch, args.seq, args.heads
    D = H * 128
    qkv = torch.randn(B * S, 3 * D, device="cuda").bfloat16()
    out = torch.empty(B * S, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, H, S, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    fwd = lambda: L.rt_kernel_attention_fwd(qkv.data_ptr(), out.data_ptr(), lse.data_ptr(), B, S, H, st)  # noqa
    fl = 4.0 * B * H * S * S / 2 * 128
    if not args.bwd:
        us = _time(fwd, args.iters)
        return {"kernel": "attention_fwd", "B": B, "S": S, "H": H, "us": us, "tflops": fl / us / 1e6}
    fwd()
    dout = torch.randn(B * S, D, device="cuda").bfloat16()
    dvec = torch.empty(B, H, S, device="cuda")
    dqkv = torch.empty(B * S, 3 * D, device="cuda", dtype=torch.bfloat16)
    cb, sb = torch.rand(64, S, device="cuda"), torch.rand(64, S, device="cuda")
    if args.impl == "tc":
        ds = torch.empty(L.rt_kernel_attention_bwd_scratch_bytes(B, S, H) // 2, device="cuda", dtype=torch.bfloat16)
        bwd = lambda: L.rt_kernel_attention_bwd_tc(  # noqa
            qkv.data_ptr(), out.data_ptr(), lse.data_ptr(), dout.data_ptr(), dvec.data_ptr(), ds.data_ptr(),
            dqkv.data_ptr(), cb.data_ptr(), sb.data_ptr(), B, S, H, st)
    else:
        bwd = lambda: L.rt_kernel_attention_bwd(  # noqa
            qkv.data_ptr(), out.data_ptr(), lse.data_ptr(), dout.data_ptr(), dvec.data_ptr(), dqkv.data_ptr(),
            cb.data_ptr(), sb.data_ptr(), B, S, H, st)
    us = _time(bwd, args.iters)
    return {"kernel": f"attention_bwd_{args.impl}", "B": B, "S": S, "H": H, "us": us, "tflops": 2.5 * fl / us / 1e6}


def bench_rmsnorm_bwd(args):
    import torch
    L = _lib.lib()
    M, D = args.m, args.d
    dy, x, res = (torch.randn(M, D, device="cuda") for _ in range(3))
    g = torch.ones(D, device="cuda")
    r = torch.rand(M, device="cuda")
    dx = torch.empty(M, D, device="cuda")
    dxb = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    dg = torch.zeros(D, device="cuda")
    part = torch.empty(L.rt_kernel_rmsnorm_bwd_partials(M) * D, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    run = lambda: L.rt_kernel_rmsnorm_bwd(dy.data_ptr(), x.data_ptr(), g.data_ptr(), r.data_ptr(),  # noqa
                                          res.data_ptr(), dx.data_ptr(), dxb.data_ptr(), 0.5, dg.data_ptr(), 0,
                                          part.data_ptr(), M, D, st)
    us = _time(run, args.iters)
    bytes_ = M * D * (4 * 4 + 2)  # read dy, x, resid; write dx (fp32) and dx (bf16)
    return {"kernel": "rmsnorm_bwd", "M": M, "D": D, "us": us, "gbs": bytes_ / us / 1e3}


def bench_rmsnorm_fwd(args):
    import torch
    L = _lib.lib()
    M, D = args.m, args.d
    x = torch.randn(M, D, device="cuda")
    g = torch.ones(D, device="cuda")
    r = torch.empty(M, device="cuda")
    out = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream
    run = lambda: L.rt_kernel_rmsnorm_fwd(x.data_ptr(), g.data_ptr(), out.data_ptr(), r.data_ptr(), M, D, st)  # noqa
    us = _time(run, args.iters)
    bytes_ = M * D * (4 + 2)  # read x (fp32), write the bf16 output
    return {"kernel": "rmsnorm_fwd", "M": M, "D": D, "us": us, "gbs": bytes_ / us / 1e3}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemm", "attention", "rmsnorm_bwd", "rmsnorm_fwd"])
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=1536)
    ap.add_argument("--d", type=int, default=1536)
    ap.add_argument("--a-mn", action="store_true")
    ap.add_argument("--b-mn", action="store_true")
    ap.add_argument("--epi", default="f32", choices=list(EPIS))
    ap.add_argument("--beta", type=int, default=0)
    ap.add_argument("--bn", type=int, default=0, help="0 auto; 128/192/256 single-CTA; -256/-128 CTA pair")
    ap.add_argument("--cublas", action="store_true", help="time torch.matmul on the same operands instead")
    ap.add_argument("--seq", type=int, default=512)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--heads", type=int, default=12)
    ap.add_argument("--bwd", action="store_true")
    ap.add_argument("--impl", default="tc", choices=["tc", "mma"], help="attention backward kernels")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    fn = {"gemm": bench_gemm, "attention": bench_attention, "rmsnorm_bwd": bench_rmsnorm_bwd,
          "rmsnorm_fwd": bench_rmsnorm_fwd}[args.kernel]
    print(json.dumps(fn(args)), flush=True)


if __name__ == "__main__":
    main()
