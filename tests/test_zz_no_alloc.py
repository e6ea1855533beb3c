"""The allocation-free attention backward (rt_kernel_attention_bwd_noalloc).

Callers that cannot allocate device memory when they run the backward pass use
this entry point: it takes its scratch from a fixed array inside the library.
This test calls it twice in a row through the C ABI, on two different inputs,
and checks each result against rt_kernel_attention_bwd (which takes its scratch
from the caller).  Both run the same kernels in the same order, so the results
must agree bit for bit; then it checks that a
size beyond the array is refused.  The file sorts last so that a run stopping
at the first failure has already run every other test.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pyoracle as po  # noqa: E402
from rustane_b200 import _lib  # noqa: E402
from rustane_b200.model import ModelConfig  # noqa: E402

pytestmark = pytest.mark.gpu
def _case(B, S, H, seed, tables):
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    D = H * 128
    g = torch.Generator(device="cuda").manual_seed(seed)
    qkv = torch.randn(B * S, 3 * D, generator=g, device="cuda").bfloat16()
    dout = torch.randn(B * S, D, generator=g, device="cuda").bfloat16()
    out = torch.empty(B * S, D, device="cuda", dtype=torch.bfloat16)
    lse2 = torch.empty(B, H, S, device="cuda")
    assert L.rt_kernel_attention_fwd(qkv.data_ptr(), out.data_ptr(), lse2.data_ptr(), B, S, H, st) == 0
    cb, sb = tables
    dvec = torch.empty(B, H, S, device="cuda")
    ref = torch.empty(B * S, 3 * D, device="cuda", dtype=torch.bfloat16)
    assert L.rt_kernel_attention_bwd(qkv.data_ptr(), out.data_ptr(), lse2.data_ptr(), dout.data_ptr(),
                                     dvec.data_ptr(), ref.data_ptr(), cb.data_ptr(), sb.data_ptr(), B, S, H, st) == 0
    got = torch.full_like(ref, float("nan"))
    assert L.rt_kernel_attention_bwd_noalloc(qkv.data_ptr(), out.data_ptr(), lse2.data_ptr(), dout.data_ptr(),
                                             got.data_ptr(), cb.data_ptr(), sb.data_ptr(), B, S, H, st) == 0
    torch.cuda.synchronize()
    return got, ref


def test_noalloc_attention_backward_matches_allocating_entry():
    S, H = 256, 2
    _, _, cb, sb = po.Oracle(ModelConfig.custom(H * 128, 256, H, 1, seq=S, vocab=256), 1).rope_tables()
    tables = (torch.from_numpy(cb).cuda(), torch.from_numpy(sb).cuda())
    for call, (B, seed) in enumerate([(2, 21), (1, 22)]):  # two calls in a row, different inputs
        got, ref = _case(B, S, H, seed, tables)
        assert torch.isfinite(got.float()).all(), call
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), call


def test_noalloc_rejects_sizes_beyond_its_array():
    L = _lib.lib()
    dummy = torch.zeros(16, device="cuda")
    p = dummy.data_ptr()
    # batch * heads * seq = 2 * 512 * 1024 > 524288: refused before any launch
    rc = L.rt_kernel_attention_bwd_noalloc(p, p, p, p, p, p, p, 2, 1024, 512, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.RT_ERR_SHAPE


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_on_a_second_device_in_the_same_process():
    """The in-library array exists once per device: a call on device 1 after calls on
    device 0 uses device 1's copy (and device 1's kernel attributes)."""
    S, H = 256, 2
    _, _, cb, sb = po.Oracle(ModelConfig.custom(H * 128, 256, H, 1, seq=S, vocab=256), 1).rope_tables()
    for dev in (0, 1):
        with torch.cuda.device(dev):
            tables = (torch.from_numpy(cb).cuda(), torch.from_numpy(sb).cuda())
            got, ref = _case(2, S, H, 23, tables)
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), dev
