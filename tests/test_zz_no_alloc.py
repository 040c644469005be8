"""The allocation-free decode attention entry point, called through its exported C symbol.

It exists for callers that cannot allocate device memory (fixed pre-planned memory budgets,
plug-in callbacks that may not call cudaMalloc, launches during someone else's graph capture):
its split-KV scratch is a fixed file-scope device array. Its output must match the regular entry
point (which takes a workspace tensor) on two calls in a row, and oversized problems must be
rejected without launching anything. This file is collected last on purpose.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 8 << 20


def _lib():
    from minisgl._native import cuda

    mod = cuda()  # loads torch's libraries and the release extension into the process first
    # the exact shared object behind the module the other assertions read (not the bounds-check
    # build, whose scratch array and device error word are separate copies)
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.msgl_attention_decode_noalloc
    P, I, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    fn.argtypes = [P, P, P, P, P, L, P, P, I, I, I, I, L, L, ctypes.c_float, I, P, I, P]
    fn.restype = ctypes.c_int
    return fn


def _setup(bs, nq, nkv, hd, seed=0):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, 900, (bs,), generator=g).tolist()
    slots = sum(lens) + 64
    kc = torch.randn(slots, nkv, hd, generator=g).to("cuda", torch.bfloat16)
    vc = torch.randn(slots, nkv, hd, generator=g).to("cuda", torch.bfloat16)
    pt = torch.zeros(bs + 1, 928, dtype=torch.int32)
    perm = torch.randperm(slots, generator=g)
    used = 0
    for b, n in enumerate(lens):
        pt[b + 1, :n] = perm[used : used + n].to(torch.int32)
        used += n
    rows = (torch.arange(bs, dtype=torch.int32) + 1).cuda()
    q = torch.randn(bs, nq, hd, generator=g).to("cuda", torch.bfloat16)
    return q, kc, vc, pt.cuda(), rows, torch.tensor(lens, dtype=torch.int32, device="cuda")


def _call(fn, o, q, kc, vc, pt, rows, kvl, splits, sinks=None):
    bs, nq, hd = q.shape
    return fn(o.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pt.data_ptr(), pt.stride(0),
              rows.data_ptr(), kvl.data_ptr(), bs, nq, kc.shape[1], hd, kc.stride(0), kc.shape[0],
              1.0 / math.sqrt(hd), -1, None if sinks is None else sinks.data_ptr(), splits,
              torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("splits", [1, 4])
def test_noalloc_matches_workspace_entry_point(splits):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from minisgl._native import cuda

    fn = _lib()
    q, kc, vc, pt, rows, kvl = _setup(bs=24, nq=40, nkv=8, hd=128)
    sinks = torch.randn(40, device="cuda")
    ws = torch.empty(24 * 40 * splits * 130 * 4, dtype=torch.uint8, device="cuda")
    expect = torch.empty_like(q)
    cuda().attention_decode(expect, q, kc, vc, pt, rows, kvl, 1.0 / math.sqrt(128), -1, sinks, splits, ws)
    from minisgl.ops import reference as ref

    cu = torch.arange(q.shape[0] + 1, dtype=torch.int32)
    fp32 = ref.paged_attention(q.cpu(), kc.cpu(), vc.cpu(), pt.cpu(), rows.cpu(), cu, kvl.cpu(),
                               1.0 / math.sqrt(128), -1, sinks.cpu())
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        out = torch.full_like(q, float("nan"))
        assert _call(fn, out, q, kc, vc, pt, rows, kvl, splits, sinks) == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float().cpu(), expect.float().cpu(), atol=2e-2, rtol=2e-2)
        torch.testing.assert_close(out.float().cpu(), fp32.float(), atol=2e-2, rtol=2e-2)
    assert cuda().get_error()[0] == 0


def test_noalloc_rejects_oversized_problem():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    fn = _lib()
    q, kc, vc, pt, rows, kvl = _setup(bs=8, nq=64, nkv=8, hd=128)
    splits = 64  # 8 * 64 * 64 * 130 * 4 bytes > 8 MiB
    assert 8 * 64 * splits * 130 * 4 > SCRATCH_BYTES
    out = torch.zeros_like(q)
    assert _call(fn, out, q, kc, vc, pt, rows, kvl, splits) == 1
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0  # nothing was launched
