"""The allocation-free paged-attention C entry point, called through its
exported C symbol, must give the same result as the regular entry point.

Callers that cannot allocate device memory (custom allocators, plugins inside
a runtime that owns all device memory, real-time paths) use that symbol; it
keeps its split-KV partials in a fixed array inside the library. The test runs
it twice in a row with different inputs, so stale scratch from the first call
would show up in the second.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from openmini_v1_b200 import _native, ops


def _close(a, b, rtol=2e-2, atol=2e-2):
    a, b = a.float(), b.float()
    err = (a - b).abs()
    bad = (err > atol + rtol * b.abs()).float().mean().item()
    assert bad < 1e-3, f"max err {err.max().item():.4g}, frac bad {bad:.4g}"


def _lib():
    lib = ctypes.CDLL(_native.C().__file__)
    fn = lib.om_paged_attention_noalloc
    P, I = ctypes.c_void_p, ctypes.c_int
    fn.argtypes = [P, I, P, P, I, I, I, P, I, P, P, I, P, I, I, I, ctypes.c_float, P, P]
    fn.restype = I
    return fn


def _case(seed, lens, Hq=16, Hkv=2, D=128, nb=256):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(nb, Hkv, 16, D, generator=g, device="cuda").bfloat16()
    vc = torch.randn(nb, Hkv, 16, D, generator=g, device="cuda").bfloat16()
    S = len(lens)
    mb = max((l + 15) // 16 for l in lens)
    perm = torch.randperm(nb, device="cuda", generator=g).to(torch.int32)
    bt = torch.zeros(S, mb, dtype=torch.int32, device="cuda")
    o = 0
    for s, l in enumerate(lens):
        n = (l + 15) // 16
        bt[s, :n] = perm[o:o + n]
        o += n
    q = torch.randn(S, Hq, D, generator=g, device="cuda").bfloat16()
    rseq = torch.arange(S, dtype=torch.int32, device="cuda")
    rctx = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, kc, vc, bt, rseq, rctx


def test_noalloc_matches_regular_entry_point_twice():
    fn = _lib()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for seed, lens in ((1, [5, 700, 1300]), (2, [2049, 33, 1, 900])):
        q, kc, vc, bt, rseq, rctx = _case(seed, lens)
        S, Hq, D = q.shape
        scale = 1 / math.sqrt(D)
        expect = ops.paged_attention(q, kc, vc, bt, rseq, rctx, Hq, scale, max_ctx=4096)
        out = torch.full((S, Hq * D), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = fn(q.data_ptr(), Hq * D, kc.data_ptr(), vc.data_ptr(), kc.shape[0], kc.shape[1], D, bt.data_ptr(),
                bt.shape[1], rseq.data_ptr(), rctx.data_ptr(), S, out.data_ptr(), Hq * D, Hq, 4096, scale,
                status.data_ptr(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert rc == 0
        assert int(status.item()) == 0
        _close(out.view(S, Hq, D), expect.view(S, Hq, D))


def test_noalloc_rejects_oversized_request():
    fn = _lib()
    q, kc, vc, bt, rseq, rctx = _case(3, [16])
    rc = fn(q.data_ptr(), 16 * 128, kc.data_ptr(), vc.data_ptr(), kc.shape[0], 2, 128, bt.data_ptr(), bt.shape[1],
            rseq.data_ptr(), rctx.data_ptr(), 4096, q.data_ptr(), 16 * 128, 16, 1 << 20, 0.1, None,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1
