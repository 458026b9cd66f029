"""The allocation-free paged-attention C entry point, called through its
exported C symbol, must give the same result as the regular entry point and as
the fp32 statement of the op.

Callers that cannot allocate device memory (custom allocators, plugins inside
a runtime that owns all device memory, real-time paths) use that symbol; it
keeps its split-KV partials in a fixed array inside the library. The test runs
it twice in a row with different inputs, so stale scratch from the first call
would show up in the second, and checks that bad inputs are reported through
the status word instead of being read past.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from openmini_v1_b200 import _native, ops
from openmini_v1_b200.ops import reference as ref

OM_ERR_BOUNDS = 5


def _close(a, b, rtol=2e-2, atol=2e-2):
    a, b = a.float(), b.float()
    err = (a - b).abs()
    tol = atol + rtol * b.abs()
    bad = (err > tol).float().mean().item()
    assert bad < 1e-3 and (err / tol).max().item() <= 8.0, f"max err {err.max().item():.4g}, frac bad {bad:.4g}"


def _lib():
    lib = ctypes.CDLL(_native.C().__file__)
    fn = lib.om_paged_attention_noalloc
    P, I = ctypes.c_void_p, ctypes.c_int
    # q, q_ld, k, v, num_blocks, Hkv, head_dim, block_tables, num_seqs, max_blocks, row_seq, row_ctx,
    # rows, out, out_ld, Hq, max_ctx, scale, status, stream
    fn.argtypes = [P, I, P, P, I, I, I, P, I, I, P, P, I, P, I, I, I, ctypes.c_float, P, P]
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


def _call(fn, q, kc, vc, bt, rseq, rctx, out, max_ctx, scale, status):
    S, Hq, D = q.shape
    return fn(q.data_ptr(), Hq * D, kc.data_ptr(), vc.data_ptr(), kc.shape[0], kc.shape[1], D, bt.data_ptr(),
              bt.shape[0], bt.shape[1], rseq.data_ptr(), rctx.data_ptr(), rseq.shape[0], out.data_ptr(), Hq * D, Hq,
              max_ctx, scale, status.data_ptr() if status is not None else None,
              torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_regular_entry_point_twice():
    fn = _lib()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for seed, lens in ((1, [5, 700, 1300]), (2, [2049, 33, 1, 900])):
        q, kc, vc, bt, rseq, rctx = _case(seed, lens)
        S, Hq, D = q.shape
        scale = 1 / math.sqrt(D)
        expect = ops.paged_attention(q, kc, vc, bt, rseq, rctx, Hq, scale, max_ctx=4096)
        oracle = ref.paged_attention(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), rseq.cpu(), rctx.cpu(), Hq, scale)
        out = torch.full((S, Hq * D), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = _call(fn, q, kc, vc, bt, rseq, rctx, out, 4096, scale, status)
        torch.cuda.synchronize()
        assert rc == 0
        assert int(status.item()) == 0
        _close(out.view(S, Hq, D), expect.view(S, Hq, D))
        _close(out.view(S, Hq, D).cpu(), oracle.view(S, Hq, D))


def test_noalloc_reports_bad_inputs_in_status():
    """An out-of-range block id, a sequence index past the block table and a context
    longer than max_ctx each set OM_ERR_BOUNDS; the call itself still succeeds."""
    fn = _lib()
    q, kc, vc, bt, rseq, rctx = _case(4, [40, 64])
    S, Hq, D = q.shape
    out = torch.empty(S, Hq * D, dtype=torch.bfloat16, device="cuda")
    cases = []
    b = bt.clone()
    b[0, 1] = kc.shape[0] + 7
    cases.append((b, rseq, rctx, 4096))
    cases.append((bt, torch.tensor([0, 5], dtype=torch.int32, device="cuda"), rctx, 4096))
    cases.append((bt, rseq, torch.tensor([40, 64 + 16], dtype=torch.int32, device="cuda"), 4096))
    cases.append((bt, rseq, torch.tensor([40, 600], dtype=torch.int32, device="cuda"), 64))
    for b, rs, rc_, mc in cases:
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        rc = _call(fn, q, kc, vc, b, rs, rc_, out, mc, 0.1, status)
        torch.cuda.synchronize()
        assert rc == 0
        assert int(status.item()) == OM_ERR_BOUNDS
        assert torch.isfinite(out.float()).all()


def test_noalloc_rejects_oversized_request():
    fn = _lib()
    q, kc, vc, bt, rseq, rctx = _case(3, [16])
    rows = torch.zeros(4096, dtype=torch.int32, device="cuda")
    out = torch.empty(4096, 16 * 128, dtype=torch.bfloat16, device="cuda")
    rc = fn(q.data_ptr(), 16 * 128, kc.data_ptr(), vc.data_ptr(), kc.shape[0], 2, 128, bt.data_ptr(), 1, bt.shape[1],
            rows.data_ptr(), rows.data_ptr(), 4096, out.data_ptr(), 16 * 128, 16, 1 << 20, 0.1, None,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    rc = fn(q.data_ptr(), 16 * 128, kc.data_ptr(), vc.data_ptr(), kc.shape[0], 2, 128, bt.data_ptr(), 1, bt.shape[1],
            rows.data_ptr(), rows.data_ptr(), 4096, out.data_ptr(), 16 * 128, 16, 2**31 - 1, 0.1, None,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1
