"""The allocation-free decode-attention entry point, called through its C symbol.

`b200_decode_attention_noalloc` is for callers that cannot allocate device
memory when they run attention (C hosts with a fixed memory budget, plugin
interfaces without an allocator, loops that cannot take cudaMalloc's implicit
synchronisation). It keeps its split-KV partials in a fixed device array in
the library instead. This test loads the symbol with ctypes (no torch in the
call path), runs it twice in a row with different inputs and split counts,
and compares each result with the regular torch-facing entry point
(`ops.decode_attention`, which uses a workspace allocated by the package).
The file is named so that pytest collects it last.
"""
import ctypes
import glob
import math
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import rlx_models_b200
    from rlx_models_b200 import ops  # noqa: F401  (loads the extension and torch's libraries)
    so = glob.glob(os.path.join(os.path.dirname(rlx_models_b200.__file__), "_C*.so"))
    assert so, "extension not built"
    lib = ctypes.CDLL(so[0])
    fn = lib.b200_decode_attention_noalloc
    P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    fn.argtypes = [P, P, P, I64, P, I, P, P, P, I, I, I, I, I, F, I, P, P]
    fn.restype = I
    return fn


def _case(dev, B, Hq, Hkv, D, lens, seed):
    g = torch.Generator().manual_seed(seed)
    maxb = max((l + 15) // 16 for l in lens)
    NB = sum((l + 15) // 16 for l in lens) + 2
    perm = torch.randperm(NB, generator=g)
    tables = torch.zeros(B, maxb, dtype=torch.int32)
    c = 0
    for b, l in enumerate(lens):
        n = (l + 15) // 16
        tables[b, :n] = perm[c:c + n].int()
        c += n
    kc = torch.randn(NB, Hkv, 16, D, generator=g).to(dev, torch.bfloat16)
    vc = torch.randn(NB, Hkv, 16, D, generator=g).to(dev, torch.bfloat16)
    q = torch.randn(B, Hq, D, generator=g).to(dev, torch.bfloat16)
    ctx = torch.tensor(lens, dtype=torch.int32, device=dev)
    return q, kc, vc, tables.to(dev), ctx


def _call(fn, q, kc, vc, tables, ctx, out, splits, scale, status, sinks=None, window=0):
    B, Hq, D = q.shape
    stream = torch.cuda.current_stream(q.device).cuda_stream
    return fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], tables.data_ptr(), tables.shape[1],
              ctx.data_ptr(), out.data_ptr(), sinks.data_ptr() if sinks is not None else None, window, B, Hq,
              kc.shape[1], D, scale, splits, status.data_ptr(), ctypes.c_void_p(stream))


def test_noalloc_matches_regular_entry_point_twice(cuda):
    from rlx_models_b200 import ops
    fn = _lib()
    status = torch.zeros(4, dtype=torch.int32, device=cuda)
    cases = [
        dict(B=5, Hq=32, Hkv=8, D=128, lens=[1, 17, 300, 999, 2047], splits=3, window=0, sinks=False, seed=1),
        dict(B=7, Hq=64, Hkv=8, D=64, lens=[5, 16, 129, 513, 64, 1000, 33], splits=2, window=128, sinks=True,
             seed=2),
    ]
    for cs in cases:
        q, kc, vc, tables, ctx = _case(cuda, cs["B"], cs["Hq"], cs["Hkv"], cs["D"], cs["lens"], cs["seed"])
        sinks = torch.randn(cs["Hq"], device=cuda) if cs["sinks"] else None
        scale = 1.0 / math.sqrt(cs["D"])
        out = torch.zeros_like(q)
        rc = _call(fn, q, kc, vc, tables, ctx, out, cs["splits"], scale, status, sinks, cs["window"])
        assert rc == 0, rc
        torch.cuda.synchronize(cuda)
        assert int(status[0]) == 0
        ref = ops.decode_attention(q, kc, vc, tables, ctx, scale=scale, sinks=sinks, window=cs["window"],
                                   splits=cs["splits"])
        rel = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
        assert rel < 2e-2, rel
        # and against the fp32 restatement of the same attention
        orc = _oracle(q, kc, vc, tables, ctx, scale, sinks, cs["window"])
        rel = ((out.float() - orc).norm() / orc.norm()).item()
        assert rel < 2e-2, rel


def _oracle(q, kc, vc, tables, ctx, scale, sinks, window):
    from rlx_models_b200.ops.reference import attention, gather_paged
    outs = []
    for b in range(q.shape[0]):
        L = int(ctx[b])
        k = gather_paged(kc, tables[b], L)
        v = gather_paged(vc, tables[b], L)
        pos = torch.arange(L, device=q.device)
        outs.append(attention(q[b:b + 1], k, v, pos[-1:], pos, scale, causal=True, window=window, sinks=sinks))
    return torch.cat(outs)


def test_noalloc_rejects_oversized_request(cuda):
    fn = _lib()
    B, Hq, Hkv, D = 64, 64, 8, 128
    q, kc, vc, tables, ctx = _case(cuda, B, Hq, Hkv, D, [32] * B, 3)
    out = torch.zeros_like(q)
    status = torch.zeros(4, dtype=torch.int32, device=cuda)
    # 64 * 64 * 2 * 130 floats > 1 << 20: rejected before any launch
    rc = _call(fn, q, kc, vc, tables, ctx, out, 2, 1.0 / math.sqrt(D), status)
    assert rc == 2
    assert torch.count_nonzero(out) == 0
