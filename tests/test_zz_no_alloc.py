"""The allocation-free C entry point ``bwn_gqa_decode_noalloc`` against the
regular ``torch.ops.bwn.gqa_decode``.

The entry point exists for callers that cannot allocate device memory (runtimes
that own all GPU memory, plugin hosts that forbid allocation after start-up,
paths that must not risk cudaMalloc's implicit synchronisation); it keeps its
split-KV scratch in a fixed device array.  This test calls it through its
exported C symbol with ctypes, twice in a row, and compares each result with the
regular op on identical inputs.  The file is named to be collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _lib():
    import bwn._C as C
    lib = ctypes.CDLL(C.__file__)
    f = lib.bwn_gqa_decode_noalloc
    P, L, I, F = ctypes.c_void_p, ctypes.c_long, ctypes.c_int, ctypes.c_float
    f.argtypes = [P, L, P, P, L, P, P, P, P, P, P, P, P, L, I, I, I, I, I, F, I, P]
    f.restype = I
    return f


def test_noalloc_matches_regular_op_twice():
    from bwn.ops import reference as R
    import bwn.ops as O

    f = _lib()
    dev = "cuda"
    B, QH, KVH, S, D = 4, 24, 4, 1024, 256
    torch.manual_seed(0)
    qg = torch.randn(B, QH, 2 * D, device=dev).bfloat16()
    kv = torch.randn(B, 2, KVH, D, device=dev).bfloat16()
    k_new, v_new = kv[:, 0], kv[:, 1]
    qn = torch.randn(D, device=dev) * 0.1
    kn = torch.randn(D, device=dev) * 0.1
    cos, sin = R.rope_table(S, 64, 1e7, device=dev)
    kc = torch.randn(B, KVH, S, D, device=dev).bfloat16()
    vc = torch.randn(B, KVH, S, D, device=dev).bfloat16()
    pos = torch.tensor([700, 3, 0, 1023], device=dev, dtype=torch.int32)

    kc_ref, vc_ref = kc.clone(), vc.clone()
    ref = O.gqa_decode(qg, k_new, v_new, qn, kn, cos, sin, kc_ref, vc_ref, pos)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.empty(B, QH * D, device=dev, dtype=torch.bfloat16)
        rc = f(qg.data_ptr(), qg.stride(0), k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), qn.data_ptr(),
               kn.data_ptr(), cos.data_ptr(), sin.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(),
               out.data_ptr(), out.stride(0), B, QH, KVH, S, 64, 1e-6, 0, stream)
        torch.cuda.synchronize()
        assert rc == 0, f"call {call}: return code {rc}"
        assert _rel(out, ref) < 2e-2, call
        assert _rel(kc, kc_ref) < 1e-2 and torch.equal(vc, vc_ref)


def test_noalloc_rejects_oversized():
    f = _lib()
    # batch * q_heads * (2 + 256) floats for one split exceeds the 1 Mi-float array
    rc = f(1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 8192, 8, 1, 64, 64, 1e-6, 1, None)
    assert rc == 2
    rc = f(1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 2, 5, 2, 64, 64, 1e-6, 1, None)
    assert rc == 1  # q_heads not a multiple of kv_heads
