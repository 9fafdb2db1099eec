"""The allocation-free C entry point ``bwn_gqa_decode_noalloc`` against the
regular ``torch.ops.bwn.gqa_decode``.

The entry point exists for callers that cannot allocate device memory (runtimes
that own all GPU memory, plugin hosts that forbid allocation after start-up,
paths that must not risk cudaMalloc's implicit synchronisation); it keeps its
split-KV scratch in a fixed device array.  These tests call it through its
exported C symbol with ctypes, twice in a row, compare each result with the
regular op on identical inputs, and read the status word through
``bwn_gqa_decode_noalloc_status``.  Both kernels are covered: the tensor-core
one (rope_dim a multiple of 16) and the CUDA-core one (rope_dim 40).  The file
is named to be collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

P, L, I, F = ctypes.c_void_p, ctypes.c_long, ctypes.c_int, ctypes.c_float


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _lib():
    import bwn._C as C
    lib = ctypes.CDLL(C.__file__)
    f = lib.bwn_gqa_decode_noalloc
    f.argtypes = [P, L, P, P, L, P, P, P, P, P, P, P, P, L, I, I, I, I, I, F, I, P]
    f.restype = I
    st = lib.bwn_gqa_decode_noalloc_status
    st.argtypes = [ctypes.POINTER(ctypes.c_int), P]
    st.restype = I
    return f, st


def _case(B, QH, KVH, S, rope, pos, seed=0):
    from bwn.ops import reference as R
    dev = "cuda"
    D = 256
    g = torch.Generator(device=dev).manual_seed(seed)
    qg = torch.randn(B, QH, 2 * D, device=dev, generator=g).bfloat16()
    kv = torch.randn(B, 2, KVH, D, device=dev, generator=g).bfloat16()
    qn = torch.randn(D, device=dev, generator=g) * 0.1
    kn = torch.randn(D, device=dev, generator=g) * 0.1
    cos, sin = R.rope_table(S, rope, 1e7, device=dev)
    kc = torch.randn(B, KVH, S, D, device=dev, generator=g).bfloat16()
    vc = torch.randn(B, KVH, S, D, device=dev, generator=g).bfloat16()
    return dict(qg=qg, k_new=kv[:, 0], v_new=kv[:, 1], qn=qn, kn=kn, cos=cos, sin=sin, kc=kc, vc=vc,
                pos=torch.tensor(pos, device=dev, dtype=torch.int32), B=B, QH=QH, KVH=KVH, S=S, rope=rope)


def _regular(c):
    import bwn.ops as O
    kc, vc = c["kc"].clone(), c["vc"].clone()
    out = O.gqa_decode(c["qg"], c["k_new"], c["v_new"], c["qn"], c["kn"], c["cos"], c["sin"], kc, vc, c["pos"])
    torch.cuda.synchronize()
    return out, kc, vc


def _noalloc(f, c, kc, vc, splits=0):
    out = torch.empty(c["B"], c["QH"] * 256, device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    rc = f(c["qg"].data_ptr(), c["qg"].stride(0), c["k_new"].data_ptr(), c["v_new"].data_ptr(), c["k_new"].stride(0),
           c["qn"].data_ptr(), c["kn"].data_ptr(), c["cos"].data_ptr(), c["sin"].data_ptr(), kc.data_ptr(),
           vc.data_ptr(), c["pos"].data_ptr(), out.data_ptr(), out.stride(0), c["B"], c["QH"], c["KVH"], c["S"],
           c["rope"], 1e-6, splits, stream)
    torch.cuda.synchronize()
    return rc, out


def _status(st):
    word = ctypes.c_int(-1)
    rc = st(ctypes.byref(word), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    return word.value


@pytest.mark.parametrize("rope", [64, 40], ids=["tensor_core", "cuda_core"])
def test_noalloc_matches_regular_op_twice(rope):
    f, st = _lib()
    c = _case(4, 24, 4, 1024, rope, [700, 3, 0, 1023])
    ref, kc_ref, vc_ref = _regular(c)
    kc, vc = c["kc"], c["vc"]
    for call in range(2):
        rc, out = _noalloc(f, c, kc, vc)
        assert rc == 0, f"call {call}: return code {rc}"
        assert _status(st) == 0, call
        assert _rel(out, ref) < 2e-2, call
        assert _rel(kc, kc_ref) < 1e-2 and torch.equal(vc, vc_ref)


def test_noalloc_split_cap():
    """batch * q_heads * (4 + 256) floats per split leaves room for 3 splits of
    the 1 Mi-float array: a request for 8 is lowered, the result is unchanged."""
    f, st = _lib()
    c = _case(64, 16, 2, 512, 64, [(37 * i) % 512 for i in range(64)], seed=1)
    ref, kc_ref, _ = _regular(c)
    kc, vc = c["kc"], c["vc"]
    for call in range(2):
        rc, out = _noalloc(f, c, kc, vc, splits=8)
        assert rc == 0 and _status(st) == 0, call
        assert _rel(out, ref) < 2e-2, call


@pytest.mark.parametrize("rope", [64, 40], ids=["tensor_core", "cuda_core"])
def test_noalloc_position_at_cache_end(rope):
    """positions s_max - 1 (the last cache row) and s_max (no such row: the row
    is inactive, nothing is written, its output is zero)."""
    f, st = _lib()
    S = 256
    c = _case(3, 8, 2, S, rope, [S - 1, S, 5], seed=2)
    kc0, vc0 = c["kc"].clone(), c["vc"].clone()
    ref, kc_ref, _ = _regular(c)
    kc, vc = c["kc"].clone(), c["vc"].clone()
    rc, out = _noalloc(f, c, kc, vc)
    assert rc == 0 and _status(st) == 0
    assert _rel(out, ref) < 2e-2
    assert torch.count_nonzero(out[1]) == 0
    # sequence 1 (position s_max) and every row other than the written ones are untouched
    assert torch.equal(kc[1], kc0[1]) and torch.equal(vc[1], vc0[1])
    assert torch.equal(kc[0, :, :S - 1], kc0[0, :, :S - 1]) and torch.equal(kc[2, :, :5], kc0[2, :, :5])
    assert torch.equal(kc[2, :, 6:], kc0[2, :, 6:])
    assert not torch.equal(kc[0, :, S - 1], kc0[0, :, S - 1])


def test_noalloc_rejects_oversized():
    f, _ = _lib()
    # batch * q_heads * (4 + 256) floats for one split exceeds the 1 Mi-float array
    rc = f(1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 8192, 8, 1, 64, 64, 1e-6, 1, None)
    assert rc == 2
    rc = f(1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 2, 5, 2, 64, 64, 1e-6, 1, None)
    assert rc == 1  # q_heads not a multiple of kv_heads
