"""Device-side bounded waits: a comm kernel waiting on a peer flag that nothing
sets gives up after its limit, reports through the status word, and leaves the
CUDA context usable (no trap, no hang)."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_flag_wait_times_out_and_reports():
    from bwn import ops as O
    from bwn.ops import _ext

    _ext.require()
    dev = torch.device("cuda", 0)
    rows, cols = 4, 256
    # a kernel that waits for every rank's flag, then reads the partials through
    # the multicast address; no peer ever signals, so it must give up and touch
    # no data (the address below is never dereferenced)
    flags = torch.zeros(2, dtype=torch.int32, device=dev)                 # peer flags nobody will set
    state = torch.zeros(8, dtype=torch.int32, device=dev)
    state[0] = 1                                                          # waiting for epoch 1
    resid = torch.randn(rows, cols, device=dev).bfloat16()
    before = resid.clone()
    w = torch.zeros(cols, device=dev)
    _ext.status_clear()
    t0 = time.perf_counter()
    torch.ops.bwn.ar_add_norm(0, rows * cols, flags.data_ptr(), 2, state, resid, w, 1e-6, 0.05)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert _ext.status() & 2, "the bounded peer wait did not report a timeout"
    with pytest.raises(RuntimeError, match="peer wait timeout"):
        O.check_status("test")
    assert _ext.status() == 0
    assert dt < 5.0
    assert torch.equal(resid, before), "a timed-out wait must leave the residual untouched"
    # the context still works: a regular kernel runs and is correct
    x = torch.randn(8, 256, device=dev).bfloat16()
    wn = torch.randn(256, device=dev) * 0.1
    y = O.rms_norm(x, wn, 1e-6)
    ref = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + wn)
    assert (y.float() - ref).abs().max() < 0.05
    assert _ext.status() == 0
