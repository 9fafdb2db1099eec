"""Op-level consistency of the CPU oracles the kernels are tested against (the
reference's ``test_gqa_stateful_cache_cpu.py`` and prefill/decode tiers):

* GQA decode writes this step's K/V row and attends over the prior rows plus
  it, so a sequence of decode steps equals causal prefill attention over the
  same tokens;
* multi-token verify (``n_tok`` query rows per cache sequence) equals that
  many sequential decode steps;
* the DeltaNet chunked prefill over S tokens equals S recurrent decode steps,
  state and conv ring included.
"""
import torch

from bwn.ops import reference as R

D, QH, KVH = 256, 4, 2


def _gqa_inputs(B, S, seed=0):
    g = torch.Generator().manual_seed(seed)
    qg = torch.randn(B, S, QH, 2 * D, generator=g)
    k = torch.randn(B, S, KVH, D, generator=g)
    v = torch.randn(B, S, KVH, D, generator=g)
    qn = torch.randn(D, generator=g) * 0.1
    kn = torch.randn(D, generator=g) * 0.1
    return qg, k, v, qn, kn


def test_decode_steps_equal_causal_prefill():
    B, S, Smax = 2, 9, 16
    qg, k, v, qn, kn = _gqa_inputs(B, S)
    cos, sin = R.rope_table(Smax, 64, 1e7)
    kc = torch.zeros(B, KVH, Smax, D)
    vc = torch.zeros_like(kc)
    outs = []
    for t in range(S):
        pos = torch.full((B,), t, dtype=torch.int32)
        outs.append(R.gqa_decode(qg[:, t], k[:, t], v[:, t], qn, kn, cos, sin, kc, vc, pos))
    dec = torch.stack(outs, 1).float()  # [B, S, QH*D]
    # the same tokens as one causal prefill: normed + roped q/k, rows written, then attention
    q, gate = qg.split(D, dim=-1)
    c, s_ = cos[:S][None, :, None], sin[:S][None, :, None]
    qr = R.apply_partial_rope(R.rms_norm(q, qn), c, s_)
    kr = R.apply_partial_rope(R.rms_norm(k, kn), c, s_)
    kc2 = torch.zeros(B, KVH, Smax, D)
    vc2 = torch.zeros_like(kc2)
    kc2[:, :, :S] = kr.transpose(1, 2)
    vc2[:, :, :S] = v.transpose(1, 2)
    att = R.attention_prefill(qr.transpose(1, 2), kc2, vc2, 0)  # [B, QH, S, D]
    pre = (att.transpose(1, 2) * torch.sigmoid(gate)).reshape(B, S, QH * D)
    assert torch.allclose(dec, pre, atol=1e-4), (dec - pre).abs().max()
    assert torch.allclose(kc[:, :, :S], kc2[:, :, :S], atol=1e-5)


def test_multi_token_verify_equals_sequential_decode():
    B, n, Smax, start = 2, 4, 16, 3
    qg, k, v, qn, kn = _gqa_inputs(B, start + n, seed=1)
    cos, sin = R.rope_table(Smax, 64, 1e7)
    kc = torch.zeros(B, KVH, Smax, D)
    vc = torch.zeros_like(kc)
    for t in range(start):  # a shared prefix
        R.gqa_decode(qg[:, t], k[:, t], v[:, t], qn, kn, cos, sin, kc, vc, torch.full((B,), t, dtype=torch.int32))
    kc_v, vc_v = kc.clone(), vc.clone()
    seq = [R.gqa_decode(qg[:, start + i], k[:, start + i], v[:, start + i], qn, kn, cos, sin, kc, vc,
                        torch.full((B,), start + i, dtype=torch.int32)) for i in range(n)]
    seq = torch.stack(seq, 1).reshape(B * n, -1)
    rows = slice(start, start + n)
    pos = (torch.arange(n) + start).repeat(B).int()
    ver = R.gqa_decode(qg[:, rows].reshape(B * n, QH, 2 * D), k[:, rows].reshape(B * n, KVH, D),
                       v[:, rows].reshape(B * n, KVH, D), qn, kn, cos, sin, kc_v, vc_v, pos, n_tok=n)
    assert torch.allclose(ver.float(), seq.float(), atol=1e-4)
    assert torch.allclose(kc_v, kc, atol=1e-6) and torch.allclose(vc_v, vc, atol=1e-6)


def test_deltanet_prefill_equals_recurrent_decode():
    B, S, KH, VH, Dk, Dv = 2, 11, 1, 2, 128, 128
    C = 2 * KH * Dk + VH * Dv
    g = torch.Generator().manual_seed(2)
    qkv = torch.randn(B, S, C, generator=g)
    a = torch.randn(B, S, VH, generator=g)
    b = torch.randn(B, S, VH, generator=g)
    z = torch.randn(B, S, VH * Dv, generator=g)
    conv_w = torch.randn(C, 4, generator=g) * 0.3
    A_log = torch.randn(VH, generator=g) * 0.5
    dt_bias = torch.randn(VH, generator=g) * 0.5
    norm_w = torch.randn(Dv, generator=g) * 0.1 + 1
    ring_p, st_p = torch.zeros(B, 4, C), torch.zeros(B, VH, Dk, Dv)
    pre = R.deltanet_prefill(qkv, a, b, z, ring_p, st_p, 0, None, conv_w, A_log, dt_bias, norm_w, KH, Dk, Dv,
                             chunk=4)
    ring_d, st_d = torch.zeros(B, 4, C), torch.zeros(B, VH, Dk, Dv)
    dec = []
    for t in range(S):
        pos = torch.full((B,), t, dtype=torch.int32)
        dec.append(R.deltanet_decode(qkv[:, t], a[:, t], b[:, t], z[:, t], ring_d, st_d, pos, conv_w, A_log,
                                     dt_bias, norm_w, KH, Dk, Dv))
    dec = torch.stack(dec, 1).float()
    err = (pre.float().reshape(dec.shape) - dec).abs().max()
    assert err < 2e-3, err
    assert torch.allclose(st_p, st_d, atol=1e-3)
    # the next decode step reads the last 3 inputs (positions S-3..S-1) from slots position % 4;
    # the fourth slot is overwritten by that step before it is read
    slots = [(S - 3 + i) % 4 for i in range(3)]
    assert torch.allclose(ring_p[:, slots], ring_d[:, slots], atol=1e-6)
