"""Shared helpers of the speculative-decoding tests (not collected)."""
import torch


def dn_params(KH, VH, device, seed=0):
    g = torch.Generator().manual_seed(seed)
    C = 2 * KH * 128 + VH * 128
    return dict(
        C=C,
        conv_w=(torch.randn(C, 4, generator=g) * 0.5).to(device),
        A_log=(torch.rand(VH, generator=g) * 2).to(device),
        dt_bias=(torch.randn(VH, generator=g) * 0.1).to(device),
        norm_w=(torch.randn(128, generator=g) * 0.1 + 1).to(device),
    )


def dn_rows(n, KH, VH, device, gen):
    """qkv, z, a, b rows ``[n, *]`` as column views of one projection output."""
    C = 2 * KH * 128 + VH * 128
    fused = torch.randn(n, C + VH * 128 + 2 * VH, generator=gen).bfloat16().to(device)
    return fused[:, :C], fused[:, C:C + VH * 128], fused[:, C + VH * 128 + VH:], fused[:, C + VH * 128:C + VH * 128 + VH]
