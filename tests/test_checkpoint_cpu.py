"""Checkpoint I/O: safetensors reader/writer, HF-layout loading for Qwen3.6
(packed / per-expert / official FP8 experts, nested prefixes) and the DeepSeek V4
FP4/FP8 preprocessing + per-rank shards."""
import json
import os

import pytest
import torch

from bwn.config import tiny_deepseek_v4, tiny_qwen36
from bwn.io import deepseek_weights as DW
from bwn.io.checkpoint import Checkpoint
from bwn.io.fp8 import dequantize_block, expand_block_scales, quantize_block
from bwn.io.qwen36_weights import synthetic_hf_globals, synthetic_hf_layer
from bwn.io.safetensors import SafeReader, save_file, save_sharded
from bwn.models.deepseek_v4 import DeepSeekV4Model, synthetic_checkpoint
from bwn.models.qwen36 import build_qwen36
from bwn.parallel.comm import Comm


def test_safetensors_roundtrip_all_dtypes(tmp_path):
    g = torch.Generator().manual_seed(0)
    ts = {
        "f32": torch.randn(3, 5, generator=g),
        "bf16": torch.randn(7, 2, generator=g).bfloat16(),
        "f16": torch.randn(4, generator=g).half(),
        "i64": torch.arange(6).reshape(2, 3),
        "i32": torch.arange(5, dtype=torch.int32),
        "u8": torch.randint(0, 255, (9,), dtype=torch.uint8, generator=g),
        "bool": torch.tensor([True, False, True]),
        "scalar": torch.tensor(3.5),
        "empty": torch.zeros(0, 4),
    }
    p = str(tmp_path / "a.safetensors")
    save_file(ts, p, metadata={"format": "pt"})
    r = SafeReader(p)
    assert sorted(r.keys()) == sorted(ts)
    assert r.metadata == {"format": "pt"}
    for k, v in ts.items():
        got = r.get(k)
        assert got.dtype == v.dtype and got.shape == v.shape and torch.equal(got, v), k


def test_safetensors_interop_with_library(tmp_path):
    st = pytest.importorskip("safetensors.torch")
    ts = {"w": torch.randn(8, 16).bfloat16(), "b": torch.randn(16)}
    mine, theirs = str(tmp_path / "mine.safetensors"), str(tmp_path / "theirs.safetensors")
    save_file(ts, mine)
    st.save_file(ts, theirs)
    lib = st.load_file(mine)
    r = SafeReader(theirs)
    for k in ts:
        assert torch.equal(lib[k], ts[k]) and torch.equal(r.get(k), ts[k])


def test_fp8_tag_kept_as_bytes(tmp_path):
    w = torch.randn(256, 128)
    w8, s = quantize_block(w)
    p = str(tmp_path / "f.safetensors")
    save_file({"x.weight": w8, "x.weight_scale_inv": s.bfloat16()}, p, dtype_tags={"x.weight": "F8_E4M3"})
    ck = Checkpoint(p, prefix="")
    assert ck.tag("x.weight") == "F8_E4M3"
    deq = ck.get("x.weight")
    ref = dequantize_block(w8, s.bfloat16().float()).bfloat16()
    assert torch.equal(deq, ref)
    kept = ck.get("x.weight", fp8="keep")
    assert torch.equal(kept.w8, w8)


def _hf_state(cfg, seed=0):
    sd = {}
    for i in range(cfg.num_layers):
        sd.update({f"layers.{i}." + k if not k.startswith("layers.") else k: v
                   for k, v in synthetic_hf_layer(cfg, i, seed, "cpu").items()})
    sd.update(synthetic_hf_globals(cfg, seed, "cpu"))
    return sd


def _strip(sd):
    return {k[len("model."):] if k.startswith("model.") else k: v for k, v in sd.items()}


@pytest.mark.parametrize("moe", [False, True])
def test_qwen36_load_from_sharded_checkpoint(tmp_path, moe):
    cfg = tiny_qwen36(moe=moe, layers=4)
    sd = _strip(_hf_state(cfg))
    on_disk = {"model.language_model." + k if k != "lm_head.weight" else k: v for k, v in sd.items()}
    if moe:  # write the per-expert layout
        for i in range(cfg.num_layers):
            p = f"model.language_model.layers.{i}.mlp.experts."
            gu, dn = on_disk.pop(p + "gate_up_proj"), on_disk.pop(p + "down_proj")
            for e in range(gu.shape[0]):
                on_disk[f"{p}{e}.gate_proj.weight"] = gu[e, :cfg.moe_inter]
                on_disk[f"{p}{e}.up_proj.weight"] = gu[e, cfg.moe_inter:]
                on_disk[f"{p}{e}.down_proj.weight"] = dn[e]
    save_sharded(on_disk, str(tmp_path), max_shard_bytes=1 << 20)
    assert len([f for f in os.listdir(tmp_path) if f.endswith(".safetensors")]) > 1
    a = build_qwen36(cfg, hf_state=sd, device="cpu")
    b = build_qwen36(cfg, checkpoint=str(tmp_path), device="cpu")
    for La, Lb in zip(a.layers, b.layers):
        assert La.keys() == Lb.keys()
        for k in La:
            assert torch.equal(La[k], Lb[k]), k
    for k in a.g:
        assert torch.equal(a.g[k], b.g[k]), k


def test_qwen36_official_fp8_experts(tmp_path):
    cfg = tiny_qwen36(moe=True, layers=4)
    sd = _strip(_hf_state(cfg))
    on_disk, tags = {}, {}
    deq = dict(sd)
    for k, v in sd.items():
        if ".mlp.experts." in k:
            continue
        on_disk[k] = v
    for i in range(cfg.num_layers):
        p = f"layers.{i}.mlp.experts."
        gu, dn = sd[p + "gate_up_proj"], sd[p + "down_proj"]
        gus, dns = [], []
        for e in range(gu.shape[0]):
            for name, w in (("gate_proj", gu[e, :cfg.moe_inter]), ("up_proj", gu[e, cfg.moe_inter:]),
                            ("down_proj", dn[e])):
                w8, s = quantize_block(w.float())
                key = f"{p}{e}.{name}.weight"
                on_disk[key], on_disk[key + "_scale_inv"] = w8, s.bfloat16()
                tags[key] = "F8_E4M3"
                d = dequantize_block(w8, s.bfloat16().float()).bfloat16()
                (gus if name != "down_proj" else dns).append(d)
        deq[p + "gate_up_proj"] = torch.stack([torch.cat(gus[2 * e:2 * e + 2]) for e in range(gu.shape[0])])
        deq[p + "down_proj"] = torch.stack(dns)
    save_file({("model." + k): v for k, v in on_disk.items()}, str(tmp_path / "model.safetensors"),
              dtype_tags={("model." + k): v for k, v in tags.items()})
    a = build_qwen36(cfg, hf_state=deq, device="cpu")
    b = build_qwen36(cfg, checkpoint=str(tmp_path), device="cpu")
    for La, Lb in zip(a.layers, b.layers):
        for k in ("experts_gate_up", "experts_down"):
            assert torch.equal(La[k], Lb[k])
    # kept fp8 (no dequantize / requantize): the same weights once dequantized
    c = build_qwen36(cfg, checkpoint=str(tmp_path), device="cpu", fp8_experts=True)
    for Lb, Lc in zip(b.layers, c.layers):
        for k in ("experts_gate_up", "experts_down"):
            assert hasattr(Lc[k], "scales16")
            assert torch.equal(Lc[k].dequant().to(torch.bfloat16), Lb[k])
    # experts sliced across two simulated ranks (tensor parallelism within experts)
    from bwn.models.qwen36 import Qwen36Model
    from bwn.io.checkpoint import Checkpoint
    from bwn.parallel.comm import Comm
    ck = Checkpoint(str(tmp_path))
    for r in range(2):
        m = Qwen36Model(cfg, Comm(None, r, 2), "cpu", torch.bfloat16, moe_sharding="tp")
        m.load_hf(ck.getter(), fp8_experts=lambda i, e0, e1, c0, w: ck.fp8_experts(f"layers.{i}.", e0, e1, c0, w))
        ref = Qwen36Model(cfg, Comm(None, r, 2), "cpu", torch.bfloat16, moe_sharding="tp").load_hf(ck.getter())
        for Lm, Lr in zip(m.layers, ref.layers):
            for k in ("experts_gate_up", "experts_down"):
                assert torch.equal(Lm[k].dequant().to(torch.bfloat16), Lr[k]), (r, k)
    ck.close()


def test_fp4_e2m1_decode_table():
    codes = torch.arange(16)
    want = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
    assert DW.decode_fp4_e2m1(codes).tolist() == want
    assert DW.decode_e8m0(torch.tensor([127, 128, 120], dtype=torch.uint8)).tolist() == [1.0, 2.0, 2.0 ** -7]


def _fp4_pack(w: torch.Tensor):
    """Quantize ``w [out, in]`` to packed E2M1 with power-of-two scales per 32."""
    out_f, in_f = w.shape
    blocks = w.reshape(out_f, in_f // 32, 32)
    amax = blocks.abs().amax(-1).clamp_min(1e-8)
    e = torch.ceil(torch.log2(amax / 6.0)).clamp(-127, 127)
    scale = torch.exp2(e)
    table = DW.decode_fp4_e2m1(torch.arange(16))
    q = (blocks / scale[..., None]).reshape(out_f, in_f)
    codes = (q[..., None] - table).abs().argmin(-1).to(torch.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    return packed.view(torch.int8), (e + 127).to(torch.uint8)


def test_deepseek_preprocess_tp2_matches_full(tmp_path):
    cfg = tiny_deepseek_v4()
    sd = synthetic_checkpoint(cfg, 0)
    src = {}
    tags = {}
    for k, v in sd.items():
        if ".experts_w" in k:  # write experts per index, FP4
            f, n = k.rsplit(".experts_", 1)
            for e in range(v.shape[0]):
                key = f"{f}.experts.{e}.{n}.weight"
                packed, sc = _fp4_pack(v[e].float())
                src[key], src[key[:-len(".weight")] + ".scale"] = packed, sc
                tags[key[:-len(".weight")] + ".scale"] = "F8_E8M0"
        elif k.endswith("wq_b.weight") or k.endswith("wo_b.weight"):  # dense FP8 with E8M0 block scales
            _, s = quantize_block(v.float())
            e8 = torch.ceil(torch.log2(s)).clamp(-127, 127)  # power-of-two block scales (E8M0)
            w8 = (v.float() / expand_block_scales(torch.exp2(e8), v.shape)).to(torch.float8_e4m3fn).view(torch.uint8)
            src[k], src[k[:-len(".weight")] + ".scale"] = w8, (e8 + 127).to(torch.uint8)
            tags[k], tags[k[:-len(".weight")] + ".scale"] = "F8_E4M3", "F8_E8M0"
        else:
            src[k] = v
    indir, outdir = tmp_path / "in", tmp_path / "out"
    os.makedirs(indir)
    save_file(src, str(indir / "model.safetensors"), dtype_tags=tags)
    cfg_json = {"n_routed_experts": cfg.n_routed_experts}
    with open(indir / "config.json", "w") as f:
        json.dump(cfg_json, f)
    DW.preprocess(str(indir), str(outdir), tp=2, mode="bf16")
    # the oracle: the full checkpoint dequantized by the same decoders
    full = {}
    r = SafeReader(str(indir / "model.safetensors"))
    for k in r.keys():
        if k.endswith(".scale"):
            continue
        full.update(DW.convert_tensor(r, k, "bf16"))
    for rank in range(2):
        comm = Comm(None, rank, 2)
        a = DeepSeekV4Model(cfg, comm).load(full)
        b = DeepSeekV4Model(cfg, comm).load_checkpoint(str(outdir))
        for La, Lb in zip(a.L, b.L):
            for k in La:
                va, vb = La[k], Lb[k]
                if isinstance(va, tuple):
                    assert all(torch.equal(x, y) for x, y in zip(va, vb)), k
                elif va is not None:
                    assert torch.equal(va, vb), (rank, k)
    # FP4 dequant is close to the original weights (E2M1 has 1 mantissa bit)
    w = sd["layers.0.ffn.experts_w1"][0].float()
    d = full["layers.0.ffn.experts.0.w1.weight"].float()
    assert (d - w).abs().max() <= w.abs().max() * 0.35
