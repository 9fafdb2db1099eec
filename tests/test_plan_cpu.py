"""The DTensor-style plan API on two gloo CPU ranks: HF ``EsmForMaskedLM``
sharded with the reference's layer plan written with torch's
``ColwiseParallel`` / ``RowwiseParallel`` objects (``contrib/esm2/run_esm.py:49-69``)
gives the unsharded model's logits and, after backward, the matching slices
of its gradients; wildcard keys, a vocab-parallel embedding and error cases."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _hf_esm():
    from transformers import EsmConfig, EsmForMaskedLM
    torch.manual_seed(0)
    cfg = EsmConfig(vocab_size=34, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                    intermediate_size=128, position_embedding_type="rotary", pad_token_id=1, mask_token_id=32,
                    token_dropout=False, hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0)
    return EsmForMaskedLM(cfg).eval()


def _rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        torch.set_num_threads(2)
        from torch.distributed.tensor.parallel import ColwiseParallel, RowwiseParallel

        from bwn.parallel.comm import Comm
        from bwn.parallel.plan import Rowwise, parallelize_module
        comm = Comm(None, rank, 2)
        full = _hf_esm()
        tp = _hf_esm()  # same seed: same weights
        plan = {"attention.self.query": ColwiseParallel(), "attention.self.key": ColwiseParallel(),
                "attention.self.value": ColwiseParallel(), "attention.output.dense": RowwiseParallel(),
                "intermediate.dense": ColwiseParallel(), "output.dense": RowwiseParallel()}
        for layer in tp.esm.encoder.layer:
            parallelize_module(layer, comm, plan)
        parallelize_module(tp, comm, {"esm.embeddings.word_embeddings": Rowwise()})
        ids = torch.randint(4, 24, (2, 10), generator=torch.Generator().manual_seed(3))
        ref = full(ids).logits
        got = tp(ids).logits
        err = float((got - ref).abs().max())
        ref.square().mean().backward()
        got.square().mean().backward()
        n = 64 // 2
        g_full = full.esm.encoder.layer[1].attention.self.query.weight.grad[rank * n:(rank + 1) * n]
        g_tp = tp.esm.encoder.layer[1].attention.self.query.weight.grad
        gerr = float((g_full - g_tp).abs().max())
        m = 128 // 2
        g_full2 = full.esm.encoder.layer[0].output.dense.weight.grad[:, rank * m:(rank + 1) * m]
        gerr = max(gerr, float((g_full2 - tp.esm.encoder.layer[0].output.dense.weight.grad).abs().max()))
        ew = tp.esm.embeddings.word_embeddings.weight
        q.put((rank, err, gerr, tuple(ew.shape)))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc(), 0.0, ()))
    finally:
        dist.destroy_process_group()


def test_reference_plan_on_hf_esm_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in ps:
        p.join(60)
    for rank, err, gerr, eshape in res:
        assert not isinstance(err, str), err
        assert err < 1e-4, (rank, err)
        assert gerr < 1e-5, (rank, gerr)
        assert eshape == (17, 64)  # vocab-parallel embedding: half the rows per rank


def test_plan_matching_and_errors():
    from bwn.parallel.comm import Comm
    from bwn.parallel.plan import _matches, _style, parallelize_module
    assert _matches("layers.*.attn.wo_b", "layers.3.attn.wo_b")
    assert not _matches("layers.*.attn.wo_b", "layers.3.attn.wo_b.inner")
    assert _style("colwise") == "colwise" and _style("Rowwise") == "rowwise"
    with pytest.raises(ValueError):
        _style("sequence")
    m = nn.Sequential(nn.Linear(8, 8), nn.ReLU())
    assert parallelize_module(m, Comm.single(), {"0": "colwise"}) is m  # one rank: unchanged
    assert isinstance(m[0], nn.Linear)
    two = Comm(None, 0, 2)  # no collective runs while sharding
    with pytest.raises(KeyError):
        parallelize_module(nn.Sequential(nn.Linear(8, 8)), two, {"missing": "colwise"})
    with pytest.raises(TypeError):
        parallelize_module(nn.Sequential(nn.ReLU()), two, {"0": "colwise"})
    s = parallelize_module(nn.Sequential(nn.Linear(8, 6), nn.Linear(6, 8)), two, {"0": "colwise", "1": "rowwise"})
    assert s[0].weight.shape == (3, 8) and s[1].weight.shape == (8, 3)
