"""Tensor-parallel Qwen3.6 on gloo CPU ranks equals the single-rank model: the
sharding math of ``tp_dims`` (DeltaNet and attention heads split, KV heads
replicated when ``tp > kv_heads``, experts partitioned ``E/tp``), the
row-parallel all-reduces, the vocab-sharded LM head and the int64-max greedy
(the reference's ``model_dims.py:99-127`` plan and ``test_moe_decode_model_device.py``
tier, run here as real ranks over gloo); the MoE runs with experts
partitioned across ranks and with every expert sliced across ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, moe, sharding, q, shard_embed=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), BWN_SHARD_EMBED="1" if shard_embed else "0")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from dataclasses import replace

        from bwn.config import tiny_qwen36
        from bwn.models.qwen36 import build_qwen36
        from bwn.parallel.comm import Comm
        torch.set_num_threads(2)  # ranks share the host's cores
        cfg = replace(tiny_qwen36(moe=moe), dn_k_heads=4, dn_v_heads=8)  # DeltaNet heads split over 4
        comm = Comm(None, rank, world)
        from bwn.parallel.topology import hosts_of, require_single_domain
        require_single_domain(comm, "test")  # every rank on this host: the collective check passes
        assert len(hosts_of(comm)) == world
        tp = build_qwen36(cfg, comm, seed=3, dtype=torch.float32, moe_sharding=sharding)
        one = build_qwen36(cfg, Comm.single(), seed=3, dtype=torch.float32)
        B, S = 3, 9
        toks = torch.randint(0, cfg.vocab, (B, S), generator=torch.Generator().manual_seed(5))
        st_tp, st_one = tp.new_state(B, 32), one.new_state(B, 32)
        h_tp, h_one = tp.prefill_hidden(toks, st_tp), one.prefill_hidden(toks, st_one)
        err = float((tp.logits(h_tp) - one.logits(h_one)).abs().max())
        ids_tp, ids_one = tp.greedy(h_tp), one.greedy(h_one)
        same = torch.equal(ids_tp, ids_one)
        for _ in range(3):
            h_tp, h_one = tp.decode_hidden(ids_tp.int(), st_tp), one.decode_hidden(ids_one.int(), st_one)
            err = max(err, float((tp.logits(h_tp) - one.logits(h_one)).abs().max()))
            ids_tp, ids_one = tp.greedy(h_tp), one.greedy(h_one)
            same = same and torch.equal(ids_tp, ids_one)
        assert tp.shard_embed == shard_embed
        if shard_embed:
            assert tp.g["embed"].shape[0] == cfg.vocab // world
        q.put((rank, err, same, tp.d.kv_heads, tp.d.q_heads))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc(), False, 0, 0))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,moe,sharding,shard_embed", [(2, False, "ep", False), (4, False, "ep", False),
                                                            (2, True, "ep", False), (4, True, "ep", False),
                                                            (4, True, "tp", False), (2, False, "ep", True)])
def test_tp_ranks_match_single_rank(world, moe, sharding, shard_embed):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, world, port, moe, sharding, q, shard_embed)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    for rank, err, same, kvh, qh in res:
        assert not isinstance(err, str), err
        assert err < 2e-3, (rank, err)
        assert same, f"rank {rank}: greedy ids differ from the single-rank model"
        assert qh * world == 4
        # 2 KV heads: split over 2 ranks, replicated (one per rank) over 4
        assert kvh == (1 if world >= 2 else 2)
