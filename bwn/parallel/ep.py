"""Expert-parallel MoE with an all-to-all over NVLink peer memory.

The reference runs expert parallelism as masked-dense expert compute on every
rank followed by an all-reduce of the partial outputs
(``contrib/qwen3.6-35b-a3b/static_decode_35b.py:811-821, 1183``).  Here each
rank owns a slice of the tokens and ``E / W`` experts, and the routed rows move:

1. ``ep_dispatch`` (``csrc/comm/ep_a2a.cu``): per-(destination, expert) counts
   are all-gathered by peer stores, every (token, slot) row is written into its
   owner's expert-major receive buffer, a flag marks completion;
2. the owner runs the grouped tcgen05 expert GEMMs (gate/up + SwiGLU, down) on
   the receive buffer, with the per-expert counts left on the device;
3. ``ep_return`` writes each output row back into its source's combine buffer
   at ``[token, slot]``;
4. ``moe_combine`` takes the router-weighted sum of the slots plus the gated
   shared expert.

No host synchronisation: the whole block is CUDA-graph capturable.  Buffers
are symmetric allocations (``torch.distributed._symmetric_memory`` maps them);
every device wait is bounded and reports through the status word.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops as O
from ..ops import _ext


class EPAllToAll:
    def __init__(self, comm, hidden: int, n_experts: int, top_k: int, max_tokens: int,
                 max_recv: int | None = None, device=None, timeout_s: float = 5.0):
        self.comm = comm
        self.W, self.rank = comm.size, comm.rank
        if n_experts % self.W:
            raise ValueError("experts must divide evenly over the ranks")
        self.H, self.k, self.E = hidden, top_k, n_experts
        self.e_local = n_experts // self.W
        self.T_max = max_tokens
        # worst case: every rank's every (token, slot) pair lands here
        self.max_recv = max_recv or self.W * max_tokens * top_k
        self.timeout_s = timeout_s
        dev = device or torch.device("cuda", torch.cuda.current_device())
        C = _ext.require()
        self.off = list(C.ep_layout(self.W, self.e_local, hidden, top_k, self.T_max, self.max_recv))
        group = comm.group or dist.group.WORLD
        from .symm import allocate
        self.buf, self.hdl = allocate(self.off[5], group, dev, "ep_all_to_all")
        self.peer_base = [int(p) for p in self.hdl.buffer_ptrs]
        self.state = torch.zeros(16 + 2 * self.e_local + 1 + self.W * self.e_local, dtype=torch.int32, device=dev)
        self.recv_x = self.buf[self.off[3]:self.off[3] + self.max_recv * hidden * 2].view(torch.bfloat16).view(
            self.max_recv, hidden)
        self.comb = self.buf[self.off[4]:self.off[4] + self.T_max * top_k * hidden * 2].view(torch.bfloat16).view(
            self.T_max * top_k, hidden)
        self.counts = self.state[16:16 + self.e_local]
        self.offsets = self.state[16 + self.e_local:16 + 2 * self.e_local + 1]
        self.pos_identity = torch.arange(self.T_max * top_k, dtype=torch.int32, device=dev)
        self.hdl.barrier()
        torch.cuda.synchronize(dev)

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor) -> None:
        O.ops().ep_dispatch(x, ids.int().contiguous(), self.peer_base, self.rank, self.e_local, self.T_max,
                            self.max_recv, self.state, self.timeout_s)

    def give_back(self, y: torch.Tensor, T: int) -> None:
        O.ops().ep_return(y, self.peer_base, self.rank, self.e_local, self.k, T, self.T_max, self.max_recv,
                          self.state, self.timeout_s)

    def moe(self, x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, gate_up: torch.Tensor, down: torch.Tensor,
            shared=None, swiglu_limit: float = 0.0) -> torch.Tensor:
        """Routed MoE output ``[T, H]`` of this rank's tokens ``x`` (routing ``w``,
        ``ids`` with global expert ids), experts of this rank in ``gate_up`` /
        ``down``; ``shared = (shared_y [T, H], shared_gate_logit [T, 1])``."""
        T = x.shape[0]
        self.dispatch(x, ids)
        if hasattr(gate_up, "scales16"):  # block-scaled fp8 experts (bwn.io.fp8.FP8Experts)
            y = O.ops().moe_grouped_ffn_w8(self.recv_x, self.counts, self.offsets, gate_up.w8, gate_up.scales16,
                                           down.w8, down.scales16, self.max_recv, swiglu_limit)
        else:
            y = O.ops().moe_grouped_ffn(self.recv_x, self.counts, self.offsets, gate_up, down, self.max_recv,
                                        swiglu_limit)
        self.give_back(y, T)
        sy, sg = shared if shared is not None else (None, None)
        sg = sg.float().reshape(-1).contiguous() if sg is not None else None
        return O.ops().moe_combine(self.comb[:T * self.k], w.float().contiguous(), self.pos_identity[:T * self.k],
                                   sy, sg)


def enable_ep_all_to_all(model, max_tokens_per_rank: int = 512, min_tokens_per_rank: int = 16) -> EPAllToAll:
    """Route a Qwen3.6 MoE model's expert layers through the NVLink all-to-all
    when a step has at least ``min_tokens_per_rank`` tokens per rank (prefill,
    large batches); smaller steps keep the all-reduce formulation, which needs
    fewer cross-GPU round trips.  The shared expert is made replicated (its
    tensor-parallel slices are all-gathered once) since each rank then runs it
    on its own token slice."""
    cfg, comm = model.cfg, model.comm
    if not cfg.is_moe or comm.size <= 1:
        raise RuntimeError("expert-parallel all-to-all needs a MoE model on more than one rank")
    from .topology import require_single_domain
    require_single_domain(comm, "expert-parallel all-to-all")
    if model.d.moe_sharding != "ep":
        raise RuntimeError("the expert-parallel all-to-all needs experts partitioned across ranks (moe_sharding='ep')")
    ep = EPAllToAll(comm, cfg.hidden, cfg.num_experts, cfg.top_k, max_tokens_per_rank, device=model.device)
    ep.min_tokens = min_tokens_per_rank
    for L in model.layers:
        L["shared_gate_up_full"] = comm.all_gather_first(L["shared_gate_up"].contiguous())
        L["shared_down_full"] = comm.all_gather_last(L["shared_down"].contiguous()).contiguous()
    model.ep_a2a = ep
    return ep


def nccl_ep_moe(comm, x, w, ids, gate_up, down, e_local: int, shared=None, swiglu_limit: float = 0.0):
    """Baseline: the same expert-parallel block with NCCL (or gloo) all-to-all
    and host-side split sizes (one device sync per call)."""
    W, rank, k, H = comm.size, comm.rank, ids.shape[1], x.shape[1]
    T = x.shape[0]
    flat = ids.reshape(-1).long()
    dst = flat // e_local
    order = torch.argsort(dst, stable=True)
    send_counts = torch.bincount(dst, minlength=W)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=comm.group)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    rows = x[(order // k)]
    meta = torch.stack([flat[order], order], 1)  # (global expert, pair index)
    r_rows = x.new_empty(sum(rc), H)
    r_meta = meta.new_empty(sum(rc), 2)
    dist.all_to_all_single(r_rows, rows.contiguous(), rc, sc, group=comm.group)
    dist.all_to_all_single(r_meta, meta.contiguous(), rc, sc, group=comm.group)
    e_loc = (r_meta[:, 0] - rank * e_local).int()
    ones = torch.ones(r_rows.shape[0], 1, device=x.device)
    y = O.moe_experts(r_rows, ones, e_loc[:, None], gate_up, down, 0, swiglu_limit=swiglu_limit) \
        if r_rows.shape[0] else r_rows
    back = x.new_empty(T * k, H)
    dist.all_to_all_single(back, y.contiguous(), sc, rc, group=comm.group)
    out_rows = x.new_empty(T * k, H)
    out_rows[order] = back
    res = (out_rows.view(T, k, H).float() * w.float()[..., None]).sum(1)
    if shared is not None:
        sy, sg = shared
        res = res + torch.sigmoid(sg.float().reshape(T, 1)) * sy.float()
    return res.to(x.dtype)
