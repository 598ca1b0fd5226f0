"""Expert-parallel LFM2-MoE block over a torch.distributed process group (one process per GPU).

The reference runs every expert of `Lfm2Engine._moEFFN` (lfm2-engine.js:413-487) in one
process.  Here the experts of a layer are sharded evenly over G ranks: rank r owns experts
[r E/G, (r+1) E/G) and its own T token rows.  One forward:

1. route the rank's tokens (`qq_moe_route`: router logits, sigmoid, top-k, weights;
   lfm2-engine.js:417-447);
2. group the (token, slot) pairs by the rank owning their expert and exchange the counts, then
   the token rows and local expert ids (all-to-all: NCCL over NVLink on GPUs, gloo in the CPU
   tests);
3. run the rank's experts on the rows it received (`qq_moe_experts`: rows regrouped by expert,
   tensor-core GEMMs);
4. send the expert outputs back with a second all-to-all;
5. combine them per token in slot order with the routing weights (`qq_moe_combine`;
   lfm2-engine.js:459-486).

The exchange is plumbing (torch.distributed); the arithmetic is the library's.  `ep_forward`
takes the three compute steps as callables so the exchange logic is testable on CPU.
"""

from __future__ import annotations

import numpy as np

from . import runtime


def plan_dispatch(idx, n_local: int, world: int):
    """(order, send_counts, pos, eid) for routed ids idx [T][k] (torch, any device):
    order  - the T*k (token, slot) pairs sorted by destination rank (stable: token order within),
    send_counts - pairs per destination rank,
    pos    - [T][k] int32: where pair (t, s) sits in `order` (and in the returned rows),
    eid    - the destination-local expert id of each pair in `order`."""
    import torch

    T, k = idx.shape
    flat = idx.reshape(-1).long()
    dest = flat // n_local
    order = torch.argsort(dest, stable=True)
    send_counts = torch.bincount(dest, minlength=world)
    pos = torch.empty_like(order)
    pos[order] = torch.arange(order.numel(), device=idx.device)
    eid = (flat[order] % n_local).to(torch.int32)
    return order, send_counts, pos.view(T, k).to(torch.int32), eid


def ep_forward(x, route_fn, experts_fn, combine_fn, n_expert: int, top_k: int, group=None):
    """The expert-parallel MoE block on this rank's rows x [T][K] (see the module docstring).
    route_fn(x) -> (idx [T][k] int32 global ids, w [T][k]); experts_fn(rows [R][K], eid [R]) ->
    [R][K]; combine_fn(rows [T*k][K], pos [T][k], w) -> [T][K]."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if n_expert % world:
        raise ValueError(f"{n_expert} experts do not shard evenly over {world} ranks")
    n_local = n_expert // world
    T, K = x.shape
    idx, w = route_fn(x)
    order, send_counts, pos, send_eid = plan_dispatch(idx, n_local, world)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    send_rows = x.index_select(0, order // top_k)
    recv_rows = x.new_empty((sum(rc), K))
    dist.all_to_all_single(recv_rows, send_rows, rc, sc, group=group)
    recv_eid = send_eid.new_empty(sum(rc))
    dist.all_to_all_single(recv_eid, send_eid, rc, sc, group=group)
    y = experts_fn(recv_rows, recv_eid)
    back = x.new_empty((T * top_k, K))
    dist.all_to_all_single(back, y.contiguous(), sc, rc, group=group)
    return combine_fn(back, pos, w)


Q8_0_BLOCK = 34  # bytes per 32 weights


def expert_slice(raw: np.ndarray, ne, e0: int, n: int):
    """Bytes and shape of experts [e0, e0 + n) of a packed Q8_0 expert tensor [K, N, E] (expert
    e at byte offset e * N * K/32 * 34, lfm2-engine.js:490-505)."""
    K, N, E = (int(v) for v in ne)
    stride = N * (K // 32) * Q8_0_BLOCK
    flat = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
    return flat[e0 * stride:(e0 + n) * stride], [K, N, n]


class EPMoEBlock:
    """One LFM2-MoE layer, experts sharded over the ranks of `group` (this process: `rank`).
    tensors: GGUF name -> (ggml type, ne, raw bytes) of the layer (`prefix` + suffix names)."""

    SUFFIX = {slot: runtime.SLOT_TENSOR_NAMES[slot]
              for slot in ("ffn_gate_inp", "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps", "exp_probs_b")}

    def __init__(self, ctx: runtime.Context, tensors: dict, prefix: str, n_expert: int, top_k: int,
                 rank: int, world: int, group=None):
        if n_expert % world:
            raise ValueError(f"{n_expert} experts do not shard evenly over {world} ranks")
        self.ctx, self.n_expert, self.top_k, self.group = ctx, n_expert, top_k, group
        self.n_local = n_expert // world
        e0 = rank * self.n_local
        self.layer = runtime.LayerDesc()
        self.layer.is_moe = 1
        self._keep = []
        for slot, suffix in self.SUFFIX.items():
            name = prefix + suffix
            if name not in tensors:
                continue
            t, ne, raw = tensors[name]
            if slot.endswith("_exps"):
                raw, ne = expert_slice(raw, ne, e0, self.n_local)
            h = ctx.upload(raw, t, ne)
            self._keep.append(h)
            self.layer.t[runtime.SLOT[slot]] = h.h.value
        self.K = int(tensors[prefix + self.SUFFIX["ffn_gate_inp"]][1][0])

    def forward(self, x):
        """x [T][K] float32 on this rank's GPU -> the MoE output rows (sum_k w_k expert_k(x))."""
        import torch

        self.ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        T, K, k = x.shape[0], self.K, self.top_k
        ctx, L = self.ctx, self.layer

        def route(xx):
            idx = torch.empty((T, k), dtype=torch.int32, device=xx.device)
            w = torch.empty((T, k), dtype=torch.float32, device=xx.device)
            ctx.moe_route(L, self.n_expert, k, xx, T, idx, w)
            return idx, w

        def experts(rows, eid):
            y = torch.empty_like(rows)
            ctx.moe_experts(L, self.n_local, rows, eid, rows.shape[0], y)
            return y

        def combine(rows, pos, w):
            out = torch.empty((T, K), dtype=torch.float32, device=rows.device)
            ctx.moe_combine(rows, pos, w, T, k, K, out)
            return out

        return ep_forward(x.contiguous(), route, experts, combine, self.n_expert, k, self.group)

    def close(self) -> None:
        for h in self._keep:
            h.free()
        self._keep = []
