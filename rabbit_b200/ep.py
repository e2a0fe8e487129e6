"""Expert parallelism for the routed-MoE layer: one process per GPU, experts split in contiguous
blocks (expert e on rank e // (E / N)), tokens owned by the rank that holds them, router and shared
expert replicated.

One forward on every rank:

1. route the rank's own tokens with the replicated router (bit-exact, same kernel as one GPU);
2. exchange counts, then token rows and their (expert, weight) slots with ``all_to_all_single``
   (variable splits), each slot sent to the rank owning its expert;
3. run the received rows through the local experts with the routing weights folded in
   (``forward_routed``: rabbit's ``apply_single_expert`` loop, src/glm52/moe.rs:463-513);
4. send the weighted expert outputs back the same way;
5. on the token's owner: ``out[t] = ((y_0 + y_1) + ... + y_{k-1}) + shared(x_t)`` in routing rank
   order with the gated shared expert last (qwen38/generate.rs:324-349), a fixed order on every
   world size.

There is no all-reduce: the only collectives are the two data exchanges (and the counts), which
the reference has no counterpart for (it runs on one host). The compute side is any object with
``route(x) -> (ids, weights)``, ``forward_routed(x, ids, weights, with_shared) -> out`` and
``hidden``/``topk``/``n_experts`` attributes: the device layer (``MoeLayer``) on GPUs.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class ExpertParallelMoe:
    def __init__(self, layer, group=None, max_rows=None):
        self.layer = layer
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if layer.n_experts % self.world:
            raise ValueError(f"{layer.n_experts} experts do not split over {self.world} ranks")
        self.per_rank = layer.n_experts // self.world
        # rows per forward_routed call: at most the layer's max_tokens
        self.max_rows = max_rows or getattr(layer, "max_tokens", None)

    def _exchange(self, send, send_counts, recv_counts):
        """Variable-split all-to-all of the leading dimension."""
        out = torch.empty((int(sum(recv_counts)),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        dist.all_to_all_single(out, send.contiguous(), [int(c) for c in recv_counts], [int(c) for c in send_counts],
                               group=self.group)
        return out

    def forward(self, x):
        """x [T_local, H] on this rank's device -> out [T_local, H] f32."""
        lay = self.layer
        T, k, H = x.shape[0], lay.topk, lay.hidden
        dev = x.device
        ids, w = lay.route(x)                                   # [T, k] rank order, bit-exact
        flat_ids = ids.reshape(-1).long()
        valid = flat_ids >= 0
        dest = torch.where(valid, flat_ids // self.per_rank, torch.full_like(flat_ids, self.world))
        order = torch.argsort(dest * (T * k) + torch.arange(T * k, device=dev), stable=True)
        order = order[: int(valid.sum())]                       # slots grouped by rank, (t, j) inside
        send_counts = torch.bincount(dest[order], minlength=self.world)[: self.world]
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        tok = order // k
        send_x = x[tok]
        send_meta = torch.stack([flat_ids[order].to(torch.float32), w.reshape(-1)[order]], dim=1)
        recv_x = self._exchange(send_x, sc, rc)
        recv_meta = self._exchange(send_meta, sc, rc)
        # the local experts: one slot per received row (the other k-1 slots empty)
        R = recv_x.shape[0]
        y = torch.empty((R, H), dtype=torch.float32, device=dev)
        if R:
            rid = torch.full((R, k), -1, dtype=torch.int32, device=dev)
            rw = torch.zeros((R, k), dtype=torch.float32, device=dev)
            rid[:, 0] = recv_meta[:, 0].round().to(torch.int32)
            rw[:, 0] = recv_meta[:, 1]
            step = self.max_rows or R
            for r0 in range(0, R, step):
                r1 = min(R, r0 + step)
                y[r0:r1] = lay.forward_routed(recv_x[r0:r1], rid[r0:r1].contiguous(), rw[r0:r1].contiguous(),
                                              with_shared=False)
        back = self._exchange(y, rc, sc)                        # rows in send order
        ys = torch.zeros((T * k, H), dtype=torch.float32, device=dev)
        ys[order] = back
        ys = ys.reshape(T, k, H)
        none_ids = torch.full((T, k), -1, dtype=torch.int32, device=dev)
        shared = lay.forward_routed(x, none_ids, torch.zeros((T, k), dtype=torch.float32, device=dev),
                                    with_shared=True)
        out = ys[:, 0].clone()
        for j in range(1, k):
            out = out + ys[:, j]
        return out + shared, ids, w
