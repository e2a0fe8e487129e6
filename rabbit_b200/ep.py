"""Expert parallelism for the routed-MoE layer: one process per GPU, experts split in contiguous
blocks (expert e on rank e // (E / N)), tokens owned by the rank that holds them, router and shared
expert replicated.

One forward on every rank:

1. route the rank's own tokens with the replicated router (bit-exact, same kernel as one GPU);
2. exchange counts, then token rows with ``all_to_all_single`` (variable splits): a token goes
   once to every rank owning at least one of its k experts, with its [k] ids and weights (slots
   of other ranks set to -1 / 0);
3. run the received rows through the local experts with the routing weights folded in
   (``forward_routed``: rabbit's ``apply_single_expert`` loop, src/glm52/moe.rs:463-513), which
   sums each row's local slots in slot order;
4. send those per-(token, rank) partial sums back the same way;
5. on the token's owner: ``out[t] = ((p_0 + p_1) + ... + p_{N-1}) + shared(x_t)`` over the ranks in
   order, the gated shared expert last (qwen38/generate.rs:324-349). The order is fixed for a
   world size; against one GPU the slot sums are only regrouped (f32 rounding).

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
        solo = group is None and not dist.is_initialized()
        self.world = 1 if solo else dist.get_world_size(group)
        self.rank = 0 if solo else dist.get_rank(group)
        self.last_exchange_bytes = 0  # bytes this rank sent in the last forward (both exchanges)
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
        """x [T_local, H] on this rank's device -> (out [T_local, H] f32, ids, weights)."""
        lay = self.layer
        T, k, H, N = x.shape[0], lay.topk, lay.hidden, self.world
        dev = x.device
        ids, w = lay.route(x)                                   # [T, k] rank order, bit-exact
        if N == 1:  # every expert local: the one-device layer
            return lay.forward_routed(x, ids, w, with_shared=True), ids, w
        dest = torch.where(ids >= 0, ids.long() // self.per_rank, torch.full_like(ids, -1, dtype=torch.long))
        # one row per (destination rank, token) that has a slot there, rank-major, token order
        hit = (dest.unsqueeze(2) == torch.arange(N, device=dev)).any(dim=1)      # [T, N]
        r_idx, t_idx = hit.t().nonzero(as_tuple=True)
        send_counts = torch.bincount(r_idx, minlength=N)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        mine = dest[t_idx] == r_idx.unsqueeze(1)                                  # slots on that rank
        send_ids = torch.where(mine, ids[t_idx], torch.full_like(ids[t_idx], -1))
        send_w = torch.where(mine, w[t_idx], torch.zeros_like(w[t_idx]))
        recv_x = self._exchange(x[t_idx], sc, rc)
        recv_ids = self._exchange(send_ids, sc, rc)
        recv_w = self._exchange(send_w, sc, rc)
        # the local experts over every received row (up to k slots each, weights folded in)
        R = recv_x.shape[0]
        y = torch.empty((R, H), dtype=torch.float32, device=dev)
        step = self.max_rows or max(R, 1)
        for r0 in range(0, R, step):
            r1 = min(R, r0 + step)
            lay.forward_routed(recv_x[r0:r1], recv_ids[r0:r1], recv_w[r0:r1], with_shared=False, out=y[r0:r1])
        back = self._exchange(y, rc, sc)                        # partial sums, in send order
        self.last_exchange_bytes = (t_idx.numel() * (H * x.element_size() + k * 8)
                                    + R * H * 4) - (sc[self.rank] * (H * x.element_size() + k * 8)
                                                    + rc[self.rank] * H * 4)
        parts = torch.zeros((N, T, H), dtype=torch.float32, device=dev)
        parts[r_idx, t_idx] = back
        shared = lay.forward_routed(x, torch.full_like(ids, -1), torch.zeros_like(w), with_shared=True)
        out = parts[0].clone()
        for r in range(1, N):
            out += parts[r]
        return out + shared, ids, w
