"""Expert parallelism for the routed-MoE layer: one process per GPU, experts split in contiguous
blocks (expert e on rank e // (E / N)), tokens owned by the rank that holds them, router and shared
expert replicated.

One forward on every rank, with no host synchronisation (every size is fixed by T and N, so no
count is read back to the host, and every step is queued on the device):

1. route the rank's own tokens with the replicated router (bit-exact, the one-GPU kernels);
2. start the exchange of every rank's token rows and their routing: ``all_gather`` of each row's
   payload -- its activation terms on the MXFP4 tensor-core path (17 bytes per 32 columns, formed
   once by the row's owner), else x [T, H] -- and of the routing row [T, 2k] (ids, and the
   weights' bits), asynchronously;
3. meanwhile compute the gated shared expert of the rank's own tokens (it needs no routing);
4. run all N*T gathered rows through the local experts (``forward_routed``: rabbit's
   ``apply_single_expert`` loop, src/glm52/moe.rs:463-513): each row sums its slots whose expert
   is resident here, in slot order; slots of other ranks' experts contribute nothing, so a row
   with no local slot costs no expert work;
5. return each owner its rows' partial sums with one equal-split ``all_to_all`` ([N, T, H] f32);
6. on the owner: ``out[t] = ((p_0 + p_1) + ... + p_{N-1}) + shared(x_t)``, ranks in order and the
   shared expert last (qwen38/generate.rs:324-349), in one kernel (``sum_rank_parts``). The order
   is fixed for a world size; against one GPU the routed slot sums are only regrouped (f32
   rounding).

The exchanges are collectives the reference has no counterpart for (it runs on one host). The
compute side is any object with ``route(x)``, ``forward_routed(x, ids, weights, with_shared, out)``,
``sum_rank_parts(parts, last)`` and ``hidden``/``topk``/``n_experts`` attributes, optionally
``row_payload(x)`` and ``forward_routed_payload(rows, ids, weights)`` for a cheaper row payload:
the device layer (``MoeLayer``) on GPUs, or a CPU stand-in for the host-side tests.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class ExpertParallelMoe:
    def __init__(self, layer, group=None):
        self.layer = layer
        self.group = group
        solo = group is None and not dist.is_initialized()
        self.world = 1 if solo else dist.get_world_size(group)
        self.rank = 0 if solo else dist.get_rank(group)
        self.last_exchange_bytes = 0  # bytes this rank sent in the last forward (both exchanges)
        if layer.n_experts % self.world:
            raise ValueError(f"{layer.n_experts} experts do not split over {self.world} ranks")
        self.per_rank = layer.n_experts // self.world
        self._gloo = not solo and dist.get_backend(group) == "gloo"

    def _all_gather(self, t):
        """[T, ...] on every rank -> [N*T, ...] in rank order (asynchronous work handle)."""
        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        if self._gloo:  # (gloo has the list form only)
            parts = list(out.chunk(self.world))
            dist.all_gather(parts, t.contiguous(), group=self.group)
            return out, None
        return out, dist.all_gather_into_tensor(out, t.contiguous(), group=self.group, async_op=True)

    def forward(self, x):
        """x [T_local, H] on this rank's device -> (out [T_local, H] f32, ids, weights)."""
        lay = self.layer
        T, k, H, N = x.shape[0], lay.topk, lay.hidden, self.world
        ids, w = lay.route(x)                                   # [T, k] rank order, bit-exact
        if N == 1:  # every expert local: the one-device layer
            self.last_exchange_bytes = 0
            return lay.forward_routed(x, ids, w, with_shared=True), ids, w
        meta = torch.cat([ids, w.view(torch.int32)], dim=1)     # [T, 2k] int32
        # what a row travels as: its activation terms where the layer has them (formed once, by
        # the row's owner), else x
        payload = lay.row_payload(x) if hasattr(lay, "row_payload") else (x,)
        gathered = [self._all_gather(p) for p in payload]
        meta_all, wm = self._all_gather(meta)
        # the shared expert of the own tokens overlaps the exchange (it needs no routing)
        shared = lay.forward_routed(x, torch.full_like(ids, -1), torch.zeros_like(w), with_shared=True)
        for work in [g[1] for g in gathered] + [wm]:
            if work is not None:
                work.wait()
        ids_all = meta_all[:, :k].contiguous()
        w_all = meta_all[:, k:].contiguous().view(torch.float32)
        rows = tuple(g[0] for g in gathered)
        if hasattr(lay, "forward_routed_payload"):
            y = lay.forward_routed_payload(rows, ids_all, w_all)             # [N*T, H] partial sums
        else:
            y = lay.forward_routed(rows[0], ids_all, w_all, with_shared=False)
        parts = torch.empty_like(y)
        dist.all_to_all_single(parts, y, group=self.group)      # block r: rank r's sums of my rows
        row_bytes = sum(q.numel() * q.element_size() for q in payload) // max(T, 1)
        self.last_exchange_bytes = (N - 1) * T * (row_bytes + 2 * k * 4 + H * 4)
        out = lay.sum_rank_parts(parts.view(N, T, H), last=shared)
        return out, ids, w
