"""Expert parallelism (rabbit_b200.ep) on CPU: world sizes 2 and 4 over gloo, the expert products done by
the oracle, against the one-process oracle layer. Covers the host side of EP: routing on the token
owner, the slot exchange and its counts, the return exchange, and the owner's fixed-order combine
with the gated shared expert last."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as orc
from rabbit_b200 import synth
from helpers import oracle_forward, oracle_routing
from refvec import rel_l2


class OracleLayer:
    """The layer interface ExpertParallelMoe drives, computed by the oracle on CPU, holding only
    the experts of one EP rank (slots naming other experts contribute nothing)."""

    def __init__(self, cfg, rank, world):
        self.cfg = cfg
        self.hidden, self.topk, self.n_experts = cfg.hidden, cfg.topk, cfg.n_experts
        per = cfg.n_experts // world
        self.lo, self.hi = rank * per, (rank + 1) * per
        self.router = synth.router_weights(cfg)
        self.experts = {e: synth.expert(cfg, e) for e in range(self.lo, self.hi)}
        self.shared = synth.expert(cfg, cfg.n_experts)
        self.gvec = synth.shared_gate(cfg)

    def _ffn(self, x, ex, inter):
        s = x.shape[0]
        g = orc.matmul_mxfp4(x, ex["gate"], ex["gate_scale"], s, self.hidden, inter)
        u = orc.matmul_mxfp4(x, ex["up"], ex["up_scale"], s, self.hidden, inter)
        h = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)
        return orc.matmul_mxfp4(h, ex["down"], ex["down_scale"], s, inter, self.hidden)

    def route(self, x):
        xn = x.numpy().astype(np.float32)
        logits = orc.matmul(xn, self.router, xn.shape[0], self.hidden, self.n_experts)
        b = synth.logit_bias(self.cfg)
        if b is not None:
            logits = (logits + b[None, :]).astype(np.float32)
        ids = np.zeros((xn.shape[0], self.topk), np.int32)
        w = np.zeros((xn.shape[0], self.topk), np.float32)
        for t in range(xn.shape[0]):
            r = orc.qwen_route(logits[t], self.topk)
            ids[t] = [i for i, _ in r]
            w[t] = [v for _, v in r]
        return torch.from_numpy(ids), torch.from_numpy(w)

    def row_payload(self, x):
        """(the payload protocol: this stand-in sends x itself, as one tensor)"""
        return (x,)

    def forward_routed_payload(self, rows, ids, w, out=None):
        return self.forward_routed(rows[0], ids, w, with_shared=False, out=out)

    def forward_routed(self, x, ids, w, with_shared=True, out=None):
        dst = out
        xn = x.numpy().astype(np.float32)
        out = np.zeros((xn.shape[0], self.hidden), np.float32)
        for t in range(xn.shape[0]):
            for j in range(self.topk):
                e = int(ids[t, j])
                if self.lo <= e < self.hi:
                    out[t] += np.float32(w[t, j]) * self._ffn(xn[t:t + 1], self.experts[e], self.cfg.inter)[0]
            if with_shared and self.cfg.shared_inter:
                gate = np.float32(1.0 / (1.0 + np.exp(-np.float32(np.dot(xn[t], self.gvec)))))
                out[t] += gate * self._ffn(xn[t:t + 1], self.shared, self.cfg.shared_inter)[0]
        if dst is not None:
            dst.copy_(torch.from_numpy(out))
            return dst
        return torch.from_numpy(out)


    def sum_rank_parts(self, parts, last=None):
        out = parts[0].clone()
        for r in range(1, parts.shape[0]):
            out += parts[r]
        return out + last if last is not None else out


class SplitPayloadLayer(OracleLayer):
    """The same layer sending each row as two tensors (its two column halves, one of them as raw
    bytes), like the device layer's terms and scales: the exchange gathers every tensor of the
    payload and the receiver reassembles the rows."""

    def row_payload(self, x):
        h = self.hidden // 2
        return (x[:, :h].contiguous(), x[:, h:].contiguous().view(torch.uint8))

    def forward_routed_payload(self, rows, ids, w, out=None):
        x = torch.cat([rows[0], rows[1].view(torch.float32)], dim=1)
        return self.forward_routed(x, ids, w, with_shared=False, out=out)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, cfg_name, t_local, results, split=False):
    from rabbit_b200.ep import ExpertParallelMoe

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = synth.CONFIGS[cfg_name]
    x = synth.activations(cfg, tokens=world * t_local)
    mine = torch.from_numpy(x[rank * t_local:(rank + 1) * t_local].copy())
    ep = ExpertParallelMoe((SplitPayloadLayer if split else OracleLayer)(cfg, rank, world))
    out, ids, w = ep.forward(mine)
    results[rank] = (out.numpy(), ids.numpy())
    dist.destroy_process_group()


@pytest.mark.parametrize("world,t_local,split", [(2, 3, False), (4, 2, False), (2, 3, True)])
def test_expert_parallel_matches_one_process(world, t_local, split):
    cfg = synth.CONFIGS["c0_tiny"]
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_run, args=(world, _free_port(), "c0_tiny", t_local, results, split), nprocs=world, join=True)
    x = synth.activations(cfg, tokens=world * t_local)
    want, want_ids, _ = oracle_forward(cfg, x)
    got = np.concatenate([results[r][0] for r in range(world)])
    got_ids = np.concatenate([results[r][1] for r in range(world)])
    assert np.array_equal(got_ids, want_ids)        # owners route exactly like one process
    assert rel_l2(got, want) < 1e-5                 # same products, fixed combine order


# ------------------------------------------------------------------------------ GPU
def _mid_cfg():
    """A c2-shaped layer (H 8192, I 2048, top-10, shared expert, Zipf skew) with 64 experts, so it
    builds in seconds and two EP halves fit beside it."""
    import dataclasses

    return dataclasses.replace(synth.CONFIGS["c2_qwen_prefill"], name="c2_mid", n_experts=64, tokens=40)


@pytest.mark.gpu
def test_forward_routed_matches_forward(cuda_ctx):
    """forward_routed with the layer's own routing is the layer forward; split into one slot per
    call and summed in slot order (the EP combine), it is the same to f32 rounding."""
    import torch

    cfg = _mid_cfg()
    L = synth.build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    x = synth.x_device(cfg, synth.activations(cfg))
    full, ids, w = L.moe_forward(x, return_routing=True)
    routed = L.forward_routed(x, ids, w)
    assert rel_l2(routed.cpu().numpy(), full.cpu().numpy()) < 1e-5
    T, k = ids.shape
    none = torch.full_like(ids, -1)
    acc = None
    for j in range(k):
        one_id, one_w = none.clone(), torch.zeros_like(w)
        one_id[:, j], one_w[:, j] = ids[:, j], w[:, j]
        y = L.forward_routed(x, one_id, one_w, with_shared=False)
        acc = y if acc is None else acc + y
    acc = acc + L.forward_routed(x, none, torch.zeros_like(w), with_shared=True)
    assert rel_l2(acc.cpu().numpy(), full.cpu().numpy()) < 1e-5
    want, _, _ = oracle_forward(cfg, synth.activations(cfg)[:4])
    assert rel_l2(routed.cpu().numpy()[:4], want) < 1e-2
    L.close()


@pytest.mark.gpu
def test_ep_halves_on_one_gpu(cuda_ctx):
    """Two EP ranks' layers (experts 0-31, 32-63) on one device: each computes only its own
    experts' slots, and the halves plus the shared expert give the one-layer output."""
    import torch

    cfg = _mid_cfg()
    full_layer = synth.build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    x = synth.x_device(cfg, synth.activations(cfg))
    full, ids, w = full_layer.moe_forward(x, return_routing=True)
    full_layer.close()
    none = torch.full_like(ids, -1)
    parts = []
    for r in range(2):
        L = synth.build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens, ep_rank=r, ep_size=2)
        parts.append(L.forward_routed(x, ids, w, with_shared=False))
        if r == 0:
            shared = L.forward_routed(x, none, torch.zeros_like(w), with_shared=True)
        L.close()
    got = parts[0] + parts[1] + shared
    assert rel_l2(got.cpu().numpy(), full.cpu().numpy()) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 7, 40])
def test_forward_routed_terms_is_forward_routed(cuda_ctx, T):
    """The payload path of expert parallelism: rows sent as their activation terms
    (rmoe_activation_terms, formed once by their owner) run through the expert loop to the same
    bits as forward_routed on x without the shared expert -- on a full layer and on one EP half."""
    import torch

    cfg = _mid_cfg()
    x = synth.x_device(cfg, synth.activations(cfg, tokens=T))
    for ep in ((0, 1), (1, 2)):
        L = synth.build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens, ep_rank=ep[0], ep_size=ep[1])
        full_layer = L if ep[1] == 1 else synth.build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
        _, ids, w = full_layer.moe_forward(x, return_routing=True)
        want = L.forward_routed(x, ids, w, with_shared=False)
        payload = L.row_payload(x)
        assert len(payload) == 2 and payload[0].dtype == torch.uint8
        assert payload[0].shape == (T, 2 * cfg.hidden) and payload[1].shape == (T, cfg.hidden // 8)
        got = L.forward_routed_payload(payload, ids, w)
        assert torch.equal(got, want)
        if full_layer is not L:
            full_layer.close()
        L.close()


def _nccl_rank(rank, world, port, results):
    import torch

    import rabbit_b200 as rb
    from rabbit_b200.ep import ExpertParallelMoe

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    cfg = _mid_cfg()
    ctx = rb.Context(rank)
    t_local = cfg.tokens // world
    L = synth.build_layer(ctx, cfg, max_tokens=cfg.tokens * cfg.topk, ep_rank=rank, ep_size=world)
    xa = synth.activations(cfg)
    x = synth.x_device(cfg, xa[rank * t_local:(rank + 1) * t_local]).cuda(rank)
    out, ids, _ = ExpertParallelMoe(L).forward(x)
    torch.cuda.synchronize()
    results[rank] = (out.cpu().numpy(), ids.cpu().numpy())
    L.close()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_expert_parallel_two_gpus():
    """ExpertParallelMoe over NCCL on 2 GPUs (one process each) against the oracle."""
    import torch

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = _mid_cfg()
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.spawn(_nccl_rank, args=(2, _free_port(), results), nprocs=2, join=True)
    x = synth.activations(cfg)
    got = np.concatenate([results[r][0] for r in range(2)])
    got_ids = np.concatenate([results[r][1] for r in range(2)])
    want_ids, _ = oracle_routing(cfg, x)
    assert np.array_equal(got_ids, want_ids)
    sel = [0, 1, 20, 39]
    want, _, _ = oracle_forward(cfg, x[sel])
    assert rel_l2(got[sel], want) < 1e-2


@pytest.mark.gpu
def test_forward_routed_one_token(cuda_ctx):
    """One token through forward_routed (the fused one-token kernel behind a one-warp dispatch,
    no front end): with the layer's own routing it is the layer forward, with and without the
    shared expert, and with half the slots dropped it is the sum of the kept slots."""
    import torch

    cfg = _mid_cfg()
    L = synth.build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    xa = synth.activations(cfg)
    for t in (0, 7):
        x = synth.x_device(cfg, xa[t:t + 1])
        full, ids, w = L.moe_forward(x, return_routing=True)
        routed = L.forward_routed(x, ids, w)
        assert rel_l2(routed.cpu().numpy(), full.cpu().numpy()) < 1e-5
        none = torch.full_like(ids, -1)
        shared = L.forward_routed(x, none, torch.zeros_like(w), with_shared=True)
        keep = torch.arange(ids.shape[1], device=ids.device) % 2 == 0
        a = L.forward_routed(x, torch.where(keep, ids, none), torch.where(keep, w, torch.zeros_like(w)),
                             with_shared=False)
        b = L.forward_routed(x, torch.where(keep, none, ids), torch.where(keep, torch.zeros_like(w), w),
                             with_shared=False)
        assert rel_l2((a + b + shared).cpu().numpy(), full.cpu().numpy()) < 1e-5
    L.close()


@pytest.mark.gpu
def test_forward_routed_repeated_expert(cuda_ctx):
    """A token whose routing names one expert in two slots gets that expert once, with the first
    slot's weight, as apply_single_expert's first-match row gather does (src/glm52/moe.rs:465-470):
    the result equals the same routing with the repeat removed, at T = 1 (one-warp dispatch) and
    T > 1 (the general dispatch)."""
    import torch

    cfg = _mid_cfg()
    L = synth.build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    xa = synth.activations(cfg)
    for t0, t1 in ((3, 4), (0, cfg.tokens)):
        x = synth.x_device(cfg, xa[t0:t1])
        _, ids, w = L.moe_forward(x, return_routing=True)
        dup_ids, dup_w = ids.clone(), w.clone()
        dup_ids[:, 3] = ids[:, 1]          # slot 3 repeats slot 1's expert with its own weight
        dup_w[:, 3] = 0.75
        ref_ids = dup_ids.clone()
        ref_ids[:, 3] = -1
        got = L.forward_routed(x, dup_ids, dup_w)
        want = L.forward_routed(x, ref_ids, dup_w)
        assert rel_l2(got.cpu().numpy(), want.cpu().numpy()) < 1e-6
    L.close()


@pytest.mark.gpu
def test_sum_rank_parts_is_rank_order(cuda_ctx):
    """rmoe_sum_rank_parts adds the ranks' partial sums in rank order and the shared expert last:
    bit-identical to the sequential sum, with and without the last term."""
    import torch

    L = synth.build_layer(cuda_ctx, synth.CONFIGS["c0_tiny"], max_tokens=4)
    g = torch.Generator(device="cuda").manual_seed(3)
    for n in (1, 2, 8):
        parts = torch.randn((n, 37, 256), device="cuda", generator=g) * 1e3
        last = torch.randn((37, 256), device="cuda", generator=g)
        want = parts[0].clone()
        for r in range(1, n):
            want = want + parts[r]
        assert torch.equal(L.sum_rank_parts(parts), want)
        assert torch.equal(L.sum_rank_parts(parts, last=last), want + last)
    L.close()
