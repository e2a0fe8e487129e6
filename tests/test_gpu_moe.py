"""Whole-layer GPU parity against the CPU oracle on the BASELINE configs: routing bit-exact,
layer output within 1e-2 relative L2 (the north star's bf16-accumulation tolerance)."""
import numpy as np
import pytest

from helpers import build_layer, hard_prefill_tokens, oracle_forward, oracle_routing, per_token_rel_l2, x_device
from rabbit_b200 import synth
from refvec import rel_l2

pytestmark = pytest.mark.gpu

OUT_RTOL = 1e-2  # relative L2 of the layer output vs the reference
# routing weights: the decode path softmaxes certified logits (within a few f32 ulps of the
# reference chain), so weights agree to ~1e-6 relative; ids are always bit-exact
W_ATOL = 2e-5


@pytest.fixture(scope="module")
def qwen_layer(cuda_ctx):
    cfg = synth.CONFIGS["c2_qwen_prefill"]
    L = build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    yield cfg, L
    L.close()


def test_c0_tiny_layer_matches_oracle(cuda_ctx):
    cfg = synth.CONFIGS["c0_tiny"]
    L = build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    x = synth.activations(cfg)
    out, ids, w = L.moe_forward(x_device(cfg, x), return_routing=True)
    want, want_ids, want_w = oracle_forward(cfg, x)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.max(np.abs(w.cpu().numpy() - want_w)) < W_ATOL
    assert rel_l2(out.cpu().numpy(), want) < OUT_RTOL
    L.close()


def test_c0_tiny_ragged_token_counts(cuda_ctx):
    """T = 1..4 on a max_tokens = 4 layer: every prefix routes and combines like the oracle."""
    cfg = synth.CONFIGS["c0_tiny"]
    L = build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    xa = synth.activations(cfg)
    for T in range(1, cfg.tokens + 1):
        x = xa[:T]
        out, ids, _ = L.moe_forward(x_device(cfg, x), return_routing=True)
        want, want_ids, _ = oracle_forward(cfg, x)
        assert np.array_equal(ids.cpu().numpy(), want_ids)
        assert rel_l2(out.cpu().numpy(), want) < OUT_RTOL
    L.close()


def test_c1_decode_one_token_matches_oracle(qwen_layer):
    cfg, L = qwen_layer
    c1 = synth.CONFIGS["c1_qwen_decode"]
    x = synth.activations(c1)
    out, ids, w = L.moe_forward(x_device(c1, x), return_routing=True)
    want, want_ids, want_w = oracle_forward(c1, x)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.max(np.abs(w.cpu().numpy() - want_w)) < W_ATOL
    assert rel_l2(out.cpu().numpy(), want) < OUT_RTOL


def test_c2_prefill_routing_exact_and_output_subset(qwen_layer):
    """All 2048 tokens route bit-exactly; the output of a token subset matches the oracle (the
    layer is per-token independent, so the subset's reference output is the same)."""
    cfg, L = qwen_layer
    x = synth.activations(cfg)
    out, ids, w = L.moe_forward(x_device(cfg, x), return_routing=True)
    want_ids, want_w = oracle_routing(cfg, x)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.max(np.abs(w.cpu().numpy() - want_w)) < 1e-6
    # the layer is per-token independent: the hard tokens' reference output is the same alone
    sel = hard_prefill_tokens(want_ids)
    assert len(sel) >= 64
    want, _, _ = oracle_forward(cfg, x[sel])
    assert rel_l2(out.cpu().numpy()[sel], want) < OUT_RTOL
    assert per_token_rel_l2(out.cpu().numpy()[sel], want).max() < OUT_RTOL


def test_c2_shaped_64_experts_every_token(cuda_ctx):
    """A C2-shaped layer (H 8192, I 2048, top-10, gated shared expert, Zipf skew) with 64 experts
    at T = 2048: every expert takes ~320 rows, i.e. ten position chunks, and every one of the
    2048 token outputs is checked against the reference (AVX-512 tier)."""
    import dataclasses

    cfg = dataclasses.replace(synth.CONFIGS["c2_qwen_prefill"], name="c2_64", n_experts=64)
    L = build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    x = synth.activations(cfg)
    out, ids, _ = L.moe_forward(x_device(cfg, x), return_routing=True)
    out = out.cpu().numpy()
    L.close()
    want, want_ids, _ = oracle_forward(cfg, x, tier="avx512")
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert per_token_rel_l2(out, want).max() < OUT_RTOL


def test_decode_router_certificate_matches_exact_routing(qwen_layer):
    """The decode front end (certified logits + exact fallback) against the exact-chain router
    on 256 single-token calls and on 32-token batches: ids identical, weights within W_ATOL."""
    import torch

    cfg, L = qwen_layer
    x = synth.activations(cfg, tokens=256, token_offset=5000)
    xd = x_device(cfg, x)
    exact_ids, exact_w = L.route(xd)  # rmoe_route: exact reference-order chains
    for t in range(64):
        _, ids, w = L.moe_forward(xd[t:t + 1], return_routing=True)
        assert torch.equal(ids, exact_ids[t:t + 1])
        assert float((w - exact_w[t:t + 1]).abs().max()) < W_ATOL
    for t0 in range(0, 256, 32):
        _, ids, w = L.moe_forward(xd[t0:t0 + 32], return_routing=True)
        assert torch.equal(ids, exact_ids[t0:t0 + 32])
        assert float((w - exact_w[t0:t0 + 32]).abs().max()) < W_ATOL
    stats = L.stats()
    assert stats["router_fallbacks"] < 0.2 * (64 + 256)


def test_host_entry_point_matches_device_path(qwen_layer):
    """rmoe_moe_forward_host (the Rust call-site signature: host slices in and out)."""
    import torch

    cfg, L = qwen_layer
    x = synth.activations(cfg, tokens=4)
    dev = L.moe_forward(x_device(cfg, x)).cpu().numpy()
    host = L.moe_forward_host(synth.f32_to_bf16_bits(x))
    assert np.array_equal(dev, host)
    pinned = torch.from_numpy(synth.f32_to_bf16_bits(x).view(np.int16)).pin_memory()
    out = L.moe_forward_host(pinned.view(torch.bfloat16))
    assert np.array_equal(dev, out)
    # pinned buffers both ways, changing between calls
    for T in (1, 4):
        xt = synth.activations(cfg, tokens=T, token_offset=77 * T)
        want = L.moe_forward(x_device(cfg, xt)).cpu().numpy()
        for _ in range(2):
            xp = torch.from_numpy(synth.f32_to_bf16_bits(xt).view(np.int16)).pin_memory()
            op = torch.empty((T, cfg.hidden), dtype=torch.float32).pin_memory()
            got = L.moe_forward_host(xp.view(torch.bfloat16), out=op)
            assert np.array_equal(want, got.numpy())


def test_graph_replays_bind_the_callers_buffers(qwen_layer):
    """Cached forward graphs read x and write out through the caller's buffers (kernel arguments
    rebound per launch; misaligned buffers go through staging): every call, in any order, gives
    the bits a fresh single call gives."""
    import torch

    cfg, L = qwen_layer
    for T in (1, 3, 40):
        xs = [x_device(cfg, synth.activations(cfg, tokens=T, token_offset=o)) for o in (0, 5000)]
        ref = [L.moe_forward(x).clone() for x in xs]
        assert not torch.equal(ref[0], ref[1])
        for _ in range(2):
            for i in (1, 0):
                out = torch.full((T, cfg.hidden), float("nan"), device="cuda")
                assert torch.equal(L.moe_forward(xs[i], out=out), ref[i])
        # a 4-byte offset view of x and of out: the staged path
        xb = torch.empty(T * cfg.hidden + 2, dtype=xs[0].dtype, device="cuda")
        xv = xb[2:].view(T, cfg.hidden)
        xv.copy_(xs[0])
        ob = torch.empty(T * cfg.hidden + 1, dtype=torch.float32, device="cuda")
        ov = ob[1:].view(T, cfg.hidden)
        L.moe_forward(xv, out=ov)
        assert torch.equal(ov, ref[0])


def test_c4_glm_int4_layer(cuda_ctx):
    cfg = synth.CONFIGS["c4_glm_int4"]
    L = build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens, scale_dtype="bf16")
    x = synth.activations(cfg)
    out, ids, w = L.moe_forward(x_device(cfg, x), return_routing=True)
    want_ids, want_w = oracle_routing(cfg, x)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.max(np.abs(w.cpu().numpy() - want_w)) < 1e-5
    sel = hard_prefill_tokens(want_ids, at_least=32)[:48]
    want, _, _ = oracle_forward(cfg, x[sel])
    assert rel_l2(out.cpu().numpy()[sel], want) < OUT_RTOL
    assert per_token_rel_l2(out.cpu().numpy()[sel], want).max() < OUT_RTOL
    L.close()


def _fused_gate_up(ex):
    """GateUp::Fused from the separate tensors: [2I, H] = gate rows, then up rows (the layout
    fuse_gate_up writes, src/expert_cache.rs:69-74)."""
    import torch

    return torch.cat([ex["gate"], ex["up"]]), torch.cat([ex["gate_scale"], ex["up_scale"]])


@pytest.mark.parametrize("name", ["c0_tiny", "c2_64"])
def test_fused_gate_up_upload_is_bit_identical(cuda_ctx, name):
    """An expert uploaded as GateUp::Fused computes exactly what the Separate upload computes
    (the reference pins the two slot kinds equal, src/glm52/moe.rs:592-626): both layouts end in
    the same device bytes, so the outputs are bit-identical on the GEMV (c0) and tensor-core
    (C2-shaped, T = 1 and T = 40) paths."""
    import dataclasses

    import torch

    if name == "c0_tiny":
        cfg = synth.CONFIGS["c0_tiny"]
        Ts = (1, cfg.tokens)
    else:
        cfg = dataclasses.replace(synth.CONFIGS["c2_qwen_prefill"], name=name, n_experts=64, tokens=40)
        Ts = (1, 40)
    sep = build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    fus = build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    for eid in range(cfg.n_experts):
        ex = synth.gpu_expert(cfg, eid)
        gu, gus = _fused_gate_up(ex)
        # overwrite with a different expert first, so a no-op upload cannot pass
        fus.upload_expert_dict(eid, synth.gpu_expert(cfg, (eid + 1) % cfg.n_experts))
        fus.upload_expert_fused(eid, gu, gus, ex["down"], ex["down_scale"])
    torch.cuda.synchronize()
    x = synth.activations(cfg)
    for T in Ts:
        xd = x_device(cfg, x[:T])
        assert torch.equal(sep.moe_forward(xd), fus.moe_forward(xd))
    with pytest.raises(Exception, match="SHAPE_MISMATCH"):
        ex = synth.gpu_expert(cfg, 0)
        gu, gus = _fused_gate_up(ex)
        fus.upload_expert_fused(0, gu[:-1], gus, ex["down"], ex["down_scale"])
    sep.close()
    fus.close()


def test_bounded_wait_reports_timeout_and_layer_recovers(cuda_ctx):
    """A wait limit far below the kernels' own run time makes a bounded device wait (the fused
    one-token kernel's wait for an expert's h, its closing grid barrier) run out: the host entry
    point returns RMOE_TIMEOUT instead of garbage with OK. With the default limit back, the next
    call succeeds and gives the bits of a call on a layer that never timed out."""
    import dataclasses

    import rabbit_b200 as rb

    cfg = dataclasses.replace(synth.CONFIGS["c2_qwen_prefill"], name="c2_64", n_experts=64, tokens=4)
    L = build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    x = synth.f32_to_bf16_bits(synth.activations(cfg, tokens=1))
    good = L.moe_forward_host(x)
    L.set_wait_limit(100)  # 100 ns: a CTA's wait for another CTA's progress runs out
    with pytest.raises(rb.RmoeError, match="TIMEOUT"):
        L.moe_forward_host(x)
    assert L.stats()["device_error_flags"] != 0
    L.set_wait_limit(0)
    again = L.moe_forward_host(x)
    assert np.array_equal(again, good)
    L.check()  # nothing pending
    # the same with pinned buffers both ways
    import torch

    xp = torch.from_numpy(x.view(np.int16)).pin_memory()
    op = torch.empty((1, cfg.hidden), dtype=torch.float32).pin_memory()
    assert np.array_equal(L.moe_forward_host(xp.view(torch.bfloat16), out=op).numpy(), good)
    L.set_wait_limit(100)
    with pytest.raises(rb.RmoeError, match="TIMEOUT"):
        L.moe_forward_host(xp.view(torch.bfloat16), out=op)
    L.set_wait_limit(0)
    assert np.array_equal(L.moe_forward_host(xp.view(torch.bfloat16), out=op).numpy(), good)
    L.check()
    L.close()


def test_shape_and_argument_errors(cuda_ctx):
    import torch

    import rabbit_b200 as rb

    cfg = synth.CONFIGS["c0_tiny"]
    L = rb.MoeLayer(cuda_ctx, cfg.hidden, cfg.inter, cfg.n_experts, cfg.topk, max_tokens=2)
    good = synth.expert(cfg, 0)
    with pytest.raises(rb.RmoeError, match="SHAPE_MISMATCH"):
        L.upload_expert(0, good["gate"][:-1], good["gate_scale"], good["up"], good["up_scale"],
                        good["down"], good["down_scale"])
    with pytest.raises(rb.RmoeError, match="INVALID_ARG"):
        L.upload_expert_dict(cfg.n_experts, good)
    with pytest.raises(rb.RmoeError, match="INVALID_ARG"):  # router never uploaded
        L.route(torch.zeros((1, cfg.hidden), device="cuda"))
    L.upload_router(synth.router_weights(cfg))
    with pytest.raises(rb.RmoeError, match="INVALID_ARG"):  # T > max_tokens
        L.route(torch.zeros((3, cfg.hidden), device="cuda"))
    with pytest.raises(rb.RmoeError, match="INVALID_ARG"):  # experts missing
        L.moe_forward(torch.zeros((1, cfg.hidden), device="cuda"))
    with pytest.raises(rb.RmoeError, match="NOT_SUPPORTED"):
        rb.MoeLayer(cuda_ctx, 100, 32, 4, 2)
    L.close()


@pytest.mark.parametrize("T", [9, 64, 200])
def test_int4_tensor_core_path_every_token(cuda_ctx, T):
    """Grouped-int4 batches above 8 tokens run on the tensor cores (weights dequantized into TMEM,
    kind::f16): a GLM-shaped layer (H 6144, I 2048, sigmoid grouped router, shared expert) with 32
    experts, every token's output against the reference within the tolerance, routing exact."""
    import dataclasses

    cfg = dataclasses.replace(synth.CONFIGS["c4_glm_int4"], name="c4_32", n_experts=32, tokens=T, n_group=4,
                              topk_group=2)
    L = build_layer(cuda_ctx, cfg, max_tokens=T, scale_dtype="bf16")
    x = synth.activations(cfg)
    out, ids, _ = L.moe_forward(x_device(cfg, x), return_routing=True)
    L.check()
    want, want_ids, _ = oracle_forward(cfg, x)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert per_token_rel_l2(out.cpu().numpy(), want).max() < OUT_RTOL
    L.close()
