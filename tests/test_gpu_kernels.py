"""GPU parity of the building blocks against the CPU oracle: the MXFP4 / int4 expert GEMMs, the
exact router matmul, the top-k selectors and the dispatch permutation. All calls go through the
C ABI (librmoe.so)."""
import numpy as np
import pytest

from oracle import oracle as orc
from rabbit_b200 import synth
from refvec import random_vec, rel_l2
from test_oracle import known_answer_i4g, known_answer_mxfp4

pytestmark = pytest.mark.gpu

# f16 HFMA2 products with f32 block accumulation: relative L2 against the f32 reference
GEMM_RTOL = 2e-3


def _t(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_known_answer_mxfp4_minus_320(cuda_ctx):  # kernels.rs:1388-1406
    import torch

    import rabbit_b200 as rb

    x, data, bs, cols = known_answer_mxfp4()
    y = torch.zeros(1, dtype=torch.float32, device="cuda")
    rb.matmul_mxfp4(y, _t(x), _t(data), _t(bs), 1, cols, 1)
    assert y.item() == -320.0


def test_known_answer_i4_grouped_nine(cuda_ctx):  # kernels.rs:1408-1428
    import torch

    import rabbit_b200 as rb

    x, b, sc = known_answer_i4g()
    y = torch.zeros(1, dtype=torch.float32, device="cuda")
    rb.matmul_i4_grouped(y, _t(x), _t(b), _t(sc), 3, 1, 6, 1)
    assert y.item() == 9.0


def test_e2m1_nibble_order_single_hot(cuda_ctx):
    """Each of the 16 codes at each of the 32 positions of a block, one at a time: checks the
    hardware E2M1 conversion and the low-nibble-first pairing against the reference table."""
    import torch

    import rabbit_b200 as rb

    cols, rows = 32, 16 * 32
    data = np.zeros((rows, 16), np.uint8)
    want = np.zeros(rows, np.float32)
    x = (np.arange(cols, dtype=np.float32) + 1.0)
    for code in range(16):
        for pos in range(32):
            r = code * 32 + pos
            data[r, pos // 2] = code << (4 * (pos % 2))
            want[r] = orc.e2m1_decode(code) * x[pos]
    bs = np.full((rows, 1), 127, np.uint8)
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    rb.matmul_mxfp4(y, _t(x), _t(data.ravel()), _t(bs.ravel()), 1, cols, rows)
    np.testing.assert_array_equal(y.cpu().numpy(), want)


@pytest.mark.parametrize("s,i,o", [(1, 256, 64), (3, 512, 100), (8, 1024, 32), (16, 96, 40),
                                   (5, 40, 7), (2, 33, 3)])
def test_matmul_mxfp4_matches_oracle(cuda_ctx, s, i, o):
    import torch

    import rabbit_b200 as rb

    w = random_vec(o * i, 1000 + i) * np.float32(4.0)
    q, bs = orc.pack_mxfp4(w, o, i)
    x = random_vec(s * i, 2000 + s).reshape(s, i)
    want = orc.matmul_mxfp4(x, q, bs, s, i, o)
    y = torch.zeros((s, o), dtype=torch.float32, device="cuda")
    rb.matmul_mxfp4(y, _t(x), _t(q), _t(bs), s, i, o)
    assert rel_l2(y.cpu().numpy(), want) < GEMM_RTOL


@pytest.mark.parametrize("s,i,o", [(1, 256, 128), (1, 8192, 256), (3, 512, 100), (8, 1024, 300),
                                   (33, 2048, 130), (2, 96, 40)])
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
def test_matmul_mxfp4_tc_matches_oracle(cuda_ctx, s, i, o, xdt):
    """tcgen05 kind::mxf4 path: weights as stored, x as a 4-term E2M1 expansion."""
    import torch

    import rabbit_b200 as rb

    w = random_vec(o * i, 1000 + i) * np.float32(4.0)
    q, bs = orc.pack_mxfp4(w, o, i)
    x = random_vec(s * i, 2000 + s).reshape(s, i)
    if xdt == "bf16":
        x = synth.round_bf16(x)
    want = orc.matmul_mxfp4(x, q, bs, s, i, o)
    y = torch.full((s, o), float("nan"), dtype=torch.float32, device="cuda")
    xd = _t(x) if xdt == "f32" else _t(x).to(torch.bfloat16)
    rb.matmul_mxfp4_tc(y, xd, _t(q), _t(bs), s, i, o)
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_l2(got, want) < GEMM_RTOL


@pytest.mark.parametrize("scale_dtype", ["f32", "bf16"])
@pytest.mark.parametrize("s,i,o,gs", [(1, 256, 64, 32), (4, 512, 48, 64), (9, 128, 16, 128),
                                      (2, 6, 3, 3)])
def test_matmul_i4_grouped_matches_oracle(cuda_ctx, s, i, o, gs, scale_dtype):
    import torch

    import rabbit_b200 as rb

    w = random_vec(o * i, 3000 + i)
    q, sc = orc.quant_int4_grouped(w, o, i, 4, gs)
    if scale_dtype == "bf16":
        sc = synth.round_bf16(sc)
    x = random_vec(s * i, 4000 + s).reshape(s, i)
    want = orc.matmul_i4_grouped(x, q, sc, gs, s, i, o)
    y = torch.zeros((s, o), dtype=torch.float32, device="cuda")
    sct = _t(sc)
    if scale_dtype == "bf16":
        sct = sct.to(torch.bfloat16)
    rb.matmul_i4_grouped(y, _t(x), _t(q), sct, gs, s, i, o)
    assert rel_l2(y.cpu().numpy(), want) < GEMM_RTOL


@pytest.mark.parametrize("s,i,o,dt", [(1, 8192, 512, "bf16"), (4, 256, 16, "f32"),
                                      (70, 512, 96, "bf16"), (130, 1000, 33, "f32"),
                                      (200, 2048, 130, "f32"), (96, 1024, 200, "mixed"),
                                      (2, 7168, 896, "bf16"), (3, 2048, 70, "mixed"), (1, 4096, 33, "f32"),
                                      (2048, 1024, 512, "mixed")])
def test_router_matmul_is_bit_exact(cuda_ctx, s, i, o, dt):
    """kernels::matmul: every element must equal the reference's sequential f32 chain."""
    import torch

    import rabbit_b200 as rb

    rng = np.random.default_rng(s * 7 + i)
    x = rng.standard_normal((s, i)).astype(np.float32)
    w = (rng.standard_normal((o, i)) * 0.02).astype(np.float32)
    if dt == "bf16":
        x, w = synth.round_bf16(x), synth.round_bf16(w)
    if dt == "mixed":  # f32 activations, bf16 router rows (the C1/C2 layers' router)
        w = synth.round_bf16(w)
    want = orc.matmul(x, w, s, i, o)
    y = torch.zeros((s, o), dtype=torch.float32, device="cuda")
    xt, wt = _t(x), _t(w)
    if dt == "bf16":
        xt, wt = xt.to(torch.bfloat16), wt.to(torch.bfloat16)
    if dt == "mixed":
        wt = wt.to(torch.bfloat16)
    rb.matmul(y, xt, wt, s, i, o)
    got = y.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _route_layer(ctx, logits_rows, topk, router="softmax", bias=None, **kw):
    """A layer whose router is the identity, so x = logits routes on exactly those logits."""
    import rabbit_b200 as rb

    T, E = logits_rows.shape
    H = max(32, ((E + 31) // 32) * 32)
    L = rb.MoeLayer(ctx, H, 32, E, topk, router=router, max_tokens=T, **kw)
    eye = np.zeros((E, H), np.float32)
    eye[np.arange(E), np.arange(E)] = 1.0
    L.upload_router(eye)
    if bias is not None:
        L.upload_router_bias(bias)
    x = np.zeros((T, H), np.float32)
    x[:, :E] = logits_rows
    return L, _t(x)


@pytest.mark.parametrize("H,E,dt", [(2048, 70, "bf16"), (7168, 896, "bf16"), (4096, 128, "f32")])
def test_one_token_route_uses_exact_logits(cuda_ctx, H, E, dt):
    """One token through a layer's router (the one-token exact kernel on the slab layout): ids in
    the reference's order and softmax weights equal to the oracle's on its exact logits."""
    import rabbit_b200 as rb

    rng = np.random.default_rng(H + E)
    w = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((1, H)).astype(np.float32)
    if dt == "bf16":
        w = synth.round_bf16(w)
    L = rb.MoeLayer(cuda_ctx, H, 32, E, 8, router="softmax", max_tokens=4)
    L.upload_router(synth.f32_to_bf16_bits(w) if dt == "bf16" else w)
    ids, wt = L.route(_t(x))
    logits = orc.matmul(x, w, 1, H, E)
    want = orc.qwen_route(logits[0], 8)
    assert ids[0].cpu().tolist() == [i for i, _ in want]
    assert np.max(np.abs(wt[0].cpu().numpy() - [v for _, v in want])) < 1e-6
    L.close()


def test_qwen_route_known_answers_on_gpu(cuda_ctx):  # qwen38/moe.rs:140-182
    L, x = _route_layer(cuda_ctx, np.array([[0.0, 2.0, -1.0, 5.0, 0.5, -3.0, 1.0, 3.0]], np.float32), 3)
    ids, w = L.route(x)
    assert ids.cpu().tolist() == [[3, 7, 1]]
    L, x = _route_layer(cuda_ctx, np.array([[1.0, 1.0, 1.0, 1.0], [0.0, 5.0, 5.0, 5.0]], np.float32), 2)
    ids, _ = L.route(x)
    assert ids.cpu().tolist() == [[0, 1], [1, 2]]


def test_qwen_route_matches_oracle_on_lcg_logits(cuda_ctx):  # qwen38/moe.rs:113-127
    from refvec import lcg_logits

    rows = np.stack([lcg_logits(512, s) for s in range(1, 6)])
    L, x = _route_layer(cuda_ctx, rows, 10)
    ids, w = L.route(x)
    for t in range(rows.shape[0]):
        want = orc.qwen_route(rows[t], 10)
        assert ids[t].cpu().tolist() == [i for i, _ in want]
        assert np.max(np.abs(w[t].cpu().numpy() - [v for _, v in want])) < 1e-6


def test_glm_grouped_route_known_answers_on_gpu(cuda_ctx):  # glm52/moe.rs:983-1007
    c = np.array([[0.1, 0.2, 9.0, 8.0, 0.3, 0.4, 7.0, 6.5]], np.float32)
    # choice = sigmoid(logit) + bias; use logits whose sigmoid keeps the order, no bias
    L, x = _route_layer(cuda_ctx, c, 3, router="sigmoid_grouped", bias=np.zeros(8, np.float32),
                        n_group=4, topk_group=2, norm_topk=False)
    ids, _ = L.route(x)
    assert ids.cpu().tolist() == [[2, 3, 6]]
    L, x = _route_layer(cuda_ctx, np.full((1, 8), 0.9, np.float32), 2, router="sigmoid_grouped",
                        bias=np.zeros(8, np.float32), n_group=4, topk_group=1, norm_topk=False)
    ids, _ = L.route(x)
    assert ids.cpu().tolist() == [[0, 1]]


def test_glm_bias_steers_selection_not_weight(cuda_ctx):  # glm52/moe.rs:920-943
    import rabbit_b200 as rb

    L = rb.MoeLayer(cuda_ctx, 32, 32, 2, 1, router="sigmoid_grouped", norm_topk=False, max_tokens=1)
    r = np.zeros((2, 32), np.float32)
    r[0, 0], r[1, 0] = 10.0, -10.0
    L.upload_router(r)
    L.upload_router_bias(np.array([0.0, 100.0], np.float32))
    x = np.zeros((1, 32), np.float32)
    x[0, 0] = 1.0
    ids, w = L.route(_t(x))
    assert ids.item() == 1
    assert abs(w.item() - 1.0 / (1.0 + np.exp(10.0))) < 1e-5


def test_glm_route_matches_oracle_c4_shape(cuda_ctx):
    """C4 routing (sigmoid + bias, 8 groups / top-4, top-8 of 256, norm, x2.5) for 512 tokens."""
    import rabbit_b200 as rb

    cfg = synth.CONFIGS["c4_glm_int4"]
    x = synth.activations(cfg)
    router = synth.router_weights(cfg)
    bias = synth.correction_bias(cfg)
    want_ids, want_w = orc.glm_route(x, router, bias, cfg.tokens, cfg.hidden, cfg.n_experts,
                                     cfg.topk, cfg.n_group, cfg.topk_group, True, cfg.routed_scale)
    import torch

    L = rb.MoeLayer(cuda_ctx, cfg.hidden, 32, cfg.n_experts, cfg.topk, router="sigmoid_grouped",
                    n_group=cfg.n_group, topk_group=cfg.topk_group, norm_topk=True,
                    routed_scale=cfg.routed_scale, fmt="int4g", max_tokens=cfg.tokens)
    L.upload_router(synth.f32_to_bf16_bits(router))
    L.upload_router_bias(bias)
    ids, w = L.route(_t(x).to(torch.bfloat16))
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.max(np.abs(w.cpu().numpy() - want_w)) < 1e-5


@pytest.mark.parametrize("T,k,E", [(1, 10, 512), (7, 2, 16), (64, 8, 256), (2048, 10, 512), (0, 4, 16)])
def test_dispatch_matches_reference_order(cuda_ctx, T, k, E):
    """unique_experts (first-occurrence order) and each expert's ascending token list."""
    import torch

    import rabbit_b200 as rb

    rng = np.random.default_rng(T * 31 + E)
    ids = np.array([rng.choice(E, k, replace=False) for _ in range(T)], np.int32).reshape(T, k)
    L = rb.MoeLayer(cuda_ctx, 32, 32, E, k, max_tokens=max(T, 1))
    res = L.dispatch(_t(ids) if T else torch.zeros((0, k), dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    counts = res["counts"].cpu().numpy()
    offsets = res["offsets"].cpu().numpy()
    perm = res["perm_token"].cpu().numpy()
    n_uniq = int(res["n_uniq"].item())
    want_uniq = orc.unique_experts(ids) if T else np.zeros(0, np.int32)
    assert n_uniq == len(want_uniq)
    assert res["uniq"].cpu().numpy()[:n_uniq].tolist() == want_uniq.tolist()
    w = np.ones((T, k), np.float32)
    for e in range(E):
        rows, _ = orc.expert_rows(ids, w, e) if T else (np.zeros(0, np.int32), None)
        assert counts[e] == len(rows)
        assert perm[offsets[e]:offsets[e] + counts[e]].tolist() == rows.tolist()


def test_synth_bytes_match_host_generator(cuda_ctx):
    import torch

    import rabbit_b200 as rb

    key = synth.stream_key(0, synth.tag(0, synth.ROLE_DATA, 5, 1))
    t = torch.empty(1000003, dtype=torch.uint8, device="cuda")
    rb.synth_bytes(t, key, 0)
    assert np.array_equal(t.cpu().numpy(), synth.uniform_bytes(key, t.numel()))
    s = torch.empty(4099, dtype=torch.uint8, device="cuda")
    rb.synth_bytes(s, key, 1, -8, -3)
    assert np.array_equal(s.cpu().numpy(), synth.e8m0_bytes(key, s.numel(), -8, -3))


@pytest.mark.gpu
@pytest.mark.parametrize("E,k,route_j,route_m", [(16, 4, 2, 12), (256, 8, 2, 12), (896, 16, 3, 24), (64, 6, 0, 6)])
def test_cache_route_matches_reference(cuda_ctx, E, k, route_j, route_m):
    """CACHE_ROUTE on the GPU (rmoe_set_route_config + rmoe_route) against the restated
    route_cache_aware: ids bit-exact, weights within 1e-6, for random residency masks, all
    resident and none resident."""
    import dataclasses

    import torch

    import rabbit_b200 as rb
    from rabbit_b200 import synth

    cfg = dataclasses.replace(synth.CONFIGS["c0_tiny"], name="cr", router="sigmoid_grouped", n_experts=E, topk=k,
                              tokens=24, hidden=256, bf16_inputs=False)
    L = rb.MoeLayer(cuda_ctx, cfg.hidden, cfg.inter, E, k, router="sigmoid_grouped", routed_scale=2.5,
                    max_tokens=cfg.tokens)
    router, bias = synth.router_weights(cfg), synth.correction_bias(cfg)
    L.upload_router(router)
    L.upload_router_bias(bias)
    x = synth.activations(cfg)
    xd = torch.from_numpy(x).cuda()
    rng = np.random.default_rng(E + k)
    for res in (None, np.ones(E, bool), np.zeros(E, bool), rng.random(E) < 0.3, rng.random(E) < 0.7):
        L.set_route_config(True, route_j, route_m, res)
        ids, w = L.route(xd)
        want_ids, want_w = orc.glm_route_cache(x, router, bias, cfg.tokens, cfg.hidden, E, k, route_j, route_m,
                                               res if res is not None else None, True, 2.5)
        assert np.array_equal(ids.cpu().numpy(), want_ids)
        assert np.max(np.abs(w.cpu().numpy() - want_w)) < 1e-6
    L.set_route_config(False)
    with pytest.raises(rb.RmoeError, match="NOT_SUPPORTED"):
        q = rb.MoeLayer(cuda_ctx, 256, 128, 16, 2, max_tokens=1)
        q.set_route_config(True)
    L.close()


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["f32", "i8", "i4", "i2", "i4_grouped", "mxfp4"])
@pytest.mark.parametrize("s,i,o", [(1, 4096, 64), (2, 4096, 33), (7, 1000, 19), (13, 64, 5), (3, 37, 4)])
def test_matmul_qt_every_kind(cuda_ctx, kind, s, i, o):
    """rmoe_matmul_qt against the restated kernels::matmul_qt for every QT kind: the integer-dot
    paths (I8 always, I4 at s >= 2) and F32 bit-exact, the float-weight paths within 2e-5 relative
    L2, the grouped / MXFP4 GEMV (f16 activations) within 2e-3."""
    import torch

    import rabbit_b200 as rb

    if kind in ("i4_grouped", "mxfp4") and i % 2:
        pytest.skip("odd widths are covered by the dedicated grouped / MXFP4 tests")
    rng = np.random.default_rng(s * 1000 + i + o)
    x = random_vec(s * i, 77 + s).reshape(s, i)
    gs = 32
    if kind == "f32":
        data, scale = random_vec(o * i, 5).reshape(o, i), np.zeros(1, np.float32)
    elif kind == "i8":
        data, scale = rng.integers(-127, 128, o * i).astype(np.int8), (rng.random(o) * 0.05).astype(np.float32)
    elif kind == "i4":
        data, scale = rng.integers(0, 256, o * ((i + 1) // 2), dtype=np.uint8), (rng.random(o) * 0.05).astype(np.float32)
    elif kind == "i2":
        data, scale = rng.integers(0, 256, o * ((i + 3) // 4), dtype=np.uint8), (rng.random(o) * 0.05).astype(np.float32)
    elif kind == "i4_grouped":
        data = rng.integers(0, 256, o * ((i + 1) // 2), dtype=np.uint8)
        scale = (rng.random(o * ((i + gs - 1) // gs)) * 0.05).astype(np.float32)
    else:
        data, scale = orc.pack_mxfp4(random_vec(o * i, 9) * np.float32(3), o, i)
    want = orc.matmul_qt(x, kind, data, scale, s, i, o, gs=gs)
    y = torch.full((s, o), float("nan"), device="cuda")
    rb.matmul_qt(y, torch.from_numpy(x).cuda(), kind, torch.from_numpy(np.ascontiguousarray(data).view(np.uint8)).cuda(),
                 torch.from_numpy(np.ascontiguousarray(scale)).cuda(), s, i, o, group_size=gs)
    got = y.cpu().numpy()
    if kind in ("f32", "i8") or (kind == "i4" and s >= 2):
        assert np.array_equal(got, want)
    elif kind in ("i4", "i2"):
        assert rel_l2(got, want) < 2e-5
    else:  # (f16 activations on the GEMV path, as the dedicated tests)
        assert rel_l2(got, want) < 2e-3


@pytest.mark.gpu
@pytest.mark.parametrize("E,k,H", [(896, 16, 7168), (256, 8, 2048), (64, 6, 1024)])
def test_few_token_sigmoid_router_matches_reference(cuda_ctx, E, k, H):
    """Few-token ungrouped sigmoid routing (the latent layers' decode case) against the restated
    glm52::moe::route on 96 tokens routed 1, 3 and 8 at a time: ids bit-exact, weights within
    1e-6."""
    import dataclasses

    import torch

    import rabbit_b200 as rb

    cfg = dataclasses.replace(synth.CONFIGS["c0_tiny"], name="cert", router="sigmoid_grouped", n_experts=E, topk=k,
                              tokens=96, hidden=H, bf16_inputs=True)
    L = rb.MoeLayer(cuda_ctx, H, 128, E, k, router="sigmoid_grouped", routed_scale=2.5, max_tokens=8)
    router, bias = synth.router_weights(cfg), synth.correction_bias(cfg)
    L.upload_router(synth.f32_to_bf16_bits(router))
    L.upload_router_bias(bias)
    x = synth.activations(cfg)
    xd = torch.from_numpy(x).cuda().to(torch.bfloat16)
    want_ids, want_w = orc.glm_route(x, router, bias, cfg.tokens, H, E, k, 1, 1, True, 2.5)
    t0 = 0
    for n in [1, 3, 8] * 8 + [1] * 24:
        if t0 + n > cfg.tokens:
            break
        ids, w = L.route(xd[t0:t0 + n])
        assert np.array_equal(ids.cpu().numpy(), want_ids[t0:t0 + n]), t0
        assert np.max(np.abs(w.cpu().numpy() - want_w[t0:t0 + n])) < 1e-6
        t0 += n
    L.close()
