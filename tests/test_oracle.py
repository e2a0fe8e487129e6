"""Pins the CPU oracle (oracle/liboracle.so) to the reference's own known-answer tests.

Each test restates one #[test] of ferrumox/rabbit v0.29.1 (cited per test) against the C
restatement. These run without a GPU.
"""
import math

import numpy as np
import pytest

from oracle import oracle as orc
from refvec import lcg_logits, random_vec, rel_l2

E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


# ---------------------------------------------------------------- quant.rs tests
def test_e2m1_decode_matches_the_spec_s_8_positive_magnitudes():  # quant.rs:858-866
    for code, want in enumerate(E2M1):
        assert orc.e2m1_decode(code) == want
        got = orc.e2m1_decode(code | 0x8)
        assert got == -want and math.copysign(1.0, got) == -1.0


def test_e2m1_encode_round_trips_every_exact_representable_value():  # quant.rs:868-875
    for code in range(16):
        v = orc.e2m1_decode(code)
        assert orc.e2m1_decode(orc.e2m1_encode(v)) == v


def test_e2m1_encode_rounds_to_nearest_and_ties_keep_lower():  # quant.rs:877-886
    assert orc.e2m1_decode(orc.e2m1_encode(2.9)) == 3.0
    assert orc.e2m1_decode(orc.e2m1_encode(5.0)) == 4.0
    assert orc.e2m1_decode(orc.e2m1_encode(-2.9)) == -3.0


def test_e8m0_decode_is_a_power_of_two_biased_by_127():  # quant.rs:888-893
    assert orc.e8m0_decode(127) == 1.0
    assert orc.e8m0_decode(128) == 2.0
    assert orc.e8m0_decode(126) == 0.5
    assert orc.e8m0_decode(131) == 16.0


def test_e8m0_decode_matches_powi_exactly_across_the_whole_valid_byte_range():  # quant.rs:895-905
    for b in range(255):
        assert orc.e8m0_decode(b) == float(np.float32(math.ldexp(1.0, b - 127))), b


def test_choose_block_scale_keeps_amax_within_e2m1_range():  # quant.rs:907-921
    assert orc.choose_block_scale(6.0) == (127, 1.0)
    assert orc.choose_block_scale(12.0) == (128, 2.0)
    b, s = orc.choose_block_scale(0.0)
    assert s == 1.0 and b != 0xFF


def test_mxfp4_fill_and_row_f32_round_trip_within_one_step():  # quant.rs:923-938
    rows, cols = 3, 40
    w = random_vec(rows * cols, 123)
    q, bs = orc.pack_mxfp4(w, rows, cols)
    for o in range(rows):
        row = orc.row_f32_mxfp4(q, bs, cols, o)
        assert np.all(np.abs(row - w[o * cols:(o + 1) * cols]) < 0.5)


def test_mxfp4_uses_a_separate_scale_per_32_element_block():  # quant.rs:940-959
    cols = 64
    w = np.ones(cols, np.float32)
    w[32:] = 100.0
    q, bs = orc.pack_mxfp4(w, 1, cols)
    row = orc.row_f32_mxfp4(q, bs, cols, 0)
    assert np.all(np.abs(row[:32] - 1.0) < 0.5)
    assert np.all(np.abs(row[32:] - 100.0) < 8.0)


def test_quant_int4_grouped_tighter_scale_for_the_low_magnitude_group():  # quant.rs:829-842
    data, scale = orc.quant_int4_grouped(np.array([100.0, 0.0, 3.0, -8.0], np.float32), 1, 4, 4, 2)
    assert scale.size == 2
    assert scale[1] == np.float32(8.0) / np.float32(7.0)
    assert data[1] == (3 + 8) | ((-7 + 8) << 4)


def test_quant_int4_grouped_trailing_partial_group():  # quant.rs:844-854
    _, scale = orc.quant_int4_grouped(np.array([1.0, 1.0, -9.0], np.float32), 1, 3, 4, 2)
    assert scale.size == 2
    assert scale[1] == np.float32(9.0) / np.float32(7.0)


# ---------------------------------------------------------------- kernels.rs tests
def test_matmul_matches_hand_computed_dot_products():  # kernels.rs:1323-1331
    x = np.array([1.0, 2.0, 3.0, -1.0, 0.5, 2.0], np.float32)
    w = np.array([1.0, 0.0, 0.0, 0.0, 1.0, 1.0], np.float32)
    y = orc.matmul(x, w, 2, 3, 2)
    assert y.ravel().tolist() == [1.0, 5.0, -1.0, 2.5]


def known_answer_mxfp4():
    """kernels.rs:1388-1406: 40 columns, block 0 at code 4 (2.0) scale 1, block 1 (8-wide tail)
    at code 7|sign (-6.0) scale 8 -> 32*2 + 8*(-48) = -320."""
    cols = 40
    data = np.zeros((cols + 1) // 2, np.uint8)
    data[0:16] = 4 | (4 << 4)
    data[16:20] = (7 | 8) | ((7 | 8) << 4)
    bs = np.array([127, 130], np.uint8)
    x = np.ones(cols, np.float32)
    return x, data, bs, cols


def test_matmul_mxfp4_matches_manual_e2m1_decode_across_two_blocks():
    x, data, bs, cols = known_answer_mxfp4()
    y = orc.matmul_mxfp4(x, data, bs, 1, cols, 1)
    assert y[0, 0] == 32.0 * 2.0 + 8.0 * -48.0 == -320.0


def known_answer_i4g():
    """kernels.rs:1408-1428: 6 columns, group 3, scales 2 and 5 -> (1-1+2)*2 + (3-2+0)*5 = 9."""
    vals = [1, -1, 2, 3, -2, 0]
    b = np.zeros(3, np.uint8)
    for i, v in enumerate(vals):
        b[i // 2] |= (v + 8) << (4 * (i % 2))
    return np.ones(6, np.float32), b, np.array([2.0, 5.0], np.float32)


def test_matmul_i4_grouped_matches_manual_nibble_unpack_across_two_groups():
    x, b, sc = known_answer_i4g()
    y = orc.matmul_i4_grouped(x, b, sc, 3, 1, 6, 1)
    assert y[0, 0] == 9.0


def test_matmul_qt_mxfp4_matches_manual_dequant_dot_product():  # kernels.rs:1570-1596
    rows, cols, s = 5, 96, 2
    w = random_vec(rows * cols, 31)
    x = random_vec(s * cols, 32)
    q, bs = orc.pack_mxfp4(w, rows, cols)
    want = np.zeros((s, rows), np.float32)
    for si in range(s):
        for oi in range(rows):
            r = orc.row_f32_mxfp4(q, bs, cols, oi)
            acc = np.float32(-0.0)
            for a, b in zip(r, x[si * cols:(si + 1) * cols]):
                acc = np.float32(acc + np.float32(a * b))
            want[si, oi] = acc
    for tier in ("scalar", "avx512"):
        if tier == "avx512" and not orc.has_avx512():
            continue
        y = orc.matmul_mxfp4(x, q, bs, s, cols, rows, tier=tier)
        assert np.all(np.abs(y - want) < 1e-3)


@pytest.mark.parametrize("cols", [1, 7, 16, 17, 32, 33, 65])
def test_matmul_mxfp4_avx512_matches_scalar_within_tolerance(cols):  # kernels.rs:1939-1958
    if not orc.has_avx512():
        pytest.skip("no AVX-512F/BW on this CPU")
    rows = 3
    w = random_vec(rows * cols, cols * 3 + 9)
    q, bs = orc.pack_mxfp4(w, rows, cols)
    x = random_vec(cols, cols * 7 + 10)
    a = orc.matmul_mxfp4(x, q, bs, 1, cols, rows)
    b = orc.matmul_mxfp4(x, q, bs, 1, cols, rows, tier="avx512")
    assert np.all(np.abs(a - b) < 1e-4)


# ---------------------------------------------------------------- qwen38/moe.rs tests
def reference_route(logits, topk):
    """qwen38/moe.rs:92-101: the four HF lines, transcribed (full softmax -> top-k -> renorm)."""
    l = np.asarray(logits, np.float32)
    mx = np.float32(np.max(l))
    ex = np.array([np.float32(math.exp(float(np.float32(v - mx)))) for v in l], np.float32)
    total = np.float32(-0.0)
    for v in ex:
        total = np.float32(total + v)
    probs = (ex / total).astype(np.float32)
    idx = sorted(range(len(probs)), key=lambda i: (-probs[i], i))[:min(topk, len(probs))]
    s = np.float32(-0.0)
    for i in idx:
        s = np.float32(s + probs[i])
    return [(i, float(probs[i] / s)) for i in idx]


def test_route_matches_the_reference_order_of_operations():  # qwen38/moe.rs:113-127
    for seed in range(1, 6):
        l = lcg_logits(512, seed)
        got = orc.qwen_route(l, 10)
        want = reference_route(l, 10)
        assert len(got) == 10
        for (gi, gw), (wi, ww) in zip(got, want):
            assert gi == wi
            assert abs(gw - ww) < 1e-6


def test_weights_sum_to_one_and_come_back_descending():  # qwen38/moe.rs:129-138
    c = orc.qwen_route(lcg_logits(64, 7), 10)
    assert abs(sum(w for _, w in c) - 1.0) < 1e-5
    assert all(a[1] >= b[1] for a, b in zip(c, c[1:]))


def test_selects_exactly_the_largest_logits():  # qwen38/moe.rs:140-147
    c = orc.qwen_route([0.0, 2.0, -1.0, 5.0, 0.5, -3.0, 1.0, 3.0], 3)
    assert [i for i, _ in c] == [3, 7, 1]
    assert c[0][1] > c[1][1] > c[2][1]


def test_routing_is_invariant_to_a_constant_logit_shift():  # qwen38/moe.rs:151-161
    l = lcg_logits(128, 11)
    a = orc.qwen_route(l, 10)
    b = orc.qwen_route(l + np.float32(17.5), 10)
    for (ai, aw), (bi, bw) in zip(a, b):
        assert ai == bi and abs(aw - bw) < 1e-6


def test_ties_break_toward_the_lower_expert_id():  # qwen38/moe.rs:163-171
    assert [i for i, _ in orc.qwen_route([1.0, 1.0, 1.0, 1.0], 2)] == [0, 1]
    assert [i for i, _ in orc.qwen_route([0.0, 5.0, 5.0, 5.0], 2)] == [1, 2]


def test_topk_at_or_above_the_expert_count_selects_every_expert():  # qwen38/moe.rs:173-182
    a = orc.qwen_route([3.0, 1.0, 2.0], 10)
    assert [i for i, _ in a] == [0, 2, 1]
    assert abs(sum(w for _, w in a) - 1.0) < 1e-6
    assert orc.qwen_route([3.0, 1.0, 2.0], 0) == []


def test_shared_expert_gate_is_a_plain_sigmoid_of_one_logit():  # qwen38/moe.rs:184-189
    assert abs(orc.sigmoid(0.0) - 0.5) < 1e-6
    assert orc.sigmoid(10.0) > 0.999
    assert orc.sigmoid(-10.0) < 0.001


# ---------------------------------------------------------------- glm52/moe.rs tests
def test_route_selection_uses_biased_score_but_weight_uses_plain_sigmoid():  # glm52/moe.rs:920-943
    ids, w = orc.glm_route(np.array([1.0, 0.0], np.float32),
                           np.array([10.0, 0.0, -10.0, 0.0], np.float32),
                           np.array([0.0, 100.0], np.float32), 1, 2, 2, 1, 1, 1, False, 1.0)
    assert ids[0, 0] == 1
    assert abs(w[0, 0] - 1.0 / (1.0 + math.exp(10.0))) < 1e-5


def test_route_norm_topk_normalizes_weights_to_sum_to_routed_scale():  # glm52/moe.rs:945-961
    router = random_vec(4 * 5, 3)
    bias = random_vec(24, 3)[20:24]
    x = random_vec(29, 3)[24:29]
    ids, w = orc.glm_route(x, router, bias, 1, 5, 4, 3, 1, 1, True, 2.0)
    assert abs(float(w.sum()) - 2.0) < 1e-5


def test_top2_sum_adds_the_two_largest_values():  # glm52/moe.rs:965-969
    assert orc.top2_sum([1.0, 5.0, 3.0, 2.0]) == 8.0
    assert orc.top2_sum([5.0, 5.0]) == 10.0


def test_top2_sum_falls_back_to_the_single_value_for_a_one_element_group():  # :971-974
    assert orc.top2_sum([7.0]) == 7.0


def test_rank_top_grouped_matches_plain_rank_top_when_n_group_is_one():  # :976-981
    c = [0.5, 3.0, 1.0, 4.0, 2.0]
    assert orc.rank_top_grouped(c, c, 2, 1, 1) == [(3, 4.0), (1, 3.0)]


def test_rank_top_grouped_keeps_only_experts_from_the_top_scoring_groups():  # :983-996
    c = [0.1, 0.2, 9.0, 8.0, 0.3, 0.4, 7.0, 6.5]
    assert [i for i, _ in orc.rank_top_grouped(c, c, 3, 4, 2)] == [2, 3, 6]


def test_rank_top_grouped_ties_keep_the_lower_group_index():  # :998-1007
    c = [0.9] * 8
    assert [i for i, _ in orc.rank_top_grouped(c, c, 2, 4, 1)] == [0, 1]


def test_unique_experts_first_occurrence_and_rows_ascending():  # glm52/moe.rs:333-344, :465-470
    ids = np.array([[5, 2], [2, 7], [9, 5]], np.int32)
    w = np.array([[0.6, 0.4], [0.3, 0.7], [0.9, 0.1]], np.float32)
    assert orc.unique_experts(ids).tolist() == [5, 2, 7, 9]
    rows, rw = orc.expert_rows(ids, w, 5)
    assert rows.tolist() == [0, 2] and np.allclose(rw, [0.6, 0.1])


# ---------------------------------------------------------------- end to end
def _mxfp4_expert(d, i, seed):
    g = random_vec(i * d, seed)
    u = random_vec(i * d, seed + 1)
    dn = random_vec(d * i, seed + 2)
    gq, gs = orc.pack_mxfp4(g, i, d)
    uq, us = orc.pack_mxfp4(u, i, d)
    dq, ds = orc.pack_mxfp4(dn, d, i)
    return {"gate": gq, "gate_scale": gs, "up": uq, "up_scale": us, "down": dq, "down_scale": ds}


def _dequant(data, bs, rows, cols):
    return np.stack([orc.row_f32_mxfp4(data, bs, cols, r) for r in range(rows)])


def test_moe_output_matches_independent_full_expert_sum():  # glm52/moe.rs:1037-1136 (Qwen form)
    e, k, d, i, s = 3, 3, 64, 32, 2
    experts = [_mxfp4_expert(d, i, 100 + 10 * n) for n in range(e)]
    shared = _mxfp4_expert(d, i, 200)
    router = random_vec(e * d, 7)
    x = random_vec(s * d, 8).reshape(s, d)
    sg = random_vec(d, 9)
    out, ids, w = orc.moe_forward_qwen(x, router, experts, e, k, i, shared=shared, shared_gate=sg)

    def silu(v):
        return v / (1.0 + np.exp(-v))

    want = np.zeros((s, d), np.float64)
    for si in range(s):
        for j in range(k):
            ex = experts[ids[si, j]]
            g = _dequant(ex["gate"], ex["gate_scale"], i, d) @ x[si]
            u = _dequant(ex["up"], ex["up_scale"], i, d) @ x[si]
            want[si] += w[si, j] * (_dequant(ex["down"], ex["down_scale"], d, i) @ (silu(g) * u))
        g = _dequant(shared["gate"], shared["gate_scale"], i, d) @ x[si]
        u = _dequant(shared["up"], shared["up_scale"], i, d) @ x[si]
        sh = _dequant(shared["down"], shared["down_scale"], d, i) @ (silu(g) * u)
        want[si] += sh / (1.0 + math.exp(-float(x[si] @ sg)))
    assert sorted(ids[0].tolist()) == [0, 1, 2]
    assert np.max(np.abs(out - want)) < 1e-4
    assert rel_l2(out, want) < 1e-5


# ---- CACHE_ROUTE (glm52::moe::cache_route_select), the reference's known answers
def test_cache_route_keeps_true_top_j_on_a_cold_cache():  # glm52/moe.rs:719-728
    choice = [0.0, 1.0, 2.0, 3.0, 4.0]
    picked = orc.cache_route_select(choice, choice, 3, 2, 5, resident=np.zeros(5, bool))
    assert [e for e, _ in picked] == [4, 3, 2]


def test_cache_route_prefers_resident_experts():  # glm52/moe.rs:731-753
    choice = [0.0, 1.0, 2.0, 3.0, 4.0]
    res = np.zeros(5, bool)
    res[[0, 1]] = True
    picked = orc.cache_route_select(choice, choice, 3, 1, 5, resident=res)
    assert [e for e, _ in picked] == [4, 1, 0]
    assert all(w == choice[e] for e, w in picked)  # a substitute keeps its own plain sigmoid


def test_cache_route_fills_resident_slots_then_falls_back():  # glm52/moe.rs:756-777
    choice = [0.0, 1.0, 2.0, 3.0, 4.0]
    res = np.zeros(5, bool)
    res[0] = True
    picked = orc.cache_route_select(choice, choice, 3, 1, 5, resident=res)
    assert [e for e, _ in picked] == [4, 0, 3]


def test_cache_route_all_resident_equals_plain_route():  # glm52/moe.rs:701-716, 780-830
    """With every expert resident (or none: the cold cache), CACHE_ROUTE selects exactly the
    ungrouped plain top-k, ids and weights bit for bit."""
    import dataclasses

    from rabbit_b200 import synth

    cfg = dataclasses.replace(synth.CONFIGS["c0_tiny"], router="sigmoid_grouped", topk=4)
    x, r, b = synth.activations(cfg), synth.router_weights(cfg), synth.correction_bias(cfg)
    i0, w0 = orc.glm_route(x, r, b, 4, 256, 16, 4, 1, 1, True, 2.5)
    for res in (None, np.ones(16, bool), np.zeros(16, bool)):
        i1, w1 = orc.glm_route_cache(x, r, b, 4, 256, 16, 4, 2, 12, res, True, 2.5)
        assert np.array_equal(i0, i1) and np.array_equal(w0, w1)


# ---- matmul_qt's other QT kinds (kernels.rs tests), replayed on the restatement
def _pack_nibbles(vals):
    b = np.zeros((len(vals) + 1) // 2, np.uint8)
    for idx, v in enumerate(vals):
        b[idx // 2] |= np.uint8((v + 8) << (4 * (idx % 2)))
    return b


def test_matmul_i4_matches_manual_nibble_unpack():  # kernels.rs:1352-1370
    vals = [3, -7, 0, 5, -2]
    y = orc.matmul_qt(np.ones(5, np.float32), "i4", _pack_nibbles(vals), np.array([2.0], np.float32), 1, 5, 1)
    assert y[0, 0] == sum(vals) * 2.0


def test_matmul_i2_matches_manual_unpack():  # kernels.rs:1373-1386
    vals = [-2, 1, 0, -1, 1]
    b = np.zeros(2, np.uint8)
    for idx, v in enumerate(vals):
        b[idx // 4] |= np.uint8((v + 2) << ((idx % 4) * 2))
    y = orc.matmul_qt(np.ones(5, np.float32), "i2", b, np.array([3.0], np.float32), 1, 5, 1)
    assert y[0, 0] == sum(vals) * 3.0


def test_dot_i8i8_and_i4i8_match_naive_sums():  # kernels.rs:1599-1621
    w = np.array([(i % 7) - 3 for i in range(40)], np.int8)
    x = np.array([(i % 5) - 2 for i in range(40)], np.int8)
    assert orc.dot_i8i8(w, x) == int(np.dot(w.astype(np.int32), x.astype(np.int32)))
    vals = [(i % 16) - 8 for i in range(41)]
    x4 = np.array([(i % 5) - 2 for i in range(41)], np.int8)
    assert orc.dot_i4i8(_pack_nibbles(vals), x4, 41) == int(np.dot(np.array(vals), x4.astype(np.int32)))


def test_qrow_i8_round_trips_close_to_original():  # kernels.rs:1624-1632
    x = random_vec(64, 5)
    q, s = orc.qrow_i8(x)
    assert np.all(np.abs(q.astype(np.float32) * s - x) < 0.02)


def test_matmul_qt_i8_idot_is_close_to_the_float_path():  # kernels.rs:1652-1673 (and :1334-1349)
    rows, cols, s = 4, 16, 2
    w = random_vec(rows * cols, 21).reshape(rows, cols)
    amax = np.abs(w).max(axis=1)
    scale = np.maximum(amax / np.float32(127), np.float32(1e-12)).astype(np.float32)
    q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    x = random_vec(s * cols, 22).reshape(s, cols)
    direct = (x @ (q.astype(np.float32) * scale[:, None]).T).astype(np.float32)
    y = orc.matmul_qt(x, "i8", q, scale, s, cols, rows)
    assert np.max(np.abs(direct - y)) < 0.05
    # integer-valued weights with scale 1 and x = 1: the IDOT path is exact (amax 127 -> scale 1)
    qi = np.array([[10, -20, 30, 127]], np.int8)
    y1 = orc.matmul_qt(np.ones(4, np.float32), "i8", qi, np.array([1.0], np.float32), 1, 4, 1)
    assert y1[0, 0] == 147.0


def test_matmul_qt_i4_gates_idot_by_seq_len():  # kernels.rs:1676-1700
    rows, cols = 3, 10
    rng = np.random.default_rng(31)
    q4 = rng.integers(0, 256, rows * 5, dtype=np.uint8)
    sc = (rng.random(rows) * 0.1).astype(np.float32)
    x1 = random_vec(cols, 32)
    y1 = orc.matmul_qt(x1, "i4", q4, sc, 1, cols, rows)  # s = 1: the float path
    want = np.zeros(rows, np.float32)
    for o in range(rows):
        a = np.float32(0)
        for k in range(0, cols, 2):
            b = q4[o * 5 + k // 2]
            a = np.float32(a + np.float32(np.float32(x1[k] * np.float32(int(b & 15) - 8))
                                          + np.float32(x1[k + 1] * np.float32(int(b >> 4) - 8))))
        want[o] = np.float32(a * sc[o])
    assert np.array_equal(y1[0], want)
    x2 = random_vec(2 * cols, 33).reshape(2, cols)  # s = 2: the integer-dot path
    y2 = orc.matmul_qt(x2, "i4", q4, sc, 2, cols, rows)
    for si in range(2):
        xq, sx = orc.qrow_i8(x2[si])
        for o in range(rows):
            d = orc.dot_i4i8(q4[o * 5:(o + 1) * 5], xq, cols)
            assert y2[si, o] == np.float32(np.float32(np.float32(d) * sc[o]) * sx)
