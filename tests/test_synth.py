"""The seeded generator (host side): determinism, value ranges, and that any slice of a stream
regenerates identically (what lets the oracle rebuild only the experts a batch touches)."""
import numpy as np

from rabbit_b200 import synth


def test_splitmix64_first_outputs():
    # SplitMix64 from state 0: the published first output is 0xE220A8397B1DCDAF
    assert int(synth.u64(0, 0, 1)[0]) == 0xE220A8397B1DCDAF


def test_uniform_bytes_cover_all_nibbles_and_are_deterministic():
    k = synth.stream_key(0, synth.tag(0, synth.ROLE_DATA, 3, synth.GATE))
    a = synth.uniform_bytes(k, 1 << 16)
    assert np.array_equal(a, synth.uniform_bytes(k, 1 << 16))
    lo, hi = a & 0xF, a >> 4
    for nib in (lo, hi):
        counts = np.bincount(nib, minlength=16)
        assert counts.min() > 0.9 * counts.mean()


def test_e8m0_bytes_stay_in_the_configured_exponent_range():
    k = synth.stream_key(0, 99)
    b = synth.e8m0_bytes(k, 10000, -8, -3)
    assert b.min() == 127 - 8 and b.max() == 127 - 3


def test_activation_token_slices_match_the_full_stream():
    cfg = synth.CONFIGS["c0_tiny"]
    full = synth.activations(cfg, tokens=6)
    part = synth.activations(cfg, tokens=3, token_offset=3)
    assert np.array_equal(full[3:], part)
    assert abs(float(full.std()) - 1.0) < 0.1


def test_bf16_rounding_is_round_to_nearest_even():
    v = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5], np.float32)
    r = synth.round_bf16(v)
    assert r.tolist() == [1.0, 1.0, 1.0 + 2 ** -6, -2.5]


def test_zipf_bias_is_a_permutation_of_log_ranks():
    cfg = synth.CONFIGS["c1_qwen_decode"]
    b = synth.logit_bias(cfg)
    want = np.sort((-1.1 * np.log(np.arange(1, 513, dtype=np.float64))).astype(np.float32))
    assert np.array_equal(np.sort(b), want)


def test_expert_layout_sizes_match_the_reference_formula():
    cfg = synth.CONFIGS["c1_qwen_decode"]
    ex = synth.expert(cfg, 7)
    total = sum(v.nbytes for v in ex.values())
    assert total == cfg.expert_bytes() == 26_738_688
    c4 = synth.CONFIGS["c4_glm_int4"]
    assert c4.expert_bytes() == 23_592_960
    assert c4.expert_bytes(scale_bytes=2) == 21_233_664
