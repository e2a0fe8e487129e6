"""The checkpoint loader (rmoe_shards_* / rmoe_load_*): .safetensors shards into the HBM expert
tables. The CPU tests restate the reference's own Shards tests (src/safetensors.rs:656-800):
multi-shard and multi-directory indexing, raw reads, missing tensors as errors, and the three
malformed-header rejections. The GPU tests load a synthetic layer written under the reference's
checkpoint tensor names and compare it with the same layer uploaded directly."""
import dataclasses
import struct

import numpy as np
import pytest

import rabbit_b200 as rb
from rabbit_b200 import synth
from st_fixture import build_safetensors, write, write_layer


def f32_bytes(vals):
    return np.asarray(vals, np.float32).tobytes()


def test_indexes_and_reads_multiple_shards(tmp_path):
    write(tmp_path / "model-00001-of-00002.safetensors",
          [("dense.weight", "F32", [2, 3], f32_bytes([1, 2, 3, 4, 5, 6]))])
    write(tmp_path / "model-00002-of-00002.safetensors",
          [("expert.0.raw", "U8", [4], bytes([10, 20, 30, 40])),
           ("half.weight", "F16", [2], bytes([0x00, 0x3C, 0x00, 0xC0])),
           ("bf16.weight", "BF16", [2], bytes([0xC0, 0x3F, 0x40, 0x40]))])
    sh = rb.Shards(str(tmp_path))
    assert len(sh) == 4
    assert sh.has("dense.weight") and not sh.has("nope.weight")
    assert sh.tensor("dense.weight") == {"dtype": "F32", "shape": [2, 3], "nbytes": 24}
    assert np.array_equal(sh.read_raw("dense.weight").view(np.float32), [1, 2, 3, 4, 5, 6])
    assert list(sh.read_raw("expert.0.raw")) == [10, 20, 30, 40]
    assert sh.tensor("bf16.weight")["dtype"] == "BF16"
    sh.close()


def test_open_multi_indexes_shards_split_across_separate_directories(tmp_path):
    d1, d2 = tmp_path / "a", tmp_path / "b"
    d1.mkdir()
    d2.mkdir()
    write(d1 / "out-00000.safetensors", [("dense.weight", "F32", [2, 3], f32_bytes([1, 2, 3, 4, 5, 6]))])
    write(d2 / "out-00001.safetensors", [("expert.0.raw", "U8", [4], bytes([10, 20, 30, 40]))])
    sh = rb.Shards(str(d1), str(d2))
    assert sh.has("dense.weight") and sh.has("expert.0.raw")
    assert list(sh.read_raw("expert.0.raw")) == [10, 20, 30, 40]


def test_missing_tensor_is_an_error_not_a_crash(tmp_path):
    write(tmp_path / "model.safetensors", [("a", "F32", [1], f32_bytes([1]))])
    sh = rb.Shards(str(tmp_path))
    with pytest.raises(rb.RmoeError, match="MISSING_TENSOR: missing tensor: does.not.exist"):
        sh.read_raw("does.not.exist")


def test_read_raw_wants_the_exact_byte_count(tmp_path):
    from rabbit_b200 import _lib

    write(tmp_path / "model.safetensors", [("a", "U8", [4], bytes([1, 2, 3, 4]))])
    sh = rb.Shards(str(tmp_path))
    buf = np.zeros(3, np.uint8)
    assert _lib.load().rmoe_shards_read_raw(sh.handle, b"a", buf.ctypes.data, 3) == 2  # SHAPE_MISMATCH


def test_open_rejects_a_header_length_claiming_to_exceed_the_file(tmp_path):
    (tmp_path / "model.safetensors").write_bytes(struct.pack("<Q", 2**64 - 1) + b"{}")
    with pytest.raises(rb.RmoeError, match="IO_ERROR: .*exceeds file size"):
        rb.Shards(str(tmp_path))


def _raw_file(path, header: dict, data: bytes):
    import json

    hb = json.dumps(header).encode()
    path.write_bytes(struct.pack("<Q", len(hb)) + hb + data)


def test_open_rejects_data_offsets_where_end_precedes_start(tmp_path):
    _raw_file(tmp_path / "model.safetensors", {"a": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}},
              f32_bytes([1]))
    with pytest.raises(rb.RmoeError, match="IO_ERROR: .*end precedes start"):
        rb.Shards(str(tmp_path))


def test_open_rejects_data_offsets_extending_past_end_of_file(tmp_path):
    _raw_file(tmp_path / "model.safetensors", {"a": {"dtype": "F32", "shape": [1024], "data_offsets": [0, 4096]}}, b"")
    with pytest.raises(rb.RmoeError, match="IO_ERROR: .*past end of file"):
        rb.Shards(str(tmp_path))


def test_header_parsing_edge_cases(tmp_path):
    """Escaped names, nested metadata, a later shard's tensor of the same name winning, an empty
    shard, and malformed JSON as an error."""
    _raw_file(tmp_path / "a.safetensors",
              {"__metadata__": {"format": "pt", "nested": {"x": [1, 2, {"y": 'z\\"}'}]}},
               "wéight\"q": {"dtype": "U8", "shape": [2], "data_offsets": [0, 2]},
               "dup": {"dtype": "U8", "shape": [1], "data_offsets": [2, 3]}}, bytes([7, 8, 9]))
    write(tmp_path / "b.safetensors", [("dup", "U8", [2], bytes([5, 6]))])
    write(tmp_path / "c.safetensors", [])
    sh = rb.Shards(str(tmp_path))
    assert list(sh.read_raw("wéight\"q")) == [7, 8]
    assert list(sh.read_raw("dup")) == [5, 6]
    (tmp_path / "d.safetensors").write_bytes(struct.pack("<Q", 5) + b'{"a":')
    with pytest.raises(rb.RmoeError, match="IO_ERROR"):
        rb.Shards(str(tmp_path))


def test_fixture_writer_matches_the_reference_layout():
    """The test writer's bytes: length prefix, JSON header, data in order."""
    raw = build_safetensors([("x", "U8", [2], bytes([1, 2])), ("y", "U8", [1], bytes([3]))])
    hl = struct.unpack("<Q", raw[:8])[0]
    assert raw[8 + hl:] == bytes([1, 2, 3])


# ------------------------------------------------------------------------------ GPU
def _tiny_glm():
    """A tiny GLM-style grouped-int4 layer (f32 .qs scales, the reference converter's format)."""
    return dataclasses.replace(synth.CONFIGS["c0_tiny"], name="tiny_glm_int4", fmt="int4g", router="sigmoid_grouped",
                               shared_gated=False, n_group=4, topk_group=2, routed_scale=2.5, topk=4)


@pytest.mark.gpu
@pytest.mark.parametrize("naming,cfg_name", [("qwen38_mxfp4", "c0_tiny"), ("kimi_k3_mxfp4", "c0_tiny"),
                                             ("glm52", "glm"), ("glm52_fused_gate_up", "glm"),
                                             ("kimi_linear", "glm"), ("kimi_k3", "glm")])
def test_loaded_layer_equals_directly_uploaded_layer(cuda_ctx, tmp_path, naming, cfg_name):
    """A layer loaded from a checkpoint (router, bias, shared expert, every routed expert, over two
    shard files) computes bit-identically to the same weights uploaded from memory, and routes
    like the reference."""
    import torch

    from helpers import build_layer, oracle_forward, x_device
    from refvec import rel_l2

    cfg = synth.CONFIGS["c0_tiny"] if cfg_name == "c0_tiny" else _tiny_glm()
    family = "qwen38" if cfg.router == "softmax" else "glm52"
    write_layer(str(tmp_path), cfg, naming, family)
    want_layer = build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    L = rb.MoeLayer(cuda_ctx, cfg.hidden, cfg.inter, cfg.n_experts, cfg.topk, shared_inter=cfg.shared_inter,
                    router=cfg.router, n_group=cfg.n_group, topk_group=cfg.topk_group, norm_topk=cfg.norm_topk,
                    routed_scale=cfg.routed_scale, fmt=cfg.fmt, group_size=cfg.group_size, scale_dtype="f32",
                    shared_gated=cfg.shared_gated, max_tokens=cfg.tokens)
    sh = rb.Shards(str(tmp_path))
    L.load_moe_weights(sh, family, 0)
    L.load_experts(sh, naming, 0)
    sh.close()
    x = synth.activations(cfg)
    got, ids, _ = L.moe_forward(x_device(cfg, x), return_routing=True)
    want = want_layer.moe_forward(x_device(cfg, x))
    assert torch.equal(got, want)
    ref, ref_ids, _ = oracle_forward(cfg, x)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    assert rel_l2(got.cpu().numpy(), ref) < 1e-2
    L.close()
    want_layer.close()


@pytest.mark.gpu
def test_loader_errors(cuda_ctx, tmp_path):
    """A truncated packed tensor is a SHAPE_MISMATCH naming it (mxfp4_from_raw's check), a plain
    float expert tensor is NOT_SUPPORTED, an absent expert is MISSING_TENSOR."""
    cfg = synth.CONFIGS["c0_tiny"]
    h, i = cfg.hidden, cfg.inter
    ex = synth.expert(cfg, 0)
    pre = "model.layers.0.mlp.experts.0."
    write(tmp_path / "model.safetensors", [
        (pre + "gate_proj.weight", "U8", [i, h // 2], ex["gate"][:-1].tobytes()),
        (pre + "gate_proj.weight_scale", "U8", [i, h // 32], ex["gate_scale"].tobytes()),
        (pre + "up_proj.weight", "U8", [i, h // 2], ex["up"].tobytes()),
        (pre + "up_proj.weight_scale", "U8", [i, h // 32], ex["up_scale"].tobytes()),
        (pre + "down_proj.weight", "U8", [h, i // 2], ex["down"].tobytes()),
        (pre + "down_proj.weight_scale", "U8", [h, i // 32], ex["down_scale"].tobytes()),
        ("model.layers.0.mlp.experts.1.gate_proj.weight", "F32", [i, h], np.zeros(i * h, np.float32).tobytes()),
    ])
    L = rb.MoeLayer(cuda_ctx, h, i, cfg.n_experts, cfg.topk, max_tokens=2)
    sh = rb.Shards(str(tmp_path))
    with pytest.raises(rb.RmoeError, match="SHAPE_MISMATCH: model.layers.0.mlp.experts.0.gate_proj.weight"):
        L.load_expert(sh, "qwen38_mxfp4", 0, 0)
    gl = rb.MoeLayer(cuda_ctx, h, i, cfg.n_experts, cfg.topk, max_tokens=2, fmt="int4g", group_size=32)
    with pytest.raises(rb.RmoeError, match="NOT_SUPPORTED: .*plain float"):
        gl.load_expert(sh, "glm52", 0, 1)
    with pytest.raises(rb.RmoeError, match="MISSING_TENSOR"):
        L.load_expert(sh, "qwen38_mxfp4", 0, 2)
    sh.close()
    L.close()
    gl.close()
