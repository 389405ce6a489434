"""Archive compiler (host encoder, no GPU): reproduces the archives the
reference's own compile_model wrote (tests/golden/make_archives.py) byte for
byte, and splits tensors into blocks by the reference's rule."""
import json

import pytest

import xksv_compile as xc
import xksv_runtime as rt
from golden.make_archives import HERE as GOLDEN, LLAMA_CONFIG, checkpoint_tensors, write_safetensors


def make_source(tmp_path, kind):
    src = tmp_path / kind
    src.mkdir()
    write_safetensors(src / "model.safetensors", checkpoint_tensors(kind))
    if kind == "llama":
        (src / "config.json").write_text(json.dumps(LLAMA_CONFIG, indent=1))
    return src


@pytest.mark.parametrize("kind", ["llama", "misc"])
@pytest.mark.parametrize("pref,tag", [("dfloat11", "tile16"), ("dfloat11-parallel", "parallel32")])
def test_host_compile_is_byte_identical_to_reference(tmp_path, kind, pref, tag):
    src = make_source(tmp_path, kind)
    out = xc.compile_checkpoint(src, tmp_path / "out.xksv", pref, encoder="host", verify=False)
    assert out.read_bytes() == (GOLDEN / f"{kind}_{tag}.xksv").read_bytes()
    assert not (tmp_path / "out.xksv.partial").exists()


def test_compile_refuses_existing_output(tmp_path):
    src = make_source(tmp_path, "misc")
    (tmp_path / "o.xksv").write_bytes(b"x")
    with pytest.raises(rt.ArchiveError, match="already exists"):
        xc.compile_checkpoint(src, tmp_path / "o.xksv", encoder="host", verify=False)


@pytest.mark.parametrize("dtype,shape,want", [
    # 1-D BF16: 4096-wide rows, 16 at a time, then the partial rows, then the tail
    ("BF16", [100000], [(0, 131072, 16, 4096), (131072, 65536, 8, 4096), (196608, 3392, 1, 1696)]),
    # wider than 32768 columns: fewer than 16 rows per 1 MiB block
    ("BF16", [20, 65536], [(0, 1 << 20, 8, 65536), (1 << 20, 1 << 20, 8, 65536), (2 << 20, 1 << 19, 4, 65536)]),
    # rows of more than 1 MiB: split as a flat tensor
    ("BF16", [1, 600000], [(i * 131072, 131072, 16, 4096) for i in range(9)]
     + [(9 * 131072, 2 * 4096 * 2, 2, 4096), (9 * 131072 + 16384, 1984 * 2, 1, 1984)]),
    ("BF16", [0, 16], []),
    ("F32", [300000], [(0, 1 << 20, 0, 0), (1 << 20, 300000 * 4 - (1 << 20), 0, 0)]),
    ("BF16", [3, 4, 5], [(0, 120, 1, 60)]),
])
def test_block_layout(dtype, shape, want):
    n = 1
    for d in shape:
        n *= d
    size = n * xc.DTYPE_SIZES[dtype]
    got = xc.block_layout(dtype, shape, size)
    assert got == want
    assert sum(b[1] for b in got) == size


def test_checkpoint_rejects_gaps(tmp_path):
    src = make_source(tmp_path, "misc")
    p = src / "model.safetensors"
    p.write_bytes(p.read_bytes() + b"\0")
    with pytest.raises(rt.ArchiveError, match="unreferenced data"):
        xc.checkpoint(src)


def _raw_safetensors(path, header, data=b""):
    hb = json.dumps(header).encode() if not isinstance(header, bytes) else header
    path.write_bytes(len(hb).to_bytes(8, "little") + hb + data)


@pytest.mark.parametrize("header,data,msg", [
    (b'{"a": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2]}, "a": {}}', b"\0\0", "duplicate JSON key: a"),
    (b'{"a": {"dtype": "BF16", "shape": [NaN], "data_offsets": [0, 2]}}', b"\0\0", "invalid JSON number"),
    ({"a": {"dtype": "Q8", "shape": [1], "data_offsets": [0, 1]}}, b"\0", "unsupported dtype Q8 for a"),
    ({"a": {"dtype": "BF16", "shape": [-1], "data_offsets": [0, 2]}}, b"\0\0", "invalid shape: a"),
    ({"a": {"dtype": "BF16", "shape": [2], "data_offsets": [0]}}, b"\0" * 4, "invalid offsets: a"),
    ({"a": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 2]}}, b"\0" * 2, "invalid tensor extent: a"),
    ({"a": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]},
      "b": {"dtype": "BF16", "shape": [2], "data_offsets": [2, 6]}}, b"\0" * 6, "overlapping or noncontiguous"),
    ({"a": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2]}}, b"\0" * 4, "unreferenced data"),
    ([1, 2], b"", "invalid Safetensors header"),
    ({"a": 7}, b"", "invalid descriptor: a"),
])
def test_checkpoint_header_checks(tmp_path, header, data, msg):
    """The Safetensors front end refuses malformed headers with the reference
    compiler's messages (python/xksv.py:30-40, 83-135)."""
    f = tmp_path / "m.safetensors"
    _raw_safetensors(f, header, data)
    with pytest.raises(rt.ArchiveError, match=msg):
        xc.checkpoint(f)


def test_checkpoint_header_length_and_shard_index(tmp_path):
    f = tmp_path / "t.safetensors"
    f.write_bytes((1 << 40).to_bytes(8, "little"))
    with pytest.raises(rt.ArchiveError, match="invalid header length"):
        xc.checkpoint(f)
    d = tmp_path / "sharded"
    d.mkdir()
    _raw_safetensors(d / "a.safetensors", {"x": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2]}}, b"\0\0")
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"x": "../a.safetensors"}}))
    with pytest.raises(rt.ArchiveError, match="invalid shard index"):
        xc.checkpoint(d)
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"y": "a.safetensors"}}))
    with pytest.raises(rt.ArchiveError, match="shard index does not match"):
        xc.checkpoint(d)
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"x": "a.safetensors"}}))
    (shard,) = xc.checkpoint(d)
    assert [t["name"] for t in shard["tensors"]] == ["x"]


@pytest.mark.parametrize("name,role", [
    ("model.embed_tokens.weight", "token_embedding"),
    ("lm_head.weight", "language_model_head"),
    ("model.visual.blocks.0.attn.qkv.weight", "vision_component"),
    ("model.layers.0.linear_attn.conv1d.weight", "deltanet_convolution"),
    ("model.layers.0.linear_attn.in_proj_qkvz.weight", "deltanet_input_projection"),
    ("model.layers.0.linear_attn.out_proj.weight", "deltanet_output_projection"),
    ("model.layers.0.linear_attn.A_log", "deltanet_state_parameter"),
    ("model.layers.0.self_attn.q_proj.weight", "attention_parameter"),
    ("model.layers.0.mlp.experts.3.down_proj.weight", "moe_expert"),
    ("model.layers.0.mlp.router.weight", "moe_router"),
    ("model.layers.0.mlp.gate_proj.weight", "feed_forward_parameter"),
    ("model.layers.0.input_layernorm.weight", "normalization_parameter"),
    ("rotary.inv_freq", "other"),
])
def test_tensor_role_labels(name, role):
    assert xc.tensor_role(name) == role
