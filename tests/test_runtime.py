"""Archive runtime host logic (no GPU): the index reader and its checks, the
plan rows built from an index, fused-layer eligibility and model assignment,
against archives compiled by the reference's own compiler
(tests/golden/make_archives.py).  The oracle decodes blocks on the CPU as the
checker of the index's digests and of the generator's seeds."""
import hashlib
import json
import struct

import numpy as np
import pytest

import xksv_runtime as rt
from golden.make_archives import HERE as GOLDEN, LLAMA_CONFIG, checkpoint_tensors
from oracle.oracle import Oracle

ARCHIVES = {
    ("llama", "tile16"): GOLDEN / "llama_tile16.xksv",
    ("llama", "parallel32"): GOLDEN / "llama_parallel32.xksv",
    ("misc", "tile16"): GOLDEN / "misc_tile16.xksv",
    ("misc", "parallel32"): GOLDEN / "misc_parallel32.xksv",
}


def read(path):
    with open(path, "rb") as f:
        index, limit = rt.load_index(f)
    return index, limit, rt.check_index(index, limit)


@pytest.mark.parametrize("key", sorted(ARCHIVES))
def test_golden_archive_index_and_blocks(key):
    """Index checks pass; every block decodes (oracle) to the generator's bytes
    and to the block digest the reference compiler stored."""
    kind, _ = key
    path = ARCHIVES[key]
    index, limit, tensors = read(path)
    data = path.read_bytes()
    src = {name: raw for name, _, _, raw in checkpoint_tensors(kind)}
    assert list(tensors) == list(src)
    oracle = Oracle()
    for name, t in tensors.items():
        assert hashlib.sha256(src[name]).hexdigest() == t["sha256"]
        pos = 0
        for b in t["blocks"]:
            blob = data[b["offset"]:b["offset"] + b["size"]]
            if b["codec"] == "raw":
                dec = blob
            elif b["codec"] == "bf16-huffman-tile16":
                dec = oracle.unpack(blob, b["rows"], b["cols"])
            else:
                dec = oracle.unpack_parallel(blob)
            assert dec == src[name][pos:pos + b["raw_size"]]
            assert hashlib.sha256(dec).hexdigest() == b["sha256"]
            pos += b["raw_size"]
        assert pos == t["size"]


def test_codec_mix_of_fixtures():
    """The fixtures cover every codec, ragged and short slabs, empty tensors."""
    seen = set()
    for path in ARCHIVES.values():
        for t in read(path)[2].values():
            seen |= {b["codec"] for b in t["blocks"]}
    assert seen == set(rt.CODECS)
    t = read(ARCHIVES["misc", "parallel32"])[2]
    assert [b["codec"] for b in t["proj.weight"]["blocks"]] == \
        ["bf16-huffman-parallel32", "bf16-huffman-parallel32", "raw"]
    assert t["misc.empty"]["blocks"] == [] and t["misc.empty"]["size"] == 0


def test_decode_entries_offsets():
    _, limit, tensors = read(ARCHIVES["misc", "tile16"])
    t = tensors["misc.rows40"]
    e = rt.decode_entries(t["blocks"], base=512)
    assert [x["dst_offset"] for x in e] == [512, 512 + 2560, 512 + 5120]
    assert [x["rows"] for x in e] == [16, 16, 8] and {x["codec"] for x in e} == {1}
    for x, b in zip(e, t["blocks"]):
        assert x["src_offset"] == b["offset"] - 16 and x["src_offset"] + x["src_size"] <= limit - 16
    raw = rt.decode_entries(tensors["misc.u8odd"]["blocks"])
    assert raw == [dict(src_offset=raw[0]["src_offset"], src_size=13, rows=0, cols=0, dst_offset=0, codec=0)]


def test_gemm_entries_rows_of_raw_blocks():
    t = read(ARCHIVES["misc", "parallel32"])[2]["proj.weight"]
    e = rt.gemm_entries(t)
    assert [(x["rows"], x["cols"], x["dst_offset"], x["codec"]) for x in e] == \
        [(16, 1536, 0, 2), (16, 1536, 16, 2), (8, 1536, 32, 0)]


def tiny_llama():
    transformers = pytest.importorskip("transformers")
    cfg = transformers.LlamaConfig(**{k: v for k, v in LLAMA_CONFIG.items()
                                      if k not in ("architectures", "model_type", "torch_dtype")})
    return transformers.LlamaForCausalLM(cfg)


def test_fused_candidates_follow_reference_rules():
    import torch
    model = tiny_llama()
    names = rt.fused_candidates(model, read(ARCHIVES["llama", "tile16"])[2])
    assert sorted(n.rsplit(".", 1)[1] for n in names) == sorted(
        ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"])
    # the parallel archive stores these narrow weights raw: nothing to fuse
    assert rt.fused_candidates(model, read(ARCHIVES["llama", "parallel32"])[2]) == []
    proj = torch.nn.Module()
    proj.proj = torch.nn.Linear(1536, 40, bias=False)
    for tag in ("tile16", "parallel32"):
        assert rt.fused_candidates(proj, read(ARCHIVES["misc", tag])[2]) == ["proj"]
    proj.proj = torch.nn.Linear(1536, 40, bias=True)
    assert rt.fused_candidates(proj, read(ARCHIVES["misc", "tile16"])[2]) == []


def test_assign_tensors_checks_names():
    import torch
    model = tiny_llama()
    src = {name: torch.frombuffer(bytearray(raw), dtype=torch.bfloat16).reshape(shape)
           for name, _, shape, raw in checkpoint_tensors("llama")}
    rt.assign_tensors(model, dict(src))
    assert torch.equal(model.lm_head.weight.view(torch.int16), src["lm_head.weight"].view(torch.int16))
    with pytest.raises(rt.ArchiveError, match="does not accept"):
        rt.assign_tensors(tiny_llama(), dict(src, **{"extra.weight": src["lm_head.weight"]}))
    partial = dict(src)
    del partial["model.norm.weight"]
    with pytest.raises(rt.ArchiveError, match="missing backend weights"):
        rt.assign_tensors(tiny_llama(), partial)


def rewrite(path, tmp_path, edit=None, head=None):
    data = bytearray(path.read_bytes())
    magic, off = struct.unpack_from("<8sQ", data, 0)
    index = json.loads(bytes(data[off:]))
    if edit:
        edit(index)
    out = bytes(data[:off]) + json.dumps(index).encode()
    if head:
        out = head(out)
    p = tmp_path / "bad.xksv"
    p.write_bytes(out)
    return p


def first_coded(index):
    for s in index["shards"]:
        for t in s["tensors"]:
            for b in t["blocks"]:
                if b["codec"] != "raw":
                    return b


@pytest.mark.parametrize("case,msg", [
    ("magic", "invalid archive header"),
    ("offset", "invalid archive header"),
    ("version", "unsupported archive"),
    ("codec", "unknown codec"),
    ("dims", "invalid compressed block dimensions"),
    ("overlap", "overlapping or unreferenced"),
    ("raw_len", "invalid raw block length"),
    ("shape", "conflicts with stored header"),
])
def test_bad_archives_rejected(tmp_path, case, msg):
    src = ARCHIVES["misc", "tile16"]
    edit = head = None
    if case == "magic":
        head = lambda d: b"XKSV\x00\x02\r\n" + d[8:]
    elif case == "offset":
        head = lambda d: d[:8] + struct.pack("<Q", 1 << 40) + d[16:]
    elif case == "version":
        edit = lambda ix: ix.update(version=2)
    elif case == "codec":
        edit = lambda ix: first_coded(ix).update(codec="zstd")
    elif case == "dims":
        edit = lambda ix: first_coded(ix).update(rows=first_coded(ix)["rows"] + 1)
    elif case == "overlap":
        edit = lambda ix: first_coded(ix).update(offset=first_coded(ix)["offset"] + 1)
    elif case == "raw_len":
        edit = lambda ix: ix["shards"][0]["tensors"][0]["blocks"][0].update(raw_size=281)
    elif case == "shape":
        edit = lambda ix: ix["shards"][0]["tensors"][0].update(shape=[10, 8])
    p = rewrite(src, tmp_path, edit, head)
    with pytest.raises(rt.ArchiveError, match=msg):
        read(p)


def test_truncated_file(tmp_path):
    p = tmp_path / "t.xksv"
    p.write_bytes(b"XKSV\x00")
    with pytest.raises(rt.ArchiveError):
        read(p)
