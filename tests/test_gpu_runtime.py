"""Archive runtime on the GPU: resident upload, device SHA-256 verification,
one-plan decode of whole archives, fused linear layers (batch 1 and batch > 1)
in a Transformers Llama, against archives compiled by the reference's own
compiler (tests/golden/make_archives.py)."""
import hashlib
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import xksv_runtime as rt  # noqa: E402
from golden.make_archives import HERE as GOLDEN, checkpoint_tensors  # noqa: E402

KINDS = [("llama", "tile16"), ("llama", "parallel32"), ("misc", "tile16"), ("misc", "parallel32")]


def path_of(kind, tag):
    return GOLDEN / f"{kind}_{tag}.xksv"


@pytest.mark.parametrize("kind,tag", KINDS)
def test_verify_and_decode_all_bit_exact(kind, tag):
    a = rt.ResidentArchive(path_of(kind, tag), "cuda:0")
    n, nbytes = a.verify()
    src = {name: raw for name, _, _, raw in checkpoint_tensors(kind)}
    assert n == len(src) and nbytes == sum(len(v) for v in src.values())
    out = a.decode_all()
    torch.cuda.synchronize()
    for name, raw in src.items():
        got = out[name].contiguous().view(torch.uint8).reshape(-1).cpu().numpy().tobytes() if raw else b""
        assert got == raw, name
        assert list(out[name].shape) == a.tensors[name]["shape"]
    # single-tensor decode agrees
    name = max(src, key=lambda k: len(src[k]))
    assert a.tensor(name).view(torch.uint8).reshape(-1).cpu().numpy().tobytes() == src[name]


def corrupt_copy(tmp_path, kind, tag, where):
    """A copy with one byte flipped in the first coded block: in its
    sign/mantissa bytes (decodes, wrong digest) or its count (header error)."""
    data = bytearray(path_of(kind, tag).read_bytes())
    off = struct.unpack_from("<Q", data, 8)[0]
    import json
    index = json.loads(bytes(data[off:]))
    b = next(b for s in index["shards"] for t in s["tensors"] for b in t["blocks"]
             if b["codec"] == "bf16-huffman-tile16")
    if where == "sm":
        data[b["offset"] + 16 + 256 + 5] ^= 0x01
    else:  # count word: the block's header no longer matches its rows x cols
        data[b["offset"]] ^= 0x01
    p = tmp_path / "corrupt.xksv"
    p.write_bytes(bytes(data))
    return p


def test_verify_detects_flipped_mantissa(tmp_path):
    a = rt.ResidentArchive(corrupt_copy(tmp_path, "misc", "tile16", "sm"), "cuda:0")
    with pytest.raises(rt.ArchiveError, match="block checksum failed"):
        a.verify()


def test_decode_reports_bad_header(tmp_path):
    a = rt.ResidentArchive(corrupt_copy(tmp_path, "misc", "tile16", "count"), "cuda:0")
    with pytest.raises(rt.ArchiveError, match="GPU block decode failed"):
        a.verify()


def test_parallel_header_checked_at_load(tmp_path):
    data = bytearray(path_of("misc", "parallel32").read_bytes())
    off = struct.unpack_from("<Q", data, 8)[0]
    import json
    index = json.loads(bytes(data[off:]))
    b = next(b for s in index["shards"] for t in s["tensors"] for b in t["blocks"]
             if b["codec"] == "bf16-huffman-parallel32")
    struct.pack_into("<Q", data, b["offset"] + 16, b["cols"] + 16)  # stored cols
    p = tmp_path / "p.xksv"
    p.write_bytes(bytes(data))
    with pytest.raises(rt.ArchiveError, match="parallel block dimensions"):
        rt.ResidentArchive(p, "cuda:0")


@pytest.mark.parametrize("tag", ["tile16", "parallel32"])
@pytest.mark.parametrize("batch", [1, 3, 16, 40])
def test_fused_weight_mixed_codecs(tag, batch):
    """proj.weight: two coded 16-row blocks and (parallel archive) a raw
    8-row block, y = x W^T for batch 1 (CUDA cores, FP32 x) and > 1."""
    a = rt.ResidentArchive(path_of("misc", tag), "cuda:0")
    a.verify()
    fw = a.fused("proj.weight")
    W = a.tensor("proj.weight").float()
    g = torch.Generator(device="cuda:0").manual_seed(batch)
    x = torch.randn(batch, 1536, device="cuda:0", generator=g)
    y = fw(x if batch > 1 else x[0])
    ref = x @ W.t() if batch > 1 else W @ x[0]
    if batch >= 4:  # tensor-core path: x rounded to BF16
        ref = x.bfloat16().float() @ W.t()
    err = float((y.float() - ref).norm() / ref.norm())
    assert err < (1e-5 if batch < 4 else 1e-2), err
    assert y.shape == ref.shape
    fw.close()


def test_fused_weights_share_one_scratch():
    """Batch >= 4 (tensor cores) on two fused weights of one archive: both borrow the
    archive's single tensor-core scratch and stay correct."""
    a = rt.ResidentArchive(path_of("llama", "tile16"), "cuda:0")
    a.verify()
    names = ["model.layers.0.mlp.gate_proj.weight", "model.layers.0.mlp.down_proj.weight"]
    fws = [a.fused(n) for n in names]
    g = torch.Generator(device="cuda:0").manual_seed(9)
    for _ in range(2):
        for n, fw in zip(names, fws):
            W = a.tensor(n).float()
            x = torch.randn(12, W.shape[1], device="cuda:0", generator=g)
            y = fw(x)
            ref = x.bfloat16().float() @ W.t()
            assert float((y - ref).norm() / ref.norm()) < 1e-2
    assert all(fw._lent is a.shared_scratch() for fw in fws if fw._scratch_need)
    for fw in fws:
        fw.close()


def test_fused_llama_matches_decoded_model():
    """load_archive builds the model from the archive's config asset, decodes
    every weight in one plan; the fused model's logits match the decoded one
    for one decode step and a 7-token prefill."""
    pytest.importorskip("transformers")
    path = path_of("llama", "tile16")
    ref_model, _, _ = rt.load_archive(path, "cuda:0")
    model, tok, archive = rt.load_archive(path, "cuda:0", fused_gemv=True)
    assert tok is None  # the fixture has no tokenizer files
    fused = [n for n, m in model.named_modules() if hasattr(m, "xksv_fused")]
    assert len(fused) == 7
    # fused weights stay compressed: their parameters hold no decoded bytes
    mods = dict(model.named_modules())
    assert all(mods[n].weight.numel() == 0 for n in fused)
    ids = torch.tensor([[3, 17, 99, 4, 64, 1, 127]], device="cuda:0")
    with torch.no_grad():
        for inp in (ids[:, :1], ids):
            want = ref_model(inp).logits.float()
            got = model(inp).logits.float()
            err = float((got - want).norm() / want.norm())
            assert err < 1e-2, err


@pytest.mark.parametrize("kind", ["llama", "misc"])
@pytest.mark.parametrize("pref,tag", [("dfloat11", "tile16"), ("dfloat11-parallel", "parallel32")])
def test_gpu_compile_is_byte_identical_to_reference(tmp_path, kind, pref, tag):
    """The GPU encoder's archive equals the one the reference's compile_model
    wrote, and passes the device verification."""
    import json
    import xksv_compile as xc
    from golden.make_archives import LLAMA_CONFIG, write_safetensors
    src = tmp_path / kind
    src.mkdir()
    write_safetensors(src / "model.safetensors", checkpoint_tensors(kind))
    if kind == "llama":
        (src / "config.json").write_text(json.dumps(LLAMA_CONFIG, indent=1))
    out = xc.compile_checkpoint(src, tmp_path / "out.xksv", pref, encoder="gpu", device="cuda:0", verify=True)
    assert out.read_bytes() == path_of(kind, tag).read_bytes()
