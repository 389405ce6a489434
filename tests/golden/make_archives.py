"""Generates the golden .xksv archives under tests/golden/ with the reference's
own compiler (python/xksv.py:197-300, compile_model) and CPU codec.

Run here, where the reference tree exists and oracle/Makefile compiles its CPU
codec into oracle/_ref/libxksv_native.so:

    make -C oracle && python tests/golden/make_archives.py

Two seeded Safetensors checkpoints are written to a temporary directory and
compiled twice each, with codec preference ``dfloat11`` (serial blocks,
"bf16-huffman-tile16") and ``dfloat11-parallel`` ("bf16-huffman-parallel32"):

* ``llama``: a one-layer Llama (hidden 64, FFN 184, 4/2 heads, vocab 128,
  untied) with config.json as an archive asset; weights N(0, 0.02) rounded to
  BF16 (round-to-nearest-even), norms 1.0.  FFN 184 gives ragged 16x16 tiles
  (184 % 16 = 8) in down_proj's columns and gate/up's rows.
* ``misc``: the archive layouts around the model weights: an F32 tensor and a
  U8 tensor of odd size (raw blocks of the compiler's non-BF16 branch), a 1-D
  BF16 tensor (one 1 x 1000 block), uniform BF16 bit patterns (stored raw
  because they do not compress, python/xksv.py:277), 40 rows (blocks of 16, 16
  and 8 rows), 3000 columns (ragged tiles), an empty tensor, an I64 tensor,
  and ``proj.weight`` [40, 1536], wide enough for the parallel codec to
  compress its 16-row blocks (the 8-row tail stays raw): the mixed-codec
  weight of the fused GEMV tests.  The Llama weights are too narrow for the
  parallel codec's per-slab tables to pay off, so that archive stores them raw.

The archive index carries the reference's SHA-256 of every block's and every
tensor's decoded bytes, which is what the GPU tests check the device decode
against; the weights themselves are regenerated from the seeds below by
``checkpoint_tensors``.
"""
import json
import os
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
# the reference tree: $XKSV_REFERENCE, else a directory named "reference"
# beside this repository's root
REF = Path(os.environ.get("XKSV_REFERENCE", ROOT.parent / "reference"))

LLAMA_CONFIG = {
    "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 64,
    "intermediate_size": 184, "num_hidden_layers": 1, "num_attention_heads": 4,
    "num_key_value_heads": 2, "vocab_size": 128, "max_position_embeddings": 64,
    "rms_norm_eps": 1e-5, "rope_theta": 10000.0, "tie_word_embeddings": False,
    "torch_dtype": "bfloat16", "hidden_act": "silu", "attention_bias": False, "mlp_bias": False,
}


def bf16_rne(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype("<u2")


def checkpoint_tensors(kind):
    """[(name, dtype, shape, little-endian bytes)] in file order, seeded."""
    rng = np.random.default_rng(7 if kind == "llama" else 8)
    out = []
    if kind == "llama":
        h, f, v, kv = 64, 184, 128, 32
        def w(name, r, c):
            out.append((name, "BF16", [r, c], bf16_rne(rng.standard_normal(r * c) * 0.02).tobytes()))
        def norm(name):
            out.append((name, "BF16", [h], bf16_rne(np.ones(h)).tobytes()))
        w("model.embed_tokens.weight", v, h)
        p = "model.layers.0."
        norm(p + "input_layernorm.weight")
        w(p + "self_attn.q_proj.weight", h, h)
        w(p + "self_attn.k_proj.weight", kv, h)
        w(p + "self_attn.v_proj.weight", kv, h)
        w(p + "self_attn.o_proj.weight", h, h)
        norm(p + "post_attention_layernorm.weight")
        w(p + "mlp.gate_proj.weight", f, h)
        w(p + "mlp.up_proj.weight", f, h)
        w(p + "mlp.down_proj.weight", h, f)
        norm("model.norm.weight")
        w("lm_head.weight", v, h)
    else:
        out.append(("misc.f32", "F32", [10, 7], rng.standard_normal(70).astype("<f4").tobytes()))
        out.append(("misc.u8odd", "U8", [13], rng.integers(0, 256, 13, dtype=np.uint8).tobytes()))
        out.append(("misc.bf16_1d", "BF16", [1000], bf16_rne(rng.standard_normal(1000)).tobytes()))
        out.append(("misc.uniform", "BF16", [16, 48],
                    rng.integers(0, 1 << 16, 16 * 48, dtype=np.uint32).astype("<u2").tobytes()))
        out.append(("misc.rows40", "BF16", [40, 80], bf16_rne(rng.standard_normal(3200) * 0.02).tobytes()))
        out.append(("misc.cols3000", "BF16", [2, 3000], bf16_rne(rng.standard_normal(6000) * 0.05).tobytes()))
        out.append(("misc.empty", "BF16", [0, 16], b""))
        out.append(("misc.i64", "I64", [5], np.arange(5, dtype="<i8").tobytes()))
        out.append(("proj.weight", "BF16", [40, 1536], bf16_rne(rng.standard_normal(40 * 1536) * 0.02).tobytes()))
    return out


def write_safetensors(path, tensors):
    header, pos = {}, 0
    for name, dtype, shape, data in tensors:
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [pos, pos + len(data)]}
        pos += len(data)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h)
        for *_, data in tensors:
            f.write(data)


def main():
    os.environ.setdefault("XKSV_LIBRARY", str(ROOT / "oracle" / "_ref" / "libxksv_native.so"))
    sys.path.insert(0, str(REF / "python"))
    import xksv  # the reference's compiler (read-only tree)

    with tempfile.TemporaryDirectory() as tmp:
        for kind in ("llama", "misc"):
            src = Path(tmp) / kind
            src.mkdir()
            write_safetensors(src / "model.safetensors", checkpoint_tensors(kind))
            if kind == "llama":
                (src / "config.json").write_text(json.dumps(LLAMA_CONFIG, indent=1))
            for pref, tag in (("dfloat11", "tile16"), ("dfloat11-parallel", "parallel32")):
                dst = HERE / f"{kind}_{tag}.xksv"
                if dst.exists():
                    dst.unlink()
                xksv.compile_model(str(src), str(dst), workers=2, codec_preference=pref)
                print(dst.name, dst.stat().st_size)


if __name__ == "__main__":
    main()
