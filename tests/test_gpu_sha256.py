"""GPU: SHA-256 (FIPS 180-4) of decoded bytes (xksv_cuda_sha256,
xksv_plan_sha256) against hashlib, the standard's worked examples, and the
reference's own block digests in the golden fixtures."""
import hashlib

import numpy as np
import pytest

from helpers import load_golden, words_for
from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def xg():
    import xksv_gpu
    assert torch.cuda.is_available()
    xksv_gpu.load()
    return xksv_gpu


def gpu_digests(xg, buf, ranges):
    d = torch.frombuffer(bytearray(buf), dtype=torch.uint8).cuda() if len(buf) else torch.zeros(1, dtype=torch.uint8, device="cuda")
    out = torch.zeros(max(1, len(ranges)) * 32, dtype=torch.uint8, device="cuda")
    xg.sha256_ranges(ranges, d.data_ptr(), out.data_ptr())
    got = out.cpu().numpy().tobytes()
    return [got[32 * i:32 * i + 32] for i in range(len(ranges))]


def test_fips_examples(xg):
    buf = b"abc" + b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq"
    ranges = [(0, 3), (3, 56), (0, 0)]
    got = gpu_digests(xg, buf, ranges)
    assert got[0].hex() == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"
    assert got[1].hex() == "248d6a61d20638b8e5c026930c3e6039a33ce45964ff2167f6ecedd419db06c1"
    assert got[2].hex() == "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"


def test_lengths_and_alignments(xg):
    rng = np.random.default_rng(1)
    buf = rng.integers(0, 256, 3 << 20, dtype=np.uint8).tobytes()
    lens = [0, 1, 3, 4, 5, 55, 56, 57, 63, 64, 65, 119, 120, 121, 127, 128, 129, 1000, 65543, 1 << 20]
    ranges = [(off, n) for n in lens for off in (0, 1, 2, 3, 6, 17)]
    got = gpu_digests(xg, buf, ranges)
    for (off, n), d in zip(ranges, got):
        assert d == hashlib.sha256(buf[off:off + n]).digest(), (off, n)


def test_plan_sha256_matches_golden_and_hashlib(xg):
    """Decode the golden slabs (both codecs) with a plan, hash on the GPU: the
    digests equal the reference's recorded SHA-256 of each slab's raw bytes."""
    cases = [g for g in load_golden() if g["serial"] is not None]
    payload, entries, out = bytearray(b"\x00"), [], 0
    want = []
    for g in cases:
        for codec, blob in ((1, g["serial"]), (2, g["parallel"])):
            if blob is None:
                continue
            entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=g["rows"],
                                cols=g["cols"], dst_offset=out + 2 * (len(entries) % 2), codec=codec))
            payload += blob
            out += g["rows"] * g["cols"] * 2 + 6
            want.append(g["sha256"])
    d_payload = torch.frombuffer(payload, dtype=torch.uint8).cuda()
    d_out = torch.zeros(out + 8, dtype=torch.uint8, device="cuda")
    plan = xg.Plan(entries)
    plan.decode(d_payload, d_out)
    dig = torch.zeros(32 * len(entries), dtype=torch.uint8, device="cuda")
    plan.sha256(d_out, dig)
    assert plan.status() == 0
    got = dig.cpu().numpy().tobytes()
    for i, w in enumerate(want):
        assert got[32 * i:32 * i + 32] == w, entries[i]
    plan.close()


def test_plan_sha256_raw_and_tensor(xg):
    """Raw slabs hash their src_size bytes; a tensor's digest is one range over
    its slabs' contiguous outputs (src/compile.cpp:483)."""
    oracle = Oracle()
    rng = np.random.default_rng(4)
    w = words_for("normal002", 48 * 1024, rng).reshape(48, 1024)
    payload, entries, raws = bytearray(), [], []
    for k, r0 in enumerate(range(0, 48, 16)):
        raw = w[r0:r0 + 16].astype("<u2").tobytes()
        codec = [0, 1, 2][k]
        blob = raw if codec == 0 else oracle.pack(raw, 16, 1024) if codec == 1 else oracle.pack_parallel(raw, 16, 1024)
        entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=16, cols=1024,
                            dst_offset=r0 * 2048, codec=codec))
        payload += blob
        raws.append(raw)
    d_payload = torch.frombuffer(payload, dtype=torch.uint8).cuda()
    d_out = torch.zeros(48 * 2048, dtype=torch.uint8, device="cuda")
    plan = xg.Plan(entries)
    plan.decode(d_payload, d_out)
    dig = torch.zeros(32 * 3, dtype=torch.uint8, device="cuda")
    plan.sha256(d_out, dig)
    assert plan.status() == 0
    got = dig.cpu().numpy().tobytes()
    for i, raw in enumerate(raws):
        assert got[32 * i:32 * i + 32] == hashlib.sha256(raw).digest()
    tensor = torch.zeros(32, dtype=torch.uint8, device="cuda")
    xg.sha256_ranges([(0, 48 * 2048)], d_out.data_ptr(), tensor.data_ptr())
    assert tensor.cpu().numpy().tobytes() == hashlib.sha256(b"".join(raws)).digest()
    plan.close()
