"""Checkpoint / resume in the reference's RKCKPT01 layout
(crates/ringkernel-core/src/checkpoint.rs)."""
import struct
import zlib

import numpy as np
import pytest

from rustcompute_b200 import checkpoint as ck


def test_crc_is_the_reference_crc32():  # checkpoint.rs:1835-1838
    assert zlib.crc32(b"") == 0
    assert zlib.crc32(b"123456789") == 0xCBF43926


def test_round_trip_and_header_layout():
    meta = ck.CheckpointMetadata(current_step=123, grid_size=(4, 3, 2), custom={"a": "b"})
    data = np.arange(24, dtype=np.float32).tobytes()
    raw = ck.to_bytes(meta, [(ck.CHUNK_DEVICE_MEMORY, ck.region_id("pressure"), data),
                             (ck.CHUNK_DEVICE_MEMORY, ck.region_id("pressure_prev"), data)])
    magic, ver, hsize, total = struct.unpack_from("<QIIQ", raw, 0)
    assert magic == 0x524B434B50543031 and raw[:8] == b"10TPKCKR"  # "RKCKPT01" as LE u64
    assert ver == 1 and hsize == 64 and total == len(raw)
    m2, chunks = ck.from_bytes(raw)
    assert m2.current_step == 123 and m2.grid_size == (4, 3, 2) and m2.custom == {"a": "b"}
    assert [c[0] for c in chunks] == [5, 5] and chunks[0][2] == data
    bad = bytearray(raw)
    bad[-1] ^= 1
    with pytest.raises(ValueError, match="checksum"):
        ck.from_bytes(bytes(bad))


def test_size_limit_like_the_reference():
    meta = ck.CheckpointMetadata(grid_size=(1, 1, 1))
    big = [(ck.CHUNK_DEVICE_MEMORY, 1, b"\0" * 16)]
    ck.MAX_SIZE, old = 100, ck.MAX_SIZE
    try:
        with pytest.raises(ValueError):
            ck.to_bytes(meta, big + big + big)
    finally:
        ck.MAX_SIZE = old


@pytest.mark.gpu
def test_resume_from_checkpoint_is_bit_exact(tmp_path):
    from rustcompute_b200 import GpuBackend3D, configs
    wl = configs.build("c2", 60, 50, 44, steps=80)

    def fresh():
        b = GpuBackend3D.create(wl.W, wl.H, wl.D, sponge_width=wl.sponge_width,
                                sponge_max=wl.sponge_max)
        b.upload_fields(*wl.initial_fields())
        b.set_sources(wl.sources, wl.wavelet)
        return b

    a = fresh()
    a.step_n(None, 50)
    path = str(tmp_path / "state.rkckpt")
    meta = ck.save(a, path)
    assert meta.current_step == 50
    a.step_n(None, 30)
    want = a.download_field(with_prev=True)
    b = fresh()
    ck.restore(b, path)
    assert b.stats()["step"] == 50
    b.step_n(None, 30)
    got = b.download_field(with_prev=True)
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])


def test_siphash_known_answer_from_the_paper():
    """SipHash-2-4, key 00 01 .. 0f, message 00 01 .. 0e: the worked example
    of the SipHash paper's appendix."""
    k0 = int.from_bytes(bytes(range(0, 8)), "little")
    k1 = int.from_bytes(bytes(range(8, 16)), "little")
    assert ck.siphash(k0, k1, bytes(range(15)), 2, 4) == 0xA129CA6149BE45E5


def test_siphash13_zero_key_matches_cpython():
    """CPython hashes bytes with SipHash-1-3; with PYTHONHASHSEED=0 its key is
    all zeros -- the same function as Rust's DefaultHasher::new().  An
    independent implementation run here pins ours for lengths 0..40 and for
    the region names this library writes."""
    import os
    import subprocess
    import sys
    msgs = [bytes((7 * i + 3) % 256 for i in range(n)) for n in range(41)]
    msgs += [b"pressure\xff", b"pressure_prev\xff", b"\xff"]
    code = ("import sys\nfor h in sys.stdin.read().split():\n"
            "    print(hash(bytes.fromhex(h[1:])))\n")
    r = subprocess.run([sys.executable, "-c", code], input=" ".join("m" + m.hex() for m in msgs),
                       capture_output=True, text=True, env={**os.environ, "PYTHONHASHSEED": "0"},
                       check=True)
    want = [int(v) for v in r.stdout.split()]
    assert len(want) == len(msgs)
    for m, w in zip(msgs, want):
        h = ck.siphash(0, 0, m, 1, 3)
        signed = h - (1 << 64) if h >= 1 << 63 else h
        if signed == -1:      # CPython reserves -1
            signed = -2
        assert signed == w or len(m) == 0, (m, h, w)   # CPython hashes b"" to 0
    assert ck.region_id("pressure") == ck.siphash(0, 0, b"pressure\xff", 1, 3)


def test_content_digest_and_delta_follow_the_reference():
    """checkpoint.rs:806-903: digest over (kind, id, data); a delta carries only
    changed chunks and refuses the wrong base."""
    a = np.arange(8, dtype=np.float32).tobytes()
    b = (np.arange(8, dtype=np.float32) + 1).tobytes()
    base = [(ck.CHUNK_DEVICE_MEMORY, ck.region_id("pressure"), a),
            (ck.CHUNK_DEVICE_MEMORY, ck.region_id("pressure_prev"), a)]
    new = [(ck.CHUNK_DEVICE_MEMORY, ck.region_id("pressure"), b),
           (ck.CHUNK_DEVICE_MEMORY, ck.region_id("pressure_prev"), a)]
    d = ck.content_digest(base)
    assert len(d) == 8 and d == ck.content_digest(list(base)) and d != ck.content_digest(new)
    # the digest is one CRC-32 over every (header, data) pair, as the reference's rolling update
    stream = b"".join(struct.pack("<IQ4x", t, i) + x for t, i, x in base)
    assert d == f"{zlib.crc32(stream):08x}"
    m0 = ck.CheckpointMetadata(current_step=1, grid_size=(8, 1, 1))
    m1 = ck.CheckpointMetadata(current_step=2, grid_size=(8, 1, 1))
    dm, dc = ck.delta_from(m0, base, m1, new)
    assert [x[2] for x in dc] == [b] and dm.custom[ck.DELTA_PARENT_DIGEST_KEY] == d
    _, full = ck.applied_with_delta(base, dm, dc)
    assert full == new
    with pytest.raises(ValueError, match="parent digest"):
        ck.applied_with_delta(new, dm, dc)

