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
    raw = ck.to_bytes(meta, [(ck.CHUNK_DEVICE_MEMORY, ck.fnv1a64("pressure"), data),
                             (ck.CHUNK_DEVICE_MEMORY, ck.fnv1a64("pressure_prev"), data)])
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
