"""Checkpoint / resume of the FDTD state in the reference's RKCKPT01 layout.

Format (crates/ringkernel-core/src/checkpoint.rs): a 64-byte little-endian
header (magic "RKCKPT01" = 0x524B434B50543031, version 1, header size,
total size, chunk count, compression 0, CRC-32/IEEE of every byte after the
header, flags, creation time in microseconds, reserved), the u32-length-
prefixed metadata (:370-415: kernel id, kernel type, current step, grid
size, tile size, HLC timestamp, custom key/value pairs), then chunks of a
32-byte header (:274-282: type, flags, uncompressed size, compressed size,
id) plus raw data.  The state of a leapfrog step is the pair (pressure,
pressure_prev) plus the step counter; both fields are stored as
DeviceMemory chunks (type 5) in z-major f32, "pressure" first.

Chunk ids: the reference hashes the region name with Rust's DefaultHasher;
here the id is the 64-bit FNV-1a hash of the name (readers select the
DeviceMemory chunks by order).  Like the reference's reader, files above
1 GiB are refused unless allow_large=True (the reference cannot read them).
"""
from __future__ import annotations

import struct
import time
import zlib
from dataclasses import dataclass, field

import numpy as np

MAGIC = 0x524B434B50543031
VERSION = 1
MAX_SIZE = 1024 * 1024 * 1024
CHUNK_DEVICE_MEMORY = 5
CHUNK_CUSTOM = 100


def fnv1a64(name: str) -> int:
    h = 0xCBF29CE484222325
    for b in name.encode():
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


@dataclass
class CheckpointMetadata:
    kernel_id: str = "wavesim3d"
    kernel_type: str = "fdtd_3d"
    current_step: int = 0
    grid_size: tuple = (0, 0, 0)
    tile_size: tuple = (128, 8, 1)
    hlc: tuple = (0, 0, 0)
    custom: dict = field(default_factory=dict)

    def to_bytes(self) -> bytes:
        def s(x: str) -> bytes:
            b = x.encode()
            return struct.pack("<I", len(b)) + b
        out = s(self.kernel_id) + s(self.kernel_type) + struct.pack("<Q", self.current_step)
        out += struct.pack("<3I", *self.grid_size) + struct.pack("<3I", *self.tile_size)
        out += struct.pack("<3Q", *self.hlc) + struct.pack("<I", len(self.custom))
        for k, v in self.custom.items():
            out += s(k) + s(v)
        return out

    @classmethod
    def from_bytes(cls, b: bytes) -> "CheckpointMetadata":
        off = 0

        def u32():
            nonlocal off
            v = struct.unpack_from("<I", b, off)[0]
            off += 4
            return v

        def u64():
            nonlocal off
            v = struct.unpack_from("<Q", b, off)[0]
            off += 8
            return v

        def st():
            nonlocal off
            n = u32()
            v = b[off:off + n].decode()
            off += n
            return v

        m = cls(kernel_id=st(), kernel_type=st(), current_step=u64())
        m.grid_size = (u32(), u32(), u32())
        m.tile_size = (u32(), u32(), u32())
        m.hlc = (u64(), u64(), u64())
        for _ in range(u32()):
            k = st()
            m.custom[k] = st()
        return m


def to_bytes(meta: CheckpointMetadata, chunks: list, allow_large: bool = False) -> bytes:
    """chunks: [(type, id, bytes)]."""
    mb = meta.to_bytes()
    total = 64 + 4 + len(mb) + sum(32 + len(d) for _, _, d in chunks)
    if total > MAX_SIZE and not allow_large:
        raise ValueError(f"checkpoint of {total} bytes exceeds the RKCKPT01 limit of {MAX_SIZE}")
    body = bytearray(struct.pack("<I", len(mb)) + mb)
    for ctype, cid, data in chunks:
        body += struct.pack("<IIQQQ", ctype, 0, len(data), len(data), cid)
        body += data
    header = struct.pack("<QIIQIIIIQ8x8x", MAGIC, VERSION, 64, total, len(chunks), 0,
                         zlib.crc32(body) & 0xFFFFFFFF, 0, int(time.time() * 1e6))
    assert len(header) == 64
    return bytes(header) + bytes(body)


def from_bytes(b: bytes, allow_large: bool = False):
    if len(b) < 64:
        raise ValueError("checkpoint too small")
    magic, ver, hsize, total, nchunks, comp, crc, flags, created = struct.unpack_from(
        "<QIIQIIIIQ", b, 0)
    if magic != MAGIC:
        raise ValueError("invalid magic number")
    if ver > VERSION:
        raise ValueError(f"unsupported version {ver}")
    if total > MAX_SIZE and not allow_large:
        raise ValueError(f"checkpoint too large: {total} bytes")
    if zlib.crc32(b[64:]) & 0xFFFFFFFF != crc:
        raise ValueError("checksum mismatch")
    if comp != 0:
        raise ValueError("compressed checkpoints are not supported")
    off = 64
    mlen = struct.unpack_from("<I", b, off)[0]
    off += 4
    meta = CheckpointMetadata.from_bytes(b[off:off + mlen])
    off += mlen
    chunks = []
    for _ in range(nchunks):
        ctype, cflags, usize, csize, cid = struct.unpack_from("<IIQQQ", b, off)
        off += 32
        chunks.append((ctype, cid, b[off:off + csize]))
        off += csize
    return meta, chunks


def save(backend, path: str, allow_large: bool = False) -> CheckpointMetadata:
    """Write the backend's (pressure, pressure_prev, step) to `path`."""
    p, pp = backend.download_field(with_prev=True)
    st = backend.stats()
    meta = CheckpointMetadata(current_step=int(st["step"]),
                              grid_size=(backend.width, backend.height, backend.depth),
                              custom={"z_begin": str(backend.z_begin), "z_end": str(backend.z_end),
                                      "layout": "z-major f32"})
    chunks = [(CHUNK_DEVICE_MEMORY, fnv1a64("pressure"), p.tobytes()),
              (CHUNK_DEVICE_MEMORY, fnv1a64("pressure_prev"), pp.tobytes())]
    with open(path, "wb") as f:
        f.write(to_bytes(meta, chunks, allow_large))
    return meta


def restore(backend, path: str, allow_large: bool = False) -> CheckpointMetadata:
    """Load `path` into the backend: both fields and the step counter."""
    with open(path, "rb") as f:
        meta, chunks = from_bytes(f.read(), allow_large)
    if tuple(meta.grid_size) != (backend.width, backend.height, backend.depth):
        raise ValueError(f"checkpoint grid {meta.grid_size} does not match the backend")
    mem = [d for t, _, d in chunks if t == CHUNK_DEVICE_MEMORY]
    if len(mem) < 2:
        raise ValueError("checkpoint lacks the pressure / pressure_prev chunks")
    p = np.frombuffer(mem[0], dtype=np.float32)
    pp = np.frombuffer(mem[1], dtype=np.float32)
    backend.upload_fields(p, pp)
    backend._chk(backend._lib.ws3d_set_step(backend._ctx, int(meta.current_step)), "set_step")
    return meta
