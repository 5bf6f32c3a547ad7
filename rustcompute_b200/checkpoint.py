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

Chunk ids: the reference ids a DeviceMemory chunk by hashing its region
name with Rust's std DefaultHasher (checkpoint.rs:600-606), which is
SipHash-1-3 with both keys zero over the name's UTF-8 bytes followed by one
0xFF byte (str's Hash writes the bytes and a 0xFF terminator).  The same id
is computed here (`region_id`, SipHash restated from Aumasson & Bernstein,
"SipHash: a fast short-input PRF", 2012), so chunk_identity (:783-797),
content_digest (:806-818) and delta diffing agree with checkpoints the
reference writes for the same region names.  restore() picks the fields by
id, and by order for files whose ids it does not know.  Like the reference's
reader, files above 1 GiB are refused unless allow_large=True (the reference
cannot read them).
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


MASK64 = 0xFFFFFFFFFFFFFFFF
DELTA_PARENT_DIGEST_KEY = "ringkernel.delta.parent_digest"   # checkpoint.rs:776


def _rotl(x: int, b: int) -> int:
    return ((x << b) | (x >> (64 - b))) & MASK64


def siphash(k0: int, k1: int, data: bytes, c_rounds: int = 1, d_rounds: int = 3) -> int:
    """SipHash-c-d of `data` under the 128-bit key (k0, k1), little-endian words,
    as the SipHash paper specifies it: four 64-bit state words initialised from
    the key and the constants "somepseudorandomlygeneratedbytes", c SipRounds
    per 8-byte message word, the last word carrying len mod 256 in its top
    byte, then 0xff xored into v2 and d SipRounds.  c = 1, d = 3 is Rust's
    DefaultHasher; c = 2, d = 4 the paper's recommended instance."""
    v0 = k0 ^ 0x736F6D6570736575
    v1 = k1 ^ 0x646F72616E646F6D
    v2 = k0 ^ 0x6C7967656E657261
    v3 = k1 ^ 0x7465646279746573

    def rounds(n):
        nonlocal v0, v1, v2, v3
        for _ in range(n):
            v0 = (v0 + v1) & MASK64
            v1 = _rotl(v1, 13) ^ v0
            v0 = _rotl(v0, 32)
            v2 = (v2 + v3) & MASK64
            v3 = _rotl(v3, 16) ^ v2
            v0 = (v0 + v3) & MASK64
            v3 = _rotl(v3, 21) ^ v0
            v2 = (v2 + v1) & MASK64
            v1 = _rotl(v1, 17) ^ v2
            v2 = _rotl(v2, 32)

    n = len(data)
    full = n - n % 8
    for i in range(0, full, 8):
        m = int.from_bytes(data[i:i + 8], "little")
        v3 ^= m
        rounds(c_rounds)
        v0 ^= m
    last = ((n & 0xFF) << 56) | int.from_bytes(data[full:], "little")
    v3 ^= last
    rounds(c_rounds)
    v0 ^= last
    v2 ^= 0xFF
    rounds(d_rounds)
    return v0 ^ v1 ^ v2 ^ v3


def region_id(name: str) -> int:
    """The reference's DeviceMemory chunk id of region `name`: Rust's
    DefaultHasher (SipHash-1-3, zero keys) over the str, i.e. its bytes and a
    0xFF terminator (checkpoint.rs:600-606)."""
    return siphash(0, 0, name.encode() + b"\xff", 1, 3)


def chunk_identity(ctype: int, cid: int):
    """(kind, id) as checkpoint.rs:783-797: the id counts for DeviceMemory and
    Custom chunks only."""
    return (ctype, cid if ctype in (CHUNK_DEVICE_MEMORY, CHUNK_CUSTOM) else None)


def content_digest(chunks: list) -> str:
    """checkpoint.rs:806-818: CRC-32/IEEE, continued over every chunk's 16-byte
    identity header (kind u32, id u64, 4 zero bytes; little-endian) and its
    data, as 8 lower-case hex digits.  chunks: [(type, id, bytes)]."""
    crc = 0
    for ctype, cid, data in chunks:
        kind, ident = chunk_identity(ctype, cid)
        crc = zlib.crc32(struct.pack("<IQ4x", kind, ident or 0), crc)
        crc = zlib.crc32(data, crc)
    return f"{crc & 0xFFFFFFFF:08x}"


def delta_from(base_meta: "CheckpointMetadata", base_chunks: list,
               new_meta: "CheckpointMetadata", new_chunks: list):
    """checkpoint.rs:829-852: the chunks of `new` whose bytes differ from the
    chunk of the same identity in `base`, or that `base` lacks; the base's
    content digest is recorded under DELTA_PARENT_DIGEST_KEY."""
    index = {chunk_identity(t, i): d for t, i, d in base_chunks}
    meta = CheckpointMetadata(**{**new_meta.__dict__, "custom": dict(new_meta.custom)})
    meta.custom[DELTA_PARENT_DIGEST_KEY] = content_digest(base_chunks)
    out = [(t, i, d) for t, i, d in new_chunks if index.get(chunk_identity(t, i)) != d]
    return meta, out


def applied_with_delta(base_chunks: list, delta_meta: "CheckpointMetadata", delta_chunks: list):
    """checkpoint.rs:862-903: base chunks replaced by the delta's chunks of
    the same identity, then the delta's new chunks; refuses a delta whose
    recorded parent digest is not the base's."""
    want = delta_meta.custom.get(DELTA_PARENT_DIGEST_KEY)
    have = content_digest(base_chunks)
    if want is not None and want != have:
        raise ValueError(f"delta parent digest mismatch: expected {want}, got {have}")
    index = {chunk_identity(t, i): (t, i, d) for t, i, d in delta_chunks}
    out, used = [], set()
    for t, i, d in base_chunks:
        key = chunk_identity(t, i)
        if key in index:
            out.append(index[key])
            used.add(key)
        else:
            out.append((t, i, d))
    out += [c for c in delta_chunks if chunk_identity(c[0], c[1]) not in used]
    return delta_meta, out


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
    chunks = [(CHUNK_DEVICE_MEMORY, region_id("pressure"), p.tobytes()),
              (CHUNK_DEVICE_MEMORY, region_id("pressure_prev"), pp.tobytes())]
    with open(path, "wb") as f:
        f.write(to_bytes(meta, chunks, allow_large))
    return meta


def restore(backend, path: str, allow_large: bool = False) -> CheckpointMetadata:
    """Load `path` into the backend: both fields and the step counter."""
    with open(path, "rb") as f:
        meta, chunks = from_bytes(f.read(), allow_large)
    if tuple(meta.grid_size) != (backend.width, backend.height, backend.depth):
        raise ValueError(f"checkpoint grid {meta.grid_size} does not match the backend")
    by_id = {i: d for t, i, d in chunks if t == CHUNK_DEVICE_MEMORY}
    pid, ppid = region_id("pressure"), region_id("pressure_prev")
    if pid in by_id and ppid in by_id:
        mem = [by_id[pid], by_id[ppid]]
    else:   # ids this reader does not know: the first two DeviceMemory chunks
        mem = [d for t, _, d in chunks if t == CHUNK_DEVICE_MEMORY]
    if len(mem) < 2:
        raise ValueError("checkpoint lacks the pressure / pressure_prev chunks")
    p = np.frombuffer(mem[0], dtype=np.float32)
    pp = np.frombuffer(mem[1], dtype=np.float32)
    backend.upload_fields(p, pp)
    backend._chk(backend._lib.ws3d_set_step(backend._ctx, int(meta.current_step)), "set_step")
    return meta
