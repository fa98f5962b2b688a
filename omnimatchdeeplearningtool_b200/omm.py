""".omm model files: the reference's parameter format, read into the named weights this package's
plans take (``InferencePlan``, ``Fp32Net``), and written back.

The layout follows the reference serializer (src/engine/om.engine.serializer.ixx:1-6 and
:174-315 for writing, :367-455 and :559-650 for reading), all integers little-endian uint32:

    "OMM\\0" | version (bit 31: encrypted) | [v >= 4: n_meta | n_meta float32]
    | n_params | params | [v >= 2: n_buffers | buffers] | crc32

with each parameter or buffer ``name_len | name | n_dims | dims | float32 data``. The checksum
is CRC-32 (IEEE, reflected, pre- and post-inverted) over every byte before it, the decrypted
ones for an encrypted file (serializer.ixx:786-792). Encryption XORs every byte after the
version word with a keystream derived from the password: an FNV-1a 64-bit hash seeds a
xorshift64 chain, each state emitting its 8 bytes low byte first (serializer.ixx:54-99).
Version 4 and 5 metadata is 8 float32 (serializer.ixx:128-140): a 42.0 marker, the model-type
hash's bit pattern, base channels, input size, classes, input channels, norm type, groups.

Names are the reference's ``Module::namedParameters()`` / ``namedBuffers()`` names
(``layer1.0.conv1.weight``, ``bn1.running_mean``, ...), which the plans use directly.
"""
import struct
import zlib
from typing import Dict, Optional, Tuple

import numpy as np

MAGIC = b"OMM\0"
ENCRYPTED = 0x80000000
META_MARKER = 42.0
_M64 = (1 << 64) - 1


class OmmError(ValueError):
    """The file is not an .omm file this reader accepts, or it is damaged."""


def _keystream(password: str, n: int) -> np.ndarray:
    """The reference's XOR keystream for `password` (serializer.ixx:54-88)."""
    h = 14695981039346656037
    for ch in password.encode("utf-8"):
        h = ((h ^ ch) * 1099511628211) & _M64
    seed = state = h
    out = bytearray()
    while len(out) < n:
        out += state.to_bytes(8, "little")
        state ^= (state << 13) & _M64
        state ^= state >> 7
        state ^= (state << 17) & _M64
        state = (state + seed) & _M64
    return np.frombuffer(bytes(out[:n]), dtype=np.uint8)


def _xor(data: bytes, password: str) -> bytes:
    a = np.frombuffer(data, dtype=np.uint8)
    return (a ^ _keystream(password, len(a))).tobytes()


def model_type_hash(name: str) -> int:
    """FNV-1a 32-bit of a model-type string (serializer.ixx:121-125)."""
    h = 2166136261
    for ch in name.encode("utf-8"):
        h = ((h ^ ch) * 16777619) & 0xFFFFFFFF
    return h


class _Reader:
    def __init__(self, data: bytes):
        self.d, self.i = data, 0

    def take(self, n: int) -> bytes:
        if self.i + n > len(self.d):
            raise OmmError(f"truncated file: need {n} bytes at offset {self.i}")
        b = self.d[self.i:self.i + n]
        self.i += n
        return b

    def u32(self) -> int:
        return struct.unpack("<I", self.take(4))[0]

    def tensors(self, count: int, what: str) -> Dict[str, np.ndarray]:
        if count > 100000:
            raise OmmError(f"unreasonable {what} count {count}")
        out: Dict[str, np.ndarray] = {}
        for _ in range(count):
            nlen = self.u32()
            if nlen > 10000:
                raise OmmError(f"unreasonable name length {nlen}")
            name = self.take(nlen).decode("utf-8")
            ndims = self.u32()
            if ndims > 16:
                raise OmmError(f"unreasonable rank {ndims} for {name}")
            shape = tuple(self.u32() for _ in range(ndims))
            numel = int(np.prod(shape, dtype=np.int64)) if shape else 1
            if numel <= 0 or numel > 500_000_000:
                raise OmmError(f"unreasonable element count {numel} for {name}")
            arr = np.frombuffer(self.take(4 * numel), dtype="<f4").reshape(shape).astype(np.float32)
            out[name] = arr
        return out


def read_omm(path: str, password: Optional[str] = None
             ) -> Tuple[Dict[str, np.ndarray], Dict[str, np.ndarray], Optional[dict]]:
    """Reads an .omm file: (parameters, buffers, metadata or None), float32 arrays by name.

    Raises OmmError for a bad magic number or version, a truncated or implausible file, a
    checksum mismatch (for an encrypted file this is also what a wrong password gives), and an
    encrypted file read without a password. The reference's loader only warns on a checksum
    mismatch (serializer.ixx:636-645); a plan built from a damaged file would silently run on
    wrong weights, so this reader refuses it."""
    with open(path, "rb") as f:
        raw = f.read()
    if len(raw) < 8 or raw[:4] != MAGIC:
        raise OmmError("not an .omm file (bad magic number)")
    vraw = struct.unpack("<I", raw[4:8])[0]
    version = vraw & ~ENCRYPTED
    if not 1 <= version <= 5:
        raise OmmError(f"unsupported .omm version {version}")
    body = raw[8:]
    if vraw & ENCRYPTED:
        if not password:
            raise OmmError("encrypted .omm file: a password is needed")
        body = _xor(body, password)
    if len(body) < 4:
        raise OmmError("truncated file")
    stored = struct.unpack("<I", body[-4:])[0]
    crc = zlib.crc32(raw[:8] + body[:-4]) & 0xFFFFFFFF
    if crc != stored:
        raise OmmError("checksum mismatch (damaged file, or a wrong password)")
    r = _Reader(body[:-4])
    meta = None
    if version >= 4:
        n_meta = r.u32()
        if n_meta > 1024:
            raise OmmError(f"unreasonable metadata count {n_meta}")
        m = np.frombuffer(r.take(4 * n_meta), dtype="<f4")
        if n_meta >= 6 and m[0] == META_MARKER:
            meta = {"model_type_hash": int(m[1:2].view("<u4")[0]), "base_channels": int(m[2]),
                    "input_size": int(m[3]), "num_classes": int(m[4]), "in_channels": int(m[5])}
            if n_meta >= 8:
                meta["norm_type"], meta["group_norm_groups"] = int(m[6]), int(m[7])
    params = r.tensors(r.u32(), "parameter")
    buffers = r.tensors(r.u32(), "buffer") if version >= 2 else {}
    if r.i != len(r.d):
        raise OmmError(f"{len(r.d) - r.i} unexpected bytes before the checksum")
    return params, buffers, meta


def load_weights(path: str, password: Optional[str] = None) -> Dict[str, np.ndarray]:
    """Parameters and buffers of an .omm file in one dict, as InferencePlan / Fp32Net take."""
    params, buffers, _ = read_omm(path, password)
    out = dict(params)
    out.update(buffers)
    return out


def write_omm(path: str, params: Dict[str, np.ndarray], buffers: Dict[str, np.ndarray],
              meta: Optional[dict] = None, version: int = 5,
              password: Optional[str] = None) -> None:
    """Writes an .omm file the reference's loader reads: versions 1-5 (metadata from version 4,
    buffers from version 2), XOR-encrypted when a password is given."""
    if not 1 <= version <= 5:
        raise ValueError("version must be 1..5")
    if version < 2 and buffers:
        raise ValueError("version 1 files hold no buffers")
    if password and len(password) > 24:
        raise ValueError("password longer than 24 characters")
    body = bytearray()
    if version >= 4:
        m = meta or {}
        v = np.array([META_MARKER, 0, m.get("base_channels", 64), m.get("input_size", 224),
                      m.get("num_classes", 2), m.get("in_channels", 3), m.get("norm_type", 0),
                      m.get("group_norm_groups", 32)], dtype="<f4")
        v[1:2] = np.array([m.get("model_type_hash", 0)], dtype="<u4").view("<f4")
        body += struct.pack("<I", 8) + v.tobytes()

    def put(tensors: Dict[str, np.ndarray]) -> None:
        body.extend(struct.pack("<I", len(tensors)))
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, dtype="<f4")
            nb = name.encode("utf-8")
            body.extend(struct.pack("<I", len(nb)) + nb + struct.pack("<I", a.ndim))
            body.extend(struct.pack(f"<{a.ndim}I", *a.shape) + a.tobytes())

    put(params)
    if version >= 2:
        put(buffers)
    head = MAGIC + struct.pack("<I", version | (ENCRYPTED if password else 0))
    body += struct.pack("<I", zlib.crc32(head + bytes(body)) & 0xFFFFFFFF)
    data = _xor(bytes(body), password) if password else bytes(body)
    with open(path, "wb") as f:
        f.write(head + data)
