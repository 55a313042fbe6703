"""The ``.dav2`` model container and seeded random-init weights.

The file layout is the reference runtime's fixed format (writer:
tools/export_model.py:94-232, reader: src/model.cpp:27-69 and 98-320): a
64-byte little-endian header, one 192-byte record per tensor (sorted by
name), an optional 128-byte derivation-metadata block, then float32 payloads
aligned to 64 bytes, each with a CRC-32 (zlib polynomial). The layout has to
stay byte-identical so that models exported for the reference load here.

No checkpoints exist on this machine, so models are built from seeded
random weights with the reference architecture's tensor names and shapes
(depth_anything_v2/dpt.py, depth_anything_v2/dinov2.py): every Linear/Conv
weight and bias, cls_token and pos_embed ~ N(0, std); LayerNorm gamma=1,
beta=0; LayerScale gamma=1.
"""
from __future__ import annotations

import hashlib
import struct
import zlib
from pathlib import Path

import numpy as np

MAGIC = b"DAV2MOD\0"
FORMAT_VERSION = 1
ENDIAN_TAG = 0x01020304
DTYPE_FLOAT32 = 1
HEADER = struct.Struct("<8sIIIIQQQQQ")
RECORD = struct.Struct("<112sII4QQQQIIQ")
METADATA = struct.Struct("<8sIIIIII32s64s")
METADATA_MAGIC = b"DAV2META"
ALIGNMENT = 64
ENCODER_IDS = {"vits": 0, "vitb": 1, "vitl": 2}
RELATIVE_CONVERTER = "dav2-export-pytorch-v1"
METRIC_CONVERTER = "dav2-export-pytorch-metric-v1"

# embedding, heads, blocks, taps, DPT features, DPT out_channels
ARCH = {
    "vits": (384, 6, 12, (2, 5, 8, 11), 64, (48, 96, 192, 384)),
    "vitb": (768, 12, 12, (2, 5, 8, 11), 128, (96, 192, 384, 768)),
    "vitl": (1024, 16, 24, (4, 11, 17, 23), 256, (256, 512, 1024, 1024)),
}


def parameter_shapes(encoder: str) -> dict[str, tuple[int, ...]]:
    """State-dict names and shapes of DepthAnythingV2(encoder)."""
    d, _, blocks, _, f, oc = ARCH[encoder]
    s: dict[str, tuple[int, ...]] = {
        "pretrained.cls_token": (1, 1, d),
        "pretrained.pos_embed": (1, 1370, d),
        "pretrained.mask_token": (1, d),
        "pretrained.patch_embed.proj.weight": (d, 3, 14, 14),
        "pretrained.patch_embed.proj.bias": (d,),
        "pretrained.norm.weight": (d,),
        "pretrained.norm.bias": (d,),
    }
    for i in range(blocks):
        p = f"pretrained.blocks.{i}"
        s[p + ".norm1.weight"] = (d,)
        s[p + ".norm1.bias"] = (d,)
        s[p + ".attn.qkv.weight"] = (3 * d, d)
        s[p + ".attn.qkv.bias"] = (3 * d,)
        s[p + ".attn.proj.weight"] = (d, d)
        s[p + ".attn.proj.bias"] = (d,)
        s[p + ".ls1.gamma"] = (d,)
        s[p + ".norm2.weight"] = (d,)
        s[p + ".norm2.bias"] = (d,)
        s[p + ".mlp.fc1.weight"] = (4 * d, d)
        s[p + ".mlp.fc1.bias"] = (4 * d,)
        s[p + ".mlp.fc2.weight"] = (d, 4 * d)
        s[p + ".mlp.fc2.bias"] = (d,)
        s[p + ".ls2.gamma"] = (d,)
    h = "depth_head"
    for i in range(4):
        s[f"{h}.projects.{i}.weight"] = (oc[i], d, 1, 1)
        s[f"{h}.projects.{i}.bias"] = (oc[i],)
    s[f"{h}.resize_layers.0.weight"] = (oc[0], oc[0], 4, 4)
    s[f"{h}.resize_layers.0.bias"] = (oc[0],)
    s[f"{h}.resize_layers.1.weight"] = (oc[1], oc[1], 2, 2)
    s[f"{h}.resize_layers.1.bias"] = (oc[1],)
    s[f"{h}.resize_layers.3.weight"] = (oc[3], oc[3], 3, 3)
    s[f"{h}.resize_layers.3.bias"] = (oc[3],)
    for i in range(4):
        s[f"{h}.scratch.layer{i + 1}_rn.weight"] = (f, oc[i], 3, 3)
    for i in range(1, 5):
        r = f"{h}.scratch.refinenet{i}"
        s[r + ".out_conv.weight"] = (f, f, 1, 1)
        s[r + ".out_conv.bias"] = (f,)
        for u in (1, 2):
            for c in (1, 2):
                s[f"{r}.resConfUnit{u}.conv{c}.weight"] = (f, f, 3, 3)
                s[f"{r}.resConfUnit{u}.conv{c}.bias"] = (f,)
    s[f"{h}.scratch.output_conv1.weight"] = (f // 2, f, 3, 3)
    s[f"{h}.scratch.output_conv1.bias"] = (f // 2,)
    s[f"{h}.scratch.output_conv2.0.weight"] = (32, f // 2, 3, 3)
    s[f"{h}.scratch.output_conv2.0.bias"] = (32,)
    s[f"{h}.scratch.output_conv2.2.weight"] = (1, 32, 1, 1)
    s[f"{h}.scratch.output_conv2.2.bias"] = (1,)
    return s


def random_state_dict(encoder: str, seed: int = 0, std: float = 0.02,
                      bias_std: float | None = None) -> dict[str, np.ndarray]:
    """Seeded random-init weights (numpy PCG64, names drawn in sorted order)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    bias_std = std if bias_std is None else bias_std
    out: dict[str, np.ndarray] = {}
    for name, shape in sorted(parameter_shapes(encoder).items()):
        if name == "pretrained.mask_token":
            out[name] = np.zeros(shape, np.float32)
        elif name.endswith("norm1.weight") or name.endswith("norm2.weight") or name == "pretrained.norm.weight":
            out[name] = np.ones(shape, np.float32)
        elif name.endswith("norm1.bias") or name.endswith("norm2.bias") or name == "pretrained.norm.bias":
            out[name] = np.zeros(shape, np.float32)
        elif name.endswith(".gamma"):
            out[name] = np.ones(shape, np.float32)
        elif name.endswith(".bias"):
            out[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(bias_std)).astype(np.float32)
        else:
            out[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
    return out


def _align(value: int) -> int:
    return (value + ALIGNMENT - 1) & ~(ALIGNMENT - 1)


def write_dav2(path, state: dict[str, np.ndarray], encoder: str,
               metric_max_depth: float = 0.0, canonical: bytes | None = None) -> int:
    """Write ``state`` as a .dav2 file; returns the file size in bytes."""
    path = Path(path)
    names = sorted(state)
    payloads = []
    for name in names:
        arr = np.ascontiguousarray(state[name], dtype=np.float32)
        if not 1 <= arr.ndim <= 4:
            raise ValueError(f"unsupported rank for {name}")
        if len(name.encode()) >= 112:
            raise ValueError(f"tensor name too long: {name}")
        payloads.append((name, arr.shape, arr))
    directory_offset = HEADER.size
    directory_bytes = len(names) * RECORD.size
    metadata_offset = directory_offset + directory_bytes
    data_offset = _align(metadata_offset + METADATA.size)
    cursor = data_offset
    records = []
    for name, shape, arr in payloads:
        cursor = _align(cursor)
        raw = arr.tobytes()
        dims = list(shape) + [0] * (4 - len(shape))
        records.append((RECORD.pack(name.encode(), DTYPE_FLOAT32, len(shape), *dims, cursor,
                                    len(raw), arr.size, zlib.crc32(raw), 0, 0), cursor, raw))
        cursor += len(raw)
    file_bytes = cursor
    header = HEADER.pack(MAGIC, FORMAT_VERSION, ENDIAN_TAG, ENCODER_IDS[encoder], len(names),
                         directory_offset, directory_bytes, data_offset, file_bytes, metadata_offset)
    metric = metric_max_depth > 0
    canonical = canonical or hashlib.sha256(b"dav2-b200 seeded random init").digest()
    meta = METADATA.pack(METADATA_MAGIC, 1, METADATA.size, FORMAT_VERSION, ENCODER_IDS[encoder],
                         1 if metric else 0,
                         struct.unpack("<I", struct.pack("<f", metric_max_depth))[0] if metric else 0,
                         canonical, (METRIC_CONVERTER if metric else RELATIVE_CONVERTER).encode())
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("wb") as f:
        f.write(header)
        for rec, _, _ in records:
            f.write(rec)
        f.write(meta)
        f.write(b"\0" * (data_offset - f.tell()))
        for _, off, raw in records:
            f.write(b"\0" * (off - f.tell()))
            f.write(raw)
        if f.tell() != file_bytes:
            raise RuntimeError("file length mismatch")
    return file_bytes


def read_dav2(path) -> tuple[int, dict[str, np.ndarray]]:
    """Minimal reader (for tests): returns (encoder id, tensors)."""
    data = Path(path).read_bytes()
    magic, ver, endian, enc, count, doff, dbytes, data_off, fbytes, _ = HEADER.unpack_from(data, 0)
    if magic != MAGIC or ver != FORMAT_VERSION or endian != ENDIAN_TAG or fbytes != len(data):
        raise ValueError("invalid DAV2 header")
    out = {}
    for i in range(count):
        rec = RECORD.unpack_from(data, doff + i * RECORD.size)
        name = rec[0].split(b"\0", 1)[0].decode()
        rank = rec[2]
        dims = rec[3:3 + rank]
        off, nbytes = rec[7], rec[8]
        arr = np.frombuffer(data, np.float32, nbytes // 4, off).reshape(dims)
        if zlib.crc32(data[off:off + nbytes]) != rec[10]:
            raise ValueError(f"CRC mismatch for {name}")
        out[name] = arr
    return enc, out
