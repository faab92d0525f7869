"""Lossless `.p12` (plamo-bf16-pack-v2) codec and archive writer.

Restates the format defined by the reference packer (scripts/pack_weights.py:19-74 for the
block codec, :89-135 for the archive layout) in this package's own code; the archive bytes are
pinned against the reference packer's output in tests/golden.

Block codec (128 bf16 values per block):
  * exponent e = (v >> 7) & 255 of every value whose low 15 bits are non-zero;
  * the block is packed when min(e) in [108, 170], max(e) < 255 and max(e) - min(e) < 15
    (scripts/pack_weights.py:26); otherwise it stays raw bf16 (256 bytes);
  * a packed block is 128 sign|mantissa bytes ((v & 127) | ((v >> 8) & 128)) followed by 64
    bytes of 4-bit exponent codes (code = e - min, 15 = signed zero), low nibble first (192 B);
  * the u32 block table holds the 64-aligned byte offset of each block in the data region,
    with min - 107 in the low six bits (0 = raw) (scripts/pack_weights.py:71-74).
Archive: 65536-byte header = <Q 65528> + compact JSON manifest padded with spaces; every
region 64-byte aligned; tensors in safetensors-header order; the input embedding skipped.
"""
from __future__ import annotations

import hashlib
import json
import struct
from pathlib import Path

import numpy as np

FORMAT = "plamo-bf16-pack-v2"
BLOCK = 128
MINIMUM_BASE = 107
HEADER = 65536
# Checkpoint digest the reference loader accepts (Sources/Plamo/Packed.swift:35).
REFERENCE_SOURCE_SHA = "7c9f0066d166c075bdbe83ada3d444e08bd7a6ee3f345f47a1f3c442aa6898c5"

_CHUNK = 1 << 18  # blocks per vectorised step (bounds temporaries to ~100 MB)


def _block_stats(blocks: np.ndarray):
    exponent = ((blocks >> 7) & 255).astype(np.uint8)
    nonzero = (blocks & 0x7FFF) != 0
    low = np.where(nonzero, exponent, np.uint8(255)).min(axis=1)
    high = np.where(nonzero, exponent, np.uint8(0)).max(axis=1)
    eligible = (low >= 108) & (low <= 170) & (high < 255) & (high.astype(np.int16) - low.astype(np.int16) < 15)
    return exponent, nonzero, low, eligible


def pack(values: np.ndarray):
    """Pack a flat uint16 array (length multiple of 128). Returns (data, offsets, minima).

    data: uint8 payload; offsets: untagged u32 byte offsets per block; minima: uint8 (0 = raw).
    Raises AssertionError if the round trip changes any bit (same guarantee as the reference).
    """
    flat = np.ascontiguousarray(values).reshape(-1)
    if flat.dtype != np.uint16 or flat.size % BLOCK:
        raise ValueError("pack expects uint16 values in whole 128-element blocks")
    blocks = flat.reshape(-1, BLOCK)
    nb = blocks.shape[0]
    eligible = np.empty(nb, dtype=bool)
    minima = np.zeros(nb, dtype=np.uint8)
    for s in range(0, nb, _CHUNK):
        _, _, low, el = _block_stats(blocks[s:s + _CHUNK])
        eligible[s:s + _CHUNK] = el
        minima[s:s + _CHUNK] = np.where(el, low, 0)
    sizes = np.where(eligible, 192, 256).astype(np.uint64)
    offsets = np.zeros(nb, dtype=np.uint32)
    if nb > 1:
        offsets[1:] = np.cumsum(sizes[:-1]).astype(np.uint32)
    total = int(sizes.sum())
    data = np.empty(total, dtype=np.uint8)
    units = data.reshape(-1, 64)  # every block is a whole number of 64-byte units
    for s in range(0, nb, _CHUNK):
        src = blocks[s:s + _CHUNK]
        el = eligible[s:s + _CHUNK]
        unit0 = (offsets[s:s + _CHUNK] // 64).astype(np.int64)
        if el.any():
            v = src[el]
            exponent = ((v >> 7) & 255).astype(np.int16)
            codes = exponent - minima[s:s + _CHUNK][el].astype(np.int16)[:, None]
            codes = np.where((v & 0x7FFF) == 0, 15, codes).astype(np.uint8)
            sm = ((v & 127) | ((v >> 8) & 128)).astype(np.uint8)
            nib = codes[:, 0::2] | (codes[:, 1::2] << 4)
            enc = np.concatenate([sm, nib], axis=1).reshape(-1, 3, 64)
            units[unit0[el][:, None] + np.arange(3)] = enc
        if (~el).any():
            raw = np.ascontiguousarray(src[~el]).view(np.uint8).reshape(-1, 4, 64)
            units[unit0[~el][:, None] + np.arange(4)] = raw
        restored = unpack(data, offsets[s:s + _CHUNK], minima[s:s + _CHUNK])
        if not np.array_equal(restored, src):
            raise AssertionError("Packing changed BF16 bits")
    return data, offsets, minima


def unpack(data: np.ndarray, offsets: np.ndarray, minima: np.ndarray) -> np.ndarray:
    """Inverse of `pack` for the given blocks: returns uint16 [len(offsets), 128]."""
    out = np.empty((len(offsets), BLOCK), dtype=np.uint16)
    packed = minima != 0
    if packed.any():
        idx = offsets[packed].astype(np.int64)[:, None] + np.arange(192)
        enc = data[idx]
        sm = enc[:, :128].astype(np.uint16)
        nib = enc[:, 128:]
        codes = np.empty((len(enc), BLOCK), dtype=np.uint16)
        codes[:, 0::2] = nib & 15
        codes[:, 1::2] = nib >> 4
        exponent = np.where(codes == 15, 0, codes + minima[packed].astype(np.uint16)[:, None])
        out[packed] = (sm & 127) | ((sm & 128) << 8) | (exponent << 7)
    if (~packed).any():
        idx = offsets[~packed].astype(np.int64)[:, None] + np.arange(256)
        out[~packed] = data[idx].view(np.uint16).reshape(-1, BLOCK)
    return out


def tag(offsets: np.ndarray, minima: np.ndarray) -> np.ndarray:
    """Block table entries: offset | (minimum - 107), 0 in the low bits for raw blocks."""
    if np.any(offsets & 63):
        raise ValueError("block offsets must be 64-byte aligned")
    if np.any((minima != 0) & ((minima < 108) | (minima > 170))):
        raise ValueError("block minimum out of range")
    return (offsets | np.where(minima != 0, minima.astype(np.uint32) - MINIMUM_BASE, 0)).astype("<u4")


def untag(entries: np.ndarray):
    entries = entries.astype(np.uint32)
    codes = entries & 63
    minima = np.where(codes != 0, codes + MINIMUM_BASE, 0).astype(np.uint8)
    return entries & ~np.uint32(63), minima


def read_safetensors_header(path: Path):
    with open(path, "rb") as f:
        length = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(length))
    return length, header


def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            chunk = f.read(1 << 24)
            if not chunk:
                break
            h.update(chunk)
    return h.hexdigest()


def write_p12(model_dir, source_sha: str | None = None) -> dict:
    """Write `model.p12` beside `model.safetensors` (same layout as the reference archive).

    `source_sha256` in the manifest is the digest of the source safetensors file; the CUDA
    loader accepts it when it matches that file (or the original checkpoint's digest).
    """
    model_dir = Path(model_dir)
    source = model_dir / "model.safetensors"
    length, header = read_safetensors_header(source)
    sha = source_sha or sha256_file(source)
    manifest = dict(format=FORMAT, block=BLOCK, minimum_base=MINIMUM_BASE, source_sha256=sha, tensors={})
    output = model_dir / "model.p12"
    part = output.with_suffix(".p12.part")
    total_raw = total_packed = compressed = blocks = 0
    try:
        with open(part, "w+b") as f:
            f.write(bytes(HEADER))

            def append(array: np.ndarray):
                f.write(bytes((-f.tell()) % 64))
                begin = f.tell() - HEADER
                f.write(np.ascontiguousarray(array).tobytes())
                return [begin, f.tell() - HEADER]

            for name, info in header.items():
                if name == "__metadata__" or name == "model.embed_tokens.weight":
                    continue
                if info["dtype"] != "BF16":
                    raise ValueError(f"{name}: only BF16 tensors can be packed")
                shape = info["shape"]
                begin, end = info["data_offsets"]
                values = np.memmap(source, dtype="<u2", mode="r", offset=8 + length + begin, shape=tuple(shape))
                record = dict(shape=shape)
                if len(shape) == 1:
                    record["raw"] = append(values)
                else:
                    data, offsets, minima = pack(values)
                    record["offsets"] = append(tag(offsets, minima))
                    record["data"] = append(data)
                    compressed += int((minima != 0).sum()); blocks += len(minima)
                    total_packed += data.nbytes + offsets.nbytes
                    total_raw += values.nbytes
                manifest["tensors"][name] = record
            manifest["payload_bytes"] = f.tell() - HEADER
            metadata = json.dumps(manifest, separators=(",", ":")).encode()
            if len(metadata) > HEADER - 8:
                raise ValueError("Packed header overflow")
            f.seek(0)
            f.write(struct.pack("<Q", HEADER - 8)); f.write(metadata); f.write(b" " * (HEADER - 8 - len(metadata)))
        part.replace(output)
    except BaseException:
        part.unlink(missing_ok=True)
        raise
    return dict(original_linear_bytes=total_raw, packed_linear_bytes=total_packed,
                archive_bytes=output.stat().st_size, compressed_blocks=compressed, blocks=blocks)


def read_p12(path):
    """Parse a `.p12` archive: returns (manifest, payload memmap)."""
    path = Path(path)
    with open(path, "rb") as f:
        count = struct.unpack("<Q", f.read(8))[0]
        manifest = json.loads(f.read(count))
    payload = np.memmap(path, dtype=np.uint8, mode="r", offset=count + 8)
    return manifest, payload


def unpack_tensor(manifest: dict, payload: np.ndarray, name: str) -> np.ndarray:
    """Reconstruct one tensor (uint16, original shape) from an archive."""
    rec = manifest["tensors"][name]
    shape = rec["shape"]
    if "raw" in rec:
        b, e = rec["raw"]
        return np.asarray(payload[b:e]).view("<u2").reshape(shape)
    ob, oe = rec["offsets"]
    db, de = rec["data"]
    offsets, minima = untag(np.asarray(payload[ob:oe]).view("<u4"))
    data = np.asarray(payload[db:de])
    return unpack(data, offsets, minima).reshape(shape)
