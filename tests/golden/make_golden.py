"""Generates the golden fixtures in tests/golden from the reference's own code.

Run where the reference checkout is available, with $PLAMO_REFERENCE pointing at it. The
reference packer (scripts/pack_weights.py) is pure numpy; importing it pulls in
`from reference import MODEL`, whose module imports `mlx.core`, so mlx is stubbed.

Fixtures:
  packer_vectors.npz  reference pack()/tag() outputs for pack_weights.self_test's bit patterns
                      (scripts/pack_weights.py:77-86) and a few seeded bf16 tensors
  micro/              a MICRO-config synthetic model (this package's writer) plus the model.p12
                      that the reference packer's main() writes for it (SOURCE_SHA and MODEL
                      patched to that model; scripts/pack_weights.py:89-142)
  packed_decode.npz   the 65536-pattern / every-(minimum, sm, code) decode vector built as in
                      Tests/PlamoTests/PackedDecodeTests.swift:8-31 (323,584 expected words),
                      expectations cross-checked with the reference numpy unpack()
  argmax_cases.json   Tests/PlamoTests/ArgmaxTests.swift:13-50 patterns with the expected index
                      from that test's own expected-value rule
"""
from __future__ import annotations

import hashlib
import importlib
import json
import os
import shutil
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REFERENCE = Path(os.environ["PLAMO_REFERENCE"]) if os.environ.get("PLAMO_REFERENCE") else None


def load_reference_packer():
    if REFERENCE is None:
        raise SystemExit("set PLAMO_REFERENCE to the reference checkout")
    mlx = types.ModuleType("mlx")
    core = types.ModuleType("mlx.core")
    mlx.core = core
    sys.modules.setdefault("mlx", mlx)
    sys.modules.setdefault("mlx.core", core)
    sys.path.insert(0, str(REFERENCE / "scripts"))
    try:
        return importlib.import_module("pack_weights")
    finally:
        sys.path.pop(0)


def load_package():
    import importlib.util
    pkg = REPO / "plamo3-0.8b-runtime_b200"
    spec = importlib.util.spec_from_file_location("plamo_b200", pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["plamo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def packer_vectors(pw):
    import torch
    vectors = {
        "all_patterns": np.arange(65536, dtype="<u2"),
        "zeros": np.zeros(256, dtype="<u2"),
        "neg_zero": np.full(128, 0x8000, dtype="<u2"),
        "mixed_sign": np.tile(np.array([0, 0x8000, 0x3F80, 0xBF80], dtype="<u2"), 64),
    }
    g = torch.Generator().manual_seed(7)
    for name, std in [("normal_002", 0.02), ("normal_1", 1.0), ("normal_1e4", 1e-4)]:
        t = (torch.randn(64 * 128, generator=g) * std).to(torch.bfloat16)
        vectors[name] = t.view(torch.int16).numpy().view(np.uint16).copy()
    # a block whose exponent span is exactly 14 (packable) and one with 15 (raw)
    span14 = np.full(128, 0x3F80, dtype="<u2"); span14[0] = (127 - 14) << 7
    span15 = np.full(128, 0x3F80, dtype="<u2"); span15[0] = (127 - 15) << 7
    vectors["span14"], vectors["span15"] = span14, span15
    out = {}
    for name, values in vectors.items():
        data, offsets, minima = pw.pack(values)
        out[f"{name}.values"] = values
        out[f"{name}.data"] = data
        out[f"{name}.offsets"] = offsets
        out[f"{name}.minima"] = minima
        out[f"{name}.entries"] = pw.tag(offsets, minima)
    np.savez_compressed(HERE / "packer_vectors.npz", **out)


def micro_model(pw, pkg):
    target = HERE / "micro"
    if target.exists():
        shutil.rmtree(target)
    pkg.synthetic.write_model(target, pkg.synthetic.MICRO, seed=0)
    source = target / "model.safetensors"
    sha = hashlib.sha256(source.read_bytes()).hexdigest()
    pw.SOURCE_SHA = sha
    pw.MODEL = target
    pw.main()  # the reference's own archive writer
    (target / "README").write_text(
        "MICRO synthetic model (seed 0). model.p12 was written by the reference packer's main()\n"
        f"with SOURCE_SHA patched to this model.safetensors ({sha}).\n")


def packed_decode_vector(pw):
    payload, offsets, expected = [], [], []
    for block in range(512):
        offsets.append(len(payload))
        for i in range(128):
            b = block * 128 + i
            payload += [b & 255, b >> 8]
            expected.append(b)
    for minimum in range(108, 171):
        for block in range(32):
            offsets.append(len(payload) | (minimum - 107))
            data = [0] * 192
            for i in range(128):
                index = block * 128 + i
                sm, code = index // 16, index % 16
                data[i] = sm
                data[128 + i // 2] |= code << ((i % 2) * 4)
                exponent = 0 if code == 15 else minimum + code
                expected.append((sm & 127) | ((sm & 128) << 8) | (exponent << 7))
            payload += data
    payload = np.array(payload, dtype=np.uint8)
    entries = np.array(offsets, dtype=np.uint32)
    expected = np.array(expected, dtype=np.uint16)
    assert expected.size == 323_584
    # cross-check with the reference numpy unpack (scripts/pack_weights.py:53-68)
    codes = entries & 63
    minima = np.where(codes != 0, codes + 107, 0).astype(np.uint8)
    ref = pw.unpack(payload, (entries & ~np.uint32(63)).astype(np.int64), minima).reshape(-1)
    assert np.array_equal(ref, expected), "reference unpack disagrees with the XCTest expectation"
    np.savez_compressed(HERE / "packed_decode.npz", payload=payload, entries=entries, expected=expected)


def argmax_cases():
    cases = []

    def to_bits(values):
        u = np.array(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)

    def expected_index(tested, row, count):
        best, index = -np.inf, 0xFFFFFFFF
        for i in range(count):
            v = tested[row * count + i]
            if v > best or (v == best and i < index):
                best, index = v, i
        return int(index)

    for count in [1, 31, 32, 33, 255, 256, 257, 1023, 1024, 1025, 107520]:
        for batch in [1, 2, 3]:
            for pattern in range(5):
                values = [float(((j * 17) % 4093) - 2046) / 32 for j in range(count * batch)]
                values = np.array(values, dtype=np.float32)
                for row in range(batch):
                    s = row * count
                    if pattern == 1:
                        values[s:s + count] = -np.inf
                    elif pattern == 2:
                        values[s:s + count] = np.nan
                    elif pattern == 3:
                        values[s:s + count] = np.where(np.arange(count) % 2 == 0, -0.0, 0.0)
                    elif pattern == 4:
                        values[s] = np.nan
                        if count > 1:
                            values[s + count - 1] = np.inf
                        if count > 257:
                            values[s + 257] = np.inf
                for compact in [False, True]:
                    bits = to_bits(values)
                    tested = (bits.astype(np.uint32) << 16).view(np.float32) if compact else values
                    if count <= 1025:
                        exp = [expected_index(tested, r, count) for r in range(batch)]
                    else:  # vectorised rule for the long rows (same semantics)
                        exp = []
                        for r in range(batch):
                            row = tested[r * count:(r + 1) * count]
                            valid = ~np.isnan(row)
                            if not valid.any():
                                exp.append(0xFFFFFFFF)
                            else:
                                m = row[valid].max()
                                exp.append(int(np.flatnonzero(valid & (row == m))[0]))
                    cases.append(dict(count=count, batch=batch, pattern=pattern, compact=compact, expected=exp))
    (HERE / "argmax_cases.json").write_text(json.dumps(cases) + "\n")


def main():
    pw = load_reference_packer()
    pkg = load_package()
    pw.self_test()
    packer_vectors(pw)
    micro_model(pw, pkg)
    packed_decode_vector(pw)
    argmax_cases()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
