"""`.p12` codec and archive parity with the reference packer (scripts/pack_weights.py)."""
import numpy as np
import pytest

from conftest import GOLDEN


@pytest.fixture(scope="module")
def vectors():
    return np.load(GOLDEN / "packer_vectors.npz")


def _names(vectors):
    return sorted({k.split(".")[0] for k in vectors.files})


def test_pack_matches_reference_vectors(pkg, vectors):
    """pack()/tag() outputs equal the reference's for every golden input (pack_weights.py:19-74)."""
    for name in _names(vectors):
        values = vectors[f"{name}.values"]
        data, offsets, minima = pkg.packing.pack(values)
        assert np.array_equal(data, vectors[f"{name}.data"]), name
        assert np.array_equal(offsets, vectors[f"{name}.offsets"]), name
        assert np.array_equal(minima, vectors[f"{name}.minima"]), name
        assert np.array_equal(pkg.packing.tag(offsets, minima), vectors[f"{name}.entries"]), name


def test_self_test_round_trip(pkg):
    """pack_weights.py:77-86: every bf16 pattern, signed zeros and mixed-sign blocks round-trip."""
    for values in [np.arange(65536, dtype="<u2"), np.zeros(256, dtype="<u2"), np.full(128, 0x8000, dtype="<u2"),
                   np.tile(np.array([0, 0x8000, 0x3F80, 0xBF80], dtype="<u2"), 64)]:
        data, offsets, minima = pkg.packing.pack(values)
        entries = pkg.packing.tag(offsets, minima)
        off, mins = pkg.packing.untag(entries)
        restored = pkg.packing.unpack(data, off, mins)
        assert np.array_equal(restored.reshape(-1), values)


def test_archive_bytes_match_reference_packer(pkg, micro_dir, tmp_path):
    """Our writer reproduces the reference main()'s archive byte for byte (pack_weights.py:89-135)."""
    import shutil
    for f in ["config.json", "config-mlx.json", "model.safetensors"]:
        shutil.copy(micro_dir / f, tmp_path / f)
    pkg.packing.write_p12(tmp_path)
    assert (tmp_path / "model.p12").read_bytes() == (micro_dir / "model.p12").read_bytes()


def test_archive_unpacks_bit_identical(pkg, micro_dir):
    manifest, payload = pkg.packing.read_p12(micro_dir / "model.p12")
    import json, struct
    raw = (micro_dir / "model.safetensors").read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])
    for name in manifest["tensors"]:
        b, e = header[name]["data_offsets"]
        src = np.frombuffer(raw[8 + n + b:8 + n + e], dtype="<u2").reshape(header[name]["shape"])
        assert np.array_equal(pkg.packing.unpack_tensor(manifest, payload, name), src), name
    assert "model.embed_tokens.weight" not in manifest["tensors"]


def test_oracle_packed_decode_golden(oracle):
    """Kernels.metal:23-31 restated: all 323,584 words of PackedDecodeTests.swift:8-31."""
    g = np.load(GOLDEN / "packed_decode.npz")
    out = oracle.packed_decode(g["payload"], g["entries"], g["expected"].size)
    assert np.array_equal(out, g["expected"])


def test_cpp_codec_matches_reference_vectors(pkg, vectors):
    """The library's C++ block codec (plamo_pack_blocks) gives the reference packer's bytes and
    tagged entries for every golden input."""
    for name in _names(vectors):
        data, entries = pkg.runtime.pack_blocks(vectors[f"{name}.values"])
        assert np.array_equal(data, vectors[f"{name}.data"]), name
        assert np.array_equal(entries, vectors[f"{name}.entries"]), name


def test_cpp_codec_round_trip(pkg):
    for values in [np.arange(65536, dtype="<u2"), np.zeros(256, dtype="<u2"), np.full(128, 0x8000, dtype="<u2"),
                   np.tile(np.array([0, 0x8000, 0x3F80, 0xBF80], dtype="<u2"), 64)]:
        data, entries = pkg.runtime.pack_blocks(values)
        off, mins = pkg.packing.untag(entries)
        assert np.array_equal(pkg.packing.unpack(data, off, mins).reshape(-1), values)
    with pytest.raises(pkg.PlamoError):
        pkg.runtime.pack_blocks(np.zeros(100, dtype="<u2"))  # not whole blocks


def test_cpp_archive_matches_reference_packer(pkg, micro_dir, tmp_path):
    """plamo_pack_p12 writes the reference main()'s archive byte for byte (pack_weights.py:89-135)."""
    import shutil
    for f in ["config.json", "config-mlx.json", "model.safetensors"]:
        shutil.copy(micro_dir / f, tmp_path / f)
    stats = pkg.runtime.pack_p12(tmp_path)
    ref = (micro_dir / "model.p12").read_bytes()
    assert (tmp_path / "model.p12").read_bytes() == ref
    assert stats["archive_bytes"] == len(ref) and 0 < stats["compressed_blocks"] <= stats["blocks"]
    assert not (tmp_path / "model.p12.part").exists()


def test_cpp_archive_matches_python_writer(pkg, tiny_dir, tmp_path):
    import shutil
    for f in ["config.json", "config-mlx.json", "model.safetensors"]:
        if (tiny_dir / f).exists():
            shutil.copy(tiny_dir / f, tmp_path / f)
    pkg.runtime.pack_p12(tmp_path, source_sha256="ab" * 32)
    py = tmp_path / "py"
    py.mkdir()
    shutil.copy(tiny_dir / "model.safetensors", py / "model.safetensors")
    pkg.packing.write_p12(py, source_sha="ab" * 32)
    assert (tmp_path / "model.p12").read_bytes() == (py / "model.p12").read_bytes()
    with pytest.raises(pkg.PlamoError):
        pkg.runtime.pack_p12(tmp_path / "missing")


def _chain_rule(entries, nbytes):
    """The validity rule of PackedFormatTests.swift:45-53, restated."""
    end = 0
    for entry in entries:
        offset = int(entry) & ~63
        size = 256 if int(entry) & 63 == 0 else 192
        if offset != end or offset > nbytes - size:
            return False
        end = offset + size
    return end == nbytes


def test_loader_chain_fuzz(pkg):
    """PackedFormatTests.swift:43-72: chains of 0..19 blocks (raw, tag 1, tag 63), every data size
    around the true end, and every entry with bits flipped; the loader's check agrees with the
    rule each time."""
    valid = pkg.runtime.p12_chain_valid
    checked = 0
    for count in range(20):
        entries, end = [], 0
        for i in range(count):
            tag = 0 if i % 3 == 0 else (1 if i % 3 == 1 else 63)
            entries.append(end | tag)
            end += 256 if tag == 0 else 192
        cases = [(entries, end)] + [(entries, b) for b in (0, max(0, end - 1), end + 1, end + 64)]
        for i in range(len(entries)):
            for change in (1, 63, 64, 256, 0xFFFFFFFF):
                bad = list(entries)
                bad[i] ^= change
                cases.append((bad, end))
        for e, nbytes in cases:
            assert valid(e, nbytes) == _chain_rule(e, nbytes), (count, e, nbytes)
            checked += 1
    assert valid([], 0) and not valid([], 64)
    assert checked > 900
