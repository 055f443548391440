"""The `.svlm` model bundle (include/svl_bundle.h, src/bundle/mod.rs) and the
bundle-or-directory model sources (src/model/source.rs), on the CPU.

The format is pinned twice: by the reference's own unit cases
(bundle/mod.rs:721-953, tests/bundle_loading.rs) and by an independent
encoder written here from the documented layout (docs/formats.md "Model
bundle": field offsets, IEEE CRC-32 over the header minus its CRC field,
SHA-256 catalog digest over the header and the section digests) with
Python's own hashlib and zlib, whose bytes the library's writer must
reproduce exactly.  The GPU half (a model loaded from a bundle embeds exactly
as from its directory, FP32 and BF16 weights) is in tests/test_gpu_bundle.py.
"""

from __future__ import annotations

import hashlib
import os
import random
import struct
import zlib

import pytest

from conftest import GOLDEN
from svl import bundle, errors
from svl.bundle import Bundle, SectionInput, SectionRole
from svl.tokenizer import Tokenizer

SAMPLE = [
    SectionInput("model.safetensors", SectionRole.Weights, b"weights"),
    SectionInput("config.json", SectionRole.Config, b"{}"),
    SectionInput("tokenizer.json", SectionRole.Tokenizer, b"tokenizer"),
]


def encode(sections, order=None, flags=0, version=1):
    """The documented layout, written independently of the library."""
    secs = sorted(sections, key=lambda s: s[0].encode()) if order is None else list(sections)
    hlen = 30 + sum(52 + len(p.encode()) for p, _, _ in secs)
    total = hlen + sum(len(d) for _, _, d in secs) + 32
    entries, off = b"", hlen
    for p, role, d in secs:
        pb = p.encode()
        entries += struct.pack("<HBBQQ", len(pb), int(role), flags, off, len(d)) + hashlib.sha256(d).digest() + pb
        off += len(d)
    head = b"SVLMDL01" + struct.pack("<HIIQ", version, hlen, len(secs), total)
    crc = zlib.crc32(head + entries) & 0xFFFFFFFF
    header = head + struct.pack("<I", crc) + entries
    digest = hashlib.sha256(header + b"".join(hashlib.sha256(d).digest() for _, _, d in secs)).digest()
    return header + b"".join(d for _, _, d in secs) + digest


def as_tuples(sections):
    return [(s.path, s.role, s.data) for s in sections]


# ---------------------------------------------------------- hashes (KATs)
@pytest.mark.parametrize("n", [0, 1, 3, 55, 56, 57, 63, 64, 65, 119, 120, 128, 1000, 1 << 20])
def test_sha256_matches_fips_180_4(n):
    data = random.Random(n).randbytes(n)
    assert bundle.sha256(data) == hashlib.sha256(data).digest()


def test_sha256_and_crc32_known_answers():
    assert bundle.sha256(b"abc").hex() == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"
    assert bundle.crc32(b"123456789") == 0xCBF43926
    for n in (0, 1, 17, 4096):
        d = random.Random(n).randbytes(n)
        assert bundle.crc32(d) == zlib.crc32(d) & 0xFFFFFFFF


# ------------------------------------------------------- layout and round trip
def test_writer_produces_the_documented_layout():
    assert Bundle.build(SAMPLE) == encode(as_tuples(SAMPLE))
    tiny = [SectionInput("config.json", SectionRole.Config, (GOLDEN / "tiny_text" / "config.json").read_bytes()),
            SectionInput("model.safetensors", SectionRole.Weights,
                         (GOLDEN / "tiny_text" / "model.safetensors").read_bytes()),
            SectionInput("nested/dir/tokenizer.json", SectionRole.Tokenizer,
                         (GOLDEN / "tokenizer" / "mini_tokenizer.json").read_bytes())]
    assert Bundle.build(tiny) == encode(as_tuples(tiny))


def test_round_trip_preserves_sections_and_sorts_paths():
    b = Bundle.parse(Bundle.build(SAMPLE))
    assert [s.path for s in b.sections()] == ["config.json", "model.safetensors", "tokenizer.json"]
    assert bytes(b.data("config.json")) == b"{}"
    assert bytes(b.data("model.safetensors")) == b"weights"
    assert bytes(b.data("tokenizer.json")) == b"tokenizer"
    assert b.data("missing") is None
    assert b.section("config.json").role == SectionRole.Config
    assert b.section("config.json").sha256 == hashlib.sha256(b"{}").digest()
    b.verify()


def test_empty_bundle_round_trips():
    b = Bundle.parse(Bundle.build([]))
    assert b.sections() == [] and b.header_len() == 30
    b.verify()


def test_parser_accepts_a_bundle_written_independently():
    b = Bundle.parse(encode([("a/b.bin", SectionRole.Other, b"\x00" * 5), ("a.txt", SectionRole.Manifest, b"")]))
    assert [s.path for s in b.sections()] == ["a.txt", "a/b.bin"]
    b.verify()


def test_duplicate_paths_are_rejected():
    with pytest.raises(errors.UsageError):
        Bundle.build([SectionInput("a", SectionRole.Other, b"1"), SectionInput("a", SectionRole.Other, b"2")])


@pytest.mark.parametrize("path", ["", "/absolute", "a//b", "a/./b", "a/../b", "a\\b", "a\0b", "a/", "..", "x" * 4097])
def test_invalid_paths_are_rejected(path):
    with pytest.raises((errors.CorruptError, errors.LimitExceededError)):
        Bundle.build([SectionInput(path, SectionRole.Other, b"x")])


# -------------------------------------------------------------- rejections
def test_corrupt_magic_version_and_lengths_are_rejected():
    good = Bundle.build(SAMPLE)
    bad = bytearray(good)
    bad[0] ^= 0xFF
    with pytest.raises(errors.CorruptError):
        Bundle.parse(bytes(bad))
    bad = bytearray(good)
    bad[8] = 2
    with pytest.raises(errors.UnsupportedError):
        Bundle.parse(bytes(bad))
    bad = bytearray(good)
    bad[18:26] = struct.pack("<Q", len(good) + 1)
    with pytest.raises(errors.CorruptError):
        Bundle.parse(bytes(bad))
    with pytest.raises(errors.CorruptError):
        Bundle.parse(good[:-1])
    with pytest.raises(errors.CorruptError):
        Bundle.parse(good[:40])


def test_header_crc_and_catalog_digest_are_checked():
    good = Bundle.build(SAMPLE)
    bad = bytearray(good)
    bad[26] ^= 0xFF
    with pytest.raises(errors.CorruptError, match="CRC"):
        Bundle.parse(bytes(bad))
    bad = bytearray(good)
    bad[-1] ^= 0xFF
    with pytest.raises(errors.CorruptError, match="digest"):
        Bundle.parse(bytes(bad))


def test_section_data_corruption_is_detected_by_verify():
    data = bytearray(Bundle.build(SAMPLE))
    off = Bundle.parse(bytes(data)).section("config.json").offset
    data[off] ^= 0xFF
    b = Bundle.parse(bytes(data))  # the structure still parses
    with pytest.raises(errors.CorruptError, match="SHA-256"):
        b.verify()


def test_flags_order_and_roles_are_checked():
    secs = as_tuples(SAMPLE)
    with pytest.raises(errors.UnsupportedError, match="flags"):
        Bundle.parse(encode(secs, flags=1))
    with pytest.raises(errors.UnsupportedError):
        Bundle.parse(encode(secs, version=7))
    unsorted = [secs[1], secs[0], secs[2]][::-1]
    with pytest.raises(errors.CorruptError, match="sorted"):
        Bundle.parse(encode(unsorted, order=True))
    with pytest.raises(errors.CorruptError, match="role"):
        Bundle.parse(encode([("x", 9, b"1")]))


def test_caps_are_limit_exceeded():
    many = [SectionInput(f"s{i:04d}", SectionRole.Other, b"") for i in range(1025)]
    with pytest.raises(errors.LimitExceededError):
        Bundle.build(many)
    head = bytearray(Bundle.build([]))
    head[14:18] = struct.pack("<I", 1025)  # declared section count above the cap (checked before the CRC)
    with pytest.raises(errors.LimitExceededError):
        Bundle.parse(bytes(head))


# ---------------------------------------------------- sources (source.rs)
def test_tokenizer_from_bundle_matches_the_directory(tmp_path):
    """tests/bundle_loading.rs:79-97."""
    path = tmp_path / "tok.svlm"
    path.write_bytes(Bundle.build([SectionInput("tokenizer.json", SectionRole.Tokenizer,
                                                (GOLDEN / "tokenizer" / "mini_tokenizer.json").read_bytes())]))
    from_bundle = bundle.load_tokenizer(path)
    from_file = Tokenizer.load(GOLDEN / "tokenizer" / "mini_tokenizer.json")
    assert from_bundle.vocab_size() == from_file.vocab_size()
    assert from_bundle.max_token_id() == from_file.max_token_id()
    for text in ["Hello world", "Bonjour le monde", "日本語", ""]:
        assert from_bundle.encode(text, True) == from_file.encode(text, True)


def test_missing_weights_section_is_corrupt(tmp_path):
    """tests/bundle_loading.rs:116-128 (fails before any device work)."""
    path = tmp_path / "incomplete.svlm"
    path.write_bytes(Bundle.build([SectionInput("config.json", SectionRole.Config,
                                                (GOLDEN / "tiny_text" / "config.json").read_bytes())]))
    with pytest.raises(errors.CorruptError, match="model.safetensors"):
        bundle.load_text_model(path)


def test_corrupt_bundle_file_is_rejected_by_the_loader(tmp_path):
    """tests/bundle_loading.rs:130-143."""
    data = bytearray(Bundle.build([SectionInput("config.json", SectionRole.Config, b"{}")]))
    data[0] ^= 0xFF
    path = tmp_path / "corrupt.svlm"
    path.write_bytes(bytes(data))
    with pytest.raises(errors.CorruptError):
        bundle.load_text_model(path)


def test_a_section_that_fails_verification_stops_the_loader(tmp_path):
    data = bytearray(Bundle.build([SectionInput("config.json", SectionRole.Config, b"{}"),
                                   SectionInput("model.safetensors", SectionRole.Weights, b"0" * 64)]))
    off = Bundle.parse(bytes(data)).section("model.safetensors").offset
    data[off + 3] ^= 1
    path = tmp_path / "tampered.svlm"
    path.write_bytes(bytes(data))
    with pytest.raises(errors.CorruptError, match="SHA-256"):
        bundle.load_text_model(path)


def test_model_file_paths_must_be_safe():
    files = bundle.ModelFiles.directory(GOLDEN)
    with pytest.raises(errors.InternalError):
        files.read("../etc/passwd", 10)
    assert not files.contains("../x") and files.contains("tiny_text/config.json")
    assert files.section_sha256("tiny_text/config.json") is None
    assert os.path.isdir(GOLDEN)


def test_random_damage_never_crashes_the_parser():
    """Every single-byte change, truncation or extension of a bundle parses to
    a typed error or to a bundle whose sections lie inside the bytes (the
    reference's parser never reads past a checked length)."""
    good = Bundle.build(SAMPLE + [SectionInput("dir/x.bin", SectionRole.Other, bytes(range(200)))])
    rnd = random.Random(11)
    for trial in range(3000):
        data = bytearray(good)
        kind = trial % 3
        if kind == 0:
            for _ in range(rnd.randint(1, 4)):
                data[rnd.randrange(len(data))] = rnd.randrange(256)
        elif kind == 1:
            del data[rnd.randrange(len(data)):]
        else:
            data += rnd.randbytes(rnd.randint(1, 64))
        try:
            b = Bundle.parse(bytes(data))
        except (errors.CorruptError, errors.UnsupportedError, errors.LimitExceededError):
            continue
        for s in b.sections():
            assert 0 <= s.offset and s.offset + len(s) <= len(data)
        try:
            b.verify()
        except errors.CorruptError:
            pass
