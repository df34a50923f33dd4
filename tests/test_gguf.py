"""The native GGUF reader (lbk_gguf_open) against the reference's own reader
and split-set tests: bridge-gguf/tests/reader.rs:200-800 and
bridge-gguf-split/tests/splits.rs:219-690, case for case where a file can
express the case, with the reference's error messages; and the Hy3 MoE block
schema checks of lbk_moe_layer_load that run before any device work
(schema.rs:200-258, checked_expert_slab :524-580, config.rs:57-109). CPU only.

Not restated: rejects_data_offset_overflow needs a reader that reports a
position near 2^64, which no file can produce.
"""

from __future__ import annotations

import ctypes
import os
import re
import struct

import numpy as np
import pytest

import lbk
from conftest import REPO
from gguf_fixture import ARRAY, BOOL, F32, I32, STRING, U8, U16, U32, U64, Fixture, Hy3Block, write_hy3

KIND = {m.group(1): int(m.group(2)) for m in
        re.finditer(r"LBK_GGUF_([A-Z0-9_]+) = (\d+)", (REPO / "include" / "lightbridge_kernels.h").read_text())}


def open_bytes(tmp_path, data: bytes, name="model.gguf", limits=None):
    p = tmp_path / name
    p.write_bytes(data)
    return lbk.Gguf(p, limits)


def failure(fn, *args):
    with pytest.raises(lbk.LbkError) as e:
        fn(*args)
    d = e.value.detail
    return e.value.status, d.bits, d.message.decode(), d


def read_err(tmp_path, data: bytes, limits=None, name="model.gguf"):
    p = tmp_path / name
    p.write_bytes(data)
    st, kind, msg, d = failure(lbk.Gguf, p, limits)
    assert st == 33, (st, msg)
    return kind, msg, d


def limits(**kw):
    lim = lbk.Gguf.default_limits()
    for k, v in kw.items():
        setattr(lim, k, v)
    return lim


# ------------------------------------------------------- reader.rs cases


def test_default_limits_are_the_reference_defaults():
    lim = lbk.Gguf.default_limits()
    assert (lim.max_dimensions, lim.max_string_bytes, lim.max_array_elements, lim.max_tensors,
            lim.max_metadata_entries, lim.max_metadata_bytes) == (4, 1 << 20, 1_000_000, 4_000_000, 1_000_000, 64 << 20)


def test_reads_minimal_little_endian_v3(tmp_path):
    with open_bytes(tmp_path, Fixture().tensor(b"x", [1], 0, 0).add_payload(bytes(32)).bytes()) as g:
        i = g.info()
        assert (i.version, i.big_endian, i.alignment, i.data_offset, i.file_len) == (3, 0, 32, 64, 96)
        ts = g.tensors()
        assert [n for n, _ in ts] == ["x"] and ts[0][1].shape == (1,)


def test_reads_exactly_aligned_tensor_directory(tmp_path):
    with open_bytes(tmp_path, Fixture().tensor(b"12345678", [1], 0, 0).add_payload(bytes(32)).bytes()) as g:
        assert (g.info().data_offset, g.info().file_len) == (64, 96)
        assert g.tensors()[0][0] == "12345678"


@pytest.mark.parametrize("records,payload,message", [
    ([(b"first", [1], 0), (b"alias", [1], 0)], 64,
     'tensor "alias" has relative payload offset 0, expected 32 for 32-byte alignment'),
    ([(b"wide", [9], 0), (b"overlap", [1], 32)], 96,
     'tensor "overlap" has relative payload offset 32, expected 64 for 32-byte alignment'),
    ([(b"first", [1], 0), (b"after-gap", [1], 64)], 96,
     'tensor "after-gap" has relative payload offset 64, expected 32 for 32-byte alignment'),
    ([(b"first", [1], 32)], 64, 'tensor "first" has relative payload offset 32, expected 0 for 32-byte alignment'),
    ([(b"second", [1], 32), (b"first", [1], 0)], 64,
     'tensor "second" has relative payload offset 32, expected 0 for 32-byte alignment'),
])
def test_rejects_directories_that_are_not_packed_in_order(tmp_path, records, payload, message):
    fx = Fixture()
    for name, dims, off in records:
        fx.tensor(name, dims, 0, off)
    kind, msg, _ = read_err(tmp_path, fx.add_payload(bytes(payload)).bytes())
    assert kind == KIND["TENSOR_OFFSET_MISMATCH"] and msg == message


def test_rejects_truncated_final_tensor_padding(tmp_path):
    kind, msg, _ = read_err(tmp_path, Fixture().tensor(b"x", [1], 0, 0).add_payload(bytes(4)).bytes())
    assert kind == KIND["TENSOR_DATA_SECTION_TRUNCATED"]
    assert msg == "GGUF tensor data section requires padded range 64..96, but physical file length is 68"


def test_rejects_overflow_while_padding_a_tensor_extent(tmp_path):
    kind, msg, _ = read_err(tmp_path, Fixture().tensor(b"huge", [2**64 - 1], 24, 0).bytes())
    assert kind == KIND["TENSOR_PADDING_OVERFLOW"]
    assert msg == 'tensor "huge" encoded byte length 18446744073709551615 overflows 32-byte padding'


def test_accepts_mixed_types_at_exact_padded_offsets_and_trailing_bytes(tmp_path):
    fx = Fixture().tensor(b"float", [1], 0, 0).tensor(b"quant", [256], 12, 32).tensor(b"bytes", [7], 24, 192)
    with open_bytes(tmp_path, fx.add_payload(bytes(231)).bytes()) as g:
        assert [t.bytes for _, t in g.tensors()] == [4, 144, 7]
        assert g.info().file_len == g.info().data_offset + 224 + 7


def test_reads_minimal_v2(tmp_path):
    with open_bytes(tmp_path, Fixture(version=2).bytes()) as g:
        assert (g.info().version, g.info().big_endian) == (2, 0)


def test_reads_byte_swapped_big_endian_file(tmp_path):
    fx = Fixture(big=True)
    fx.meta(b"answer", U32, fx.u32(42))
    with open_bytes(tmp_path, fx.bytes()) as g:
        assert g.info().big_endian == 1
        assert g.metadata("answer") == 42


def test_rejects_bad_magic_and_unsupported_versions(tmp_path):
    bad = bytearray(Fixture().bytes())
    bad[:4] = b"NOPE"
    kind, msg, _ = read_err(tmp_path, bytes(bad))
    assert kind == KIND["BAD_MAGIC"] and msg == "bad GGUF magic bytes [78, 79, 80, 69]"
    for v in (1, 4):
        kind, msg, d = read_err(tmp_path, Fixture(version=v).bytes())
        assert kind == KIND["UNSUPPORTED_VERSION"] and msg == f"unsupported GGUF version {v}" and d.actual == v


def test_rejects_truncated_scalars_strings_arrays_and_tensor_records(tmp_path):
    fx = Fixture()
    scalar = Fixture().meta(b"k", U64, bytes(7)).bytes()[:44]
    string_value = Fixture().meta(b"k", STRING, fx.u64(4) + b"abc").bytes()[:48]
    array_value = Fixture().meta(b"k", ARRAY, fx.array(U32, bytes(3), 1)).bytes()[:52]
    tensor = Fixture().tensor(b"x", [1], 0, 0).bytes()[:56]
    for data in (scalar, string_value, array_value, tensor):
        kind, msg, _ = read_err(tmp_path, data)
        assert kind == KIND["TRUNCATED"] and msg.startswith("GGUF is truncated while reading "), msg


def test_enforces_metadata_tensor_string_and_array_limits(tmp_path):
    kind, msg, _ = read_err(tmp_path, Fixture().bytes(0, 2), limits(max_metadata_entries=1))
    assert kind == KIND["LIMIT_EXCEEDED"] and msg.startswith("metadata entries count 2")
    kind, msg, _ = read_err(tmp_path, Fixture().bytes(2, 0), limits(max_tensors=1))
    assert kind == KIND["LIMIT_EXCEEDED"] and msg.startswith("tensors count 2")
    fx = Fixture()
    kind, msg, _ = read_err(tmp_path, fx.meta(b"four", U32, fx.u32(1)).bytes(), limits(max_string_bytes=3))
    assert kind == KIND["LIMIT_EXCEEDED"] and msg == "string bytes count 4 exceeds configured limit 3"
    fx = Fixture()
    kind, msg, _ = read_err(tmp_path, fx.meta(b"k", ARRAY, fx.array(U8, b"\x01\x02", 2)).bytes(),
                            limits(max_array_elements=1))
    assert kind == KIND["LIMIT_EXCEEDED"] and msg.startswith("array elements count 2")


def test_metadata_budget_charges_string_and_array_payloads(tmp_path):
    fx = Fixture()
    kind, msg, _ = read_err(tmp_path, fx.meta(b"k", STRING, fx.string(b"abc")).bytes(), limits(max_metadata_bytes=3))
    assert kind == KIND["LIMIT_EXCEEDED"] and msg.startswith("metadata bytes count")
    fx = Fixture()
    kind, msg, _ = read_err(tmp_path, fx.meta(b"k", ARRAY, fx.array(U32, bytes([0, 0, 0, 0, 1, 0, 0, 0]), 2)).bytes(),
                            limits(max_metadata_bytes=8))
    assert kind == KIND["LIMIT_EXCEEDED"] and msg.startswith("metadata bytes count")
    kind, msg, _ = read_err(tmp_path, Fixture().tensor(b"name", [1], 0, 0).add_payload(bytes(4)).bytes(),
                            limits(max_metadata_bytes=11))
    assert kind == KIND["LIMIT_EXCEEDED"] and msg == "metadata bytes count 12 exceeds configured limit 11"


def test_array_element_limit_is_aggregate_across_the_file(tmp_path):
    fx = Fixture()
    fx.meta(b"a", ARRAY, fx.array(U8, b"\x01\x02", 2)).meta(b"b", ARRAY, fx.array(U8, b"\x03\x04", 2))
    kind, msg, d = read_err(tmp_path, fx.bytes(), limits(max_array_elements=3))
    assert kind == KIND["LIMIT_EXCEEDED"] and (d.expected, d.actual) == (3, 4)


def test_array_minimum_encoding_must_fit_remaining_metadata_budget(tmp_path):
    fx = Fixture()
    data = fx.meta(b"k", ARRAY, fx.array(U64, b"", 4)).bytes()[:49]
    kind, msg, d = read_err(tmp_path, data, limits(max_metadata_bytes=50))
    assert kind == KIND["LIMIT_EXCEEDED"] and (d.expected, d.actual) == (50, 57)


def test_truncated_maximum_array_reports_truncation(tmp_path):
    fx = Fixture()
    kind, _, _ = read_err(tmp_path, fx.meta(b"k", ARRAY, fx.array(U8, b"", 1_000_000)).bytes()[:49])
    assert kind == KIND["TRUNCATED"]


def test_rejects_invalid_utf8_boolean_and_metadata_type(tmp_path):
    fx = Fixture()
    kind, msg, _ = read_err(tmp_path, fx.meta(b"\xff", U32, fx.u32(1)).bytes())
    assert kind == KIND["INVALID_UTF8"] and msg == "invalid UTF-8 in metadata key"
    kind, msg, _ = read_err(tmp_path, Fixture().meta(b"k", BOOL, b"\x02").bytes())
    assert kind == KIND["INVALID_BOOLEAN"] and msg == "invalid GGUF boolean byte 2"
    kind, msg, _ = read_err(tmp_path, Fixture().meta(b"k", 99, b"").bytes())
    assert kind == KIND["UNKNOWN_VALUE_TYPE"] and msg == "unknown GGUF metadata value type 99"


def test_rejects_recursive_array_type(tmp_path):
    fx = Fixture()
    kind, msg, _ = read_err(tmp_path, fx.meta(b"k", ARRAY, fx.array(ARRAY, b"", 0)).bytes())
    assert kind == KIND["NESTED_ARRAY"] and msg == "GGUF arrays may not contain arrays"


def test_rejects_unknown_ggml_type_and_invalid_dimension_counts(tmp_path):
    kind, msg, _ = read_err(tmp_path, Fixture().tensor(b"x", [1], 5, 0).add_payload(bytes(4)).bytes())
    assert kind == KIND["UNKNOWN_GGML_TYPE"] and msg == "unknown ggml type discriminant 5"
    fx = Fixture()
    fx.tensors.append(fx.string(b"x") + fx.u32(0) + fx.u32(0) + fx.u64(0))
    kind, msg, d = read_err(tmp_path, fx.bytes())
    assert kind == KIND["INVALID_DIMENSION_COUNT"] and d.actual == 0
    kind, msg, d = read_err(tmp_path, Fixture().tensor(b"x", [1, 1, 1, 1, 1], 0, 0).add_payload(bytes(4)).bytes())
    assert kind == KIND["INVALID_DIMENSION_COUNT"] and d.actual == 5
    assert msg == "tensor dimension count 5 is outside GGML's supported 1..=4 dimensions"


def test_rejects_quantized_row_block_mismatch_and_zero_dimensions(tmp_path):
    kind, msg, _ = read_err(tmp_path, Fixture().tensor(b"q", [31], 2, 0).bytes())
    assert kind == KIND["NOT_BLOCK_ALIGNED"] and msg == "Q4_0 requires a leading dimension divisible by 32, got 31"
    kind, msg, _ = read_err(tmp_path, Fixture().tensor(b"z", [4, 0], 0, 0).bytes())
    assert kind == KIND["ZERO_TENSOR_DIMENSION"] and msg == "tensor dimension 1 is zero"


def test_rejects_tensor_range_beyond_physical_file_length(tmp_path):
    kind, msg, _ = read_err(tmp_path, Fixture().tensor(b"x", [1], 0, 0).bytes())
    assert kind == KIND["TENSOR_OUT_OF_BOUNDS"] and msg == "tensor byte range 64..68 exceeds file length 64"


def test_rejects_duplicate_metadata_and_invalid_alignment(tmp_path):
    fx = Fixture()
    fx.meta(b"k", U32, fx.u32(1)).meta(b"k", U32, fx.u32(2))
    kind, msg, _ = read_err(tmp_path, fx.bytes())
    assert kind == KIND["DUPLICATE_METADATA_KEY"] and msg == 'duplicate GGUF metadata key "k"'
    for a in (0, 3):
        fx = Fixture()
        kind, msg, _ = read_err(tmp_path, fx.meta(b"general.alignment", U32, fx.u32(a)).bytes())
        assert kind == KIND["INVALID_ALIGNMENT"] and msg == f"general.alignment must be a positive u32 power of two, got {a}"
    fx = Fixture()
    kind, msg, _ = read_err(tmp_path, fx.meta(b"general.alignment", U64, fx.u64(32)).bytes())
    assert kind == KIND["ALIGNMENT_WRONG_TYPE"] and msg == "general.alignment must have type U32, got U64"


def test_typed_getters_distinguish_missing_keys_from_wrong_types(tmp_path):
    fx = Fixture()
    fx.meta(b"name", STRING, fx.string(b"hy3")).meta(b"enabled", BOOL, b"\x01")
    with open_bytes(tmp_path, fx.bytes()) as g:
        assert g.metadata("name") == "hy3" and g.metadata("enabled") is True
        st, kind, msg, _ = failure(g.metadata, "missing")
        assert (st, kind, msg) == (33, KIND["METADATA_MISSING"], 'missing GGUF metadata key "missing"')
        buf = ctypes.create_string_buffer(8)
        assert lbk.lib.lbk_gguf_metadata_string(g.ptr, b"enabled", buf, 8, None) == 33
        d = lbk.last_error()
        assert d.bits == KIND["METADATA_WRONG_TYPE"]
        assert d.message.decode() == 'GGUF metadata key "enabled" has type Bool, expected String'


def test_rejects_caller_dimension_limit_above_ggml_maximum(tmp_path):
    kind, msg, _ = read_err(tmp_path, Fixture().bytes(), limits(max_dimensions=5))
    assert kind == KIND["INVALID_DIMENSION_LIMIT"] and msg == "configured dimension limit 5 exceeds GGML's maximum of four"


def test_metadata_values_of_every_scalar_type(tmp_path):
    fx = Fixture()
    fx.meta(b"u8", 0, b"\xfe").meta(b"i8", 1, b"\xfe").meta(b"u16", 2, struct.pack("<H", 65000))
    fx.meta(b"i16", 3, struct.pack("<h", -3)).meta(b"i32", 5, struct.pack("<i", -70000))
    fx.meta(b"f32", 6, struct.pack("<f", 2.826)).meta(b"i64", 11, struct.pack("<q", -(2**40)))
    fx.meta(b"f64", 12, struct.pack("<d", 1e-300)).meta(b"u64", U64, fx.u64(2**63 + 5))
    fx.meta(b"arr", ARRAY, fx.array(STRING, fx.string(b"a") + fx.string(b"bc"), 2))
    with open_bytes(tmp_path, fx.bytes()) as g:
        assert g.metadata("u8") == 254 and g.metadata("i8") == -2 and g.metadata("u16") == 65000
        assert g.metadata("i16") == -3 and g.metadata("i32") == -70000 and g.metadata("i64") == -(2**40)
        assert g.metadata("f32") == float(np.float32(2.826)) and g.metadata("f64") == 1e-300
        assert g.metadata("u64") == 2**63 + 5
        assert g.metadata("arr") == ("array", STRING, 2)


# ------------------------------------------------------- splits.rs cases


def split_fixture(ordinal=None, count=None, tensors=(), split_count=None, version=3, big=False, alignment=None,
                  extra=()):
    fx = Fixture(version=version, big=big)
    if alignment is not None:
        fx.meta(b"general.alignment", U32, fx.u32(alignment))
        fx.alignment = alignment
    if ordinal is not None:
        fx.meta(b"split.no", U16, fx.u16(ordinal)).meta(b"split.count", U16, fx.u16(count))
    if split_count is not None:
        fx.meta(b"split.tensors.count", I32, fx.i32(split_count))
    for key, ty, val in extra:
        fx.meta(key, ty, val)
    payload = 0
    for name, off in tensors:
        fx.tensor(name, [1], 0, off)
        payload = max(payload, off + fx.alignment)
    return fx.add_payload(bytes(payload)).bytes()


def write(d, name, data):
    p = d / name
    p.write_bytes(data)
    return p


def split_err(entry):
    st, kind, msg, d = failure(lbk.Gguf, entry)
    return kind, msg


def test_opens_an_ordinary_non_numbered_single_file(tmp_path):
    with lbk.Gguf(write(tmp_path, "model.gguf", split_fixture(tensors=[(b"only", 0)]))) as g:
        assert g.info().shard_count == 1 and [n for n, _ in g.tensors()] == ["only"]


def test_accepts_any_numbered_member_and_orders_shards_by_ordinal(tmp_path):
    write(tmp_path, "name-00003-of-00003.gguf", split_fixture(2, 3, [(b"third", 0)]))
    write(tmp_path, "name-00001-of-00003.gguf", split_fixture(0, 3, [(b"first", 0)]))
    write(tmp_path, "name-00002-of-00003.gguf", split_fixture(1, 3, [(b"second", 0)]))
    with lbk.Gguf(tmp_path / "name-00003-of-00003.gguf") as g:
        assert g.info().shard_count == 3
        ts = g.tensors()
        assert [n for n, _ in ts] == ["first", "second", "third"] and [t.shard for _, t in ts] == [0, 1, 2]


@pytest.mark.parametrize("files,entry,kind", [
    ([("name-00001-of-00003.gguf", 0, 3), ("name-00003-of-00003.gguf", 2, 3)], 0, "MISSING_SHARD"),
    ([("name-00000-of-00003.gguf", 0, 3)], 0, "INVALID_NUMBERED_FILENAME"),
    ([("name-00004-of-00003.gguf", 3, 3)], 0, "INVALID_NUMBERED_FILENAME"),
    ([("name-00001-of-00002.gguf", 0, 2), ("name-00002-of-00003.gguf", 1, 3)], 0, "MISSING_SHARD"),
    ([("name-00001-of-00002.gguf", 0, 2), ("name-00002-of-00002.gguf", 0, 2)], 0, "SPLIT_METADATA_DISAGREEMENT"),
    ([("name-00001-of-00002.gguf", 1, 2), ("name-00002-of-00002.gguf", 1, 2)], 0, "SPLIT_METADATA_DISAGREEMENT"),
    ([("name-00001-of-00002.gguf", 0, 3), ("name-00002-of-00002.gguf", 1, 2)], 0, "SPLIT_METADATA_DISAGREEMENT"),
    ([("model-00001-of-65536.gguf", None, None)], 0, "INVALID_NUMBERED_FILENAME"),
    ([("name-00001-of-00002.gguf", None, None), ("name-00002-of-00002.gguf", 1, 2)], 0, "MISSING_SPLIT_METADATA"),
])
def test_rejects_bad_numbered_sets(tmp_path, files, entry, kind):
    paths = [write(tmp_path, n, split_fixture(o, c)) for n, o, c in files]
    k, msg = split_err(paths[entry])
    assert k == KIND[kind], msg


def test_split_metadata_disagreement_names_the_key(tmp_path):
    e = write(tmp_path, "name-00001-of-00002.gguf", split_fixture(0, 3))
    write(tmp_path, "name-00002-of-00002.gguf", split_fixture(1, 2))
    assert split_err(e)[1].endswith('metadata "split.count" does not match its filename')


def test_rejects_aggregate_tensor_count_disagreement(tmp_path):
    e = write(tmp_path, "name-00001-of-00002.gguf", split_fixture(0, 2, [(b"one", 0)], split_count=3))
    write(tmp_path, "name-00002-of-00002.gguf", split_fixture(1, 2, [(b"two", 0)], split_count=3))
    assert split_err(e) == (KIND["AGGREGATE_TENSOR_DIRECTORY_DISAGREEMENT"],
                            "split.tensors.count does not match the aggregate tensor directory")


def test_rejects_different_declared_aggregate_counts_between_shards(tmp_path):
    e = write(tmp_path, "model-00001-of-00002.gguf", split_fixture(0, 2, [(b"one", 0)], split_count=2))
    write(tmp_path, "model-00002-of-00002.gguf", split_fixture(1, 2, [(b"two", 0)], split_count=3))
    assert split_err(e)[0] == KIND["AGGREGATE_TENSOR_COUNT_DISAGREEMENT"]


def test_accepts_a_matching_aggregate_count(tmp_path):
    e = write(tmp_path, "model-00001-of-00002.gguf", split_fixture(0, 2, [(b"one", 0)], split_count=2))
    write(tmp_path, "model-00002-of-00002.gguf", split_fixture(1, 2, [(b"two", 0)], split_count=2))
    with lbk.Gguf(e) as g:
        assert g.info().tensor_count == 2 and g.tensor("two").shard == 1


def test_rejects_duplicate_tensor_names_across_shards(tmp_path):
    e = write(tmp_path, "name-00001-of-00002.gguf", split_fixture(0, 2, [(b"same", 0)]))
    write(tmp_path, "name-00002-of-00002.gguf", split_fixture(1, 2, [(b"same", 0)]))
    assert split_err(e) == (KIND["DUPLICATE_TENSOR_NAME"], 'duplicate tensor name "same" across GGUF shards')


@pytest.mark.parametrize("offset", [8, 4])
def test_rejects_a_misplaced_first_tensor_offset_at_the_parser_boundary(tmp_path, offset):
    fx = Fixture().tensor(b"bad", [1], 0, offset)
    k, msg = split_err(write(tmp_path, "model.gguf", fx.add_payload(bytes(offset + 32)).bytes()))
    assert k == KIND["TENSOR_OFFSET_MISMATCH"]
    assert msg == f'tensor "bad" has relative payload offset {offset}, expected 0 for 32-byte alignment'


def test_rejects_non_file_input(tmp_path):
    assert split_err(tmp_path)[0] == KIND["NOT_A_FILE"]


def test_ignores_similarly_named_unrelated_siblings(tmp_path):
    e = write(tmp_path, "name-00001-of-00002.gguf", split_fixture(0, 2))
    write(tmp_path, "name-00002-of-00002.gguf", split_fixture(1, 2))
    write(tmp_path, "name-00003-of-00003.gguf", split_fixture(2, 3))
    with lbk.Gguf(e) as g:
        assert g.info().shard_count == 2


def test_rejects_wrongly_typed_required_split_metadata(tmp_path):
    fx = Fixture()
    fx.meta(b"split.no", U32, fx.u32(0)).meta(b"split.count", U16, fx.u16(2))
    e = write(tmp_path, "typed-00001-of-00002.gguf", fx.bytes())
    write(tmp_path, "typed-00002-of-00002.gguf", split_fixture(1, 2))
    assert split_err(e) == (KIND["METADATA_WRONG_TYPE"], 'GGUF metadata key "split.no" has type U32, expected U16')


def test_rejects_symlinks_that_escape_the_entry_parent(tmp_path):
    inside, outside = tmp_path / "in", tmp_path / "out"
    inside.mkdir()
    outside.mkdir()
    target = write(outside, "model.gguf", split_fixture())
    os.symlink(target, inside / "model.gguf")
    assert split_err(inside / "model.gguf")[0] == KIND["SHARD_ESCAPES_PARENT"]
    t1 = write(outside, "model-00001-of-00002.gguf", split_fixture(0, 2))
    write(outside, "model-00002-of-00002.gguf", split_fixture(1, 2))
    os.symlink(t1, inside / "model-00001-of-00002.gguf")
    assert split_err(inside / "model-00001-of-00002.gguf")[0] == KIND["SHARD_ESCAPES_PARENT"]
    d = tmp_path / "set"
    d.mkdir()
    e = write(d, "model-00001-of-00002.gguf", split_fixture(0, 2))
    os.symlink(outside / "model-00002-of-00002.gguf", d / "model-00002-of-00002.gguf")
    assert split_err(e)[0] == KIND["SHARD_ESCAPES_PARENT"]


def test_treats_non_five_digit_split_like_names_as_ordinary_files(tmp_path):
    with lbk.Gguf(write(tmp_path, "model-1-of-2.gguf", split_fixture(tensors=[(b"only", 0)]))) as g:
        assert g.info().shard_count == 1


def test_rejects_single_file_optional_split_metadata_that_contradicts_ordinal_or_count(tmp_path):
    assert split_err(write(tmp_path, "ordinal.gguf", split_fixture(1, 1)))[1].endswith(
        'metadata "split.no" does not match its filename')
    assert split_err(write(tmp_path, "count.gguf", split_fixture(0, 2)))[1].endswith(
        'metadata "split.count" does not match its filename')


def test_rejects_negative_or_wrongly_typed_aggregate_tensor_counts(tmp_path):
    assert split_err(write(tmp_path, "negative.gguf", split_fixture(split_count=-1)))[0] == \
        KIND["NEGATIVE_AGGREGATE_TENSOR_COUNT"]
    fx = Fixture()
    k, msg = split_err(write(tmp_path, "wrong-type.gguf", fx.meta(b"split.tensors.count", U32, fx.u32(1)).bytes()))
    assert (k, msg) == (KIND["METADATA_WRONG_TYPE"], 'GGUF metadata key "split.tensors.count" has type U32, expected I32')


@pytest.mark.parametrize("second,message", [
    (dict(version=2), "has version 2, expected common version 3"),
    (dict(big=True), "has endianness Big, expected common endianness Little"),
    (dict(alignment=64), "has alignment 64, expected common alignment 32"),
])
def test_rejects_heterogeneous_shards(tmp_path, second, message):
    e = write(tmp_path, "model-00001-of-00002.gguf", split_fixture(0, 2))
    s = write(tmp_path, "model-00002-of-00002.gguf", split_fixture(1, 2, **second))
    k, msg = split_err(e)
    assert msg == f'GGUF shard "{os.path.realpath(s)}" {message}'


def test_accepts_shards_with_different_metadata_counts(tmp_path):
    fx = Fixture()
    e = write(tmp_path, "model-00001-of-00002.gguf", split_fixture(0, 2, extra=[(b"extra", U32, fx.u32(7))]))
    write(tmp_path, "model-00002-of-00002.gguf", split_fixture(1, 2))
    with lbk.Gguf(e) as g:
        assert g.info().metadata_count == 3 and g.metadata("extra") == 7


# ------------------------------------------------------- Hy3 MoE block schema

H, FF, E, K = 256, 256, 4, 2
T_IQ2, T_IQ3, T_Q4, T_Q8 = lbk.TYPE_IQ2_S, lbk.TYPE_IQ3_S, lbk.TYPE_Q4_K, lbk.TYPE_Q8_K


def small_block(rng, down=T_IQ3):
    return Hy3Block(rng, H, FF, E, T_IQ2, T_IQ2, down, T_IQ2, T_IQ2, down)


def load_err(gguf, block=0, first=0, count=0):
    p = ctypes.c_void_p()
    st = lbk.lib.lbk_moe_layer_load(None, gguf.ptr, block, first, count, None, ctypes.byref(p))
    d = lbk.last_error()
    return st, d.bits, d.message.decode()


def test_hy3_set_exposes_the_schema_tensors_and_slabs(tmp_path):
    rng = np.random.default_rng(1)
    blocks = {1: small_block(rng), 2: small_block(rng, T_IQ2)}
    entry = write_hy3(tmp_path, H, FF, E, K, blocks, block_count=3, shards=2)
    with lbk.Gguf(entry) as g:
        assert g.info().shard_count == 2 and g.info().tensor_count == 16
        assert g.metadata("general.architecture") == "hy_v3"
        assert g.metadata("hy_v3.expert_weights_scale") == float(np.float32(2.826))
        assert g.metadata("tokenizer.ggml.tokens") == ("array", STRING, 3)
        t = g.tensor("blk.2.ffn_down_exps.weight")
        assert (t.shape, t.type, t.shard) == ((FF, H, E), T_IQ2, 1)
        assert t.bytes == E * H * (FF // 256) * 82
        # expert e is the e-th slab of the stacked payload (checked_expert_slab)
        raw = (tmp_path / "hy3-00002-of-00002.gguf").read_bytes()
        slab = t.bytes // E
        assert raw[t.offset + 3 * slab:t.offset + 4 * slab] == blocks[2].experts[3][2].tobytes()
        r = g.tensor("blk.1.ffn_gate_inp.weight")
        assert r.shape == (H, E) and np.array_equal(
            np.frombuffer((tmp_path / "hy3-00001-of-00002.gguf").read_bytes()[r.offset:r.offset + r.bytes], np.float32),
            blocks[1].router.reshape(-1))


def test_layer_load_validates_the_block_before_device_work(tmp_path):
    rng = np.random.default_rng(2)
    entry = write_hy3(tmp_path, H, FF, E, K, {0: small_block(rng)}, block_count=2)
    with lbk.Gguf(entry) as g:
        # a valid block reaches the device step, which needs a context
        assert load_err(g)[:2] == (15, 0)
        assert load_err(g, block=2)[1] == KIND["BLOCK_OUT_OF_RANGE"]
        assert load_err(g, block=1) == (33, KIND["MISSING_TENSOR"], 'missing tensor "blk.1.exp_probs_b"')
        assert load_err(g, first=4)[1] == KIND["EXPERT_RANGE"]
        assert load_err(g, first=1, count=4)[1] == KIND["EXPERT_RANGE"]
        assert load_err(g, first=1, count=3)[:2] == (15, 0)


def _schema_case(tmp_path, rng, mutate, name="case"):
    """A one-block set whose metadata / tensors `mutate` edits."""
    d = tmp_path / name
    d.mkdir()
    b = small_block(rng)
    ts = b.tensors(0, H, FF, E)
    meta = {"general.architecture": (STRING, b"hy_v3"), "hy_v3.block_count": (U32, 1), "hy_v3.embedding_length": (U32, H),
            "hy_v3.expert_feed_forward_length": (U32, FF), "hy_v3.expert_shared_feed_forward_length": (U32, FF),
            "hy_v3.expert_count": (U32, E), "hy_v3.expert_used_count": (U32, K),
            "hy_v3.expert_weights_scale": (F32, 2.826)}
    ts = [list(t) for t in ts]
    mutate(meta, ts)
    fx = Fixture()
    enc = {STRING: fx.string, U32: fx.u32, F32: fx.f32, U64: fx.u64, BOOL: fx.u8}
    for k, (ty, v) in meta.items():
        fx.meta(k.encode(), ty, enc[ty](v))
    off = 0
    for name_, dims, ty, payload in ts:
        fx.tensor(name_.encode(), dims, ty, off)
        padded = (len(payload) + 31) // 32 * 32
        fx.add_payload(payload + bytes(padded - len(payload)))
        off += padded
    p = d / "m.gguf"
    p.write_bytes(fx.bytes())
    with lbk.Gguf(p) as g:
        return load_err(g)


def test_layer_load_schema_errors(tmp_path):
    rng = np.random.default_rng(3)

    def arch(m, t):
        m["general.architecture"] = (STRING, b"llama")

    def wrong_type(m, t):
        m["hy_v3.expert_count"] = (U64, E)

    def missing(m, t):
        del m["hy_v3.expert_used_count"]

    def scale_inf(m, t):
        m["hy_v3.expert_weights_scale"] = (F32, float("inf"))

    def shared_width(m, t):
        m["hy_v3.expert_shared_feed_forward_length"] = (U32, 512)

    def q8_gate(m, t):  # a ggml type the device path does not compute
        t[2][2] = T_Q8
        t[2][3] = bytes(E * FF * 292)

    def router_f16(m, t):
        t[1][2] = 1
        t[1][3] = t[1][3][: len(t[1][3]) // 2]

    def shape(m, t):
        t[4][1] = [FF, H, E // 2]
        t[4][3] = t[4][3][: len(t[4][3]) // 2]

    cases = [(arch, "METADATA_VALUE"), (wrong_type, "METADATA_WRONG_TYPE"), (missing, "METADATA_MISSING"),
             (scale_inf, "NON_FINITE_METADATA"), (shared_width, "SHARED_WIDTH"), (q8_gate, "TENSOR_TYPE"),
             (router_f16, "TENSOR_TYPE"), (shape, "TENSOR_SHAPE")]
    for i, (fn, kind) in enumerate(cases):
        st, k, msg = _schema_case(tmp_path, rng, fn, f"c{i}")
        assert (st, k) == (33, KIND[kind]), (fn.__name__, msg)
    st, k, msg = _schema_case(tmp_path, rng, wrong_type, "msg")
    assert msg == 'GGUF metadata key "hy_v3.expert_count" has type U64, expected U32'
