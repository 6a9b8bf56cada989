"""GGUF parsing: the reference reader's own test cases on the oracle.

crates/det-gguf/src/lib.rs:586-845 builds small GGUF byte strings and
checks which `GgufError` each one raises.  The same byte strings go through
the oracle's reader (oracle/ref_gguf.c) on the CPU and, on a GPU, through
the library's loader (det_model_load, detllm_b200/csrc/model.cpp), which
reports every parse error as the reference's ModelError::Gguf.
"""
import struct

import pytest


def header(n_tensors, n_kv):
    return b"GGUF" + struct.pack("<IQQ", 3, n_tensors, n_kv)


def string(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def u32_kv(key, value):
    return string(key) + struct.pack("<II", 4, value)


def tensor_info(name, offset=0):
    # one dimension of 1 element, F32
    return string(name) + struct.pack("<IQIQ", 1, 1, 0, offset)


def array_header(key, elem_ty, n):
    return string(key) + struct.pack("<IIQ", 9, elem_ty, n)


def pad(b):
    return b + b"\0" * (-len(b) % 32)


@pytest.fixture(scope="module")
def parse(oracle):
    return oracle.gguf_parse_error


def test_rejects_bad_magic(parse):
    assert parse(b"nope") == "bad magic"


def test_rejects_missing_aligned_tensor_data_region(parse):
    b = header(0, 0)
    assert parse(b) == "truncated"
    assert parse(pad(b)) == "ok"


def test_metadata_prefix_without_tensor_payload_is_truncated(parse):
    assert parse(header(1, 1) + u32_kv("answer", 42) + tensor_info("weight")) == "truncated"


def test_rejects_impossible_counts_before_allocating(parse):
    assert parse(b"GGUF" + struct.pack("<IQQ", 3, 2**64 - 1, 0)) == "truncated"
    huge = header(0, 1) + string("huge") + struct.pack("<IIQ", 9, 0, 2**64 - 1)
    assert parse(huge) == "truncated"


def test_rejects_duplicate_metadata_keys_and_tensor_names(parse):
    assert parse(header(0, 2) + u32_kv("dup", 1) + u32_kv("dup", 2)) == "duplicate metadata key"
    assert parse(header(2, 0) + tensor_info("dup") + tensor_info("dup")) == "duplicate tensor name"


def test_rejects_overlapping_or_out_of_bounds_tensor_data(parse):
    overlapping = pad(header(2, 0) + tensor_info("a", 0) + tensor_info("b", 2)) + b"\0" * 6
    assert parse(overlapping) == "invalid tensor offset"
    out_of_bounds = pad(header(1, 0) + tensor_info("a", 4)) + b"\0" * 4
    assert parse(out_of_bounds) == "truncated"
    in_bounds = pad(header(2, 0) + tensor_info("a", 0) + tensor_info("b", 4)) + b"\0" * 8
    assert parse(in_bounds) == "ok"


def test_rejects_noncanonical_bool_metadata_values(parse):
    assert parse(header(0, 1) + string("flag") + struct.pack("<IB", 7, 2)) == "invalid bool"
    assert parse(header(0, 1) + array_header("flags", 7, 3) + bytes([0, 1, 2])) == "invalid bool"


def test_parses_all_supported_metadata_array_types(parse):
    b = header(0, 12)
    b += array_header("u8s", 0, 2) + bytes([1, 2])
    b += array_header("i8s", 1, 2) + bytes([255, 2])
    b += array_header("u16s", 2, 2) + struct.pack("<HH", 1, 2)
    b += array_header("i16s", 3, 2) + struct.pack("<hh", -1, 2)
    b += array_header("u32s", 4, 2) + struct.pack("<II", 1, 2)
    b += array_header("i32s", 5, 2) + struct.pack("<ii", -1, 2)
    b += array_header("f32s", 6, 2) + struct.pack("<ff", 1.5, -2.25)
    b += array_header("bools", 7, 2) + bytes([0, 1])
    b += array_header("strings", 8, 2) + string("a") + string("bc")
    b += array_header("u64s", 10, 2) + struct.pack("<QQ", 1, 2)
    b += array_header("i64s", 11, 2) + struct.pack("<qq", -1, 2)
    b += array_header("f64s", 12, 2) + struct.pack("<dd", 1.5, -2.25)
    assert parse(pad(b)) == "ok"


def test_rejects_unsupported_version_and_value_type(parse):
    assert parse(pad(b"GGUF" + struct.pack("<IQQ", 4, 0, 0))) == "unsupported version"
    assert parse(pad(header(0, 1) + string("x") + struct.pack("<I", 13))) == "unsupported value type"


@pytest.mark.gpu
def test_library_loader_refuses_the_same_files():
    """det_model_load on each malformed file returns DET_ERR_GGUF (8), as
    F32Llama::from_gguf maps every GgufError (det-model :2158-2163); a
    well-formed file without metadata lacks general.architecture (7)."""
    import detllm_b200 as D

    assert D.device_count() > 0, "gpu tests need a CUDA device"
    bad = [
        b"nope",
        header(0, 0),
        header(1, 1) + u32_kv("answer", 42) + tensor_info("weight"),
        b"GGUF" + struct.pack("<IQQ", 3, 2**64 - 1, 0),
        header(0, 2) + u32_kv("dup", 1) + u32_kv("dup", 2),
        header(2, 0) + tensor_info("dup") + tensor_info("dup"),
        pad(header(2, 0) + tensor_info("a", 0) + tensor_info("b", 2)) + b"\0" * 6,
        pad(header(1, 0) + tensor_info("a", 4)) + b"\0" * 4,
        header(0, 1) + string("flag") + struct.pack("<IB", 7, 2),
        pad(b"GGUF" + struct.pack("<IQQ", 4, 0, 0)),
    ]
    for i, b in enumerate(bad):
        with pytest.raises(D.DetError) as e:
            D.Model(b)
        assert e.value.code == 8, i
    with pytest.raises(D.DetError) as e:
        D.Model(pad(header(0, 0)))
    assert e.value.code == 7
