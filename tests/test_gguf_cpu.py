"""The GGUF v3 reader of the C ABI (beacon_cuda_gguf_*) on the CPU, pinned
by the reference's own parser tests (crates/beacon-format/src/tests.rs:18-190:
parse_synthetic_gguf, extract_model_config_from_gguf) on the same bytes, and
its error cases (header.rs:17-47, tensor_info.rs, metadata.rs). No GPU."""
import numpy as np
import pytest

from gguf_writer import F32, STRING, U32, GgufBuilder


def reference_test_file(path, **kw):
    """build_test_gguf (tests.rs:18-105): two f32 tensors, Llama metadata."""
    b = GgufBuilder(pad_tensors=False, **kw)
    b.add_kv("general.architecture", STRING, "llama")
    b.add_kv("llama.embedding_length", U32, 64)
    b.add_kv("llama.block_count", U32, 2)
    b.add_kv("llama.attention.head_count", U32, 4)
    b.add_kv("llama.attention.head_count_kv", U32, 2)
    b.add_kv("llama.feed_forward_length", U32, 128)
    b.add_kv("llama.context_length", U32, 512)
    b.add_kv("llama.rope.freq_base", F32, 10000.0)
    b.add_kv("llama.attention.layer_norm_rms_epsilon", F32, 1e-5)
    b.add_kv("tokenizer.ggml.bos_token_id", U32, 1)
    b.add_kv("tokenizer.ggml.eos_token_id", U32, 2)
    b.add_tensor("weight_a", (3, 2), "F32", np.arange(1, 7, dtype=np.float32))    # GGUF dims [2, 3]
    b.add_tensor("weight_b", (2, 3), "F32", np.arange(7, 13, dtype=np.float32))   # GGUF dims [3, 2]
    return b.write(path)


@pytest.fixture(scope="module")
def gg():
    from beacon_cuda.gguf import GgufFile
    return GgufFile


def test_parse_synthetic_gguf(tmp_path, gg):
    """tests.rs:133-169."""
    from beacon_cuda import _lib as L
    f = gg(reference_test_file(tmp_path / "t.gguf"))
    assert f.version == 3
    ts = f.tensors
    assert [t.name for t in ts] == ["weight_a", "weight_b"]
    assert ts[0].shape == (3, 2) and ts[1].shape == (2, 3)        # dims reversed to row-major
    assert ts[0].dtype == L.DTYPE_F32 and ts[1].dtype == L.DTYPE_F32
    assert ts[0].nbytes == 24 and ts[1].nbytes == 24
    assert ts[0].data().view(np.float32).tolist() == [1, 2, 3, 4, 5, 6]
    assert ts[1].data().view(np.float32).tolist() == [7, 8, 9, 10, 11, 12]


def test_extract_model_config_from_gguf(tmp_path, gg):
    """tests.rs:171-190."""
    f = gg(reference_test_file(tmp_path / "t.gguf"))
    c = f.model_config()
    assert (c["hidden_size"], c["num_layers"], c["num_heads"], c["num_kv_heads"]) == (64, 2, 4, 2)
    assert (c["intermediate_size"], c["head_dim"], c["max_context"]) == (128, 16, 512)
    assert abs(c["rope_theta"] - 10000.0) < 1e-3 and abs(c["rms_norm_eps"] - 1e-5) < 1e-8
    assert f.get_int("tokenizer.ggml.bos_token_id") == 1 and f.get_int("tokenizer.ggml.eos_token_id") == 2
    assert f.get_string("general.architecture") == "llama"
    assert f.model_config(max_context=77)["max_context"] == 77     # the caller's cache size wins


def test_alignment_and_metadata_types(tmp_path, gg):
    """general.alignment moves the data section; every scalar type and arrays parse."""
    from gguf_writer import ARRAY, BOOL, F64, I8, I16, I64, U8, U16, U64
    b = GgufBuilder(alignment=64)
    b.add_kv("general.alignment", U32, 64)
    for k, t, v in [("a.u8", U8, 200), ("a.i8", I8, -5), ("a.u16", U16, 60000), ("a.i16", I16, -30000),
                    ("a.u64", U64, 1 << 40), ("a.i64", I64, -(1 << 40)), ("a.b", BOOL, 1), ("a.f64", F64, 0.25)]:
        b.add_kv(k, t, v)
    b.add_kv("tokenizer.ggml.tokens", ARRAY, (STRING, ["a", "bb", "ccc"]))
    b.add_tensor("x", (5,), "F32", np.arange(5, dtype=np.float32))
    f = gg(b.write(tmp_path / "a.gguf"))
    assert f.get_int("a.u8") == 200 and f.get_int("a.i8") == -5 and f.get_int("a.u16") == 60000
    assert f.get_int("a.i16") == -30000 and f.get_int("a.u64") == 1 << 40 and f.get_int("a.i64") == -(1 << 40)
    assert f.get_int("a.b") == 1 and f.get_float("a.f64") == 0.25
    assert f.get_array_len("tokenizer.ggml.tokens") == 3
    assert f.tensors[0].data().view(np.float32).tolist() == [0, 1, 2, 3, 4]


def test_gguf_errors(tmp_path, gg):
    from beacon_cuda import EngineError, ShapeMismatch
    from beacon_cuda import _lib as L
    good = open(reference_test_file(tmp_path / "t.gguf"), "rb").read()
    bad_magic = tmp_path / "m.gguf"
    bad_magic.write_bytes(b"GGML" + good[4:])
    with pytest.raises(EngineError) as e:
        gg(str(bad_magic))
    assert e.value.status == L.ERR_INVALID_ARGUMENT
    v2 = tmp_path / "v.gguf"
    v2.write_bytes(good[:4] + (2).to_bytes(4, "little") + good[8:])
    with pytest.raises(EngineError) as e:
        gg(str(v2))
    assert e.value.status == L.ERR_UNSUPPORTED_DTYPE
    with pytest.raises(ShapeMismatch):                 # truncated: data beyond the end of the file
        (tmp_path / "tr.gguf").write_bytes(good[:-8])
        gg(str(tmp_path / "tr.gguf"))
    with pytest.raises(ShapeMismatch):                 # truncated inside the metadata
        (tmp_path / "tm.gguf").write_bytes(good[:40])
        gg(str(tmp_path / "tm.gguf"))
    with pytest.raises(EngineError):
        gg(str(tmp_path / "missing.gguf"))
