"""The safetensors reader (crates/graph/src/checkpoint.rs:1-191, its tests :193-): tensors read a
tensor at a time as their storage gives them, gathers of rows, joins along rows, and refusals."""

import struct

import numpy as np
import pytest

import __graft_entry__ as entry

entry.load_package()
from tgtts_v4_b200 import checkpoint  # noqa: E402
from tgtts_v4_b200 import synthetic as syn  # noqa: E402


def test_tensors_come_back_as_stored(tmp_path):
    rng = np.random.default_rng(0)
    f32 = rng.standard_normal((3, 5), dtype=np.float32)
    f16 = rng.standard_normal((4,)).astype(np.float16)
    bf = syn.bf16_bits(rng.standard_normal((2, 8), dtype=np.float32))
    path = tmp_path / "w.safetensors"
    checkpoint.save(path, {"a.f32": f32, "b.f16": f16, "c.bf16": bf})
    with checkpoint.Checkpoint(path) as ck:
        assert ck.names() == ["a.f32", "b.f16", "c.bf16"]
        assert ck.shape("c.bf16") == [2, 8] and ck.shape("nope") is None
        np.testing.assert_array_equal(ck.tensor("a.f32"), f32)
        np.testing.assert_array_equal(ck.tensor("b.f16"), f16.astype(np.float32))
        got = ck.tensor("c.bf16")
        assert got.dtype == np.uint16
        np.testing.assert_array_equal(got, bf)


def test_a_gather_reads_the_rows_the_whole_tensor_holds(tmp_path):
    # Quarters, which bfloat16 holds exactly (checkpoint.rs's own test).
    rows = (np.arange(12, dtype=np.float32) / 4 - 1.5).reshape(4, 3)
    path = tmp_path / "g.safetensors"
    checkpoint.save(path, {"emb": syn.bf16_bits(rows)})
    with checkpoint.Checkpoint(path) as ck:
        whole = syn.bf16_to_f32(ck.tensor("emb"))
        np.testing.assert_array_equal(whole, rows)
        got = syn.bf16_to_f32(ck.gather("emb", [3, 0, 3]))
        np.testing.assert_array_equal(got, rows[[3, 0, 3]])
        with pytest.raises(checkpoint.CheckpointError):
            ck.gather("emb", [4])


def test_rows_join_and_refusals(tmp_path):
    a = np.ones((2, 4), np.float32)
    b = np.full((3, 4), 2.0, np.float32)
    c = np.zeros((1, 5), np.float32)
    path = tmp_path / "r.safetensors"
    checkpoint.save(path, {"a": a, "b": b, "c": c})
    with checkpoint.Checkpoint(path) as ck:
        j = ck.rows(["a", "b"])
        assert j.shape == (5, 4) and np.all(j[:2] == 1) and np.all(j[2:] == 2)
        with pytest.raises(checkpoint.CheckpointError):
            ck.rows(["a", "c"])
        with pytest.raises(checkpoint.CheckpointError):
            ck.tensor("missing")
    # A header that claims more bytes than the tensor's shape, and an unknown dtype.
    for dtype, shape, offs in (("F32", [2, 2], [0, 12]), ("I8", [4], [0, 4])):
        h = ('{"t": {"dtype": "%s", "shape": %s, "data_offsets": %s}}' % (dtype, shape, offs)).encode()
        bad = tmp_path / f"bad_{dtype}.safetensors"
        bad.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 16)
        with checkpoint.Checkpoint(bad) as ck, pytest.raises(checkpoint.CheckpointError):
            ck.tensor("t")
    huge = tmp_path / "huge.safetensors"
    huge.write_bytes(struct.pack("<Q", 200 << 20))
    with pytest.raises(checkpoint.CheckpointError):
        checkpoint.Checkpoint(huge)
