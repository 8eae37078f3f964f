"""The C-ABI library: it loads, it exports every entry point include/tgcuda.h declares, and its
host logic (shape byte model, placements, RoPE tables, config checks) holds tgtts-v4's known
answers. Nothing here launches a kernel."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import oracle

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "tgcuda.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(tg_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_entry_point(pkg):
    lib = pkg.library()
    names = declared_functions()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # The Python layer types every one of them, and nothing it types is undeclared.
    assert sorted(pkg.SIGNATURES) == names
    assert lib.tg_abi_version() == 1


def test_without_a_gpu_a_context_fails_loudly(pkg):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(pkg.NoDeviceError):
        pkg.Context(0)


def test_weight_bytes_of_the_base_lm(pkg):
    # crates/graph/src/decode.rs:946-947: VoxCPM2's base LM, 28 layers of (2048, 6144, 16, 2, 128)
    # in f16, reads 2,642,644,992 bytes of weights a step.
    s = pkg.Shape(hidden=2048, inner=6144, heads=16, kv_heads=2, head_dim=128, layers=28, capacity=1024)
    assert s.weight_bytes(2) == 2_642_644_992
    # The 0.5B-shaped backbone: 24 x 14,942,208 projection weights plus gains, in bf16.
    s5 = pkg.Shape(hidden=1024, inner=4096, heads=16, kv_heads=2, head_dim=64, layers=24, capacity=2048)
    assert s5.weight_bytes(2) == 2 * (24 * (14_942_208 + 2 * 1024) + 1024)
    # Keys and values read at position p (decode.rs:137-141): 2 x kv x hd x 2 bytes per position
    # and layer, over positions 0 .. p in whole chunks of 32, at most the capacity.
    per = 24 * 2 * 2 * 64 * 2
    assert s5.cache_bytes(639, 2) == per * 640
    assert s5.cache_bytes(512, 2) == per * 544
    assert s5.cache_bytes(2047, 2) == per * 2048
    assert pkg.Shape(hidden=1024, inner=4096, heads=16, kv_heads=2, head_dim=64, layers=24,
                     capacity=160).cache_bytes(150, 2) == per * 160


def test_placement_words_and_refusals(pkg):
    # crates/graph/src/decode.rs:1073-1092.
    batch = pkg.Batch(rows=3, slots=4)
    at = lambda p, s: pkg.Row(p, s)  # noqa: E731
    assert batch.placement([at(5, 2), None, at(0, 0)], 64) == [5, 0xFFFFFFFF, 0, 2, 0xFFFFFFFF, 0]
    assert pkg.Batch.ONE.placement([at(7, 0)], 64) == [7]
    for rows in ([at(5, 2), at(9, 2), None], [at(64, 0), None, None], [at(1, 4), None, None]):
        with pytest.raises(pkg.ShapeError):
            batch.placement(rows, 64)
    with pytest.raises(pkg.ShapeError):
        batch.placement([None, None], 64)


def test_rope_tables_are_the_oracles_bit_for_bit(pkg):
    s = pkg.Shape(hidden=1024, inner=4096, heads=16, kv_heads=2, head_dim=64, layers=1, capacity=256)
    cos, sin = s.rope_tables()
    oc, os_ = oracle.rope_tables(64, 256, 10000.0)
    assert np.array_equal(cos, oc) and np.array_equal(sin, os_)
    # decode.rs:1232-1242.
    assert np.all(cos[0] == 1) and np.all(sin[0] == 0)
    assert cos[1, 0] == np.float32(np.cos(1.0)) and sin[1, 0] == np.float32(np.sin(1.0))
    f = pkg.Shape(hidden=32, inner=48, heads=4, kv_heads=2, head_dim=8, layers=1, capacity=64,
                  rope_factors=[0.99, 1.6, 3.4, 8.9])
    fc, fs = f.rope_tables()
    oc, os_ = oracle.rope_tables(8, 64, 10000.0, [0.99, 1.6, 3.4, 8.9])
    assert np.array_equal(fc, oc) and np.array_equal(fs, os_)


def _config(pkg, **kw):
    d = dict(hidden_size=2048, intermediate_size=6144, num_attention_heads=16, num_key_value_heads=2,
             num_hidden_layers=28, rms_norm_eps=1e-5, rope_theta=10000, kv_channels=128,
             max_position_embeddings=32768,
             rope_scaling={"type": "longrope", "short_factor": [1.0] * 64,
                           "original_max_position_embeddings": 32768},
             use_mup=False)
    d.update(kw)
    return pkg.LmConfig.from_dict(d)


def test_shape_new_refuses_what_voxcpm2_does_not_use(pkg):
    # crates/graph/src/decode.rs:84-126 and :1030-1071.
    s = pkg.Shape.new(_config(pkg), 8, 64)
    assert (s.hidden, s.head_dim, s.layers, s.capacity, s.rope) == (2048, 128, 8, 64, True)
    with pytest.raises(pkg.ShapeError):
        pkg.Shape.new(_config(pkg, use_mup=True), 8, 64)
    dynamic = {"type": "dynamic", "short_factor": [1.0] * 64, "original_max_position_embeddings": 32768}
    with pytest.raises(pkg.ShapeError):
        pkg.Shape.new(_config(pkg, rope_scaling=dynamic), 8, 64)
    # Refused only where it would be used: a stack without RoPE takes it.
    assert not pkg.Shape.new(_config(pkg, rope_scaling=dynamic, no_rope=True), 8, 64).rope
    with pytest.raises(pkg.ShapeError):
        pkg.Shape.new(_config(pkg), 29, 64)
    with pytest.raises(pkg.ShapeError):
        pkg.Shape.new(_config(pkg), 8, 40000)
    # A config without use_mup is taken as upstream takes it: with muP, refused.
    d = _config(pkg).__dict__.copy()
    del d["use_mup"]
    with pytest.raises(pkg.ShapeError):
        pkg.Shape.new(pkg.LmConfig.from_dict(d), 8, 64)


def test_synthetic_weights_are_seeded_and_bf16_valued(syn):
    a = syn.make_weights(syn.TINY, seed=0, layers=1)
    b = syn.make_weights(syn.TINY, seed=0, layers=1)
    assert all(np.array_equal(a[k], b[k]) for k in a)
    w = syn.make_weights(syn.S05B, seed=0, layers=1)
    q = w["layers.0.self_attn.q_proj.weight"]
    assert q.shape == (1024, 1024) and np.array_equal(q, syn.bf16_round(q))
    assert abs(float(q.std()) - 0.02) < 1e-3
    assert np.all(w["norm.weight"] == 1)


def test_the_ctypes_structs_match_the_c_header(pkg, tmp_path):
    """Every struct the Python binding mirrors has the C header's size and field offsets (gcc on
    include/tgcuda.h), so that a params field added on one side cannot go unnoticed."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    structs = {"tg_params": pkg.TgParams, "tg_shape": pkg.TgShape, "tg_row": pkg.TgRow, "tg_run": pkg.TgRun,
               "tg_request": pkg.TgRequest, "tg_binding": pkg.TgBinding, "tg_dispatch": pkg.TgDispatch,
               "tg_region": pkg.TgRegion, "tg_local_tuning": pkg.TgLocalTuning}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "tgcuda.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    root = Path(__file__).resolve().parent.parent
    subprocess.run(["gcc", "-std=c11", "-I", str(root / "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {}
    for line in out:
        if line:
            cname, field, value = line.split()
            got[(cname, field)] = int(value)
    for cname, py in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for field, _ in py._fields_:
            assert got[(cname, field)] == getattr(py, field).offset, (cname, field)


def test_the_per_step_calls_marshal_their_arrays_without_a_gpu(pkg, syn):
    """Decoder.step_rows, step_rows_n, set_rows and output pass their arrays as addresses: with no
    decoder behind them the library refuses the call (InvalidError) before it reads any of them,
    which shows the arguments reach it as the header declares them."""
    dec = object.__new__(pkg.Decoder)
    dec.handle = None
    dec.batch = pkg.Batch(2, 2)
    dec.shape = syn.shape_of(syn.TINY, capacity=64)
    x = np.zeros((2, dec.shape.hidden), np.float32)
    rows = [pkg.Row(3, 0), None]
    for call in (lambda: dec.step_rows(rows, x), lambda: dec.step_rows_n(rows[:1], x[:1]),
                 lambda: dec.set_rows(rows, x), lambda: dec.output()):
        with pytest.raises(pkg.InvalidError, match="null"):
            call()


def test_the_no_alloc_attention_refuses_bad_shapes_before_touching_a_device(pkg):
    """tg_attention_decode_noalloc checks its shape before any CUDA call, so on a machine without a
    GPU a shape it cannot run comes back as TG_ESHAPE (no heads, heads not a multiple of the KV
    heads, an unsupported head width) and never reaches a device. The pointers are 16-byte
    aligned stand-ins that nothing dereferences."""
    shape = pkg.Shape(hidden=1024, inner=4096, heads=16, kv_heads=2, head_dim=64, layers=1, capacity=256)
    fake = 0x10000
    for field, value in (("heads", 0), ("heads", 15), ("head_dim", 96), ("rows", 0), ("kv_heads", 0)):
        p = pkg.params(shape, "bf16", rows=4, slots=4)
        setattr(p, field, value)
        with pytest.raises(pkg.ShapeError):
            pkg.attention_decode_noalloc(p, fake, fake, fake, fake, fake, 0)
