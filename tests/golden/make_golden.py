"""Writes the fixtures under tests/golden/.

reference_testkit.json: the values tgtts-v4's own testkit fixture holds
(crates/testkit/tests/fixtures/testkit.safetensors, made by fixtures/testkit.py from upstream
VoxCPM's `rms_layernorm` and torch's roundings), read from the reference tree when it is present:

- "rms_layernorm": upstream's rms_layernorm([[3, 4]], [1, 2], eps=0), which
  crates/testkit/tests/testkit.rs:57-68 checks against [3/sqrt(12.5), 8/sqrt(12.5)];
- "bf16": the bf16 bytes torch stores for [1.0, -2.5, 0.1, 3.14159] (testkit.rs:45-55), the
  round-to-nearest-even the synthetic bf16 weights must follow.

oracle_tiny.npz: the CPU oracle's own outputs for BASELINE config 1 (seeded weights and inputs,
32-position prefill then 16 decode steps feeding back), so that a change to the oracle shows. These
are not from the reference: tgtts-v4 keeps no backbone goldens in its tree.

Run: python tests/golden/make_golden.py [path to the reference tree]
"""

import json
import struct
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def read_safetensors(path: Path) -> dict:
    raw = path.read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])
    body = raw[8 + n:]
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        a, b = info["data_offsets"]
        out[name] = (info["dtype"], info["shape"], body[a:b])
    return out


def reference_fixture(reference: Path) -> None:
    path = reference / "crates/testkit/tests/fixtures/testkit.safetensors"
    t = read_safetensors(path)
    dtype, shape, data = t["rms_layernorm"]
    assert dtype == "F32"
    rms = np.frombuffer(data, np.float32).reshape(shape)
    dtype, shape, data = t["bf16"]
    assert dtype == "BF16"
    fixture = {
        "source": "crates/testkit/tests/fixtures/testkit.safetensors (fixtures/testkit.py)",
        "rms_layernorm": {"x": [[3.0, 4.0]], "g": [1.0, 2.0], "eps": 0.0,
                          "out": rms.tolist(), "out_bits": rms.view(np.uint32).tolist()},
        "bf16": {"values": [1.0, -2.5, 0.1, 3.14159], "bytes": list(data)},
    }
    (HERE / "reference_testkit.json").write_text(json.dumps(fixture, indent=1) + "\n")


def oracle_tiny() -> None:
    sys.path.insert(0, str(ROOT))
    import __graft_entry__ as entry
    import oracle

    entry.load_package()
    from tgtts_v4_b200 import synthetic as syn

    cfg = syn.TINY
    shape = syn.shape_of(cfg, capacity=64)
    w = syn.make_weights(cfg, seed=0)
    stack = oracle.OracleStack(shape, w, slots=1, threads=4)
    x = syn.make_inputs(32, cfg.hidden, seed=1)
    pre = stack.prefill(0, x)
    h = pre[-1]
    steps = []
    for t in range(16):
        h = stack.decode_step([(32 + t, 0)], h[None])[0]
        steps.append(h)
    np.savez_compressed(HERE / "oracle_tiny.npz", prefill=pre, decode=np.stack(steps))


if __name__ == "__main__":
    # The reference's checkout, when given (its testkit fixture is read from it); the oracle's own
    # golden is written either way.
    ref = Path(sys.argv[1]) if len(sys.argv) > 1 else None
    if ref is not None and ref.exists():
        reference_fixture(ref)
    oracle_tiny()
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".json", ".npz")))
