"""tgtts-v4_b200: the B200 (sm_100a) runtime for the MiniCPM-4 stack that tgtts-v4's `graph` crate
drives, from Python.

A thin ctypes layer over `lib/libtgcuda.so` (declared in `include/tgcuda.h`), named after the
graph crate's types so that code and tests read like the crate's own:

- `LmConfig` / `Shape.new` (crates/graph/src/decode.rs:30-126), `Shape.weight_bytes`,
  `Shape.rope_tables` (decode.rs:127-168);
- `Batch`, `Row`, `Batch.placement` (decode.rs:171-235);
- `Decoder` (decode.rs:778-913): `with_batch`, `load`, `step`, `step_rows`, `set_rows`, `start`,
  `wait`, `output`, `timings`, plus the KV-cache reads and slot copies the prompt cache uses;
- `Prefill` (prefill.rs:415-504): `run`, `max_rows`, and `run_batch` for several prompts at once.

Errors mirror `graph::Error`: a `ShapeError` for shapes and placements the kernels cannot run,
raised before anything is launched. There is no CPU path: without the built library or a B200,
constructing a `Context` raises.
"""

from __future__ import annotations

import ctypes
import json
import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Iterable, Mapping, Optional, Sequence

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "lib" / "libtgcuda.so"

SPARE = 0xFFFFFFFF
# The positions attention_split takes per block, fixed in the kernels (decode.rs:26 has 32 for
# the Vulkan kernels; these take 64).
CHUNK = 64

# ---- errors (crates/graph/src/lib.rs:41-59) ---------------------------------------------------


class Error(Exception):
    """A failure of the runtime, with its status code."""

    status = -1

    def __init__(self, message: str, status: Optional[int] = None):
        super().__init__(message)
        if status is not None:
            self.status = status


class InvalidError(Error):
    status = 1


class ShapeError(Error):
    status = 2


class CudaError(Error):
    status = 3


class OutOfMemoryError(Error):
    status = 4


class TimeoutError(Error):  # noqa: A001 - the runtime's own timeout, as vulkan::Error names it
    status = 5


class NotFiniteError(Error):
    status = 6


class KernelError(Error):
    status = 7


class NoDeviceError(Error):
    status = 8


_ERRORS = {c.status: c for c in (InvalidError, ShapeError, CudaError, OutOfMemoryError,
                                  TimeoutError, NotFiniteError, KernelError, NoDeviceError)}

# ---- the library ---------------------------------------------------------------------------------

F32, BF16, F16 = 0, 1, 2
DTYPES = {"f32": F32, "fp32": F32, "float32": F32, "bf16": BF16, "bfloat16": BF16, "f16": F16,
          "float16": F16}
RES_DEVICE, RES_UPLOAD, RES_READBACK = 0, 1, 2

KERNELS = {
    "rmsnorm": 0, "gemv_qkv_rope": 1, "attention_split": 2, "attention_combine": 3,
    "gemv_residual": 4, "gemv_gate_up": 5, "stream_read": 6, "norm_rows": 7, "add_norm_rows": 8,
    "rope_rows": 9, "attention_rows": 10, "silu_mul_rows": 11, "gemm": 12,
    "gemm_silu": 14, "attention_rows_tc": 15, "gemm_qkv_rope": 16, "gemv_linear": 17,
    "local_norm": 18, "local_partial": 19, "local_gate_up": 20, "local_attention": 21,
    "local_add_norm": 22, "local_rows": 23, "local_embed": 24, "cfm_noise": 25, "dit_euler": 26,
}


class TgShape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in
                ("hidden", "inner", "heads", "kv_heads", "head_dim", "layers", "capacity")] + [
        ("eps", ctypes.c_float), ("rope_theta", ctypes.c_float), ("residual_scale", ctypes.c_float),
        ("rope", ctypes.c_uint32), ("rope_factors", ctypes.POINTER(ctypes.c_double))]


class TgRow(ctypes.Structure):
    _fields_ = [("position", ctypes.c_uint32), ("slot", ctypes.c_uint32)]


class TgRun(ctypes.Structure):
    _fields_ = [("start", ctypes.c_uint32), ("len", ctypes.c_uint32), ("slot", ctypes.c_uint32)]


class TgRequest(ctypes.Structure):
    _fields_ = [("slot", ctypes.c_uint32), ("len", ctypes.c_uint32), ("steps", ctypes.c_uint32),
                ("start", ctypes.c_uint32)]


class TgParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in
                ("dtype", "hidden", "inner", "heads", "kv_heads", "head_dim", "capacity", "rows",
                 "slots")] + [("eps", ctypes.c_float), ("residual_scale", ctypes.c_float)] + [
        (n, ctypes.c_uint32) for n in ("rope", "normed_f32", "m", "n", "k", "k1", "offset", "stride",
                                       "act")] + [("levels", ctypes.c_float)] + [
        (n, ctypes.c_uint32) for n in ("parts", "seqs", "first", "at", "copied", "flags", "frames",
                                       "feat")] + [("dt", ctypes.c_float)]


class TgLocalTuning(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in ("qkv_parts", "o_parts", "down_parts")]


class TgBinding(ctypes.Structure):
    _fields_ = [("mem", ctypes.c_void_p), ("offset", ctypes.c_uint64), ("bytes", ctypes.c_uint64)]


class TgDispatch(ctypes.Structure):
    _fields_ = [("kernel", ctypes.c_uint32), ("params", ctypes.POINTER(TgParams)),
                ("bindings", ctypes.POINTER(TgBinding)), ("n_bindings", ctypes.c_uint32),
                ("label", ctypes.c_char_p)]


class TgRegion(ctypes.Structure):
    _fields_ = [("src_offset", ctypes.c_uint64), ("dst_offset", ctypes.c_uint64),
                ("bytes", ctypes.c_uint64)]


# Every entry point include/tgcuda.h declares: name -> (restype, argtypes).
_P, _U32, _U64, _I, _SZ = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_size_t
_FP, _DP = ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_double)
SIGNATURES = {
    "tg_last_error": (ctypes.c_char_p, []),
    "tg_abi_version": (_U32, []),
    "tg_ctx_create": (_I, [_I, ctypes.POINTER(_P)]),
    "tg_ctx_destroy": (_I, [_P]),
    "tg_ctx_synchronize": (_I, [_P, _U64]),
    "tg_ctx_info": (_I, [_P, ctypes.c_char_p, _SZ, ctypes.POINTER(_I)]),
    "tg_ctx_stream": (_P, [_P]),
    "tg_ctx_selftest_wait": (_I, [_P, _U64]),
    "tg_mem_alloc": (_I, [_P, _U64, _I, ctypes.POINTER(_P)]),
    "tg_mem_free": (_I, [_P]),
    "tg_mem_size": (_U64, [_P]),
    "tg_mem_device_ptr": (_P, [_P]),
    "tg_mem_write": (_I, [_P, _U64, _P, _U64]),
    "tg_mem_read": (_I, [_P, _U64, _P, _U64]),
    "tg_mem_fill": (_I, [_P, _U64, _U32, _U64]),
    "tg_copy_regions": (_I, [_P, _P, _P, ctypes.POINTER(TgRegion), _SZ]),
    "tg_dispatch_once": (_I, [_P, ctypes.POINTER(TgDispatch), _DP]),
    "tg_program_create": (_I, [_P, ctypes.POINTER(TgDispatch), _SZ, _I, ctypes.POINTER(_P)]),
    "tg_program_destroy": (_I, [_P]),
    "tg_program_start": (_I, [_P]),
    "tg_program_wait": (_I, [_P, _U64]),
    "tg_program_elapsed_ns": (_I, [_P, _DP]),
    "tg_program_timings": (_I, [_P, _DP, _SZ]),
    "tg_shape_weight_bytes": (_U64, [ctypes.POINTER(TgShape), _U32]),
    "tg_shape_cache_bytes": (_U64, [ctypes.POINTER(TgShape), _U32, _U32]),
    "tg_shape_rope_tables": (_I, [ctypes.POINTER(TgShape), _FP, _FP]),
    "tg_batch_placement": (_I, [_U32, _U32, ctypes.POINTER(TgRow), _U32,
                                ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32)]),
    "tg_decoder_create": (_I, [_P, ctypes.POINTER(TgShape), _U32, _U32, _I, _I, ctypes.POINTER(_P)]),
    "tg_decoder_destroy": (_I, [_P]),
    "tg_decoder_load": (_I, [_P, ctypes.c_char_p, _P, _U64, _I]),
    # The per-step entry points take their host arrays as addresses (c_void_p from an int), which
    # costs the caller less per call than a typed pointer object.
    "tg_decoder_step_rows": (_I, [_P, ctypes.POINTER(TgRow), _P, _P]),
    "tg_decoder_set_rows": (_I, [_P, ctypes.POINTER(TgRow), _P]),
    "tg_decoder_set_rows_n": (_I, [_P, _U32, ctypes.POINTER(TgRow), _P]),
    "tg_decoder_step_rows_n": (_I, [_P, _U32, ctypes.POINTER(TgRow), _P, _P]),
    "tg_decoder_start": (_I, [_P]),
    "tg_decoder_wait": (_I, [_P, _U64]),
    "tg_decoder_output": (_I, [_P, _P]),
    "tg_decoder_step_device": (_I, [_P, ctypes.POINTER(ctypes.c_uint32), _P, _P]),
    "tg_decoder_elapsed_ns": (_I, [_P, _DP]),
    "tg_decoder_timings": (_I, [_P, _DP, _SZ, ctypes.POINTER(_SZ)]),
    "tg_decoder_dispatch_label": (_I, [_P, _SZ, ctypes.c_char_p, _SZ]),
    "tg_decoder_read_cache": (_I, [_P, _U32, _U32, _U32, _U32, _U32, _FP]),
    "tg_decoder_copy_slot": (_I, [_P, _U32, _U32, _U32]),
    "tg_decoder_prefix_bytes": (_U64, [_P, _U32]),
    "tg_decoder_copy_out": (_I, [_P, _U32, _U32, _P, _U64]),
    "tg_decoder_copy_in": (_I, [_P, _U32, _U32, _P, _U64]),
    "tg_decoder_weight_bytes": (_U64, [_P]),
    "tg_decoder_retune": (_I, [_P, _I, _I]),
    "tg_decoder_persistent": (_I, [_P]),
    "tg_decoder_tensor": (_I, [_P]),
    "tg_decoder_set_tensor": (_I, [_P, _I]),
    "tg_prefill_create": (_I, [_P, _U32, _I, ctypes.POINTER(_P)]),
    "tg_prefill_destroy": (_I, [_P]),
    "tg_prefill_run": (_I, [_P, _U32, _U32, _FP, _U32, _FP]),
    "tg_prefill_run_batch": (_I, [_P, ctypes.POINTER(TgRun), _U32, _FP, _FP]),
    "tg_prefill_run_batch_device": (_I, [_P, ctypes.POINTER(TgRun), _U32, _P, _P]),
    "tg_prefill_elapsed_ns": (_I, [_P, _DP]),
    "tg_prefill_timings": (_I, [_P, _DP, _SZ, ctypes.POINTER(_SZ)]),
    "tg_prefill_dispatch_label": (_I, [_P, _SZ, ctypes.c_char_p, _SZ]),
    "tg_prefill_max_rows": (_U32, [_P]),
    "tg_attention_decode_noalloc": (_I, [ctypes.POINTER(TgParams), _P, _P, _P, _P, _P, _P]),
    "tg_server_create": (_I, [_P, _P, ctypes.POINTER(_P)]),
    "tg_server_destroy": (_I, [_P]),
    "tg_server_start": (_I, [_P, ctypes.POINTER(TgRequest), _U32, _FP]),
    "tg_server_step": (_I, [_P, _FP, ctypes.POINTER(_U32), ctypes.POINTER(_U32), _FP]),
    "tg_server_under_way": (_I, [_P, ctypes.POINTER(_U32), ctypes.POINTER(_U32)]),
    "tg_server_request": (_I, [_P, _U32, ctypes.POINTER(_U32), ctypes.POINTER(_U32), ctypes.POINTER(_U32)]),
    "tg_server_finish": (_I, [_P, _U32]),
    "tg_server_last_output": (_I, [_P, _U32, _FP]),
    "tg_server_sync": (_I, [_P, _U64]),
    "tg_sampler_create": (_I, [_P, ctypes.POINTER(TgShape), _U32, _U32, _U32, _U32,
                               ctypes.POINTER(TgLocalTuning), _I, ctypes.POINTER(_P)]),
    "tg_sampler_destroy": (_I, [_P]),
    "tg_sampler_load": (_I, [_P, ctypes.c_char_p, _P, _U64, _I]),
    "tg_sampler_sample": (_I, [_P, _P, _FP, _FP, _FP, _FP]),
    "tg_sampler_sample_device": (_I, [_P, _P, _P, _P, _P, _P]),
    "tg_sampler_wait": (_I, [_P, _U64]),
    "tg_sampler_steps": (_I, [_P, _FP, _FP, _SZ, ctypes.POINTER(_SZ)]),
    "tg_sampler_elapsed_ns": (_I, [_P, _DP]),
    "tg_sampler_timings": (_I, [_P, _DP, _SZ, ctypes.POINTER(_SZ)]),
    "tg_sampler_dispatch_label": (_I, [_P, _SZ, ctypes.c_char_p, _SZ]),
    "tg_sampler_weight_bytes": (_U64, [_P]),
    "tg_cfm_schedule": (_I, [_U32, _FP]),
    "tg_cfm_euler_steps": (_I, [_U32, _FP, _FP, _SZ, ctypes.POINTER(_SZ)]),
    "tg_encoder_create": (_I, [_P, ctypes.POINTER(TgShape), _U32, _U32, _U32,
                               ctypes.POINTER(TgLocalTuning), _I, ctypes.POINTER(_P)]),
    "tg_encoder_destroy": (_I, [_P]),
    "tg_encoder_load": (_I, [_P, ctypes.c_char_p, _P, _U64, _I]),
    "tg_encoder_encode": (_I, [_P, _FP, _P]),
    "tg_encoder_encode_device": (_I, [_P, _P, _P]),
    "tg_encoder_wait": (_I, [_P, _U64]),
    "tg_encoder_elapsed_ns": (_I, [_P, _DP]),
    "tg_encoder_timings": (_I, [_P, _DP, _SZ, ctypes.POINTER(_SZ)]),
    "tg_encoder_dispatch_label": (_I, [_P, _SZ, ctypes.c_char_p, _SZ]),
    "tg_encoder_weight_bytes": (_U64, [_P]),
}

_lib: Optional[ctypes.CDLL] = None


def library() -> ctypes.CDLL:
    """The loaded libtgcuda.so with every entry point typed. Raises when it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise Error(f"{LIB_PATH} is not built: run __graft_entry__.build() (nvcc, sm_100a)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int) -> None:
    """Raises the error a status names, with the library's message."""
    if status != 0:
        msg = library().tg_last_error().decode(errors="replace")
        raise _ERRORS.get(status, Error)(msg, status)


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(_FP)


# ---- config and shape (crates/graph/src/decode.rs:30-168) ---------------------------------------


@dataclass
class LmConfig:
    """What a step reads of VoxCPM2's `lm_config` (decode.rs:30-63)."""

    hidden_size: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    num_hidden_layers: int
    rms_norm_eps: float
    rope_theta: float
    max_position_embeddings: int
    rope_scaling: Mapping
    kv_channels: Optional[int] = None
    use_mup: bool = True  # as upstream assumes when it is missing (decode.rs:55-57)
    no_rope: bool = False
    # The residual branch scale BASELINE's configs use (scale_depth / sqrt(layers)); 1.0 is
    # tgtts-v4's. Not a field of upstream's config.
    residual_scale: float = 1.0

    @classmethod
    def from_dict(cls, d: Mapping) -> "LmConfig":
        keys = {f for f in cls.__dataclass_fields__}
        return cls(**{k: v for k, v in d.items() if k in keys})

    @classmethod
    def from_json(cls, text: str) -> "LmConfig":
        return cls.from_dict(json.loads(text))


@dataclass
class Shape:
    """The shapes a step is recorded at (decode.rs:66-83), plus the residual scale."""

    hidden: int
    inner: int
    heads: int
    kv_heads: int
    head_dim: int
    layers: int
    capacity: int
    eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_factors: Optional[Sequence[float]] = None
    rope: bool = True
    residual_scale: float = 1.0

    @staticmethod
    def new(config: LmConfig, layers: int, capacity: int) -> "Shape":
        """Shape::new (decode.rs:84-126): refuses what VoxCPM2 does not use."""
        if config.use_mup:
            raise ShapeError("use_mup")
        rope = config.rope_scaling
        kind = rope.get("type")
        if not config.no_rope and (
                kind != "longrope"
                or config.max_position_embeddings != rope.get("original_max_position_embeddings")):
            raise ShapeError(
                f"rope_scaling {kind!r} from {rope.get('original_max_position_embeddings')} "
                f"positions to {config.max_position_embeddings}")
        if layers > config.num_hidden_layers:
            raise ShapeError(f"{layers} of {config.num_hidden_layers} layers")
        if capacity > config.max_position_embeddings:
            raise ShapeError(
                f"a cache of {capacity} past {config.max_position_embeddings} positions")
        head_dim = config.kv_channels or config.hidden_size // config.num_attention_heads
        return Shape(hidden=config.hidden_size, inner=config.intermediate_size,
                     heads=config.num_attention_heads, kv_heads=config.num_key_value_heads,
                     head_dim=head_dim, layers=layers, capacity=capacity,
                     eps=float(np.float32(config.rms_norm_eps)),
                     rope_theta=float(np.float32(config.rope_theta)),
                     rope_factors=list(rope.get("short_factor", [])) or None,
                     rope=not config.no_rope, residual_scale=config.residual_scale)

    def _c(self):
        s = TgShape(self.hidden, self.inner, self.heads, self.kv_heads, self.head_dim, self.layers,
                    self.capacity, self.eps, self.rope_theta, self.residual_scale, int(self.rope),
                    None)
        keep = None
        if self.rope_factors is not None:
            if len(self.rope_factors) != self.head_dim // 2:
                raise ShapeError(f"{len(self.rope_factors)} rope factors for head_dim {self.head_dim}")
            keep = (ctypes.c_double * len(self.rope_factors))(*self.rope_factors)
            s.rope_factors = ctypes.cast(keep, _DP)
        return s, keep

    @property
    def qkv_rows(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    def weight_bytes(self, bytes_per_weight: int = 2) -> int:
        """Shape::weight_bytes (decode.rs:127-133), at `bytes_per_weight` per value."""
        s, _keep = self._c()
        return int(library().tg_shape_weight_bytes(ctypes.byref(s), bytes_per_weight))

    def cache_bytes(self, position: int, bytes_per_value: int = 2) -> int:
        """The bytes of keys and values a step at `position` reads over every layer."""
        s, _keep = self._c()
        return int(library().tg_shape_cache_bytes(ctypes.byref(s), position, bytes_per_value))

    def rope_tables(self) -> tuple[np.ndarray, np.ndarray]:
        """Shape::rope_tables (decode.rs:143-168): cos, sin, [capacity][head_dim / 2] f32."""
        s, _keep = self._c()
        cos = np.zeros((self.capacity, self.head_dim // 2), np.float32)
        sin = np.zeros_like(cos)
        check(library().tg_shape_rope_tables(ctypes.byref(s), _fptr(cos), _fptr(sin)))
        return cos, sin


# ---- batches (decode.rs:171-235) ------------------------------------------------------------------


@dataclass(frozen=True)
class Row:
    """Where a row of a batch runs: at a position of its request's cache slot."""

    position: int
    slot: int = 0


@dataclass(frozen=True)
class Batch:
    """How many requests a step runs at once, and the slots of the KV cache they are kept in."""

    rows: int
    slots: int

    def words(self) -> int:
        return 2 * self.rows if self.slots > 1 else self.rows

    def placement(self, rows: Sequence[Optional[Row]], capacity: int) -> list[int]:
        """Batch::placement (decode.rs:198-227): each row's position, then its slot when there is
        more than one; a spare row (None) gets u32::MAX. Refuses two rows in one slot."""
        if len(rows) != self.rows:
            raise ShapeError(f"{len(rows)} rows for a batch of {self.rows}")
        c_rows = _rows(rows)
        words = (ctypes.c_uint32 * (2 * self.rows))()
        n = ctypes.c_uint32()
        check(library().tg_batch_placement(self.rows, self.slots, c_rows, capacity, words,
                                           ctypes.byref(n)))
        return list(words[: n.value])


Batch.ONE = Batch(1, 1)  # type: ignore[attr-defined]


def _rows(rows: Sequence[Optional[Row]]):
    arr = (TgRow * len(rows))()
    for i, r in enumerate(rows):
        arr[i] = TgRow(SPARE, 0) if r is None else TgRow(r.position, r.slot)
    return arr


# ---- context ---------------------------------------------------------------------------------------


class Context:
    """A CUDA device with its own stream (vulkan::Context, crates/vulkan/src/context.rs:198-240)."""

    def __init__(self, device: int = 0):
        self._lib = library()
        h = ctypes.c_void_p()
        check(self._lib.tg_ctx_create(device, ctypes.byref(h)))
        self.handle = h
        self.device = device
        name = ctypes.create_string_buffer(256)
        sms = ctypes.c_int()
        check(self._lib.tg_ctx_info(h, name, 256, ctypes.byref(sms)))
        self.name = name.value.decode()
        self.sm_count = sms.value

    @property
    def stream(self) -> int:
        """The context's cudaStream_t, as an integer (for torch.cuda.ExternalStream)."""
        return int(self._lib.tg_ctx_stream(self.handle) or 0)

    def synchronize(self, timeout_ns: int = 0) -> None:
        check(self._lib.tg_ctx_synchronize(self.handle, timeout_ns))

    def selftest_wait(self, limit_ns: int) -> None:
        """Runs the kernels' bounded waits on things that never come (tg_ctx_selftest_wait):
        raises KernelError once both have given up after `limit_ns`."""
        check(self._lib.tg_ctx_selftest_wait(self.handle, limit_ns))

    def close(self) -> None:
        if self.handle:
            self._lib.tg_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Memory:
    """A buffer by residence (vulkan::Memory / Buffer)."""

    def __init__(self, ctx: Context, nbytes: int, residence: int = RES_DEVICE):
        self.ctx = ctx
        h = ctypes.c_void_p()
        check(library().tg_mem_alloc(ctx.handle, nbytes, residence, ctypes.byref(h)))
        self.handle = h
        self.nbytes = nbytes

    @property
    def device_ptr(self) -> int:
        return int(library().tg_mem_device_ptr(self.handle) or 0)

    def write(self, data: np.ndarray, offset: int = 0) -> None:
        a = np.ascontiguousarray(data)
        check(library().tg_mem_write(self.handle, offset, a.ctypes.data, a.nbytes))

    def read(self, dtype, count: int, offset: int = 0) -> np.ndarray:
        out = np.empty(count, dtype)
        check(library().tg_mem_read(self.handle, offset, out.ctypes.data, out.nbytes))
        return out

    def fill(self, word: int, nbytes: Optional[int] = None, offset: int = 0) -> None:
        check(library().tg_mem_fill(self.handle, offset, word, self.nbytes if nbytes is None else nbytes))

    def free(self) -> None:
        if self.handle:
            library().tg_mem_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def params(shape: Shape, dtype: str, rows: int = 0, slots: int = 1, **extra) -> TgParams:
    """The params struct a kernel-table dispatch takes, from a shape."""
    p = TgParams(dtype=DTYPES[dtype], hidden=shape.hidden, inner=shape.inner, heads=shape.heads,
                 kv_heads=shape.kv_heads, head_dim=shape.head_dim, capacity=shape.capacity,
                 rows=rows, slots=slots, eps=shape.eps, residual_scale=shape.residual_scale,
                 rope=int(shape.rope))
    for k, v in extra.items():
        setattr(p, k, v)
    return p


def dispatch_once(ctx: Context, kernel: str, p: TgParams,
                  bindings: Sequence[tuple[Memory, int, int]], label: str = "") -> float:
    """Context::dispatch (crates/vulkan/src/context.rs:520): one kernel of the table, run and
    waited for; returns its GPU time in ns. `bindings` are (buffer, offset, bytes)."""
    b = (TgBinding * len(bindings))(*[TgBinding(m.handle, o, n) for m, o, n in bindings])
    d = TgDispatch(KERNELS[kernel], ctypes.pointer(p), b, len(bindings), label.encode())
    ns = ctypes.c_double()
    check(library().tg_dispatch_once(ctx.handle, ctypes.byref(d), ctypes.byref(ns)))
    return ns.value


class Program:
    """A chain of kernel-table dispatches captured once into a CUDA graph (vulkan::Recording):
    `dispatches` are (kernel name, params, [(buffer, offset, bytes)], label)."""

    def __init__(self, ctx: Context, dispatches, timed: bool = False):
        self.ctx = ctx
        keep = []
        arr = (TgDispatch * len(dispatches))()
        for i, (kernel, p, bindings, label) in enumerate(dispatches):
            b = (TgBinding * len(bindings))(*[TgBinding(m.handle, o, n) for m, o, n in bindings])
            pp = ctypes.pointer(p)
            lab = label.encode()
            keep += [b, pp, lab]
            arr[i] = TgDispatch(KERNELS[kernel], pp, b, len(bindings), lab)
        h = ctypes.c_void_p()
        check(library().tg_program_create(ctx.handle, arr, len(dispatches), int(timed), ctypes.byref(h)))
        self.handle = h
        self.n = len(dispatches)

    def start(self) -> None:
        check(library().tg_program_start(self.handle))

    def wait(self, timeout_ns: int = 0) -> None:
        check(library().tg_program_wait(self.handle, timeout_ns))

    def run(self) -> None:
        self.start()
        self.wait()

    def elapsed_ns(self) -> float:
        ns = ctypes.c_double()
        check(library().tg_program_elapsed_ns(self.handle, ctypes.byref(ns)))
        return ns.value

    def timings(self) -> list[float]:
        ns = (ctypes.c_double * self.n)()
        check(library().tg_program_timings(self.handle, ns, self.n))
        return list(ns)

    def close(self) -> None:
        if getattr(self, "handle", None):
            library().tg_program_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def attention_decode_noalloc(p: TgParams, q_ptr: int, k_ptr: int, v_ptr: int, at_ptr: int,
                             out_ptr: int, stream: int = 0) -> None:
    """Decode attention (split + combine) with its partials in the library's fixed scratch array:
    nothing is allocated. All pointers are device addresses; the work is enqueued on `stream`."""
    check(library().tg_attention_decode_noalloc(ctypes.byref(p), ctypes.c_void_p(q_ptr),
                                                ctypes.c_void_p(k_ptr), ctypes.c_void_p(v_ptr),
                                                ctypes.c_void_p(at_ptr), ctypes.c_void_p(out_ptr),
                                                ctypes.c_void_p(stream)))


# ---- decoder (decode.rs:778-913) ---------------------------------------------------------------------

WEIGHT_NAMES = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                "mlp.down_proj.weight", "input_layernorm.weight",
                "post_attention_layernorm.weight")


class Decoder:
    """A MiniCPM-4 stack's decode step on the GPU, with its weights and KV cache, recorded once
    for a batch of `rows` rows in a cache of `slots` slots (Decoder::with_batch)."""

    def __init__(self, ctx: Context, shape: Shape, rows: int = 1, slots: Optional[int] = None,
                 dtype: str = "bf16", timed: bool = False):
        self.ctx, self.shape = ctx, shape
        self.batch = Batch(rows, rows if slots is None else slots)
        self.dtype = dtype
        s, self._keep = shape._c()
        self._shape_c = s
        h = ctypes.c_void_p()
        check(library().tg_decoder_create(ctx.handle, ctypes.byref(s), self.batch.rows,
                                          self.batch.slots, DTYPES[dtype], int(timed),
                                          ctypes.byref(h)))
        self.handle = h
        self._out = np.zeros((rows, shape.hidden), np.float32)

    @classmethod
    def with_batch(cls, ctx, shape, batch: Batch, dtype="bf16", timed=False) -> "Decoder":
        return cls(ctx, shape, batch.rows, batch.slots, dtype, timed)

    def load(self, weights: Mapping[str, np.ndarray], prefix: str = "") -> None:
        """Decoder::load (decode.rs:808-820): every weight of the stack by its upstream name
        (after `prefix`), from f32 arrays, or uint16 arrays holding bf16 bits."""
        names = [f"layers.{l}.{w}" for l in range(self.shape.layers) for w in WEIGHT_NAMES]
        names.append("norm.weight")
        for name in names:
            key = prefix + name
            if key not in weights:
                raise Error(f"checkpoint: no tensor {key}")
            self.load_tensor(name, weights[key])

    def load_checkpoint(self, path, prefix: str = "") -> None:
        """Decoder::load from a safetensors file (crates/graph/src/checkpoint.rs): every weight of
        the stack by its upstream name after `prefix`, read a tensor at a time."""
        from .checkpoint import Checkpoint

        with Checkpoint(path) as ck:
            names = [f"layers.{l}.{w}" for l in range(self.shape.layers) for w in WEIGHT_NAMES]
            names.append("norm.weight")
            for name in names:
                if ck.shape(prefix + name) is None:
                    raise Error(f"checkpoint: no tensor {prefix + name}")
                self.load_tensor(name, ck.tensor(prefix + name))

    def load_tensor(self, name: str, values: np.ndarray) -> None:
        a = np.ascontiguousarray(values)
        if a.dtype == np.uint16:
            src = BF16
        else:
            a = np.ascontiguousarray(a, dtype=np.float32)
            src = F32
        check(library().tg_decoder_load(self.handle, name.encode(), a.ctypes.data, a.size, src))

    def step(self, position: int, x: np.ndarray) -> np.ndarray:
        """Decoder::step: batch 1 at `position` of slot 0."""
        return self.step_rows([Row(position, 0)], x)

    def step_rows(self, rows: Sequence[Optional[Row]], x: np.ndarray) -> np.ndarray:
        """Decoder::step_rows (decode.rs:849-853): x [rows][hidden] -> outputs after the final
        norm, [rows][hidden]; a spare row's is meaningless."""
        x = self._x(x)
        out = np.empty((self.batch.rows, self.shape.hidden), np.float32)
        check(library().tg_decoder_step_rows(self.handle, self._c_rows(rows), x.ctypes.data, out.ctypes.data))
        return out

    def step_rows_n(self, rows: Sequence[Optional[Row]], x: np.ndarray) -> np.ndarray:
        """A step of len(rows) <= batch rows, run by the smallest row bucket that holds them
        (generator.rs:115-123, :306-330): x [n][hidden] -> [n][hidden]."""
        n = len(rows)
        if not 1 <= n <= self.batch.rows:
            raise ShapeError(f"{n} rows in a decoder of {self.batch.rows}")
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        if x.size != n * self.shape.hidden:
            raise ShapeError(f"{x.size} values for {n} rows of {self.shape.hidden}")
        out = np.empty((n, self.shape.hidden), np.float32)
        check(library().tg_decoder_step_rows_n(self.handle, n, _rows(rows), x.ctypes.data, out.ctypes.data))
        return out

    def set_input(self, position: int, x: np.ndarray) -> None:
        """Decoder::set_input (decode.rs:841-845): the next run's input at batch 1, `x` the hidden
        state of `position` in slot 0."""
        self.set_rows([Row(position, 0)], x)

    def set_rows(self, rows: Sequence[Optional[Row]], x: np.ndarray) -> None:
        x = self._x(x)
        check(library().tg_decoder_set_rows(self.handle, self._c_rows(rows), x.ctypes.data))

    def start(self) -> None:
        check(library().tg_decoder_start(self.handle))

    def wait(self, timeout_ns: int = 0) -> None:
        check(library().tg_decoder_wait(self.handle, timeout_ns))

    def output(self) -> np.ndarray:
        out = np.empty((self.batch.rows, self.shape.hidden), np.float32)
        check(library().tg_decoder_output(self.handle, out.ctypes.data))
        return out

    def step_device(self, words: Sequence[int], x_ptr: int, out_ptr: int) -> None:
        """A step over device-resident x and out (pointers to [rows][hidden] f32)."""
        w = (ctypes.c_uint32 * len(words))(*words)
        check(library().tg_decoder_step_device(self.handle, w, ctypes.c_void_p(x_ptr),
                                               ctypes.c_void_p(out_ptr)))

    def elapsed_ns(self) -> float:
        ns = ctypes.c_double()
        check(library().tg_decoder_elapsed_ns(self.handle, ctypes.byref(ns)))
        return ns.value

    def labels(self) -> list[str]:
        n = ctypes.c_size_t()
        check(library().tg_decoder_timings(self.handle, None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(64)
        out = []
        for i in range(n.value):
            check(library().tg_decoder_dispatch_label(self.handle, i, buf, 64))
            out.append(buf.value.decode())
        return out

    def timings(self) -> list[tuple[str, float]]:
        """Each dispatch's label and GPU time in ns in the last step (when created timed)."""
        labels = self.labels()
        ns = (ctypes.c_double * len(labels))()
        check(library().tg_decoder_timings(self.handle, ns, len(labels), None))
        return list(zip(labels, list(ns)))

    def prefix_bytes(self, count: int) -> int:
        return int(library().tg_decoder_prefix_bytes(self.handle, count))

    def copy_out(self, slot: int, count: int, mem: "Memory", offset: int = 0) -> None:
        """Positions [0, count) of the slot's keys and values into `mem` (a kept prefix)."""
        check(library().tg_decoder_copy_out(self.handle, slot, count, mem.handle, offset))

    def copy_in(self, slot: int, count: int, mem: "Memory", offset: int = 0) -> None:
        """A kept prefix from `mem` into positions [0, count) of the slot."""
        check(library().tg_decoder_copy_in(self.handle, slot, count, mem.handle, offset))

    def read_cache(self, layer: int, slot: int, kind: str, first: int, count: int) -> np.ndarray:
        """Keys ("k") or values ("v") of positions [first, first + count) of a slot, as f32
        [kv_heads][count][head_dim]."""
        out = np.empty((self.shape.kv_heads, count, self.shape.head_dim), np.float32)
        check(library().tg_decoder_read_cache(self.handle, layer, slot, 0 if kind == "k" else 1,
                                              first, count, _fptr(out)))
        return out

    def copy_slot(self, src: int, dst: int, count: int) -> None:
        """Copies positions [0, count) of every layer's cache from slot `src` to slot `dst`."""
        check(library().tg_decoder_copy_slot(self.handle, src, dst, count))

    def weight_bytes(self) -> int:
        return int(library().tg_decoder_weight_bytes(self.handle))

    def retuned(self, persistent: bool, timed: bool = False) -> "Decoder":
        """Decoder::retuned (decode.rs:874-890): the step recorded again, as one persistent launch
        or as six kernels a layer (the same results bit for bit), over the same weights and cache."""
        check(library().tg_decoder_retune(self.handle, int(persistent), int(timed)))
        return self

    @property
    def persistent(self) -> bool:
        return bool(library().tg_decoder_persistent(self.handle))

    @property
    def tensor(self) -> bool:
        """True when the projections run on tcgen05 (bf16 decoders of 16 rows or more)."""
        return bool(library().tg_decoder_tensor(self.handle))

    def with_tensor(self, on: bool = True, split_k: bool = False) -> "Decoder":
        """Records the step again with its projections on tcgen05 (or as GEMVs); returns self. On
        tcgen05 they run as the prefill's GEMMs, or with `split_k` as split-K clusters over hi/lo
        activations."""
        check(library().tg_decoder_set_tensor(self.handle, 2 if (on and split_k) else int(on)))
        return self

    @property
    def split_k(self) -> bool:
        """True when the tcgen05 projections run as split-K clusters (not as the prefill's GEMMs)."""
        return bool(library().tg_decoder_tensor(self.handle) == 2)

    def _x(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        if x.size != self.batch.rows * self.shape.hidden:
            raise ShapeError(f"{x.size} values for {self.batch.rows} rows of {self.shape.hidden}")
        return x

    def _c_rows(self, rows: Sequence[Optional[Row]]):
        if len(rows) != self.batch.rows:
            raise ShapeError(f"{len(rows)} rows for a batch of {self.batch.rows}")
        return _rows(rows)

    def close(self) -> None:
        if getattr(self, "handle", None):
            library().tg_decoder_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Prefill:
    """A stack's prefill on the GPU: programs over a Decoder's weights, tables and cache for runs
    of up to `max_rows` positions at once (Prefill::new, prefill.rs:431-461)."""

    def __init__(self, decoder: Decoder, max_rows: int, timed: bool = False):
        self.decoder = decoder
        h = ctypes.c_void_p()
        check(library().tg_prefill_create(decoder.handle, max_rows, int(timed), ctypes.byref(h)))
        self.handle = h

    def max_rows(self) -> int:
        return int(library().tg_prefill_max_rows(self.handle))

    def run(self, start: int, x: np.ndarray, slot: int = 0) -> np.ndarray:
        """Prefill::run (prefill.rs:473-503): x [len][hidden] of positions start.. into `slot`;
        returns the outputs after the final norm, [len][hidden]."""
        h = self.decoder.shape.hidden
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        if x.size == 0 or x.size % h:
            raise ShapeError(f"{x.size} values from position {start}")
        n = x.size // h
        out = np.empty((n, h), np.float32)
        check(library().tg_prefill_run(self.handle, start, slot, _fptr(x), n, _fptr(out)))
        return out

    def run_batch(self, runs: Sequence[tuple[int, int, int]], x: np.ndarray) -> np.ndarray:
        """Several runs (start, len, slot) at once, their rows of x in order."""
        h = self.decoder.shape.hidden
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        total = sum(r[1] for r in runs)
        if x.size != total * h:
            raise ShapeError(f"{x.size} values for {total} rows of {h}")
        c = (TgRun * len(runs))(*[TgRun(*r) for r in runs])
        out = np.empty((total, h), np.float32)
        check(library().tg_prefill_run_batch(self.handle, c, len(runs), _fptr(x), _fptr(out)))
        return out

    def run_batch_device(self, runs: Sequence[tuple[int, int, int]], x_ptr: int, out_ptr: int) -> None:
        c = (TgRun * len(runs))(*[TgRun(*r) for r in runs])
        check(library().tg_prefill_run_batch_device(self.handle, c, len(runs),
                                                    ctypes.c_void_p(x_ptr), ctypes.c_void_p(out_ptr)))

    def elapsed_ns(self) -> float:
        ns = ctypes.c_double()
        check(library().tg_prefill_elapsed_ns(self.handle, ctypes.byref(ns)))
        return ns.value

    def timings(self) -> list[tuple[str, float]]:
        n = ctypes.c_size_t()
        check(library().tg_prefill_timings(self.handle, None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(64)
        labels = []
        for i in range(n.value):
            check(library().tg_prefill_dispatch_label(self.handle, i, buf, 64))
            labels.append(buf.value.decode())
        ns = (ctypes.c_double * n.value)()
        check(library().tg_prefill_timings(self.handle, ns, n.value, None))
        return list(zip(labels, list(ns)))

    def close(self) -> None:
        if getattr(self, "handle", None):
            library().tg_prefill_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Server:
    """Continuous batching over a decoder (a row per slot) and its prefill (generator.rs:99-352):
    requests hold slots, each step runs every request under way packed into rows by the smallest
    row bucket that holds them, requests are admitted between steps by a prefill. A request's next
    input is its last output, fed back on the GPU, unless the step is given inputs."""

    def __init__(self, decoder: Decoder, prefill: "Prefill"):
        self.decoder, self.prefill = decoder, prefill
        h = ctypes.c_void_p()
        check(library().tg_server_create(decoder.handle, prefill.handle, ctypes.byref(h)))
        self.handle = h

    def start(self, requests: Sequence[tuple], x: np.ndarray) -> None:
        """Generator::start for (slot, len, steps[, start]) requests, the rows of each prompt
        from its start (positions already in the slot, a kept prefix copied in) in x, in order."""
        hdim = self.decoder.shape.hidden
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        reqs = [tuple(r) + (0,) * (4 - len(r)) for r in requests]
        total = sum(r[1] - r[3] for r in reqs)
        if x.size != total * hdim:
            raise ShapeError(f"{x.size} values for {total} prompt rows of {hdim}")
        c = (TgRequest * max(len(reqs), 1))(*[TgRequest(*r) for r in reqs])
        check(library().tg_server_start(self.handle, c, len(requests), _fptr(x)))

    def step(self, x: Optional[np.ndarray] = None, read: bool = True):
        """One step of every request under way: (slots, outputs [n][hidden]) when `read`, else
        (slots, None) with the step only enqueued."""
        hdim = self.decoder.shape.hidden
        under = self.under_way()
        n = len(under)
        xp = None
        if x is not None:
            x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
            if x.size != n * hdim:
                raise ShapeError(f"{x.size} values for {n} rows under way")
            xp = _fptr(x)
        slots = (ctypes.c_uint32 * max(n, 1))()
        out = np.empty((n, hdim), np.float32) if read else None
        got = ctypes.c_uint32()
        check(library().tg_server_step(self.handle, xp, ctypes.byref(got), slots,
                                       _fptr(out) if read and n else None))
        return list(slots)[:got.value], out

    def under_way(self) -> list[int]:
        n = ctypes.c_uint32()
        check(library().tg_server_under_way(self.handle, None, ctypes.byref(n)))
        slots = (ctypes.c_uint32 * max(n.value, 1))()
        check(library().tg_server_under_way(self.handle, slots, ctypes.byref(n)))
        return list(slots)[:n.value]

    def request(self, slot: int) -> tuple[bool, int, int]:
        """(held, position of the next step, steps left) of the slot's request."""
        held, pos, left = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
        check(library().tg_server_request(self.handle, slot, ctypes.byref(held), ctypes.byref(pos),
                                          ctypes.byref(left)))
        return bool(held.value), pos.value, left.value

    def finish(self, slot: int) -> None:
        check(library().tg_server_finish(self.handle, slot))

    def last_output(self, slot: int) -> np.ndarray:
        out = np.empty(self.decoder.shape.hidden, np.float32)
        check(library().tg_server_last_output(self.handle, slot, _fptr(out)))
        return out

    def sync(self, timeout_ns: int = 0) -> None:
        check(library().tg_server_sync(self.handle, timeout_ns))

    def close(self) -> None:
        if getattr(self, "handle", None):
            library().tg_server_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
