"""ctypes front of the CPU oracle (oracle/wsp_oracle.c).

TEST INFRASTRUCTURE ONLY.  tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg import this module as the checker; the product package
``whispereacp_b200`` never does.

Besides the decoder itself this module restates the reference's fixture
generator for its small synthetic decoder, ``syntheticDecoderFile``
(Tests/Decoder/Common.h:66-169): the tensors in the order the reference draws
them, each from ``spreadValues`` (Tests/Kernels/Common.h:79-88) under a seed
that starts at 2000 and counts up, the layer-norm gains from
``shiftedValues`` (Tests/Encoder/Common.h:148-156).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "liboracle.so")


def build() -> None:
    """Compile liboracle.so (and the reference libraries where the checkout is)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


class CShape(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int) for name in (
        "width", "heads", "layers", "feed_forward_width", "vocabulary_size",
        "max_positions", "cross_positions")]


_F = ctypes.POINTER(ctypes.c_float)
_D = ctypes.POINTER(ctypes.c_double)
_I32 = ctypes.POINTER(ctypes.c_int32)
_U32 = ctypes.POINTER(ctypes.c_uint32)


def _declare(l: ctypes.CDLL) -> None:
    l.wspo_reference_decode.argtypes = [ctypes.POINTER(CShape), ctypes.POINTER(_F), _F,
                                        ctypes.c_int, _I32, ctypes.c_int, _D, _D, ctypes.c_int]
    l.wspo_session_new.argtypes = [ctypes.POINTER(CShape), ctypes.POINTER(_F), ctypes.c_int]
    l.wspo_session_new.restype = ctypes.c_void_p
    l.wspo_session_free.argtypes = [ctypes.c_void_p]
    l.wspo_session_begin.argtypes = [ctypes.c_void_p, _F, ctypes.c_int]
    l.wspo_session_step.argtypes = [ctypes.c_void_p, _I32, ctypes.c_int, _D, _D]
    l.wspo_session_position.argtypes = [ctypes.c_void_p]
    l.wspo_masked_argmax_f64.argtypes = [_D, _F, ctypes.c_int, ctypes.c_int, _U32]
    l.wspo_masked_argmax_f32.argtypes = [_F, _F, ctypes.c_int, ctypes.c_int, _U32]
    l.wspo_spread_values.argtypes = [_F, ctypes.c_int, ctypes.c_uint32, ctypes.c_float]
    l.wspo_shifted_values.argtypes = [_F, ctypes.c_int, ctypes.c_uint32, ctypes.c_float]
    l.wspo_synthetic_encoder_output.argtypes = [_F, ctypes.c_int, ctypes.c_int]
    l.wspo_pack_half.argtypes = [ctypes.c_float]
    l.wspo_pack_half.restype = ctypes.c_uint16
    l.wspo_half_to_float.argtypes = [ctypes.c_uint16]
    l.wspo_half_to_float.restype = ctypes.c_float
    l.wspo_pack_bfloat16.argtypes = [ctypes.c_float]
    l.wspo_pack_bfloat16.restype = ctypes.c_uint16


def _ptr(array: np.ndarray, ctype):
    return array.ctypes.data_as(ctypes.POINTER(ctype))


@dataclass(frozen=True)
class Shape:
    """DecoderShape (Lib/WhisperEACP/Decoder/DecoderShape.h:20-83)."""
    width: int
    heads: int
    layers: int
    feed_forward_width: int
    vocabulary_size: int
    max_positions: int
    cross_positions: int

    def c(self) -> CShape:
        return CShape(self.width, self.heads, self.layers, self.feed_forward_width,
                      self.vocabulary_size, self.max_positions, self.cross_positions)


# smallDecoderShape, Tests/Decoder/Common.h:45-54.
SMALL_SHAPE = Shape(width=8, heads=2, layers=2, feed_forward_width=16,
                    vocabulary_size=24, max_positions=16, cross_positions=6)

# The prompt the reference's small-shape tests decode (DecoderTests.cpp:34-37).
SMALL_PROMPT = [5, 17, 3, 11]


def decoder_tensor_names(layers: int) -> list[str]:
    """HF tensor names in the oracle's flat order (wsp_oracle.h)."""
    names = ["model.decoder.embed_tokens.weight", "model.decoder.embed_positions.weight",
             "model.decoder.layer_norm.weight", "model.decoder.layer_norm.bias"]
    for layer in range(layers):
        p = f"model.decoder.layers.{layer}."
        for attention, norm in (("self_attn", "self_attn_layer_norm"),
                                ("encoder_attn", "encoder_attn_layer_norm")):
            names += [p + norm + ".weight", p + norm + ".bias",
                      p + attention + ".q_proj.weight", p + attention + ".q_proj.bias",
                      p + attention + ".k_proj.weight",
                      p + attention + ".v_proj.weight", p + attention + ".v_proj.bias",
                      p + attention + ".out_proj.weight", p + attention + ".out_proj.bias"]
        names += [p + "final_layer_norm.weight", p + "final_layer_norm.bias",
                  p + "fc1.weight", p + "fc1.bias", p + "fc2.weight", p + "fc2.bias"]
    return names


def tensor_extents(shape: Shape, name: str) -> tuple[int, ...]:
    d, f = shape.width, shape.feed_forward_width
    if name.endswith("embed_tokens.weight"):
        return (shape.vocabulary_size, d)
    if name.endswith("embed_positions.weight"):
        return (shape.max_positions, d)
    if name.endswith("fc1.weight"):
        return (f, d)
    if name.endswith("fc1.bias"):
        return (f,)
    if name.endswith("fc2.weight"):
        return (d, f)
    if name.endswith("proj.weight"):
        return (d, d)
    return (d,)


def spread_values(count: int, seed: int, value_range: float) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().wspo_spread_values(_ptr(out, ctypes.c_float), count, seed, value_range)
    return out


def shifted_values(count: int, seed: int, value_range: float) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().wspo_shifted_values(_ptr(out, ctypes.c_float), count, seed, value_range)
    return out


def synthetic_encoder_output(positions: int, width: int) -> np.ndarray:
    out = np.empty(positions * width, dtype=np.float32)
    lib().wspo_synthetic_encoder_output(_ptr(out, ctypes.c_float), positions, width)
    return out.reshape(positions, width)


def synthetic_decoder_tensors(shape: Shape, first_seed: int = 2000) -> dict[str, np.ndarray]:
    """syntheticDecoderFile's float tensors (Tests/Decoder/Common.h:66-169)."""
    seed = first_seed
    tensors: dict[str, np.ndarray] = {}

    def draw(name: str, value_range: float, shifted: bool = False) -> None:
        nonlocal seed
        extents = tensor_extents(shape, name)
        count = int(np.prod(extents))
        generate = shifted_values if shifted else spread_values
        tensors[name] = generate(count, seed, value_range).reshape(extents)
        seed += 1

    draw("model.decoder.embed_tokens.weight", 0.3)
    draw("model.decoder.embed_positions.weight", 0.3)
    for layer in range(shape.layers):
        p = f"model.decoder.layers.{layer}."
        for attention, norm in (("self_attn", "self_attn_layer_norm"),
                                ("encoder_attn", "encoder_attn_layer_norm")):
            draw(p + norm + ".weight", 0.2, shifted=True)
            draw(p + norm + ".bias", 0.2)
            draw(p + attention + ".q_proj.weight", 0.5)
            draw(p + attention + ".q_proj.bias", 0.2)
            draw(p + attention + ".k_proj.weight", 0.5)
            draw(p + attention + ".v_proj.weight", 0.5)
            draw(p + attention + ".v_proj.bias", 0.2)
            draw(p + attention + ".out_proj.weight", 0.5)
            draw(p + attention + ".out_proj.bias", 0.2)
        draw(p + "final_layer_norm.weight", 0.2, shifted=True)
        draw(p + "final_layer_norm.bias", 0.2)
        draw(p + "fc1.weight", 0.5)
        draw(p + "fc1.bias", 0.2)
        draw(p + "fc2.weight", 0.5)
        draw(p + "fc2.bias", 0.2)
    draw("model.decoder.layer_norm.weight", 0.2, shifted=True)
    draw("model.decoder.layer_norm.bias", 0.2)
    return tensors


class _Tensors:
    """Keeps contiguous float32 copies alive and hands out the pointer array."""

    def __init__(self, shape: Shape, tensors: dict[str, np.ndarray]):
        names = decoder_tensor_names(shape.layers)
        self.arrays = [np.ascontiguousarray(tensors[n], dtype=np.float32) for n in names]
        self.pointers = (_F * len(names))(*[_ptr(a, ctypes.c_float) for a in self.arrays])


def reference_decode(shape: Shape, tensors: dict[str, np.ndarray], encoder: np.ndarray,
                     tokens, threads: int = 1, cross_rows: int | None = None):
    """referenceDecode (Tests/Decoder/Common.h:360-468): (hidden, logits) in double."""
    held = _Tensors(shape, tensors)
    encoder = np.ascontiguousarray(encoder, dtype=np.float32)
    rows = cross_rows if cross_rows is not None else shape.cross_positions
    ids = np.ascontiguousarray(tokens, dtype=np.int32)
    hidden = np.empty((len(ids), shape.width))
    logits = np.empty((len(ids), shape.vocabulary_size))
    status = lib().wspo_reference_decode(ctypes.byref(shape.c()), held.pointers,
                                         _ptr(encoder, ctypes.c_float), rows,
                                         _ptr(ids, ctypes.c_int32), len(ids),
                                         _ptr(hidden, ctypes.c_double),
                                         _ptr(logits, ctypes.c_double), threads)
    if status != 0:
        raise ValueError("the oracle refused this decode")
    return hidden, logits


class Session:
    """The KV-cached oracle: begin() once per window, then step()s."""

    def __init__(self, shape: Shape, tensors: dict[str, np.ndarray], threads: int = 1):
        self.shape = shape
        self._held = _Tensors(shape, tensors)
        self._shape_c = shape.c()
        self._handle = lib().wspo_session_new(ctypes.byref(self._shape_c),
                                              self._held.pointers, threads)
        if not self._handle:
            raise MemoryError("oracle session")

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle:
            lib().wspo_session_free(handle)
            self._handle = None

    def begin(self, encoder: np.ndarray, cross_rows: int | None = None) -> None:
        self._encoder = np.ascontiguousarray(encoder, dtype=np.float32)
        rows = cross_rows if cross_rows is not None else self.shape.cross_positions
        if lib().wspo_session_begin(self._handle, _ptr(self._encoder, ctypes.c_float), rows) != 0:
            raise ValueError("the oracle refused this sequence start")

    def step(self, tokens, want_logits: bool = True):
        ids = np.ascontiguousarray(tokens, dtype=np.int32)
        hidden = np.empty((len(ids), self.shape.width))
        logits = np.empty((len(ids), self.shape.vocabulary_size)) if want_logits else None
        status = lib().wspo_session_step(
            self._handle, _ptr(ids, ctypes.c_int32), len(ids), _ptr(hidden, ctypes.c_double),
            _ptr(logits, ctypes.c_double) if logits is not None else None)
        if status != 0:
            raise ValueError("the oracle refused this step")
        return hidden, logits

    @property
    def position(self) -> int:
        return lib().wspo_session_position(self._handle)


def masked_argmax(logits: np.ndarray, mask: np.ndarray | None = None) -> np.ndarray:
    """ArgmaxTests.cpp:20-35 (first maximum among unsuppressed; none -> 0)."""
    logits = np.atleast_2d(logits)
    rows, length = logits.shape
    out = np.empty(rows, dtype=np.uint32)
    mask_ptr = None
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.float32)
        mask_ptr = _ptr(mask, ctypes.c_float)
    if logits.dtype == np.float64:
        data = np.ascontiguousarray(logits)
        lib().wspo_masked_argmax_f64(_ptr(data, ctypes.c_double), mask_ptr, rows, length,
                                     _ptr(out, ctypes.c_uint32))
    else:
        data = np.ascontiguousarray(logits, dtype=np.float32)
        lib().wspo_masked_argmax_f32(_ptr(data, ctypes.c_float), mask_ptr, rows, length,
                                     _ptr(out, ctypes.c_uint32))
    return out


def pack_half(values: np.ndarray) -> np.ndarray:
    flat = np.asarray(values, dtype=np.float32).ravel()
    return np.array([lib().wspo_pack_half(float(v)) for v in flat], dtype=np.uint16)


def pack_bfloat16(values: np.ndarray) -> np.ndarray:
    flat = np.asarray(values, dtype=np.float32).ravel()
    return np.array([lib().wspo_pack_bfloat16(float(v)) for v in flat], dtype=np.uint16)
