"""The decoder token loop's host interface, over the C ABI of include/wsp_decoder.h.

The names and argument meanings follow WhisperEACP's own classes so that a
test written against the reference reads the same here:

  DecoderShape   Lib/WhisperEACP/Decoder/DecoderShape.h:20-83
  Decoder        Lib/WhisperEACP/Decoder/Decoder.h:49-127 (prepare, beginSequence,
                 step, position, crossPositions, hiddenStates)
  DecoderWeights Lib/WhisperEACP/Decoder/DecoderWeights.h:25-160 (tensors by
                 their HuggingFace names)
  Argmax         Lib/WhisperEACP/Kernels/Argmax.h:207-262
  greedy search  Lib/WhisperEACP/Whisper/Whisper.cpp:148-254, 1361-1449

What the reference has no notion of is the batch: ``windows`` independent
30 s windows decoded in lockstep, each with its own caches.  ``windows=1`` is
the reference's behaviour.  Errors surface as the reference's do: ModelError
for shapes and capacities, raised before anything runs on the GPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._native import (CGeneration, CShape, KERNEL_CLASSES, TRACE_SECTIONS, LogicError, ModelError,
                      WSP_BFLOAT16, WSP_FLOAT16, WSP_FLOAT32, check, library)

__all__ = ["DecoderShape", "Decoder", "StepResult", "ModelError", "LogicError", "argmax", "argmax_no_alloc",
           "STORAGE"]

STORAGE = {"float16": WSP_FLOAT16, "bfloat16": WSP_BFLOAT16}


@dataclass(frozen=True)
class DecoderShape:
    """Every extent one decoder is built against (DecoderShape.h:20-31)."""
    width: int
    heads: int
    layers: int
    feed_forward_width: int
    vocabulary_size: int
    max_positions: int
    cross_positions: int

    def head_width(self) -> int:
        return self.width // self.heads

    def c(self) -> CShape:
        return CShape(self.width, self.heads, self.layers, self.feed_forward_width,
                      self.vocabulary_size, self.max_positions, self.cross_positions)

    @staticmethod
    def from_config(config: dict, cross_positions: int = 1500) -> "DecoderShape":
        """DecoderShape::fromConfig (DecoderShape.cpp:7-17) over HF config.json keys."""
        return DecoderShape(config["d_model"], config["decoder_attention_heads"],
                            config["decoder_layers"], config["decoder_ffn_dim"],
                            config["vocab_size"], config["max_target_positions"], cross_positions)


@dataclass
class StepResult:
    """One step's outputs (Tests/Decoder/Common.h:519-524)."""
    hidden: np.ndarray | None   # [windows, tokens, width]
    logits: np.ndarray | None   # [windows, tokens, vocabulary]
    argmax: np.ndarray          # [windows, tokens]


def _pointer(array: np.ndarray):
    return ctypes.c_void_p(array.ctypes.data)


_DTYPES = {np.dtype(np.float32): WSP_FLOAT32, np.dtype(np.float16): WSP_FLOAT16}


class Decoder:
    """A CUDA decoder for `windows` windows on one device (Decoder.h:49-127)."""

    PRODUCTS = {"auto": 0, "mma": 1, "tcgen05": 2}

    def __init__(self, shape: DecoderShape, windows: int = 1, device: int = 0,
                 storage: str = "float16", products: str = "auto"):
        """products: "auto" (the faster form for the window count), "mma"
        (mma.sync tiles) or "tcgen05" (tensor-memory tiles)."""
        if storage not in STORAGE:
            raise ValueError(f"storage must be one of {sorted(STORAGE)}")
        if products not in self.PRODUCTS:
            raise ValueError(f"products must be one of {sorted(self.PRODUCTS)}")
        self.shape = shape
        self.windows = windows
        self.device = device
        self.storage = storage
        self._lib = library()
        handle = ctypes.c_void_p()
        self._shape_c = shape.c()
        check(self._lib.wsp_decoder_create_products(ctypes.byref(self._shape_c), device, windows,
                                                    STORAGE[storage], self.PRODUCTS[products],
                                                    ctypes.byref(handle)))
        self._handle = handle
        self._generation = None

    def close(self) -> None:
        if getattr(self, "_handle", None):
            self._lib.wsp_decoder_destroy(self._handle)
            self._handle = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ------------------------------------------------------------- weights

    def set_tensor(self, name: str, values: np.ndarray, dtype: int | None = None) -> None:
        """One checkpoint tensor by its HuggingFace name (DecoderWeights.cpp:74-178).

        float32 and float16 arrays are passed as they are; ``dtype=WSP_BFLOAT16``
        marks a uint16 array holding bfloat16 bits.
        """
        values = np.ascontiguousarray(values)
        if dtype is None:
            if values.dtype not in _DTYPES:
                values = values.astype(np.float32)
            dtype = _DTYPES[values.dtype]
        extents = (ctypes.c_int64 * max(1, values.ndim))(*values.shape)
        check(self._lib.wsp_decoder_set_tensor(self._handle, name.encode(), dtype, extents,
                                               values.ndim, _pointer(values)))

    NARROWING = {"round": 0, "exact": 1}

    def set_narrowing(self, mode: str) -> None:
        """"round" (the default: nearest even) or "exact" (the reference's
        ExactHalf rule: a projection that does not narrow to the storage type
        unchanged is refused with ModelError naming it)."""
        if mode not in self.NARROWING:
            raise ValueError(f"narrowing must be one of {sorted(self.NARROWING)}")
        check(self._lib.wsp_decoder_set_narrowing(self._handle, self.NARROWING[mode]))

    def narrowing(self) -> tuple[int, float]:
        """(tensors narrowed inexactly so far, the largest change of a value)."""
        tensors, largest = ctypes.c_int(), ctypes.c_double()
        check(self._lib.wsp_decoder_narrowing(self._handle, ctypes.byref(tensors), ctypes.byref(largest)))
        return tensors.value, largest.value

    def load_weights(self, tensors: dict[str, np.ndarray]) -> None:
        """Every decoder tensor of a checkpoint (a safetensors file's dict)."""
        for name, values in tensors.items():
            self.set_tensor(name, values)
        check(self._lib.wsp_decoder_check_weights(self._handle))

    # ----------------------------------------------------------- sequences

    def begin_sequence(self, encoder_rows, cross_positions: int = 0) -> None:
        """Decoder::beginSequence for every window (Decoder.h:67-73).

        encoder_rows: float32 [windows, cross_positions, width] (numpy), or a
        device pointer (int) to the same.
        """
        check(self._lib.wsp_decoder_begin_sequence(self._handle, self._rows_pointer(encoder_rows),
                                                   cross_positions))

    def step(self, tokens, logits: bool = True, hidden: bool = True) -> StepResult:
        """Decoder::step: appends tokens [windows, n] to every window (Decoder.h:75-98)."""
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32).reshape(self.windows, -1))
        n = ids.shape[1]
        out_logits = np.empty((self.windows, n, self.shape.vocabulary_size), np.float32) if logits else None
        out_hidden = np.empty((self.windows, n, self.shape.width), np.float32) if hidden else None
        out_argmax = np.empty((self.windows, n), np.uint32)
        check(self._lib.wsp_decoder_step(
            self._handle, _pointer(ids), n,
            _pointer(out_logits) if logits else None,
            _pointer(out_hidden) if hidden else None,
            _pointer(out_argmax)))
        return StepResult(out_hidden, out_logits, out_argmax)

    @property
    def position(self) -> int:
        value = ctypes.c_int()
        check(self._lib.wsp_decoder_position(self._handle, ctypes.byref(value)))
        return value.value

    @property
    def cross_positions(self) -> int:
        value = ctypes.c_int()
        check(self._lib.wsp_decoder_cross_positions(self._handle, ctypes.byref(value)))
        return value.value

    # ------------------------------------------------------ greedy search

    def set_generation(self, prompt, first_step_mask=None, later_step_mask=None,
                       maximum_tokens: int | None = None, end_of_text: int = 50256,
                       stop_at_end_of_text: bool = True) -> None:
        """The generation config Whisper::load builds (Whisper.cpp:148-254)."""
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        if maximum_tokens is None:
            maximum_tokens = self.shape.max_positions - len(prompt)
        v = self.shape.vocabulary_size
        first = np.ascontiguousarray(first_step_mask if first_step_mask is not None else np.zeros(v),
                                     dtype=np.float32)
        later = np.ascontiguousarray(later_step_mask if later_step_mask is not None else np.zeros(v),
                                     dtype=np.float32)
        if first.shape != (v,) or later.shape != (v,):
            raise ModelError(f"suppression masks must hold {v} entries")
        config = CGeneration(prompt.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), len(prompt),
                             first.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                             later.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                             maximum_tokens, end_of_text, 1 if stop_at_end_of_text else 0)
        check(self._lib.wsp_decoder_set_generation(self._handle, ctypes.byref(config)))
        self._generation = (len(prompt), maximum_tokens)

    def step_limit(self) -> int:
        prompt_length, maximum_tokens = self._require_generation()
        return min(maximum_tokens, self.shape.max_positions - prompt_length + 1)

    def transcribe(self, encoder_rows, cross_positions: int = 0) -> list[np.ndarray]:
        """Whisper::decodeTranscript for every window: one token id array each."""
        limit = self.step_limit()
        tokens = np.zeros((self.windows, limit), np.uint32)
        counts = np.zeros(self.windows, np.int32)
        check(self._lib.wsp_decoder_transcribe(self._handle, self._rows_pointer(encoder_rows),
                                               cross_positions, _pointer(tokens), _pointer(counts)))
        return [tokens[b, :counts[b]].copy() for b in range(self.windows)]

    def enqueue_transcribe(self, encoder_rows, steps: int, cross_positions: int = 0) -> None:
        check(self._lib.wsp_decoder_enqueue_transcribe(self._handle, self._rows_pointer(encoder_rows),
                                                       cross_positions, steps))

    def read_transcript(self) -> list[np.ndarray]:
        limit = self.step_limit()
        tokens = np.zeros((self.windows, limit), np.uint32)
        counts = np.zeros(self.windows, np.int32)
        check(self._lib.wsp_decoder_read_transcript(self._handle, _pointer(tokens), _pointer(counts)))
        return [tokens[b, :counts[b]].copy() for b in range(self.windows)]

    # -------------------------------------------------------- measurement

    @property
    def stream(self) -> int:
        """The cudaStream_t every launch of this decoder goes to."""
        return self._lib.wsp_decoder_stream(self._handle) or 0

    def synchronize(self) -> None:
        check(self._lib.wsp_decoder_synchronize(self._handle))

    def step_launches(self) -> int:
        value = ctypes.c_int()
        check(self._lib.wsp_decoder_step_launches(self._handle, ctypes.byref(value)))
        return value.value

    def phase_ms(self) -> dict:
        """Milliseconds of the last transcription's phases (CUDA events on the
        decoder's stream): sequence start, prompt launch, later-steps launch."""
        ms = (ctypes.c_float * 3)()
        check(self._lib.wsp_decoder_phase_ms(self._handle, ms))
        return {"sequence_start": ms[0], "prompt": ms[1], "steps": ms[2]}

    def time_barriers(self, count: int = 40) -> float:
        """Mean microseconds of one grid barrier of the decode kernel."""
        value = ctypes.c_float()
        check(self._lib.wsp_decoder_time_barriers(self._handle, count, ctypes.byref(value)))
        return value.value

    def trace_cycles(self) -> dict[str, float]:
        """CTA 0's clock cycles per step in each section, from the last time_kernels."""
        values = (ctypes.c_double * len(TRACE_SECTIONS))()
        check(self._lib.wsp_decoder_trace_cycles(self._handle, values, len(TRACE_SECTIONS)))
        return {name: values[i] for i, name in enumerate(TRACE_SECTIONS)}

    def op_times(self) -> list[tuple[int, float]]:
        """(kind, microseconds) of each op of the step, from the last time_kernels."""
        count = ctypes.c_int()
        check(self._lib.wsp_decoder_op_times(self._handle, None, None, 0, ctypes.byref(count)))
        us = (ctypes.c_float * max(1, count.value))()
        kinds = (ctypes.c_int * max(1, count.value))()
        check(self._lib.wsp_decoder_op_times(self._handle, us, kinds, count.value, ctypes.byref(count)))
        return [(kinds[i], us[i]) for i in range(count.value)]

    def time_kernels(self, steps: int) -> dict[str, tuple[float, int]]:
        """Mean ms per launch and launches per step of each kernel class."""
        ms = (ctypes.c_float * len(KERNEL_CLASSES))()
        launches = (ctypes.c_int * len(KERNEL_CLASSES))()
        check(self._lib.wsp_decoder_time_kernels(self._handle, steps, ms, launches))
        return {name: (ms[i], launches[i]) for i, name in enumerate(KERNEL_CLASSES)}

    # -------------------------------------------------------------- helpers

    def _require_generation(self):
        if self._generation is None:
            raise LogicError("set_generation has not been called")
        return self._generation

    def _rows_pointer(self, rows):
        if isinstance(rows, int):
            return ctypes.c_void_p(rows)
        rows = np.ascontiguousarray(rows, dtype=np.float32)
        expected = self.windows * self.shape.cross_positions * self.shape.width
        if rows.size != expected:
            raise ModelError(f"encoder rows hold {rows.size} floats; the decoder reads "
                             f"{self.windows} x {self.shape.cross_positions} x {self.shape.width}")
        self._rows_keepalive = rows
        return _pointer(rows)


def argmax(logits_pointer: int, mask_pointer: int | None, out_pointer: int, row_count: int,
           row_length: int, stream: int = 0) -> None:
    """Argmax::encode over device buffers (Argmax.h:207-262, Argmax.cpp:47-80)."""
    check(library().wsp_argmax(ctypes.c_void_p(logits_pointer),
                               ctypes.c_void_p(mask_pointer) if mask_pointer else None,
                               ctypes.c_void_p(out_pointer), row_count, row_length,
                               ctypes.c_void_p(stream) if stream else None))


def argmax_no_alloc(logits_pointer: int, mask_pointer: int | None, out_pointer: int, row_count: int,
                    row_length: int, stream: int = 0) -> None:
    """argmax without allocating device memory (wsp_argmax_no_alloc): scratch
    is a fixed array inside the library, at most 65536 row groups
    (rows x ceil(length / 2048)).  Queues the work on `stream` and returns
    without waiting.  Calls that overlap on one device race on the scratch;
    calls on one stream are ordered."""
    check(library().wsp_argmax_no_alloc(ctypes.c_void_p(logits_pointer),
                                        ctypes.c_void_p(mask_pointer) if mask_pointer else None,
                                        ctypes.c_void_p(out_pointer), row_count, row_length,
                                        ctypes.c_void_p(stream) if stream else None))
