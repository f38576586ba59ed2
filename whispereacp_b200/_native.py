"""Loads libwsp_b200.so, the CUDA decoder behind include/wsp_decoder.h.

There is no fallback: without the built library, importing the package's
decoder raises, so nothing can silently run a CPU path in its place.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(HERE, "libwsp_b200.so")

WSP_OK = 0
WSP_MODEL_ERROR = 1
WSP_LOGIC_ERROR = 2
WSP_INVALID_ARGUMENT = 3
WSP_CUDA_ERROR = 4
WSP_OUT_OF_MEMORY = 5

WSP_FLOAT32 = 0
WSP_FLOAT16 = 1
WSP_BFLOAT16 = 2

TRACE_SECTIONS = ("wait", "compute", "barrier", "epilogue", "norm", "attention", "ops", "query", "join",
                  "out_projection", "self_item", "logits", "norm_load", "norm_rest", "logits_tiles",
                  "logits_fold")

KERNEL_CLASSES = ("embed", "layer_norm", "projection", "self_attention", "cross_attention",
                  "attention_combine", "logits_argmax", "argmax_final", "other")


class ModelError(RuntimeError):
    """WSP::ModelError: a shape, capacity or tensor the model cannot take."""


class LogicError(RuntimeError):
    """std::logic_error: the API used out of order."""


class CudaError(RuntimeError):
    """A CUDA failure inside the library."""


class CShape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "width", "heads", "layers", "feed_forward_width", "vocabulary_size",
        "max_positions", "cross_positions")]


class CGeneration(ctypes.Structure):
    _fields_ = [("prompt", ctypes.POINTER(ctypes.c_uint32)),
                ("prompt_length", ctypes.c_int32),
                ("first_step_mask", ctypes.POINTER(ctypes.c_float)),
                ("later_step_mask", ctypes.POINTER(ctypes.c_float)),
                ("maximum_tokens", ctypes.c_int32),
                ("end_of_text", ctypes.c_uint32),
                ("stop_at_end_of_text", ctypes.c_int32)]


class CEncoderShape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "mel_bins", "width", "heads", "layers", "feed_forward_width", "input_frames")]


# Every entry point include/wsp_decoder.h and include/wsp_encoder.h declare,
# with its ctypes signature.
_P = ctypes.c_void_p
_I = ctypes.c_int
SIGNATURES = {
    "wsp_last_error": ([], ctypes.c_char_p),
    "wsp_abi_version": ([], _I),
    "wsp_device_count": ([ctypes.POINTER(_I)], _I),
    "wsp_decoder_create": ([ctypes.POINTER(CShape), _I, _I, _I, ctypes.POINTER(_P)], _I),
    "wsp_decoder_create_products": ([ctypes.POINTER(CShape), _I, _I, _I, _I, ctypes.POINTER(_P)], _I),
    "wsp_decoder_destroy": ([_P], None),
    "wsp_decoder_set_tensor": ([_P, ctypes.c_char_p, _I, ctypes.POINTER(ctypes.c_int64), _I, _P], _I),
    "wsp_decoder_check_weights": ([_P], _I),
    "wsp_decoder_set_narrowing": ([_P, _I], _I),
    "wsp_decoder_narrowing": ([_P, ctypes.POINTER(_I), ctypes.POINTER(ctypes.c_double)], _I),
    "wsp_decoder_begin_sequence": ([_P, _P, _I], _I),
    "wsp_decoder_step": ([_P, _P, _I, _P, _P, _P], _I),
    "wsp_decoder_position": ([_P, ctypes.POINTER(_I)], _I),
    "wsp_decoder_cross_positions": ([_P, ctypes.POINTER(_I)], _I),
    "wsp_decoder_set_generation": ([_P, ctypes.POINTER(CGeneration)], _I),
    "wsp_decoder_transcribe": ([_P, _P, _I, _P, _P], _I),
    "wsp_decoder_enqueue_transcribe": ([_P, _P, _I, _I], _I),
    "wsp_decoder_read_transcript": ([_P, _P, _P], _I),
    "wsp_decoder_stream": ([_P], _P),
    "wsp_decoder_synchronize": ([_P], _I),
    "wsp_decoder_time_kernels": ([_P, _I, _P, _P], _I),
    "wsp_decoder_time_barriers": ([_P, _I, ctypes.POINTER(ctypes.c_float)], _I),
    "wsp_decoder_trace_cycles": ([_P, ctypes.POINTER(ctypes.c_double), _I], _I),
    "wsp_decoder_op_times": ([_P, _P, _P, _I, _P], _I),
    "wsp_decoder_step_launches": ([_P, ctypes.POINTER(_I)], _I),
    "wsp_decoder_phase_ms": ([_P, ctypes.POINTER(ctypes.c_float)], _I),
    "wsp_argmax": ([_P, _P, _P, _I, _I, _P], _I),
    "wsp_argmax_no_alloc": ([_P, _P, _P, _I, _I, _P], _I),
    "wsp_encoder_create": ([ctypes.POINTER(CEncoderShape), _I, _I, ctypes.POINTER(_P)], _I),
    "wsp_encoder_destroy": ([_P], None),
    "wsp_encoder_set_tensor": ([_P, ctypes.c_char_p, _I, ctypes.POINTER(ctypes.c_int64), _I, _P], _I),
    "wsp_encoder_set_filters": ([_P, _P], _I),
    "wsp_encoder_check_weights": ([_P], _I),
    "wsp_encoder_log_mel": ([_P, _P, _I, _P], _I),
    "wsp_encoder_encode": ([_P, _P, _P], _I),
    "wsp_encoder_encode_samples": ([_P, _P, _I, _P], _I),
}

_lib = None


def library() -> ctypes.CDLL:
    """The loaded CUDA library; raises ImportError if it was never built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIBRARY_PATH):
            raise ImportError(
                f"{LIBRARY_PATH} is missing: build it with `make -C whispereacp_b200` "
                "(or __graft_entry__.build()); there is no CPU fallback")
        lib = ctypes.CDLL(LIBRARY_PATH)
        for name, (args, result) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = result
        _lib = lib
    return _lib


def check(status: int) -> None:
    """Raises the Python counterpart of a wsp_status."""
    if status == WSP_OK:
        return
    text = (library().wsp_last_error() or b"").decode(errors="replace")
    if status == WSP_MODEL_ERROR:
        raise ModelError(text)
    if status == WSP_LOGIC_ERROR:
        raise LogicError(text)
    if status == WSP_INVALID_ARGUMENT:
        raise ValueError(text)
    if status == WSP_OUT_OF_MEMORY:
        raise MemoryError(text)
    raise CudaError(text)
