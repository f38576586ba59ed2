"""B200-native decoder token loop for Whisper (the WhisperEACP decode path).

The compute lives in libwsp_b200.so (CUDA, sm_100a) behind the C ABI of
include/wsp_decoder.h; this package is the host-side mirror of the
reference's Decoder / Argmax / greedy-search interface over that ABI.
"""
from ._native import CudaError, LogicError, ModelError, library  # noqa: F401
from .decoder import Decoder, DecoderShape, StepResult, argmax, argmax_no_alloc  # noqa: F401

__all__ = ["Decoder", "DecoderShape", "StepResult", "ModelError", "LogicError", "CudaError",
           "argmax", "argmax_no_alloc", "library"]
