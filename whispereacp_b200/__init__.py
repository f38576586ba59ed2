"""B200-native decoder token loop for Whisper (the WhisperEACP decode path),
with the audio front end (log-mel spectrogram and encoder) that feeds it.

The compute lives in libwsp_b200.so (CUDA, sm_100a) behind the C ABI of
include/wsp_decoder.h and include/wsp_encoder.h; this package is the
host-side mirror of the reference's Decoder / Argmax / greedy-search and
Encoder / MelSpectrogram interfaces over that ABI.
"""
from ._native import CudaError, LogicError, ModelError, library  # noqa: F401
from .decoder import Decoder, DecoderShape, StepResult, argmax, argmax_no_alloc  # noqa: F401
from .encoder import Encoder, EncoderShape  # noqa: F401

__all__ = ["Decoder", "DecoderShape", "StepResult", "Encoder", "EncoderShape", "ModelError", "LogicError",
           "CudaError", "argmax", "argmax_no_alloc", "library"]
