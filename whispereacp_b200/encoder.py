"""The audio front end's host interface, over the C ABI of include/wsp_encoder.h.

  EncoderShape    Lib/WhisperEACP/Encoder/EncoderShape.h:16-65
  Encoder         Lib/WhisperEACP/Encoder/Encoder.h (prepare, encode)
  EncoderWeights  Lib/WhisperEACP/Encoder/EncoderWeights.h (tensors by their
                  HuggingFace names, model.encoder.*)
  MelSpectrogram  Lib/WhisperEACP/Mel/MelSpectrogram.h (the normalised log-mel)
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._native import CEncoderShape, WSP_FLOAT16, WSP_FLOAT32, check, library
from .decoder import STORAGE

__all__ = ["EncoderShape", "Encoder"]

SAMPLES_PER_FRAME = 160


@dataclass(frozen=True)
class EncoderShape:
    """The encoder's extents; input_frames mel frames become input_frames / 2 positions."""
    mel_bins: int
    width: int
    heads: int
    layers: int
    feed_forward_width: int
    input_frames: int = 3000

    @property
    def positions(self) -> int:
        return (self.input_frames - 1) // 2 + 1

    @staticmethod
    def from_config(config: dict) -> "EncoderShape":
        return EncoderShape(config["num_mel_bins"], config["d_model"], config["encoder_attention_heads"],
                            config["encoder_layers"], config["encoder_ffn_dim"], 2 * config["max_source_positions"])

    def c(self) -> CEncoderShape:
        return CEncoderShape(self.mel_bins, self.width, self.heads, self.layers, self.feed_forward_width,
                             self.input_frames)


def _pointer(array: np.ndarray):
    return ctypes.c_void_p(array.ctypes.data)


class Encoder:
    """Encoder + MelSpectrogram on one CUDA device."""

    def __init__(self, shape: EncoderShape, device: int = 0, storage: str = "float16"):
        self._lib = library()
        self.shape = shape
        self._handle = ctypes.c_void_p()
        c = shape.c()
        check(self._lib.wsp_encoder_create(ctypes.byref(c), device, STORAGE[storage], ctypes.byref(self._handle)))

    def close(self) -> None:
        if self._handle:
            self._lib.wsp_encoder_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        self.close()

    def set_tensor(self, name: str, values: np.ndarray) -> None:
        values = np.ascontiguousarray(values, np.float32)
        extents = (ctypes.c_int64 * values.ndim)(*values.shape)
        check(self._lib.wsp_encoder_set_tensor(self._handle, name.encode(), WSP_FLOAT32, extents, values.ndim,
                                               _pointer(values)))

    def load_weights(self, tensors: dict[str, np.ndarray]) -> None:
        for name, values in tensors.items():
            self.set_tensor(name, values)
        check(self._lib.wsp_encoder_check_weights(self._handle))

    def set_filters(self, filters: np.ndarray) -> None:
        filters = np.ascontiguousarray(filters, np.float32)
        if filters.shape != (self.shape.mel_bins, 201):
            raise ValueError(f"a filterbank is [{self.shape.mel_bins}][201]")
        check(self._lib.wsp_encoder_set_filters(self._handle, _pointer(filters)))

    def log_mel(self, samples: np.ndarray) -> np.ndarray:
        samples = np.ascontiguousarray(samples, np.float32)
        out = np.empty((self.shape.mel_bins, self.shape.input_frames), np.float32)
        check(self._lib.wsp_encoder_log_mel(self._handle, _pointer(samples), samples.size, _pointer(out)))
        return out

    def encode(self, mel: np.ndarray) -> np.ndarray:
        mel = np.ascontiguousarray(mel, np.float32)
        if mel.shape != (self.shape.mel_bins, self.shape.input_frames):
            raise ValueError(f"a log-mel is [{self.shape.mel_bins}][{self.shape.input_frames}]")
        out = np.empty((self.shape.positions, self.shape.width), np.float32)
        check(self._lib.wsp_encoder_encode(self._handle, _pointer(mel), _pointer(out)))
        return out

    def encode_samples(self, samples: np.ndarray) -> np.ndarray:
        samples = np.ascontiguousarray(samples, np.float32)
        out = np.empty((self.shape.positions, self.shape.width), np.float32)
        check(self._lib.wsp_encoder_encode_samples(self._handle, _pointer(samples), samples.size, _pointer(out)))
        return out
