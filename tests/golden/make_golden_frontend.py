"""Writes tests/golden/reference_frontend.npz from the reference's own code.

Run where the WhisperEACP checkout is (it needs oracle/_ref/libref_frontend.so,
which oracle/Makefile compiles from the reference's sources):

    make -C oracle REF=<reference checkout> && python tests/golden/make_golden_frontend.py

The mel spectrograms come out of the reference's scalar mel
(Tests/Mel/ScalarMel.h, scalar::melSpectrogram), the encoder rows out of its
scalar encoder (Tests/Encoder/Common.h:569-677, referenceEncode) on its own
test input (syntheticMel).  The audio, filterbank and weights are drawn by
oracle.frontend's seeded generators; their checksums are stored so a drift
in the draws is caught before a comparison.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import frontend as FE  # noqa: E402

F = ctypes.POINTER(ctypes.c_float)
D = ctypes.POINTER(ctypes.c_double)
I = ctypes.POINTER(ctypes.c_int)

# The mel cases: 48 frames (7680 samples) of 80 bands; the second recording
# is 5000 samples, silence after it.
MEL_FRAMES, MEL_BINS = 48, 80
SHORT_SAMPLES = 5000
# The encoder case: Whisper's 64-wide heads, 64 input frames (32 positions).
ENCODER = dict(mel_bins=80, width=128, heads=2, layers=2, ffn=256, input_frames=64)


def load_reference():
    ref = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_frontend.so"))
    ref.ref_mel_spectrogram.argtypes = [F, ctypes.c_int, F, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, D]
    ref.ref_encode.argtypes = [I, ctypes.POINTER(F), F, D]
    ref.ref_synthetic_mel.argtypes = [ctypes.c_int, ctypes.c_int, F]
    return ref


def ref_mel(ref, samples, filters, frames):
    samples = np.ascontiguousarray(samples, np.float32)
    filters = np.ascontiguousarray(filters, np.float32)
    out = np.empty((filters.shape[0], frames))
    ref.ref_mel_spectrogram(samples.ctypes.data_as(F), samples.size, filters.ctypes.data_as(F), 400, 160, frames,
                            filters.shape[0], out.ctypes.data_as(D))
    return out


def ref_encode(ref, tensors, mel, e):
    names = FE.encoder_tensor_names(e["layers"])
    positions = (e["input_frames"] - 1) // 2 + 1
    held = [np.ascontiguousarray(tensors[n][:positions] if "embed_positions" in n else tensors[n], np.float32)
            for n in names]
    pointers = (F * len(held))(*[h.ctypes.data_as(F) for h in held])
    fields = (ctypes.c_int * 6)(e["mel_bins"], e["width"], e["heads"], e["layers"], e["ffn"], e["input_frames"])
    mel = np.ascontiguousarray(mel, np.float32)
    out = np.empty((positions, e["width"]))
    ref.ref_encode(fields, pointers, mel.ctypes.data_as(F), out.ctypes.data_as(D))
    return out


def checksum(arrays) -> float:
    return float(sum(np.asarray(a, np.float64).sum() for a in arrays))


def main():
    ref = load_reference()
    filters = FE.synthetic_filters(MEL_BINS)
    audio = FE.synthetic_audio(MEL_FRAMES * 160)
    short = np.zeros(MEL_FRAMES * 160, np.float32)
    short[:SHORT_SAMPLES] = FE.synthetic_audio(SHORT_SAMPLES, seed=4)
    e = ENCODER
    positions = (e["input_frames"] - 1) // 2 + 1
    tensors = FE.synthetic_encoder_tensors(e["mel_bins"], e["width"], e["layers"], e["ffn"], positions)
    mel = np.empty((e["mel_bins"], e["input_frames"]), np.float32)
    ref.ref_synthetic_mel(e["mel_bins"], e["input_frames"], mel.ctypes.data_as(F))
    np.savez_compressed(
        os.path.join(ROOT, "tests", "golden", "reference_frontend.npz"),
        mel_audio=ref_mel(ref, audio, filters, MEL_FRAMES),
        mel_short=ref_mel(ref, short, filters, MEL_FRAMES),
        encoder_mel=mel,
        encoder_rows=ref_encode(ref, tensors, mel, e),
        inputs_checksum=np.array([checksum([filters]), checksum([audio]), checksum([short]),
                                  checksum(tensors.values())]),
    )


if __name__ == "__main__":
    main()
