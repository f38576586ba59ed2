"""Writes tests/golden/reference_decoder.npz from the reference's own code.

Run where the WhisperEACP checkout is (it needs oracle/_ref/, which
oracle/Makefile compiles from the reference's sources):

    make -C oracle REF=<reference checkout> && python tests/golden/make_golden.py

Every array in the fixture comes out of the reference's scalar test decoder
(Tests/Decoder/Common.h:258-500 with Tests/Encoder/Common.h:390-507) or its
fp16 narrowing (Lib/WhisperEACP/Core/Utils/Half.cpp), compiled from the
reference's lines.  The inputs are the reference's own test inputs:
smallDecoderShape, syntheticDecoderFile's seeds, syntheticEncoderOutput, the
prompts of Tests/Decoder/DecoderTests.cpp.  The weights are drawn by
oracle.synthetic_decoder_tensors, whose draws are themselves checked here
against the reference's spreadValues.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

F = ctypes.POINTER(ctypes.c_float)
D = ctypes.POINTER(ctypes.c_double)
I = ctypes.POINTER(ctypes.c_int)

# A shape with Whisper's 64-wide heads, small enough for the scalar reference.
MID_SHAPE = O.Shape(width=128, heads=2, layers=2, feed_forward_width=512, vocabulary_size=300,
                    max_positions=32, cross_positions=40)
MID_TOKENS = [250, 7, 99, 3, 281, 12]


def load_reference():
    ref = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_decoder.so"))
    ref.ref_decode.argtypes = [I, ctypes.POINTER(F), F, I, ctypes.c_int, D, D]
    ref.ref_spread_values.argtypes = [F, ctypes.c_int, ctypes.c_uint, ctypes.c_float]
    ref.ref_synthetic_encoder_output.argtypes = [F, ctypes.c_int, ctypes.c_int]
    half = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_half.so"))
    half.ref_pack_half.argtypes = [ctypes.c_float]
    half.ref_pack_half.restype = ctypes.c_uint16
    return ref, half


def ref_decode(ref, shape, tensors, encoder, tokens):
    held = O._Tensors(shape, tensors)
    fields = (ctypes.c_int * 7)(shape.width, shape.heads, shape.layers, shape.feed_forward_width,
                                shape.vocabulary_size, shape.max_positions, shape.cross_positions)
    encoder = np.ascontiguousarray(encoder, np.float32)
    ids = np.ascontiguousarray(tokens, np.int32)
    hidden = np.empty((len(ids), shape.width))
    logits = np.empty((len(ids), shape.vocabulary_size))
    ref.ref_decode(fields, held.pointers, encoder.ctypes.data_as(F), ids.ctypes.data_as(I), len(ids),
                   hidden.ctypes.data_as(D), logits.ctypes.data_as(D))
    return hidden, logits


def main() -> None:
    ref, half = load_reference()
    out = {}

    spread = np.empty(2048, np.float32)
    ref.ref_spread_values(spread.ctypes.data_as(F), spread.size, 2000, 0.3)
    out["spread_2000_0p3"] = spread

    shape = O.SMALL_SHAPE
    tensors = O.synthetic_decoder_tensors(shape)
    encoder = np.empty((shape.cross_positions, shape.width), np.float32)
    ref.ref_synthetic_encoder_output(encoder.ctypes.data_as(F), shape.cross_positions, shape.width)
    out["small_encoder"] = encoder

    # Decoder/promptMatchesReference and cachedStepsMatchTheReference.
    out["small_prompt_hidden"], out["small_prompt_logits"] = ref_decode(
        ref, shape, tensors, encoder, O.SMALL_PROMPT)

    # Decoder/mixedStepsAndASecondSequence: -0.5 e + 0.25, tokens {7, 2, 9}.
    second = (-0.5 * encoder + 0.25).astype(np.float32)
    out["small_second_hidden"], out["small_second_logits"] = ref_decode(
        ref, shape, tensors, second, [7, 2, 9])

    # Decoder/reducedCrossPositionsMatchTheShorterShape: 3 of 6 rows, prompt + its first id.
    shorter = O.Shape(**{**shape.__dict__, "cross_positions": shape.cross_positions // 2})
    reduced = np.empty((shorter.cross_positions, shape.width), np.float32)
    ref.ref_synthetic_encoder_output(reduced.ctypes.data_as(F), shorter.cross_positions, shape.width)
    out["small_reduced_hidden"], out["small_reduced_logits"] = ref_decode(
        ref, shorter, tensors, reduced, O.SMALL_PROMPT + [O.SMALL_PROMPT[0]])

    # A shape with 64-wide heads.
    mid = O.synthetic_decoder_tensors(MID_SHAPE, first_seed=7000)
    mid_encoder = np.empty((MID_SHAPE.cross_positions, MID_SHAPE.width), np.float32)
    ref.ref_synthetic_encoder_output(mid_encoder.ctypes.data_as(F), MID_SHAPE.cross_positions,
                                     MID_SHAPE.width)
    out["mid_hidden"], out["mid_logits"] = ref_decode(ref, MID_SHAPE, mid, mid_encoder, MID_TOKENS)

    # fp16 narrowing of the reference (Half.cpp): normals, subnormals, ties, overflow.
    probes = np.concatenate([
        spread,
        np.array([0.0, -0.0, 1.0, -2.5, 65504.0, 65520.0, 65519.0, 1e6, -1e6, 6.1035156e-05,
                  5.9604645e-08, 2.9802322e-08, 2.9802326e-08, 1e-9, 1.0009766, 1.0004883,
                  1.0014648, 3.1415927, np.inf, -np.inf], np.float32),
        (np.arange(-2000, 2000, dtype=np.float32) * 1.2345e-3),
    ]).astype(np.float32)
    out["half_probes"] = probes
    out["half_bits"] = np.array([half.ref_pack_half(float(v)) for v in probes], np.uint16)

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_decoder.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
