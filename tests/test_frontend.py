"""The audio front end: the log-mel spectrogram and the encoder.

CPU: the numpy restatement (oracle/frontend.py) against the reference's own
scalar mel (Tests/Mel/ScalarMel.h) and scalar encoder (Tests/Encoder/
Common.h:569-677), through tests/golden/reference_frontend.npz.

GPU (through include/wsp_encoder.h):
  - the normalised log-mel within 1e-4 of the oracle, the bound of the
    reference's own MelSpectrogramTests.cpp:116, for a full recording and a
    short one with silence after it;
  - the encoder rows against the oracle on the same 16-bit weights: max-abs
    within 1e-4 on LayerNorm-ed rows (|x| up to ~5) -- the products carry
    the rows as 16-bit hi + lo pairs, the attention is fp32 -- for the
    reference's own test input (64 frames) and for a whole 30 s window of
    base.en's width (1500 positions, 8 heads);
  - samples -> rows equals log_mel then encode; the refusals.
"""
import os

import numpy as np
import pytest

from oracle import frontend as FE

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_frontend.npz")
MEL_TOLERANCE = 1e-4
ROWS_TOLERANCE = 1e-4
SMALL = dict(mel_bins=80, width=128, heads=2, layers=2, ffn=256, input_frames=64)


def golden():
    return np.load(GOLDEN)


def test_golden_inputs_are_the_ones_drawn_here():
    g = golden()
    positions = (SMALL["input_frames"] - 1) // 2 + 1
    tensors = FE.synthetic_encoder_tensors(SMALL["mel_bins"], SMALL["width"], SMALL["layers"], SMALL["ffn"], positions)
    short = np.zeros(48 * 160, np.float32)
    short[:5000] = FE.synthetic_audio(5000, seed=4)
    sums = [FE.synthetic_filters(80).astype(np.float64).sum(), FE.synthetic_audio(48 * 160).astype(np.float64).sum(),
            short.astype(np.float64).sum(), sum(t.astype(np.float64).sum() for t in tensors.values())]
    np.testing.assert_allclose(sums, g["inputs_checksum"], rtol=0, atol=1e-9)


def test_oracle_mel_matches_the_reference_scalar_mel():
    g = golden()
    filters = FE.synthetic_filters(80)
    mel = FE.mel_spectrogram(FE.synthetic_audio(48 * 160), filters, frames=48)
    assert np.abs(mel - g["mel_audio"]).max() < 1e-11
    short = np.zeros(48 * 160, np.float32)
    short[:5000] = FE.synthetic_audio(5000, seed=4)
    assert np.abs(FE.mel_spectrogram(short, filters, frames=48) - g["mel_short"]).max() < 1e-11


def test_oracle_encoder_matches_the_reference_scalar_encoder():
    g = golden()
    positions = (SMALL["input_frames"] - 1) // 2 + 1
    tensors = FE.synthetic_encoder_tensors(SMALL["mel_bins"], SMALL["width"], SMALL["layers"], SMALL["ffn"], positions)
    rows = FE.encode(tensors, g["encoder_mel"], SMALL["heads"], SMALL["layers"])
    assert np.abs(rows - g["encoder_rows"]).max() < 1e-11


def rounded(tensors: dict, storage: str) -> dict:
    """The weights as the CUDA encoder holds them (products' matrices 16-bit)."""
    from tests.helpers import round_to
    out = {}
    for name, values in tensors.items():
        matrix = name.endswith(("proj.weight", "fc1.weight", "fc2.weight", "conv1.weight", "conv2.weight"))
        out[name] = round_to(storage, values) if matrix else values
    return out


def make_encoder(shape_args, tensors, filters=None, storage="float16"):
    from whispereacp_b200 import Encoder, EncoderShape
    shape = EncoderShape(shape_args["mel_bins"], shape_args["width"], shape_args["heads"], shape_args["layers"],
                         shape_args["ffn"], shape_args["input_frames"])
    encoder = Encoder(shape, storage=storage)
    encoder.load_weights(tensors)
    if filters is not None:
        encoder.set_filters(filters)
    return encoder


@pytest.mark.gpu
def test_log_mel_matches_the_oracle():
    g = golden()
    filters = FE.synthetic_filters(80)
    args = dict(SMALL, input_frames=48)
    positions = (48 - 1) // 2 + 1
    tensors = FE.synthetic_encoder_tensors(80, SMALL["width"], SMALL["layers"], SMALL["ffn"], positions)
    encoder = make_encoder(args, tensors, filters)
    full = encoder.log_mel(FE.synthetic_audio(48 * 160))
    worst = np.abs(full - g["mel_audio"]).max()
    print(f"  log-mel max-abs {worst:.3g}")
    assert worst <= MEL_TOLERANCE
    # A shorter recording: the rest of the window is silence.
    short = encoder.log_mel(FE.synthetic_audio(5000, seed=4))
    assert np.abs(short - g["mel_short"]).max() <= MEL_TOLERANCE


@pytest.mark.gpu
@pytest.mark.parametrize("storage", ["float16", "bfloat16"])
def test_encoder_matches_the_oracle_on_the_reference_input(storage):
    g = golden()
    positions = (SMALL["input_frames"] - 1) // 2 + 1
    tensors = FE.synthetic_encoder_tensors(SMALL["mel_bins"], SMALL["width"], SMALL["layers"], SMALL["ffn"], positions)
    held = rounded(tensors, storage)
    encoder = make_encoder(SMALL, tensors, storage=storage)
    rows = encoder.encode(g["encoder_mel"])
    expected = FE.encode(held, g["encoder_mel"], SMALL["heads"], SMALL["layers"])
    worst = np.abs(rows - expected).max()
    print(f"  encoder {storage} max-abs {worst:.3g} (rows up to {np.abs(expected).max():.2f})")
    assert worst <= ROWS_TOLERANCE


@pytest.mark.gpu
def test_encoder_over_a_whole_window_at_base_width():
    """1500 positions, 8 heads of 64, 512 wide: every tile shape the products
    and the attention meet at base.en, two layers."""
    args = dict(mel_bins=80, width=512, heads=8, layers=2, ffn=2048, input_frames=3000)
    tensors = FE.synthetic_encoder_tensors(80, 512, 2, 2048, 1500, seed=11, scale=0.03)
    filters = FE.synthetic_filters(80)
    encoder = make_encoder(args, tensors, filters)
    audio = FE.synthetic_audio(16000 * 12, seed=12)  # 12 s, then silence
    mel = encoder.log_mel(audio)
    expected_mel = FE.mel_spectrogram(np.pad(audio, (0, 480000 - audio.size)), filters, frames=3000)
    assert np.abs(mel - expected_mel).max() <= MEL_TOLERANCE
    rows = encoder.encode(mel)
    expected = FE.encode(rounded(tensors, "float16"), mel, 8, 2)
    worst = np.abs(rows - expected).max()
    print(f"  base-width encoder max-abs {worst:.3g}")
    assert worst <= ROWS_TOLERANCE
    # samples -> rows in one call equals the two calls.
    np.testing.assert_array_equal(encoder.encode_samples(audio), rows)


@pytest.mark.gpu
def test_the_refusals():
    from whispereacp_b200 import Encoder, EncoderShape, ModelError
    with pytest.raises(ModelError, match="64-wide"):
        Encoder(EncoderShape(80, 96, 2, 1, 256, 64))
    positions = 32
    tensors = FE.synthetic_encoder_tensors(80, 128, 1, 256, positions)
    encoder = Encoder(EncoderShape(80, 128, 2, 1, 256, 64))
    with pytest.raises(ModelError, match="no tensor model.encoder.conv1.weight"):
        encoder.encode(np.zeros((80, 64), np.float32))
    with pytest.raises(ModelError, match="wrong shape"):
        encoder.set_tensor("model.encoder.conv1.weight", np.zeros((128, 80, 2), np.float32))
    with pytest.raises(ModelError, match="not one this encoder reads"):
        encoder.set_tensor("model.encoder.layers.0.mlp.weight", np.zeros(4, np.float32))
    encoder.load_weights(tensors)
    with pytest.raises(ModelError, match="no mel filterbank"):
        encoder.log_mel(np.zeros(1000, np.float32))
    encoder.set_filters(FE.synthetic_filters(80))
    with pytest.raises(ModelError, match="2 to 10240 samples"):
        encoder.log_mel(np.zeros(64 * 160 + 1, np.float32))
