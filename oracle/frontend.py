"""CPU restatement of WhisperEACP's audio front end, in float64 numpy: test
infrastructure only (the checker of the CUDA front end), never part of the
product.  Pinned bit-for-bit-close (1e-12) against the reference's own
scalar code built into oracle/_ref/libref_frontend.so, through the golden
vectors in tests/golden/reference_frontend.npz.

Follows (paths within eyalamirmusic/WhisperEACP):
  periodic_hann, reflect_padded, stft_power, log_mel, normalise,
  mel_spectrogram        Tests/Mel/ScalarMel.h (scalar::*)
  gelu, conv1d, layer_norm, linear, attention, encode
                         Tests/Encoder/Common.h:390-677 (referenceGelu,
                         referenceConv1d, referenceLayerNorm, referenceLinear,
                         referenceAttention, referenceEncode)
"""
from __future__ import annotations

import math

import numpy as np

EPSILON = float(np.float32(1e-5))  # LayerNorm::whisperEpsilon, a float widened


def periodic_hann(length: int) -> np.ndarray:
    n = np.arange(length, dtype=np.float64)
    return 0.5 * (1.0 - np.cos(2.0 * math.pi * n / length))


def reflect_padded(samples: np.ndarray, pad: int) -> np.ndarray:
    """numpy's "reflect": mirrored about the first and last sample."""
    return np.pad(np.asarray(samples, np.float64), pad, mode="reflect")


def stft_power(samples, window, fft_length: int, hop_length: int, frames: int) -> np.ndarray:
    """[frames][bins] power of the textbook DFT of each windowed frame."""
    bins = fft_length // 2 + 1
    padded = reflect_padded(samples, fft_length // 2)
    starts = np.arange(frames) * hop_length
    framed = padded[starts[:, None] + np.arange(fft_length)[None, :]] * window[None, :]
    angle = 2.0 * math.pi * np.outer(np.arange(bins), np.arange(fft_length)) / fft_length
    real = framed @ np.cos(angle).T
    imaginary = -(framed @ np.sin(angle).T)
    return real * real + imaginary * imaginary


def log_mel(power: np.ndarray, filters: np.ndarray) -> np.ndarray:
    """[mels][frames]: log10(max(filters . power, 1e-10))."""
    total = np.asarray(filters, np.float64) @ power.T
    return np.log10(np.maximum(total, 1e-10))


def normalise(values: np.ndarray) -> np.ndarray:
    peak = values.max()
    return (np.maximum(values, peak - 8.0) + 4.0) / 4.0


def mel_spectrogram(samples, filters, fft_length=400, hop_length=160, frames=3000) -> np.ndarray:
    window = periodic_hann(fft_length)
    power = stft_power(np.asarray(samples, np.float32), window, fft_length, hop_length, frames)
    return normalise(log_mel(power, np.asarray(filters, np.float32)))


def gelu(x: np.ndarray) -> np.ndarray:
    from scipy.special import erf
    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def conv1d(x: np.ndarray, weight: np.ndarray, bias: np.ndarray, stride: int) -> np.ndarray:
    """[out][length'] from channel-major [in][length], kernel 3, padding 1."""
    channels_in, length = x.shape
    out_length = (length + 2 - 3) // stride + 1
    padded = np.zeros((channels_in, length + 2))
    padded[:, 1:-1] = x
    w = np.asarray(weight, np.float64)  # [out][in][3]
    taps = np.stack([padded[:, t + stride * np.arange(out_length)] for t in range(3)], axis=-1)  # [in][out_len][3]
    return np.tensordot(w, taps, axes=([1, 2], [0, 2])) + np.asarray(bias, np.float64)[:, None]


def layer_norm(rows: np.ndarray, weight, bias) -> np.ndarray:
    mean = rows.mean(axis=1, keepdims=True)
    centred = rows - mean
    variance = (centred * centred).sum(axis=1, keepdims=True) / rows.shape[1]
    return centred / np.sqrt(variance + EPSILON) * np.asarray(weight, np.float64) + np.asarray(bias, np.float64)


def linear(x: np.ndarray, weight, bias=None) -> np.ndarray:
    out = x @ np.asarray(weight, np.float64).T
    return out if bias is None else out + np.asarray(bias, np.float64)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, heads: int) -> np.ndarray:
    positions, width = q.shape
    d = width // heads
    out = np.empty_like(q)
    for h in range(heads):
        cols = slice(h * d, (h + 1) * d)
        scores = (q[:, cols] @ k[:, cols].T) / math.sqrt(d)
        scores = np.exp(scores - scores.max(axis=1, keepdims=True))
        out[:, cols] = (scores @ v[:, cols]) / scores.sum(axis=1, keepdims=True)
    return out


def encode(tensors: dict, mel: np.ndarray, heads: int, layers: int) -> np.ndarray:
    """referenceEncode: mel [mel_bins][frames] -> rows [positions][width]."""
    t = {k: np.asarray(v, np.float64) for k, v in tensors.items()}
    e = "model.encoder."
    x = gelu(conv1d(np.asarray(mel, np.float64), t[e + "conv1.weight"], t[e + "conv1.bias"], 1))
    x = gelu(conv1d(x, t[e + "conv2.weight"], t[e + "conv2.bias"], 2))
    positions = x.shape[1]
    h = x.T + t[e + "embed_positions.weight"][:positions]
    for i in range(layers):
        p = f"{e}layers.{i}."
        n = layer_norm(h, t[p + "self_attn_layer_norm.weight"], t[p + "self_attn_layer_norm.bias"])
        q = linear(n, t[p + "self_attn.q_proj.weight"], t[p + "self_attn.q_proj.bias"])
        k = linear(n, t[p + "self_attn.k_proj.weight"])
        v = linear(n, t[p + "self_attn.v_proj.weight"], t[p + "self_attn.v_proj.bias"])
        h = h + linear(attention(q, k, v, heads), t[p + "self_attn.out_proj.weight"], t[p + "self_attn.out_proj.bias"])
        n = layer_norm(h, t[p + "final_layer_norm.weight"], t[p + "final_layer_norm.bias"])
        f = gelu(linear(n, t[p + "fc1.weight"], t[p + "fc1.bias"]))
        h = h + linear(f, t[p + "fc2.weight"], t[p + "fc2.bias"])
    return layer_norm(h, t[e + "layer_norm.weight"], t[e + "layer_norm.bias"])


# ------------------------------------------------------------ test inputs

# The seeded inputs live with the package's other synthetic inputs (the
# bench draws them too); re-exported here under the names the tests use.
from whispereacp_b200.synthetic import (encoder_extents, encoder_tensor_names,  # noqa: E402,F401
                                        synthetic_audio, synthetic_encoder_tensors, synthetic_filters)
