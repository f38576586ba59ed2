"""Seeded synthetic models and inputs for the benchmark configurations.

No checkpoint or dataset is available offline, so every configuration runs on
random-init weights of the named architecture: N(0, 0.02) for every matrix,
embedding and bias, layer-norm gains 1 and offsets 0; encoder outputs N(0, 1).
Normals come from an explicit Box-Muller transform over numpy's PCG64
uniforms, seeded per tensor from a CRC of its name, so the values do not
depend on any library's normal sampler.
"""
from __future__ import annotations

import math
import os
import zlib
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np

from .decoder import DecoderShape

START_OF_TRANSCRIPT = 50257
NO_TIMESTAMPS = 50362
END_OF_TEXT = 50256
LEADING_SPACE = 220


@dataclass(frozen=True)
class RunConfig:
    """One benchmark configuration (the decoder part of it)."""
    name: str
    shape: DecoderShape
    windows: int          # windows on one GPU
    storage: str          # 16-bit type of weights, activations and caches
    prompt: tuple         # prompt token ids
    steps: int            # sampled steps per window (the prompt step included)
    description: str


def _shape(d, heads, layers, vocab=51864):
    return DecoderShape(width=d, heads=heads, layers=layers, feed_forward_width=4 * d,
                        vocabulary_size=vocab, max_positions=448, cross_positions=1500)


ENGLISH_PROMPT = (START_OF_TRANSCRIPT, NO_TIMESTAMPS)
# A multilingual four-special-token prompt: start, language, task, no-timestamps.
MULTILINGUAL_PROMPT = (50258, 50259, 50360, 50364)

CONFIGS = {
    "tiny_en_b1": RunConfig("tiny_en_b1", _shape(384, 6, 4), 1, "float16", ENGLISH_PROMPT, 224,
                            "tiny.en decoder, 1 window"),
    "base_en_b1": RunConfig("base_en_b1", _shape(512, 8, 6), 1, "float16", ENGLISH_PROMPT, 224,
                            "base.en decoder, 1 window"),
    "small_en_b32": RunConfig("small_en_b32", _shape(768, 12, 12), 32, "float16", ENGLISH_PROMPT, 224,
                              "small.en decoder, 32 windows, fp16"),
    "medium_en_b64": RunConfig("medium_en_b64", _shape(1024, 16, 24), 64, "bfloat16", ENGLISH_PROMPT,
                               224, "medium.en decoder, 64 windows, bf16"),
    "large_v3_b128": RunConfig("large_v3_b128", _shape(1280, 20, 32, vocab=51866), 128, "bfloat16",
                               MULTILINGUAL_PROMPT, 444, "large-v3 decoder, 128 windows, bf16"),
}


def _seed(name: str, base_seed: int) -> int:
    return (zlib.crc32(name.encode()) ^ (base_seed * 0x9E3779B1)) & 0xFFFFFFFF


def box_muller(count: int, seed: int, std: float = 1.0) -> np.ndarray:
    """count normals N(0, std^2) from PCG64 uniforms, cos branch of Box-Muller."""
    rng = np.random.Generator(np.random.PCG64(seed))
    u1 = 1.0 - rng.random(count)  # (0, 1]
    u2 = rng.random(count)
    return (std * np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)).astype(np.float32)


def decoder_tensor_extents(shape: DecoderShape) -> dict[str, tuple[int, ...]]:
    """Every decoder tensor of a HuggingFace Whisper checkpoint, with its extents."""
    d, f = shape.width, shape.feed_forward_width
    out = {"model.decoder.embed_tokens.weight": (shape.vocabulary_size, d),
           "model.decoder.embed_positions.weight": (shape.max_positions, d),
           "model.decoder.layer_norm.weight": (d,), "model.decoder.layer_norm.bias": (d,)}
    for layer in range(shape.layers):
        p = f"model.decoder.layers.{layer}."
        for attention, norm in (("self_attn", "self_attn_layer_norm"),
                                ("encoder_attn", "encoder_attn_layer_norm")):
            out[p + norm + ".weight"] = (d,)
            out[p + norm + ".bias"] = (d,)
            for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
                out[p + attention + "." + proj + ".weight"] = (d, d)
                if proj != "k_proj":
                    out[p + attention + "." + proj + ".bias"] = (d,)
        out[p + "final_layer_norm.weight"] = (d,)
        out[p + "final_layer_norm.bias"] = (d,)
        out[p + "fc1.weight"] = (f, d)
        out[p + "fc1.bias"] = (f,)
        out[p + "fc2.weight"] = (d, f)
        out[p + "fc2.bias"] = (d,)
    return out


def normal_weights(shape: DecoderShape, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Random-init decoder: N(0, std) everywhere but layer norms (gain 1, offset 0).

    Each tensor has its own generator, so the tensors are drawn on several
    threads at once (numpy releases the GIL while it fills and transforms)."""
    def draw(item):
        name, extents = item
        count = int(np.prod(extents))
        if "layer_norm" in name:
            return name, np.full(extents, 1.0 if name.endswith("weight") else 0.0, np.float32)
        return name, box_muller(count, _seed(name, seed), std).reshape(extents)

    items = list(decoder_tensor_extents(shape).items())
    with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as pool:
        return dict(pool.map(draw, items))


def encoder_output(windows: int, positions: int, width: int, seed: int = 1) -> np.ndarray:
    """Seeded N(0, 1) stand-in for the encoder's output, [windows, positions, width]."""
    return box_muller(windows * positions * width, _seed("encoder_output", seed)).reshape(
        windows, positions, width)


def teacher_tokens(count: int, seed: int = 2, high: int = END_OF_TEXT) -> np.ndarray:
    """Seeded uniform token ids in [0, high] for teacher-forced steps."""
    rng = np.random.Generator(np.random.PCG64(_seed("teacher_tokens", seed)))
    return rng.integers(0, high + 1, size=count, dtype=np.int64).astype(np.uint32)


def suppression_masks(vocabulary: int, seed: int = 3) -> tuple[np.ndarray, np.ndarray]:
    """(first-step mask, later-step mask) in the shape of Whisper's generation config.

    The later mask suppresses 90 ids -- <|startoftranscript|> and 89 seeded ids
    below <|endoftext|> -- at every step; the first mask adds the two
    begin-suppress ids, a leading space and <|endoftext|>
    (Tests/Whisper/WhisperTests.cpp:171-213 states the rule).
    """
    rng = np.random.Generator(np.random.PCG64(_seed("suppress_tokens", seed)))
    candidates = np.setdiff1d(np.arange(1, END_OF_TEXT), [LEADING_SPACE])
    ids = np.concatenate([[START_OF_TRANSCRIPT], rng.choice(candidates, 89, replace=False)])
    later = np.zeros(vocabulary, np.float32)
    later[ids[ids < vocabulary]] = 1.0
    first = later.copy()
    first[[LEADING_SPACE, END_OF_TEXT]] = 1.0
    return first, later


# --------------------------------------------- the audio front end's inputs

def encoder_tensor_names(layers: int) -> list[str]:
    e = "model.encoder."
    names = [e + "conv1.weight", e + "conv1.bias", e + "conv2.weight", e + "conv2.bias",
             e + "embed_positions.weight", e + "layer_norm.weight", e + "layer_norm.bias"]
    for i in range(layers):
        p = f"{e}layers.{i}."
        names += [p + s for s in ("self_attn_layer_norm.weight", "self_attn_layer_norm.bias",
                                  "self_attn.q_proj.weight", "self_attn.q_proj.bias", "self_attn.k_proj.weight",
                                  "self_attn.v_proj.weight", "self_attn.v_proj.bias", "self_attn.out_proj.weight",
                                  "self_attn.out_proj.bias", "final_layer_norm.weight", "final_layer_norm.bias",
                                  "fc1.weight", "fc1.bias", "fc2.weight", "fc2.bias")]
    return names


def encoder_extents(name: str, mel_bins: int, width: int, ffn: int, positions: int) -> tuple[int, ...]:
    tail = name.split(".", 2)[2] if name.startswith("model.encoder.") else name
    if tail.startswith("layers."):
        tail = tail.split(".", 2)[2]
    table = {
        "conv1.weight": (width, mel_bins, 3), "conv2.weight": (width, width, 3),
        "embed_positions.weight": (positions, width),
        "self_attn.q_proj.weight": (width, width), "self_attn.k_proj.weight": (width, width),
        "self_attn.v_proj.weight": (width, width), "self_attn.out_proj.weight": (width, width),
        "fc1.weight": (ffn, width), "fc1.bias": (ffn,), "fc2.weight": (width, ffn),
    }
    return table.get(tail, (width,))


def synthetic_encoder_tensors(mel_bins: int, width: int, layers: int, ffn: int, positions: int,
                              seed: int = 7, scale: float = 0.05) -> dict[str, np.ndarray]:
    """Seeded weights in the ranges a trained encoder's sit in: matrices and
    biases N(0, scale), LayerNorm gains 1 + N(0, scale), offsets N(0, scale),
    the positional rows N(0, 0.5)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for name in encoder_tensor_names(layers):
        shape = encoder_extents(name, mel_bins, width, ffn, positions)
        values = rng.normal(0.0, 0.5 if "embed_positions" in name else scale, size=shape)
        if name.endswith("norm.weight"):
            values = 1.0 + values
        out[name] = values.astype(np.float32)
    return out


def synthetic_filters(mel_bins: int, bins: int = 201, seed: int = 5) -> np.ndarray:
    """Triangular filters over the bins, like a mel filterbank's shape."""
    centres = np.linspace(1.0, bins - 2.0, mel_bins + 2)
    b = np.arange(bins, dtype=np.float64)
    out = np.zeros((mel_bins, bins))
    for m in range(mel_bins):
        lo, mid, hi = centres[m], centres[m + 1], centres[m + 2]
        up = (b - lo) / max(mid - lo, 1e-9)
        down = (hi - b) / max(hi - mid, 1e-9)
        out[m] = np.maximum(0.0, np.minimum(up, down)) * 2.0 / max(hi - lo, 1e-9)
    return out.astype(np.float32)


def synthetic_audio(count: int, seed: int = 3) -> np.ndarray:
    """Three seeded sinusoids (100-4000 Hz) and N(0, 0.05) noise at 16 kHz,
    clipped to [-1, 1]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    t = np.arange(count) / 16000.0
    x = np.zeros(count)
    for _ in range(3):
        x += rng.uniform(0.1, 0.4) * np.sin(2 * math.pi * rng.uniform(100, 4000) * t + rng.uniform(0, 2 * math.pi))
    x += rng.normal(0.0, 0.05, count)
    return np.clip(x, -1.0, 1.0).astype(np.float32)
