"""Shared pieces of the GPU parity tests: rounding the oracle's inputs to what
the CUDA path stores, building decoders, and the error measures."""
from __future__ import annotations

import numpy as np

from oracle import oracle as O

# The 16-bit tensors the CUDA decoder narrows (every projection matrix and the
# token table); biases, layer norms and the positional table stay fp32.
NARROWED = ("proj.weight", "fc1.weight", "fc2.weight", "embed_tokens.weight")


def round_to(storage: str, values: np.ndarray) -> np.ndarray:
    values = np.asarray(values, dtype=np.float32)
    if storage == "float16":
        return values.astype(np.float16).astype(np.float32)
    bits = values.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    return rounded.astype(np.uint32).view(np.float32)


def stored_tensors(tensors: dict, storage: str) -> dict:
    """The tensors as the CUDA path holds them, widened back to fp32 for the oracle."""
    return {name: (round_to(storage, v) if name.endswith(NARROWED) else v)
            for name, v in tensors.items()}


def shape_of(o: O.Shape):
    from whispereacp_b200 import DecoderShape
    return DecoderShape(**o.__dict__)


def make_decoder(oshape: O.Shape, tensors: dict, storage: str = "float16", windows: int = 1,
                 products: str = "auto"):
    from whispereacp_b200 import Decoder
    decoder = Decoder(shape_of(oshape), windows=windows, storage=storage, products=products)
    decoder.load_weights(tensors)
    return decoder


def worst_error(actual, expected) -> float:
    """worstError, Tests/Encoder/Common.h:731-749: max |a - e| / (1 + |e|)."""
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    return float(np.max(np.abs(actual - expected) / (1.0 + np.abs(expected))))


def max_abs(actual, expected) -> float:
    return float(np.max(np.abs(np.asarray(actual, np.float64) - np.asarray(expected, np.float64))))


def top2_margin(logits: np.ndarray, mask: np.ndarray | None = None) -> np.ndarray:
    """Per row: largest minus second-largest unsuppressed logit."""
    logits = np.atleast_2d(np.asarray(logits, np.float64)).copy()
    if mask is not None:
        logits[:, np.asarray(mask) != 0] = -np.inf
    part = np.sort(logits, axis=1)
    return part[:, -1] - part[:, -2]
