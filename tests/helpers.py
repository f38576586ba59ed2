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
    # round to nearest even on the top 16 bits (finite values: the sum
    # cannot wrap below the NaN patterns)
    bits = values.view(np.uint32)
    rounded = (bits + np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return rounded.view(np.float32)


def stored_tensors(tensors: dict, storage: str) -> dict:
    """The tensors as the CUDA path holds them, widened back to fp32 for the oracle."""
    from concurrent.futures import ThreadPoolExecutor
    import os

    def one(item):
        name, v = item
        return name, (round_to(storage, v) if name.endswith(NARROWED) else v)

    with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as pool:
        return dict(pool.map(one, tensors.items()))


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
