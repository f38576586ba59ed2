"""Every benchmark architecture's decoder against the oracle, at the sizes
the configurations run: small.en (fp16, 32 windows), medium.en (bf16, 64
windows, both product forms), large-v3 (bf16, vocabulary 51866, 20 heads,
the 4-token multilingual prompt) over a whole 448-position window, and
large-v3 at 128 windows, where the decoder picks the tcgen05 products by
itself.  tiny.en runs configuration C1 as stated: the prompt, then 224
teacher-forced steps.

Teacher forcing as the reference's decoder tests do it (Tests/Decoder/
DecoderTests.cpp:117-148): a prompt step, then one token a step; each
window's logits against the double-precision oracle (Tests/Decoder/
Common.h:360-468) on the same 16-bit weights and the same encoder rows.
Logits must agree within max-abs 2e-2, and every row's greedy id must equal
the oracle's wherever the oracle's top-2 margin exceeds 5e-2.

Past 224 keys a single window's self attention leaves its one-round-trip
form for the general one (scores, then weights, then values over the whole
row); the 226- and 448-position runs go through it.
"""
import functools
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import make_decoder, max_abs, stored_tensors, top2_margin
from whispereacp_b200 import synthetic as S

pytestmark = pytest.mark.gpu

LOGIT_MAX_ABS = 2e-2
MARGIN = 5e-2
THREADS = max(1, min(32, os.cpu_count() or 1))


def oracle_shape(shape) -> O.Shape:
    return O.Shape(**shape.__dict__)


@functools.lru_cache(maxsize=1)
def model(config: str, storage: str, seed: int):
    """The configuration's random-init weights as the CUDA path stores them."""
    run = S.CONFIGS[config]
    return stored_tensors(S.normal_weights(run.shape, seed=seed), storage)


def teacher_ids(windows: int, prompt, steps: int, seed: int) -> np.ndarray:
    ids = np.empty((windows, len(prompt) + steps), np.uint32)
    ids[:, :len(prompt)] = prompt
    for b in range(windows):
        ids[b, len(prompt):] = S.teacher_tokens(steps, seed=seed + b)
    return ids


def run_teacher_forced(config: str, storage: str, windows: int, steps: int, checked,
                       products: str = "auto", seed: int = 70):
    """Decodes `windows` windows teacher-forced (prompt, then `steps` single
    tokens) and checks the windows in `checked` against the oracle."""
    run = S.CONFIGS[config]
    shape = run.shape
    tensors = model(config, storage, seed)
    encoders = S.encoder_output(windows, shape.cross_positions, shape.width, seed=seed + 1)
    ids = teacher_ids(windows, run.prompt, steps, seed + 2)
    p = len(run.prompt)

    decoder = make_decoder(oracle_shape(shape), tensors, storage, windows=windows, products=products)
    decoder.begin_sequence(encoders)
    logits = np.empty((len(checked), p + steps, shape.vocabulary_size), np.float32)
    argmax = np.empty((len(checked), p + steps), np.uint32)
    cols = [slice(0, p)] + [slice(k, k + 1) for k in range(p, p + steps)]
    for cut in cols:
        result = decoder.step(ids[:, cut], hidden=False)
        logits[:, cut] = result.logits[list(checked)]
        argmax[:, cut] = result.argmax[list(checked)]
    assert decoder.position == p + steps
    decoder.close()

    worst, decided = 0.0, 0
    for i, b in enumerate(checked):
        _, expected = O.reference_decode(oracle_shape(shape), tensors, encoders[b], ids[b], threads=THREADS)
        err = max_abs(logits[i], expected)
        worst = max(worst, err)
        assert err <= LOGIT_MAX_ABS, (b, err, int(np.argmax(np.max(np.abs(logits[i] - expected), axis=1))))
        wanted = O.masked_argmax(expected)
        margins = top2_margin(expected)
        sure = margins > MARGIN
        wrong = np.nonzero(sure & (argmax[i] != wanted))[0]
        assert wrong.size == 0, (b, wrong[:8], margins[wrong[:8]])
        decided += int(sure.sum())
    print(f"  {config} {storage} {windows} windows ({products}): {p + steps} positions, "
          f"logits max-abs {worst:.3g}, {decided} greedy ids decided by the margin")
    return worst


def test_tiny_en_configuration_c1():
    """C1 as stated: tiny.en, the prompt [50257, 50362], then 224 teacher-forced
    steps (226 positions, so the last steps attend over more than 224 keys)."""
    run_teacher_forced("tiny_en_b1", "float16", windows=1, steps=224, checked=[0])


@pytest.mark.parametrize("storage", ["float16", "bfloat16"])
def test_base_en_past_224_keys(storage):
    """base.en at batch 1, the bench's single-window path, out to 240 positions."""
    run_teacher_forced("base_en_b1", storage, windows=1, steps=238, checked=[0])


def test_small_en_one_window():
    run_teacher_forced("small_en_b32", "float16", windows=1, steps=24, checked=[0])


def test_small_en_thirty_two_windows():
    """Configuration C3's batch: 32 windows, fp16."""
    run_teacher_forced("small_en_b32", "float16", windows=32, steps=5, checked=[0, 13, 31])


def test_medium_en_one_window():
    run_teacher_forced("medium_en_b64", "bfloat16", windows=1, steps=24, checked=[0])


@pytest.mark.parametrize("products", ["auto", "tcgen05"])
def test_medium_en_sixty_four_windows(products):
    """Configuration C4's batch: 64 windows, bf16, with the products the
    decoder picks (mma.sync at 64 windows) and with tcgen05 forced."""
    run_teacher_forced("medium_en_b64", "bfloat16", windows=64, steps=5, checked=[0, 37, 63],
                       products=products)


def test_large_v3_whole_window():
    """large-v3, one window: the 4-token prompt, then 444 single-token steps --
    all 448 positions of the self-attention cache."""
    run_teacher_forced("large_v3_b128", "bfloat16", windows=1, steps=444, checked=[0])


def test_large_v3_128_windows_pick_the_tensor_core_products():
    """Configuration C5's batch: 128 windows, where the decoder's own choice is
    the tcgen05 products; three windows checked against the oracle."""
    run_teacher_forced("large_v3_b128", "bfloat16", windows=128, steps=3, checked=[0, 64, 127])
