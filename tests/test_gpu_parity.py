"""The tiny.en and base.en decoders against the oracle (random-init weights).

Teacher forcing: the English prompt [50257, 50362], then seeded uniform ids
in [0, 50256], through the CUDA decoder and the double-precision oracle
(Tests/Decoder/Common.h:360-468) on the same 16-bit weights.  Logits must
agree within max-abs 2e-2 (16-bit weights, fp32 accumulation), and every
greedy id must equal the oracle's wherever the oracle's top-2 margin
exceeds 5e-2.  The greedy search is checked by
replaying the GPU's own transcript through the oracle: each id it chose
must be the oracle's masked argmax wherever the masked margin exceeds 5e-2.
"""
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


def check_tokens(gpu_ids, oracle_logits, mask=None):
    expected = O.masked_argmax(oracle_logits, mask)
    margins = top2_margin(oracle_logits, mask)
    decided = margins > MARGIN
    mismatches = np.nonzero(decided & (np.asarray(gpu_ids) != expected))[0]
    assert mismatches.size == 0, f"rows {mismatches[:8]} differ with margins {margins[mismatches[:8]]}"
    return int(decided.sum())


@pytest.mark.parametrize("config,storage,steps", [
    ("tiny_en_b1", "float16", 24),
    ("tiny_en_b1", "bfloat16", 12),
    ("base_en_b1", "float16", 12),
])
def test_teacher_forced_steps_match_the_oracle(config, storage, steps):
    run = S.CONFIGS[config]
    shape = run.shape
    tensors = stored_tensors(S.normal_weights(shape, seed=11), storage)
    encoder = S.encoder_output(1, shape.cross_positions, shape.width, seed=12)
    ids = [*run.prompt, *S.teacher_tokens(steps, seed=13)]

    session = O.Session(oracle_shape(shape), tensors, threads=THREADS)
    session.begin(encoder[0])
    decoder = make_decoder(oracle_shape(shape), tensors, storage)
    decoder.begin_sequence(encoder)

    p = len(run.prompt)
    worst = 0.0
    decided = 0
    chunks = [ids[:p]] + [[t] for t in ids[p:]]
    for chunk in chunks:
        hidden, logits = session.step(chunk)
        result = decoder.step([chunk])
        worst = max(worst, max_abs(result.logits[0], logits))
        assert max_abs(result.logits[0], logits) <= LOGIT_MAX_ABS
        decided += check_tokens(result.argmax[0], logits)
    print(f"  {config} {storage}: {len(ids)} positions, logits max-abs {worst:.3g}, "
          f"{decided} greedy ids decided by the margin")


@pytest.mark.parametrize("config,storage,steps", [("tiny_en_b1", "float16", 40), ("base_en_b1", "bfloat16", 16)])
def test_greedy_transcript_follows_the_oracle(config, storage, steps):
    run = S.CONFIGS[config]
    shape = run.shape
    tensors = stored_tensors(S.normal_weights(shape, seed=21), storage)
    encoder = S.encoder_output(1, shape.cross_positions, shape.width, seed=22)
    first, later = S.suppression_masks(shape.vocabulary_size)

    decoder = make_decoder(oracle_shape(shape), tensors, storage)
    decoder.set_generation(run.prompt, first, later, maximum_tokens=steps,
                           end_of_text=S.END_OF_TEXT, stop_at_end_of_text=False)
    transcript = decoder.transcribe(encoder)[0]
    assert len(transcript) == steps

    session = O.Session(oracle_shape(shape), tensors, threads=THREADS)
    session.begin(encoder[0])
    _, logits = session.step(list(run.prompt))
    decided = check_tokens([transcript[0]], logits[-1:], first)
    for k in range(1, steps):
        _, logits = session.step([int(transcript[k - 1])])
        decided += check_tokens([transcript[k]], logits, later)
    print(f"  greedy {config}: {steps} ids, {decided} decided by the margin")


def test_transcript_stops_at_end_of_text():
    """decodeTranscript's stop rule (Whisper.cpp:1420-1436): the transcript ends
    before the first end-of-text id, whichever step produced it."""
    run = S.CONFIGS["tiny_en_b1"]
    shape = run.shape
    tensors = stored_tensors(S.normal_weights(shape, seed=31), "float16")
    encoder = S.encoder_output(1, shape.cross_positions, shape.width, seed=32)
    decoder = make_decoder(oracle_shape(shape), tensors)
    decoder.set_generation(run.prompt, maximum_tokens=20, stop_at_end_of_text=False)
    full = decoder.transcribe(encoder)[0]
    assert len(full) == 20
    stop_id = int(full[5])
    first_at = int(np.nonzero(full == stop_id)[0][0])
    decoder.set_generation(run.prompt, maximum_tokens=20, end_of_text=stop_id, stop_at_end_of_text=True)
    stopped = decoder.transcribe(encoder)[0]
    assert np.array_equal(stopped, full[:first_at])


def test_batched_windows_follow_the_oracle():
    """Four windows decoded in lockstep: each window's transcript, replayed
    through the oracle on its own encoder rows, is the oracle's greedy choice
    wherever the margin decides it."""
    run = S.CONFIGS["tiny_en_b1"]
    shape = run.shape
    tensors = stored_tensors(S.normal_weights(shape, seed=41), "float16")
    encoders = S.encoder_output(4, shape.cross_positions, shape.width, seed=42)
    first, later = S.suppression_masks(shape.vocabulary_size)
    batched = make_decoder(oracle_shape(shape), tensors, windows=4)
    batched.set_generation(run.prompt, first, later, maximum_tokens=12, stop_at_end_of_text=False)
    together = batched.transcribe(encoders)
    for b in range(4):
        session = O.Session(oracle_shape(shape), tensors, threads=THREADS)
        session.begin(encoders[b])
        _, logits = session.step(list(run.prompt))
        check_tokens([together[b][0]], logits[-1:], first)
        for k in range(1, 12):
            _, logits = session.step([int(together[b][k - 1])])
            check_tokens([together[b][k]], logits, later)


@pytest.mark.parametrize("products", ["mma", "tcgen05"])
def test_wide_batched_windows_follow_the_oracle(products):
    """Forty windows of a 1024-wide decoder with the full vocabulary: 32 KB
    weight-stream stages leave room for fewer stages than warps, the logits
    run as two row tiles with each warp owning every seventh vocabulary tile;
    both product forms.
    Each window's
    transcript, replayed through the oracle, is its greedy choice wherever
    the margin decides it."""
    from whispereacp_b200.decoder import DecoderShape
    shape = DecoderShape(width=1024, heads=16, layers=1, feed_forward_width=1024, vocabulary_size=51864,
                         max_positions=32, cross_positions=24)
    windows, steps = 40, 5
    prompt = S.CONFIGS["medium_en_b64"].prompt
    tensors = stored_tensors(S.normal_weights(shape, seed=51), "float16")
    encoders = S.encoder_output(windows, shape.cross_positions, shape.width, seed=52)
    first, later = S.suppression_masks(shape.vocabulary_size)
    batched = make_decoder(oracle_shape(shape), tensors, windows=windows, products=products)
    batched.set_generation(prompt, first, later, maximum_tokens=steps, stop_at_end_of_text=False)
    together = batched.transcribe(encoders)
    decided = 0
    for b in range(windows):
        session = O.Session(oracle_shape(shape), tensors, threads=THREADS)
        session.begin(encoders[b])
        _, logits = session.step(list(prompt))
        decided += check_tokens([together[b][0]], logits[-1:], first)
        for k in range(1, steps):
            _, logits = session.step([int(together[b][k - 1])])
            decided += check_tokens([together[b][k]], logits, later)
    assert decided > windows * steps // 2


@pytest.mark.parametrize("storage", ["float16", "bfloat16"])
def test_tensor_core_products_match_the_oracle(storage):
    """Thirty-two windows with the products as tcgen05 tiles (128 weight rows
    against every window's row, accumulated in tensor memory, split along K
    and joined).  Teacher-forced
    logits of every window match its own oracle sequence within max-abs 2e-2."""
    run = S.CONFIGS["tiny_en_b1"]
    shape = run.shape
    windows = 32
    tensors = stored_tensors(S.normal_weights(shape, seed=61), storage)
    encoders = S.encoder_output(windows, shape.cross_positions, shape.width, seed=62)
    rng = np.random.default_rng(63)
    ids = rng.integers(0, 50256, size=(windows, 5)).astype(np.uint32)
    ids[:, :2] = run.prompt
    decoder = make_decoder(oracle_shape(shape), tensors, storage, windows=windows, products="tcgen05")
    decoder.begin_sequence(encoders)
    steps = [decoder.step(ids[:, :2])] + [decoder.step(ids[:, k:k + 1]) for k in range(2, 5)]
    worst = 0.0
    for b in range(0, windows, 5):
        session = O.Session(oracle_shape(shape), tensors, threads=THREADS)
        session.begin(encoders[b])
        chunks = [list(ids[b, :2])] + [[int(ids[b, k])] for k in range(2, 5)]
        for result, chunk in zip(steps, chunks):
            _, logits = session.step([int(t) for t in chunk])
            err = max_abs(result.logits[b], logits)
            worst = max(worst, err)
            assert err <= LOGIT_MAX_ABS, (b, err)
            check_tokens(result.argmax[b], logits)
    print(f"  tensor-core products {storage}: logits max-abs {worst:.3g}")
