"""The CPU oracle, pinned before anything is checked against it.

The fixture tests/golden/reference_decoder.npz was written by the reference's
own scalar test decoder, compiled from its sources (tests/golden/make_golden.py);
the oracle must reproduce it to the last bit.  The self-checks after it are
the reference's own tests of that decoder (Tests/Decoder/
ReferenceDecoderTests.cpp:45-155), run on the oracle.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.golden.make_golden import MID_SHAPE, MID_TOKENS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def small():
    shape = O.SMALL_SHAPE
    return shape, O.synthetic_decoder_tensors(shape), O.synthetic_encoder_output(
        shape.cross_positions, shape.width)


def test_spread_values_are_the_references(golden):
    assert np.array_equal(O.spread_values(2048, 2000, 0.3), golden["spread_2000_0p3"])


def test_synthetic_encoder_output_is_the_references(golden):
    shape = O.SMALL_SHAPE
    assert np.array_equal(O.synthetic_encoder_output(shape.cross_positions, shape.width),
                          golden["small_encoder"])


def test_prompt_decoding_is_bit_identical(golden):
    shape, tensors, encoder = small()
    hidden, logits = O.reference_decode(shape, tensors, encoder, O.SMALL_PROMPT)
    assert np.array_equal(hidden, golden["small_prompt_hidden"])
    assert np.array_equal(logits, golden["small_prompt_logits"])


def test_second_sequence_is_bit_identical(golden):
    shape, tensors, encoder = small()
    second = (-0.5 * encoder + 0.25).astype(np.float32)
    hidden, logits = O.reference_decode(shape, tensors, second, [7, 2, 9])
    assert np.array_equal(hidden, golden["small_second_hidden"])
    assert np.array_equal(logits, golden["small_second_logits"])


def test_reduced_cross_positions_is_bit_identical(golden):
    shape, tensors, _ = small()
    rows = shape.cross_positions // 2
    encoder = O.synthetic_encoder_output(rows, shape.width)
    hidden, logits = O.reference_decode(shape, tensors, encoder, O.SMALL_PROMPT + [O.SMALL_PROMPT[0]],
                                        cross_rows=rows)
    assert np.array_equal(hidden, golden["small_reduced_hidden"])
    assert np.array_equal(logits, golden["small_reduced_logits"])


def test_sixty_four_wide_heads_are_bit_identical(golden):
    tensors = O.synthetic_decoder_tensors(MID_SHAPE, first_seed=7000)
    encoder = O.synthetic_encoder_output(MID_SHAPE.cross_positions, MID_SHAPE.width)
    hidden, logits = O.reference_decode(MID_SHAPE, tensors, encoder, MID_TOKENS, threads=4)
    assert np.array_equal(hidden, golden["mid_hidden"])
    assert np.array_equal(logits, golden["mid_logits"])


def test_cached_steps_equal_the_whole_prompt():
    """Decoder/cachedStepsMatchTheReference, on the oracle's two forms: bit-identical."""
    shape, tensors, encoder = small()
    hidden, logits = O.reference_decode(shape, tensors, encoder, O.SMALL_PROMPT)
    session = O.Session(shape, tensors)
    session.begin(encoder)
    first_h, first_l = session.step(O.SMALL_PROMPT[:2])
    rows_h, rows_l = [first_h], [first_l]
    for token in O.SMALL_PROMPT[2:]:
        h, l = session.step([token])
        rows_h.append(h)
        rows_l.append(l)
    assert session.position == len(O.SMALL_PROMPT)
    assert np.array_equal(np.vstack(rows_h), hidden)
    assert np.array_equal(np.vstack(rows_l), logits)


def test_threads_do_not_change_the_answer():
    tensors = O.synthetic_decoder_tensors(MID_SHAPE, first_seed=7000)
    encoder = O.synthetic_encoder_output(MID_SHAPE.cross_positions, MID_SHAPE.width)
    serial = O.reference_decode(MID_SHAPE, tensors, encoder, MID_TOKENS, threads=1)
    threaded = O.reference_decode(MID_SHAPE, tensors, encoder, MID_TOKENS, threads=8)
    assert np.array_equal(serial[1], threaded[1])


def test_session_refuses_a_step_past_the_window():
    shape, tensors, encoder = small()
    session = O.Session(shape, tensors)
    session.begin(encoder)
    session.step([i % shape.vocabulary_size for i in range(shape.max_positions)], want_logits=False)
    with pytest.raises(ValueError):
        session.step([1])
    assert session.position == shape.max_positions


# --- the reference's self-checks (ReferenceDecoderTests.cpp) -------------------------------

def test_reference_is_finite():
    shape, tensors, encoder = small()
    hidden, logits = O.reference_decode(shape, tensors, encoder, O.SMALL_PROMPT)
    assert hidden.shape == (4, shape.width) and logits.shape == (4, shape.vocabulary_size)
    assert np.isfinite(hidden).all() and np.isfinite(logits).all()


def test_reference_is_causal():
    shape, tensors, encoder = small()
    tokens = list(O.SMALL_PROMPT)
    before = O.reference_decode(shape, tensors, encoder, tokens)
    tokens[2] = (tokens[2] + 7) % shape.vocabulary_size
    after = O.reference_decode(shape, tensors, encoder, tokens)
    assert np.array_equal(before[0][:2], after[0][:2])
    assert np.array_equal(before[1][:2], after[1][:2])
    assert not np.array_equal(before[0][2], after[0][2])


def test_reference_logits_are_tied():
    shape, tensors, encoder = small()
    hidden, logits = O.reference_decode(shape, tensors, encoder, O.SMALL_PROMPT)
    table = tensors["model.decoder.embed_tokens.weight"].astype(np.float64)
    expected = hidden[1] @ table.T
    assert np.all(np.abs(logits[1] - expected) <= 1e-12 * (1 + np.abs(expected)))


def test_reference_reads_the_encoder():
    shape, tensors, encoder = small()
    before = O.reference_decode(shape, tensors, encoder, O.SMALL_PROMPT)
    altered = encoder.copy()
    altered[0, 0] += 1.0
    after = O.reference_decode(shape, tensors, altered, O.SMALL_PROMPT)
    assert before[0][0, 0] != after[0][0, 0]


# --- masked argmax, Tests/Kernels/ArgmaxTests.cpp known answers ------------------------------

ROW = 37


def hand_built_rows():
    i = np.arange(ROW, dtype=np.float32)
    rows = np.stack([-i, -np.abs(i - 18.0), i, np.where((i == 5) | (i == 29), 4.0, i * 0.01)])
    return rows.astype(np.float32)


def test_argmax_finds_the_maximum():
    assert list(O.masked_argmax(hand_built_rows())) == [0, 18, ROW - 1, 5]


def test_argmax_skips_the_suppressed_maximum():
    logits = (np.arange(ROW, dtype=np.float32) * 0.5)
    logits[7], logits[23] = 100.0, 50.0
    mask = np.zeros(ROW, np.float32)
    assert O.masked_argmax(logits, mask)[0] == 7
    mask[7] = 1
    assert O.masked_argmax(logits, mask)[0] == 23
    mask[23] = 1
    assert O.masked_argmax(logits, mask)[0] == ROW - 1


def test_argmax_takes_the_only_token_left():
    logits = (1000.0 - np.arange(ROW)).astype(np.float32)
    logits[11] = -1000.0
    mask = np.ones(ROW, np.float32)
    mask[11] = 0
    assert O.masked_argmax(logits, mask)[0] == 11


def test_argmax_of_an_all_suppressed_row_is_zero():
    assert O.masked_argmax(np.ones(ROW, np.float32), np.ones(ROW, np.float32))[0] == 0


def test_argmax_over_the_vocabulary():
    logits = O.spread_values(51864, 51864, 4.0)
    logits[50361], logits[318] = 900.0, 800.0
    assert O.masked_argmax(logits)[0] == 50361
    mask = np.zeros(51864, np.float32)
    mask[50361] = 1
    assert O.masked_argmax(logits, mask)[0] == 318


# --- number formats -------------------------------------------------------------------------

def test_half_narrowing_matches_the_references(golden):
    ours = O.pack_half(golden["half_probes"])
    assert np.array_equal(ours, golden["half_bits"])


def test_half_narrowing_matches_numpy():
    values = O.spread_values(4096, 99, 70000.0)
    with np.errstate(over="ignore"):
        expected = values.astype(np.float16).view(np.uint16)
    assert np.array_equal(O.pack_half(values), expected)


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libref_decoder.so")),
                    reason="the reference's decoder library is built only where its checkout is")
def test_oracle_equals_the_compiled_reference_on_a_fresh_input():
    from tests.golden.make_golden import load_reference, ref_decode
    ref, _ = load_reference()
    tensors = O.synthetic_decoder_tensors(MID_SHAPE, first_seed=9100)
    encoder = (O.spread_values(MID_SHAPE.cross_positions * MID_SHAPE.width, 31, 1.5)
               .reshape(MID_SHAPE.cross_positions, MID_SHAPE.width))
    tokens = [3, 141, 59, 26, 53, 58, 97, 93]
    expected = ref_decode(ref, MID_SHAPE, tensors, encoder, tokens)
    got = O.reference_decode(MID_SHAPE, tensors, encoder, tokens, threads=4)
    assert np.array_equal(got[0], expected[0]) and np.array_equal(got[1], expected[1])
