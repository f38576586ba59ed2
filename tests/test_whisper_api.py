"""Whisper::load / prepare / transcribe / transcribeText through
include/wsp_whisper.hpp, on a synthetic HuggingFace repository
(tests/whisper_repo.py).

On the CPU: the header compiles into a program against the library; load
reads the four files; the generation config is the reference's
(Whisper.cpp:148-254: prompt [decoder_start_token_id, <|notimestamps|>],
suppress_tokens at every step, begin_suppress_tokens at the first, limit
max_target_positions - prompt); the multilingual prompt puts the language
and task tokens between the two; Tokenizer::decode drops special tokens and
maps the byte-level spellings back to UTF-8, checked against a restatement
and against the `tokenizers` library's ByteLevel decoder; the refusals carry
the reference's messages; audioContextForSamples rounds as
Whisper.cpp:450-460 does.

On the GPU: transcribe through the header equals the Python binding's
transcript under the same generation config (bit-for-bit: the same kernels),
window by window, at the whole window and at a reduced audio context, and
each id is the oracle's masked argmax wherever the margin decides it.
"""
import json
import os
import subprocess

import numpy as np
import pytest

from tests import whisper_repo as R

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCE = os.path.join(ROOT, "tests", "cpp", "whisper_test.cpp")
LIBRARY_DIR = os.path.join(ROOT, "whispereacp_b200")
MARGIN = 5e-2


def compile_program(out_dir) -> str:
    program = os.path.join(str(out_dir), "whisper_test")
    try:
        subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        SOURCE, "-L", LIBRARY_DIR, "-lwsp_b200", f"-Wl,-rpath,{LIBRARY_DIR}", "-o", program],
                       check=True, capture_output=True, text=True)
    except subprocess.CalledProcessError as e:
        pytest.fail(e.stderr)
    return program


@pytest.fixture(scope="module")
def program(tmp_path_factory):
    return compile_program(tmp_path_factory.mktemp("whisper_program"))


@pytest.fixture(scope="module")
def repo(tmp_path_factory):
    return R.write_repo(str(tmp_path_factory.mktemp("whisper_repo")))


def run(program, *args, expect=0):
    result = subprocess.run([program, *map(str, args)], capture_output=True, text=True, timeout=600)
    assert result.returncode == expect, result.stdout + result.stderr
    return result.stdout


def fields(output: str) -> dict[str, str]:
    out = {}
    for line in output.splitlines():
        key, _, value = line.partition(":")
        out.setdefault(key, []).append(value.strip())
    return out


def ids_of(value: str) -> list[int]:
    return [int(x) for x in value.split()]


def test_load_builds_the_reference_generation_config(program, repo):
    f = fields(run(program, "inspect", repo.directory))
    s = repo.shape
    assert ids_of(f["shape"][0]) == [s.width, s.heads, s.layers, s.feed_forward_width, s.vocabulary_size,
                                      s.max_positions, s.cross_positions]
    assert ids_of(f["prompt"][0]) == [repo.token("<|startoftranscript|>"), repo.token("<|notimestamps|>")]
    first, later = R.masks(repo)
    assert ids_of(f["later"][0]) == list(np.nonzero(later)[0])
    assert ids_of(f["first"][0]) == list(np.nonzero(first)[0])
    assert int(f["maximum"][0]) == s.max_positions - 2


def test_the_multilingual_prompt(program, repo):
    f = fields(run(program, "inspect", repo.directory, "de", "translate"))
    assert ids_of(f["prompt"][0]) == [repo.token(t) for t in
                                      ("<|startoftranscript|>", "<|de|>", "<|translate|>", "<|notimestamps|>")]
    assert int(f["maximum"][0]) == repo.shape.max_positions - 4
    f = fields(run(program, "inspect", repo.directory, "ja"))
    assert ids_of(f["prompt"][0])[1:3] == [repo.token("<|ja|>"), repo.token("<|transcribe|>")]
    out = run(program, "inspect", repo.directory, "xx", expect=1)
    assert "no language token <|xx|>" in out


def test_decode_drops_special_tokens_and_returns_utf8(program, repo):
    rng = np.random.default_rng(5)
    words = [repo.texts.index(R.spell(w)) for w in ("the", " fellow", " café", " 日本", "語", " 🎙", " привет", "!")]
    for trial in range(6):
        ids = list(rng.choice(words, size=12))
        ids.insert(int(rng.integers(0, 12)), repo.token("<|notimestamps|>"))
        ids.append(repo.token("<|endoftext|>"))
        f = fields(run(program, "inspect", repo.directory, "--", *ids))
        expected = R.decode(repo.texts, repo.first_added, ids)
        assert bytes.fromhex(f["text"][0]) == expected
        # and the tokenizers library's own ByteLevel decoder on the same file
        tokenizers = pytest.importorskip("tokenizers")
        hf = tokenizers.Tokenizer.from_file(os.path.join(repo.directory, "tokenizer.json"))
        assert hf.decode([int(i) for i in ids], skip_special_tokens=True) == expected.decode("utf-8")


def test_decode_of_single_bytes_and_ids_outside_the_vocabulary(program, repo):
    # bytes of a multi-byte character spelled one id at a time, then an id
    # past the vocabulary, which decode skips
    ids = list("é".encode("utf-8")) + [ord("a"), len(repo.texts) + 5]
    f = fields(run(program, "inspect", repo.directory, "--", *ids))
    assert bytes.fromhex(f["text"][0]) == "éa".encode("utf-8")


def test_audio_context_for_samples(program, repo):
    f = fields(run(program, "inspect", repo.directory))
    # 1 s + 2.5 s margin = 175 positions -> 192, held at the 448 floor; 20 s
    # + 2.5 s = 1125 -> 1152; 40 s is past the window
    assert ids_of(f["context"][0]) == [448, 1152, 1500]


def test_a_reduced_audio_context_is_not_run_through_the_front_end(program, repo):
    """The reference's encoder computes a reduced context's positions itself
    (Whisper.h:382-402); the CUDA front end encodes whole windows, so
    transcribe_samples refuses a reduced context instead of answering
    differently.  Zero and the whole window pass that check (and then stop
    at the missing prepare)."""
    out = run(program, "context-samples", repo.directory, 16)
    assert "encodes whole windows" in out and "audio context of 16 positions" in out
    for whole in (0, repo.config["max_source_positions"]):
        out = run(program, "context-samples", repo.directory, whole)
        assert "has not been prepared" in out, out


@pytest.mark.parametrize("change,message", [
    (lambda d: os.remove(os.path.join(d, "tokenizer.json")), "has no tokenizer.json"),
    (lambda d: os.remove(os.path.join(d, "preprocessor_config.json")), "has no preprocessor_config.json"),
    (lambda d: edit_config(d, lambda c: c.pop("d_model")), "config.json field 'd_model' is missing"),
    (lambda d: edit_config(d, lambda c: c.update(decoder_layers=0)), "field 'decoder_layers' must be positive"),
    (lambda d: edit_config(d, lambda c: c.update(d_model=129)), "does not divide into the encoder head count"),
    (lambda d: edit_config(d, lambda c: c.update(model_type="bart")), "describes a 'bart' model"),
    (lambda d: edit_config(d, lambda c: c.update(vocab_size=1.5)), "is not a whole 64-bit integer"),
    (lambda d: edit_config(d, lambda c: c["suppress_tokens"].append(10 ** 6)),
     "suppresses token 1000000, which is outside the vocabulary"),
    (lambda d: edit_tokenizer(d, lambda t: t["added_tokens"].pop(10)), "names no <|notimestamps|> token"),
    (lambda d: edit_tokenizer(d, lambda t: t["model"].pop("merges")), "tokenizer.json has no 'merges'"),
    (lambda d: open(os.path.join(d, "config.json"), "w").write("{\"d_model\": 12,"), "config.json is not valid JSON"),
    (lambda d: truncate(os.path.join(d, "model.safetensors")), "do not fit its shape or the file"),
    (lambda d: edit_preprocessor(d, lambda c: c.pop("hop_length")),
     "preprocessor_config.json field 'hop_length' is missing"),
    (lambda d: edit_preprocessor(d, lambda c: c["mel_filters"][3].pop()), "mel_filters is ragged"),
    (lambda d: edit_preprocessor(d, lambda c: c["mel_filters"].pop()), "mel_filters is not 80 x 201"),
    (lambda d: edit_preprocessor(d, lambda c: c.update(n_fft=401)), "n_fft is not a positive even number"),
])
def test_load_refuses_with_the_reference_messages(program, tmp_path, change, message):
    repo = R.write_repo(str(tmp_path / "repo"), width=64, layers=1, seed=3)
    change(repo.directory)
    out = run(program, "refuse", repo.directory)
    assert message in out, out


def edit_config(directory, edit):
    path = os.path.join(directory, "config.json")
    config = json.load(open(path))
    edit(config)
    json.dump(config, open(path, "w"))


def edit_preprocessor(directory, edit):
    path = os.path.join(directory, "preprocessor_config.json")
    config = json.load(open(path))
    edit(config)
    json.dump(config, open(path, "w"))


def edit_tokenizer(directory, edit):
    path = os.path.join(directory, "tokenizer.json")
    tokenizer = json.load(open(path, encoding="utf-8"))
    edit(tokenizer)
    json.dump(tokenizer, open(path, "w", encoding="utf-8"), ensure_ascii=False)


def truncate(path):
    size = os.path.getsize(path)
    with open(path, "r+b") as f:
        f.truncate(size - 64)


def test_a_transposed_filterbank_is_read_mel_major(program, tmp_path):
    """PreprocessorConfig accepts mel_filters as [bins][mels] too
    (PreprocessorConfig.cpp:66-76)."""
    repo = R.write_repo(str(tmp_path / "repo"), width=64, layers=1, seed=5)
    edit_preprocessor(repo.directory, lambda c: c.update(mel_filters=np.asarray(c["mel_filters"]).T.tolist()))
    run(program, "inspect", repo.directory)


def test_without_end_of_text_the_decoder_start_comes_from_the_tokenizer(program, tmp_path):
    repo = R.write_repo(str(tmp_path / "repo"), width=64, layers=1, seed=4)
    edit_config(repo.directory, lambda c: c.pop("decoder_start_token_id"))
    f = fields(run(program, "inspect", repo.directory))
    assert ids_of(f["prompt"][0])[0] == repo.token("<|startoftranscript|>")


@pytest.mark.gpu
@pytest.mark.parametrize("storage,context", [("f16", 0), ("bf16", 24)])
def test_transcribe_through_the_header(program, repo, tmp_path, storage, context):
    from oracle import oracle as O
    from tests.helpers import stored_tensors, top2_margin
    from whispereacp_b200 import Decoder, synthetic as S

    windows = 3
    s = repo.shape
    encoder = S.encoder_output(windows, s.cross_positions, s.width, seed=93)
    path = tmp_path / "encoder.bin"
    path.write_bytes(np.ascontiguousarray(encoder, np.float32).tobytes())
    f = fields(run(program, "transcribe", repo.directory, path, windows, storage, context))
    assert f["ok"] == [""]
    got = [ids_of(v) for v in f["ids"]]
    texts = [bytes.fromhex(v) for v in f["text"]]

    first, later = R.masks(repo)
    prompt = [repo.token("<|startoftranscript|>"), repo.token("<|notimestamps|>")]
    end_of_text = repo.token("<|endoftext|>")
    decoder = Decoder(s, windows=windows, storage="float16" if storage == "f16" else "bfloat16")
    decoder.load_weights(repo.tensors)
    decoder.set_generation(prompt, first, later, maximum_tokens=s.max_positions - 2, end_of_text=end_of_text)
    expected = decoder.transcribe(encoder, cross_positions=context)
    for b in range(windows):
        assert got[b] == [int(x) for x in expected[b]]
        assert texts[b] == R.decode(repo.texts, repo.first_added, got[b])

    # Each id against the oracle's masked argmax on the same 16-bit weights.
    oshape = R.oracle_shape(repo)
    positions = context or s.cross_positions
    if context:
        oshape = O.Shape(**{**s.__dict__, "cross_positions": context})
    tensors = stored_tensors(repo.tensors, "float16" if storage == "f16" else "bfloat16")
    decided = 0
    for b in range(windows):
        session = O.Session(oshape, tensors)
        session.begin(encoder[b, :positions])
        chunk = prompt
        for k, token in enumerate(got[b][:8]):
            _, logits = session.step(chunk)
            mask = first if k == 0 else later
            row = logits[-1:]
            if top2_margin(row, mask)[0] > MARGIN:
                assert token == int(O.masked_argmax(row, mask)[0])
                decided += 1
            chunk = [token]
    assert decided > 0


@pytest.mark.gpu
def test_transcribe_samples_through_the_header(program, repo, tmp_path):
    """Whisper::transcribe on recordings: the header's spectrogram, encoder and
    greedy search give the ids the Python bindings give by the same route
    (Encoder.encode_samples, then Decoder.transcribe), window by window."""
    from oracle import frontend as FE
    from whispereacp_b200 import Decoder, Encoder, EncoderShape

    windows, count = 2, 9000
    audio = np.stack([FE.synthetic_audio(count, seed=70 + b) for b in range(windows)])
    path = tmp_path / "audio.bin"
    path.write_bytes(np.ascontiguousarray(audio, np.float32).tobytes())
    f = fields(run(program, "samples", repo.directory, path, windows, count))
    assert f["ok"] == [""]
    got = [ids_of(v) for v in f["ids"]]

    encoder = Encoder(EncoderShape.from_config(repo.config))
    encoder.load_weights(repo.encoder)
    encoder.set_filters(repo.filters)
    rows = np.stack([encoder.encode_samples(audio[b]) for b in range(windows)])
    first, later = R.masks(repo)
    prompt = [repo.token("<|startoftranscript|>"), repo.token("<|notimestamps|>")]
    decoder = Decoder(repo.shape, windows=windows)
    decoder.load_weights(repo.tensors)
    decoder.set_generation(prompt, first, later, maximum_tokens=repo.shape.max_positions - 2,
                           end_of_text=repo.token("<|endoftext|>"))
    expected = decoder.transcribe(rows)
    for b in range(windows):
        assert got[b] == [int(x) for x in expected[b]]
        assert bytes.fromhex(f["text"][b]) == R.decode(repo.texts, repo.first_added, got[b])
