"""A synthetic HuggingFace Whisper repository on disk, in the layout
Whisper::load reads (Lib/WhisperEACP/Whisper/Whisper.cpp:121-132):
config.json, preprocessor_config.json, tokenizer.json and model.safetensors.

The vocabulary is byte-level BPE as Whisper's is: the first 256 ids are the
256 bytes spelled in GPT-2's printable alphabet, then words (ASCII, accented,
CJK and emoji, some with a leading space) spelled the same way, then the
added <|...|> tokens.  No merges are needed to decode.  The decoder tensors
are random-init, rounded to the storage type and kept in fp32 containers, as
Whisper's own checkpoints hold fp16 values in fp32.
"""
from __future__ import annotations

import json
import os

import numpy as np

from oracle import frontend as FE
from oracle import oracle as O
from tests.helpers import round_to, stored_tensors
from whispereacp_b200 import synthetic as S
from whispereacp_b200.decoder import DecoderShape


def bytes_to_unicode() -> dict[int, str]:
    """GPT-2's byte-level alphabet (the published bytes_to_unicode): bytes
    33-126, 161-172 and 174-255 spell themselves, the other 68 take code
    points 256, 257, ... in byte order."""
    printable = [*range(33, 127), *range(161, 173), *range(174, 256)]
    table, extra = {}, 0
    for b in range(256):
        if b in printable:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


BYTE_SPELLING = bytes_to_unicode()
BYTE_OF = {c: b for b, c in BYTE_SPELLING.items()}

WORDS = ["the", "and", "so", "my", "fellow", "Americans", "ask", "not", "what", "your", "country", "can",
         "do", "for", "you", "café", "naïve", "Übermaß", "señor", "日本", "語", "音声", "認識", "🎙", "🙂",
         "Ωμέγα", "привет", "!", ",", ".", "?", "'s", "'t", "20", "2026"]

SPECIALS = ["<|endoftext|>", "<|startoftranscript|>", "<|en|>", "<|de|>", "<|ja|>", "<|translate|>",
            "<|transcribe|>", "<|startoflm|>", "<|startofprev|>", "<|nocaptions|>", "<|notimestamps|>",
            "<|0.00|>", "<|0.02|>", "<|0.04|>"]


def spell(text: str) -> str:
    return "".join(BYTE_SPELLING[b] for b in text.encode("utf-8"))


def vocabulary() -> tuple[list[str], int]:
    """Every token's spelling by id, and the id of the first added token."""
    texts = [BYTE_SPELLING[b] for b in range(256)]
    for word in WORDS:
        for form in (word, " " + word):
            if spell(form) not in texts:
                texts.append(spell(form))
    first_added = len(texts)
    return texts + SPECIALS, first_added


def decode(texts: list[str], first_added: int, ids) -> bytes:
    """Tokenizer::decode (Tokenizer/Tokenizer.cpp:369-398): the non-special
    tokens' spellings joined and mapped back to bytes."""
    spelled = "".join(texts[i] for i in ids if 0 <= i < first_added)
    return bytes(BYTE_OF[c] for c in spelled if c in BYTE_OF)


class Repo:
    """The repository's contents, as the tests need them again."""

    def __init__(self, directory: str, shape: DecoderShape, tensors: dict, texts: list[str], first_added: int,
                 config: dict):
        self.directory = directory
        self.shape = shape
        self.tensors = tensors
        self.texts = texts
        self.first_added = first_added
        self.config = config

    def token(self, text: str) -> int:
        return self.texts.index(text)


def write_repo(directory: str, width: int = 128, heads: int = 2, layers: int = 2, target_positions: int = 32,
               source_positions: int = 40, storage: str = "float16", seed: int = 91, **overrides) -> Repo:
    from safetensors.numpy import save_file

    os.makedirs(directory, exist_ok=True)
    texts, first_added = vocabulary()
    v = len(texts)
    end_of_text = texts.index("<|endoftext|>")
    start = texts.index("<|startoftranscript|>")
    config = {
        "model_type": "whisper", "num_mel_bins": 80, "d_model": width, "encoder_layers": 2,
        "decoder_layers": layers, "encoder_attention_heads": heads, "decoder_attention_heads": heads,
        "encoder_ffn_dim": 4 * width, "decoder_ffn_dim": 4 * width, "max_source_positions": source_positions,
        "max_target_positions": target_positions, "vocab_size": v, "activation_function": "gelu",
        "scale_embedding": False, "bos_token_id": end_of_text, "eos_token_id": end_of_text,
        "pad_token_id": end_of_text, "decoder_start_token_id": start,
        "suppress_tokens": [1, 2, 7, texts.index(spell(" the")), texts.index("<|startoflm|>")],
        "begin_suppress_tokens": [texts.index(spell(" ")), end_of_text],
        "forced_decoder_ids": None, "torch_dtype": "float32",
    }
    config.update(overrides)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(config, f, indent=2)
    filters = FE.synthetic_filters(80)
    with open(os.path.join(directory, "preprocessor_config.json"), "w") as f:
        json.dump({"feature_size": 80, "hop_length": 160, "n_fft": 400, "n_samples": 480000,
                   "sampling_rate": 16000, "chunk_length": 30, "nb_max_frames": 3000,
                   "mel_filters": filters.astype(np.float64).tolist()}, f)
    tokenizer = {
        "version": "1.0", "truncation": None, "padding": None,
        "added_tokens": [{"id": first_added + k, "content": t, "single_word": False, "lstrip": False,
                          "rstrip": False, "normalized": False, "special": True} for k, t in enumerate(SPECIALS)],
        "normalizer": None,
        "pre_tokenizer": {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True, "use_regex": True},
        "post_processor": None,
        "decoder": {"type": "ByteLevel", "add_prefix_space": True, "trim_offsets": True, "use_regex": True},
        "model": {"type": "BPE", "dropout": None, "unk_token": None, "continuing_subword_prefix": "",
                  "end_of_word_suffix": "", "fuse_unk": False, "byte_fallback": False, "ignore_merges": False,
                  "vocab": {t: i for i, t in enumerate(texts[:first_added])}, "merges": []},
    }
    with open(os.path.join(directory, "tokenizer.json"), "w", encoding="utf-8") as f:
        json.dump(tokenizer, f, ensure_ascii=False)

    shape = DecoderShape(width=width, heads=heads, layers=layers, feed_forward_width=4 * width,
                         vocabulary_size=v, max_positions=target_positions, cross_positions=source_positions)
    tensors = stored_tensors(S.normal_weights(shape, seed=seed), storage)
    stored = {k: np.ascontiguousarray(t, np.float32) for k, t in tensors.items()}
    # The encoder (its matrices fp16 values in fp32 containers, as a
    # checkpoint's), and an integer buffer the loader reads past.
    encoder = FE.synthetic_encoder_tensors(80, width, config["encoder_layers"], config["encoder_ffn_dim"],
                                           source_positions, seed=seed + 1)
    encoder = {k: (round_to(storage, v) if v.ndim > 1 and "embed_positions" not in k else v) for k, v in encoder.items()}
    stored.update(encoder)
    stored["model.encoder.position_ids"] = np.arange(source_positions, dtype=np.int64)
    save_file(stored, os.path.join(directory, "model.safetensors"))
    repo = Repo(directory, shape, tensors, texts, first_added, config)
    repo.encoder = encoder
    repo.filters = filters
    return repo


def masks(repo: Repo) -> tuple[np.ndarray, np.ndarray]:
    """buildSuppressionMasks (Whisper.cpp:227-254) from the repo's config."""
    later = np.zeros(repo.shape.vocabulary_size, np.float32)
    later[repo.config["suppress_tokens"]] = 1.0
    first = later.copy()
    first[repo.config["begin_suppress_tokens"]] = 1.0
    return first, later


def oracle_shape(repo: Repo) -> O.Shape:
    return O.Shape(**repo.shape.__dict__)
