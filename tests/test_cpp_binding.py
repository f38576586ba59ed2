"""The C++ side of the boundary: include/wsp_decoder.hpp (CudaDecoder) and
include/wsp_net.hpp (CudaNet, the CUDA backend behind the Net op interface,
Lib/WhisperEACP/Net/Net.h:110-171), compiled with g++ into a program that
only reaches the library through them.

On the CPU the program is compiled, so a header that drifts from the library
fails here.  On the GPU it runs: the decoder's own recording sequence
(Decoder.cpp:121-177, restated in tests/cpp/net_decoder_test.cpp) through
CudaNet, the same inputs through CudaDecoder, and the refusals; logits
against the oracle within max-abs 2e-2.
"""
import os
import struct
import subprocess

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import stored_tensors
from whispereacp_b200 import synthetic as S
from whispereacp_b200.decoder import DecoderShape

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCE = os.path.join(ROOT, "tests", "cpp", "net_decoder_test.cpp")
LIBRARY_DIR = os.path.join(ROOT, "whispereacp_b200")

SHAPE = DecoderShape(width=128, heads=2, layers=2, feed_forward_width=512, vocabulary_size=2000,
                     max_positions=24, cross_positions=40)


def compile_program(out_dir) -> str:
    program = os.path.join(str(out_dir), "net_decoder_test")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    SOURCE, "-L", LIBRARY_DIR, "-lwsp_b200", f"-Wl,-rpath,{LIBRARY_DIR}", "-o", program],
                   check=True, capture_output=True, text=True)
    return program


def test_the_cpp_headers_compile_against_the_library(tmp_path):
    try:
        compile_program(tmp_path)
    except subprocess.CalledProcessError as e:
        pytest.fail(e.stderr)


def write_fixture(path, shape, storage, tensors, encoder, prompt, tokens, logits):
    with open(path, "wb") as f:
        f.write(b"WSPF")
        f.write(struct.pack("<7i", shape.width, shape.heads, shape.layers, shape.feed_forward_width,
                            shape.vocabulary_size, shape.max_positions, shape.cross_positions))
        f.write(struct.pack("<i", 1 if storage == "float16" else 2))
        f.write(struct.pack("<i", len(tensors)))
        for name, values in tensors.items():
            values = np.ascontiguousarray(values, np.float32)
            f.write(struct.pack("<i", len(name)) + name.encode())
            f.write(struct.pack("<i", values.ndim) + struct.pack(f"<{values.ndim}q", *values.shape))
            f.write(values.tobytes())
        f.write(np.ascontiguousarray(encoder, np.float32).tobytes())
        f.write(struct.pack("<i", len(prompt)) + np.asarray(prompt, np.uint32).tobytes())
        f.write(struct.pack("<i", len(tokens)) + np.asarray(tokens, np.uint32).tobytes())
        f.write(np.ascontiguousarray(logits, np.float32).tobytes())


@pytest.mark.gpu
@pytest.mark.parametrize("storage", ["float16", "bfloat16"])
def test_the_decoder_through_cuda_net(tmp_path, storage):
    program = compile_program(tmp_path)
    tensors = stored_tensors(S.normal_weights(SHAPE, seed=81), storage)
    encoder = S.encoder_output(1, SHAPE.cross_positions, SHAPE.width, seed=82)[0]
    prompt = [1990, 1991, 7]
    tokens = [int(t) for t in S.teacher_tokens(9, seed=83, high=1989)]
    _, logits = O.reference_decode(O.Shape(**SHAPE.__dict__), tensors, encoder, prompt + tokens)
    fixture = tmp_path / "fixture.bin"
    write_fixture(fixture, SHAPE, storage, tensors, encoder, prompt, tokens, logits)
    run = subprocess.run([program, str(fixture)], capture_output=True, text=True, timeout=300)
    print(run.stdout)
    assert run.returncode == 0, run.stdout + run.stderr
    assert run.stdout.strip().endswith("ok")
