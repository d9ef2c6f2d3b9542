"""The C++ host interface (include/stt_b200.hpp, the mirror of the stt-wasm types over the C ABI)
from a compiled program, tests/cpp_host.cpp, linked against libsttb200.so.  Only calls that need no
device run here; the header is compiled whole, so every wrapper is type-checked against the C ABI."""
import json
import os
import subprocess

import pytest

from conftest import GOLDEN, REPO
import stt_b200

LIBDIR = os.path.dirname(stt_b200.LIB_PATH)


@pytest.fixture(scope="module")
def cpp_host(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("cpp_host") / "cpp_host")
    subprocess.check_call(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-pedantic",
                           "-I", os.path.join(REPO, "include"), os.path.join(REPO, "tests", "cpp_host.cpp"),
                           "-L", LIBDIR, "-lsttb200", "-Wl,-rpath," + LIBDIR, "-o", exe])
    return exe


def run(exe, *args):
    r = subprocess.run([exe, *args], capture_output=True, timeout=120)
    assert r.returncode == 0, r.stderr.decode()
    return r.stdout.decode("utf-8")


def test_config_defaults(cpp_host):
    # SttConfig::default, crates/stt-wasm/src/lib.rs:60-80
    assert run(cpp_host, "config").split() == ["16", "2048", "16", "16", "5632", "8000", "8001", "32", "2049", "6",
                                               "100000.0", "4096", "750", "3", "8000"]


def test_from_shards_raises_the_loader_error(cpp_host):
    out = run(cpp_host, "load", os.path.join(GOLDEN, "tiny_ref.gguf")).rstrip("\n")
    assert out == "-2 stt_model_load_gguf: text_emb.weight width 256 != hidden_size 2048"


def test_from_q4_bytes_checks_the_byte_count(cpp_host):
    # Q4Tensor::from_q4_bytes (gguf.rs:418-432): 2 x 64 weights are 4 blocks of 18 bytes
    out = run(cpp_host, "q4bad").rstrip("\n")
    assert out == "-2 stt_q4_tensor_create: Q4_0 byte count mismatch: expected 72 for 4 blocks, got 71"


def test_spm_decoder(cpp_host):
    cases = json.load(open(os.path.join(GOLDEN, "spm_cases.json"), encoding="utf-8"))["cases"]
    for c in cases:
        vocab, text = run(cpp_host, "spm", os.path.join(GOLDEN, "spm_tiny.model"), *map(str, c["ids"])).split("\n", 1)
        assert vocab == "400"
        assert text[:-1] == c["text"], c["what"]
