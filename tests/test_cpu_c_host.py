"""The C ABI from a compiled C99 program (tests/c_host.c) linked against libsttb200.so: the header
compiles as C, and the calls that need no device behave as through the Python binding."""
import json
import os
import subprocess

import pytest

from conftest import GOLDEN, REPO
import stt_b200

LIBDIR = os.path.dirname(stt_b200.LIB_PATH)


@pytest.fixture(scope="module")
def c_host(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("c_host") / "c_host")
    subprocess.check_call(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
                           "-I", os.path.join(REPO, "include"), os.path.join(REPO, "tests", "c_host.c"),
                           "-L", LIBDIR, "-lsttb200", "-Wl,-rpath," + LIBDIR, "-o", exe])
    return exe


def run(exe, *args):
    r = subprocess.run([exe, *args], capture_output=True, timeout=120)
    assert r.returncode == 0, r.stderr.decode()
    return r.stdout.decode("utf-8")


def test_default_config_from_c(c_host):
    # SttConfig::default, crates/stt-wasm/src/lib.rs:60-80
    assert run(c_host, "config").split() == ["16", "2048", "16", "16", "5632", "8000", "8001", "32", "2049", "6",
                                             "100000.0", "4096", "750", "3", "8000"]


def test_loader_errors_from_c(c_host):
    # the tiny checkpoint (d_model 256) under the default config (hidden_size 2048): a format error
    rc, msg = run(c_host, "load", os.path.join(GOLDEN, "tiny_ref.gguf")).rstrip("\n").split(" ", 1)
    assert int(rc) == -2 and msg == "text_emb.weight width 256 != hidden_size 2048"


def test_detokeniser_from_c(c_host):
    cases = json.load(open(os.path.join(GOLDEN, "spm_cases.json"), encoding="utf-8"))["cases"]
    for c in cases:
        if not c["ids"]:
            continue
        vocab, text = run(c_host, "spm", os.path.join(GOLDEN, "spm_tiny.model"),
                          *map(str, c["ids"])).split("\n", 1)
        assert vocab == "400"
        assert text[:-1] == c["text"], c["what"]
