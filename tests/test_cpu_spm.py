"""SentencePiece detokeniser (the step after the decode path): libsttb200's stt_spm_* against the
restatement of crates/stt-wasm/src/tokenizer.rs in oracle/spm_oracle.py and the committed
fixtures of tests/golden/make_spm_golden.py.  Host only."""
import ctypes as C
import json
import os
import random

import numpy as np
import pytest

import stt_b200
from oracle import spm_oracle as S
from stt_b200._lib import STT_E_FORMAT, STT_E_INVALID_ARG, lib

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def model_bytes():
    return open(os.path.join(GOLDEN, "spm_tiny.model"), "rb").read()


@pytest.fixture(scope="module")
def golden():
    return json.load(open(os.path.join(GOLDEN, "spm_cases.json"), encoding="utf-8"))


@pytest.fixture(scope="module")
def dec(model_bytes):
    d = stt_b200.SpmDecoder.from_bytes(model_bytes)
    yield d
    d.close()


def _create(data: bytes):
    buf = np.frombuffer(data, dtype=np.uint8) if data else np.zeros(1, np.uint8)
    h = C.c_void_p()
    rc = lib().stt_spm_decoder_create(buf.ctypes.data_as(C.POINTER(C.c_uint8)), len(data), C.byref(h))
    return rc, (stt_b200.SpmDecoder(h) if rc == 0 else None)


# ---- protobuf building blocks for hand-made models
def varint(v):
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        out.append(b | (0x80 if v else 0))
        if not v:
            return bytes(out)


def field(num, wire, payload=b""):
    return varint(num << 3 | wire) + payload


def ld(num, data):
    return field(num, 2, varint(len(data)) + data)


def entry(*parts):
    return ld(1, b"".join(parts))


def test_oracle_is_pinned_to_sentencepiece(model_bytes, golden):
    spm = pytest.importorskip("sentencepiece")
    sp = spm.SentencePieceProcessor(model_proto=model_bytes)
    assert S.parse_vocab(model_bytes) == [sp.id_to_piece(i) for i in range(sp.get_piece_size())] == golden["pieces"]
    for c in golden["cases"]:
        if c["what"] == "encoded text":
            assert c["text"] == " " + sp.decode(c["ids"])


def test_oracle_reproduces_the_fixtures(golden):
    for c in golden["cases"]:
        assert S.decode(golden["pieces"], c["ids"]) == c["text"], c["what"]


def test_vocabulary_and_pieces(dec, golden):
    assert dec.vocab_len() == len(golden["pieces"]) == 400
    assert [dec.piece(i) for i in range(dec.vocab_len())] == golden["pieces"]


def test_decode_matches_fixtures(dec, golden):
    for c in golden["cases"]:
        assert dec.decode(c["ids"]) == c["text"], c["what"]


def test_decode_random_sequences_matches_oracle(dec, golden):
    vocab = golden["pieces"]
    byte_ids = [i for i, p in enumerate(vocab) if S.byte_piece_value(p) is not None]
    word_ids = [i for i, p in enumerate(vocab) if S.byte_piece_value(p) is None]
    rng = random.Random(3)
    for _ in range(3000):
        n = rng.randint(0, 24)
        ids = []
        for _ in range(n):
            r = rng.random()
            ids.append(rng.choice(byte_ids) if r < 0.55 else rng.choice(word_ids) if r < 0.85
                       else rng.choice([0, 3, 400, 401, 2 ** 31, 2 ** 32 - 1]))
        assert dec.decode(ids) == S.decode(vocab, ids), ids


def test_hand_made_models_match_oracle():
    models = [
        b"",
        # unknown top-level fields of every wire type around the pieces
        field(2, 0, varint(300)) + entry(ld(1, "▁a".encode())) + field(3, 1, b"\0" * 8) + field(4, 5, b"\0" * 4)
        + ld(5, b"xyz") + entry(ld(1, b"b")),
        # unknown fields inside an entry (score f32, type varint), a repeated piece field: the last wins
        entry(ld(1, b"first"), field(2, 5, b"\0\0\x80?"), field(3, 0, varint(6)), ld(1, b"last")),
        # an entry without a piece field, invalid UTF-8 piece bytes, byte pieces of both accepted forms
        entry(field(3, 0, b"\x01")) + entry(ld(1, b"\xff\xfeok\xe2\x96")) + entry(ld(1, b"<0x+F>"))
        + entry(ld(1, b"<0x41>")) + entry(ld(1, b"<0xg1>")) + entry(ld(1, b"<0x-1>")) + entry(ld(1, "<0xé>".encode())),
        # a wire type the walk does not know (3, 4, 6, 7): one byte skipped
        field(6, 3) + b"\x00" + entry(ld(1, b"c")) + field(7, 7) + entry(ld(1, b"d")),
        # an over-long varint tag (shift past bit 63) and a tag cut off at the end of the file
        b"\xff" * 11 + b"\x00" + entry(ld(1, b"e")) + b"\x80",
        # a skipped length-delimited field longer than the rest of the file ends the walk
        entry(ld(1, b"f")) + field(9, 2, varint(10 ** 6)) + b"tail",
    ]
    for m in models:
        rc, d = _create(m)
        assert rc == 0, lib().stt_last_error()
        vocab = S.parse_vocab(m)
        assert [d.piece(i) for i in range(d.vocab_len())] == vocab
        for ids in ([], list(range(len(vocab))), list(range(len(vocab)))[::-1] * 2):
            assert d.decode(ids) == S.decode(vocab, ids)
        d.close()


def test_truncated_entries_are_format_errors(model_bytes):
    for m in (ld(1, b"abc")[:-1], entry(ld(1, b"abc"))[:-1], model_bytes[:20],
              entry(field(1, 2, varint(50) + b"short"))):
        with pytest.raises(ValueError):
            S.parse_vocab(m)
        rc, _ = _create(m)
        assert rc == STT_E_FORMAT
        assert "runs past" in lib().stt_last_error().decode()


def test_corrupted_models_agree_with_oracle(model_bytes):
    rng = random.Random(11)
    ok = bad = 0
    for _ in range(400):
        m = bytearray(model_bytes)
        for _ in range(rng.randint(1, 6)):
            m[rng.randrange(len(m))] = rng.randrange(256)
        m = bytes(m[:rng.randint(len(m) // 2, len(m))])
        try:
            vocab = S.parse_vocab(m)
        except ValueError:
            vocab = None
        rc, d = _create(m)
        if vocab is None:
            assert rc == STT_E_FORMAT
            bad += 1
            continue
        assert rc == 0
        assert [d.piece(i) for i in range(d.vocab_len())] == vocab
        ids = [rng.randrange(len(vocab) + 2) for _ in range(40)] if vocab else []
        assert d.decode(ids) == S.decode(vocab, ids)
        d.close()
        ok += 1
    assert ok > 20 and bad > 20


def test_output_buffer_protocol(dec, golden):
    case = next(c for c in golden["cases"] if c["what"] == "encoded text")
    ids = np.array(case["ids"], dtype=np.uint32)
    want = case["text"].encode("utf-8")
    p = ids.ctypes.data_as(C.POINTER(C.c_uint32))
    n = C.c_size_t(12345)
    assert lib().stt_spm_decode(dec._h, p, ids.size, None, 0, C.byref(n)) == 0 and n.value == len(want)
    small = C.create_string_buffer(len(want))
    assert lib().stt_spm_decode(dec._h, p, ids.size, small, len(want), C.byref(n)) == STT_E_INVALID_ARG
    assert n.value == len(want)
    exact = C.create_string_buffer(len(want) + 1)
    assert lib().stt_spm_decode(dec._h, p, ids.size, exact, len(want) + 1, C.byref(n)) == 0
    assert exact.raw == want + b"\0"
    assert lib().stt_spm_piece(dec._h, 400, None, 0, C.byref(n)) == STT_E_INVALID_ARG
    assert lib().stt_spm_piece(dec._h, -1, None, 0, C.byref(n)) == STT_E_INVALID_ARG
    assert lib().stt_spm_decode(None, p, ids.size, None, 0, C.byref(n)) == STT_E_INVALID_ARG


def test_load_reads_the_file(model_bytes, tmp_path):
    f = tmp_path / "tok.model"
    f.write_bytes(model_bytes)
    d = stt_b200.SpmDecoder.load(str(f))
    assert d.vocab_len() == 400
    d.close()


def test_per_token_decoding_concatenates(dec, golden):
    # The reference keeps each piece's leading space so that a host decoding token by token, as the
    # stream emits them, gets the same text as decoding the whole sequence (tokenizer.rs:187-190).
    # That holds for every sequence without byte-fallback pieces; a multi-byte character split over
    # byte pieces only decodes once its run is complete.
    vocab = golden["pieces"]
    for c in golden["cases"]:
        ids = c["ids"]
        if any(0 <= i < len(vocab) and S.byte_piece_value(vocab[i]) is not None for i in ids):
            continue
        assert "".join(dec.decode([i]) for i in ids) == dec.decode(ids) == c["text"]
