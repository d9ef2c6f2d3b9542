"""Generates the SentencePiece fixtures of tests/test_cpu_spm.py.

  spm_tiny.model   a 400-piece unigram model with byte fallback, trained here by the
                   `sentencepiece` package on seeded pseudo-words (no real corpus); special ids
                   laid out as the reference's decoder expects them: 0 end of stream, 3 padding
  spm_cases.json   the model's pieces as `sentencepiece` reports them (id_to_piece), and token-id
                   sequences with the text the reference's decoding rules give
                   (crates/stt-wasm/src/tokenizer.rs:150-192, restated in oracle/spm_oracle.py)

The expected texts come from the restatement, which this script first checks against
`sentencepiece` where the two agree by construction: the vocabulary, and the decoded text of
encoded input (the reference keeps the leading space of the first word).

Run: python tests/golden/make_spm_golden.py
"""
import io
import json
import os
import random
import sys

import sentencepiece as spm

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle import spm_oracle as S  # noqa: E402

SYLLABLES = ["ba", "lo", "mi", "tre", "sou", "ré", "çà", "ün", "qua", "del", "por", "fi", "zé", "ou", "an", "est",
             "le", "la"]


def sentences(rng, n):
    return [" ".join("".join(rng.choice(SYLLABLES) for _ in range(rng.randint(1, 4)))
                     for _ in range(rng.randint(3, 12))) for _ in range(n)]


def main():
    rng = random.Random(20240611)
    buf = io.BytesIO()
    spm.SentencePieceTrainer.train(
        sentence_iterator=iter(sentences(rng, 3000)), model_writer=buf, vocab_size=400, model_type="unigram",
        byte_fallback=True, eos_id=0, unk_id=1, bos_id=2, pad_id=3, character_coverage=1.0,
        normalization_rule_name="identity", num_threads=1, minloglevel=2)
    model = buf.getvalue()
    sp = spm.SentencePieceProcessor(model_proto=model)
    pieces = [sp.id_to_piece(i) for i in range(sp.get_piece_size())]
    vocab = S.parse_vocab(model)
    assert vocab == pieces, "restated vocabulary walk differs from sentencepiece"
    byte_id = {S.byte_piece_value(p): i for i, p in enumerate(pieces) if S.byte_piece_value(p) is not None}
    assert sorted(byte_id) == list(range(256))

    cases = []
    # encoded text: words of the training alphabet, unseen letters (byte fallback) and multi-byte characters
    texts = sentences(rng, 20) + ["bonjour le monde", "漢字 かな 🙂 ok", "naïve café", "x", "ré-été 2024"]
    for t in texts:
        ids = sp.encode(t)
        assert sp.decode(ids) == t
        got = S.decode(vocab, ids)
        assert got == " " + t, (t, got)        # the reference keeps the first word's leading space
        cases.append({"what": "encoded text", "ids": ids, "text": got})
    enc = sp.encode("漢字")
    b = [i for i in enc if S.byte_piece_value(vocab[i]) is not None]
    word = sp.encode("lo")
    special = [
        ("empty", []),
        ("ids 0 and 3 skipped", [0] + sp.encode("ba lo") + [3, 3, 0] + word),
        ("ids past the vocabulary skipped", [400, 2 ** 32 - 1] + word + [10 ** 6]),
        ("control pieces kept as text", [1, 2] + word),
        ("byte run across a skipped padding id", b[:2] + [3] + b[2:]),
        ("truncated byte run dropped", b[:2] + word),
        ("byte run split by a piece: both halves dropped", b[:1] + word + b[1:3]),
        ("lone continuation byte dropped", [byte_id[0x80]] + word + [byte_id[0x41]]),
        ("surrogate encoding dropped", [byte_id[0xED], byte_id[0xA0], byte_id[0x80]] + word),
        ("ascii bytes kept", [byte_id[c] for c in b"Hi!"]),
        ("U+2581 from bytes becomes a space", [byte_id[0xE2], byte_id[0x96], byte_id[0x81]] + word),
    ]
    for what, ids in special:
        cases.append({"what": what, "ids": [int(i) for i in ids], "text": S.decode(vocab, ids)})
    with open(os.path.join(HERE, "spm_tiny.model"), "wb") as f:
        f.write(model)
    with open(os.path.join(HERE, "spm_cases.json"), "w") as f:
        json.dump({"sentencepiece": spm.__version__, "pieces": pieces, "cases": cases}, f, ensure_ascii=False,
                  indent=0)
    print(f"spm_tiny.model: {len(model)} bytes, {len(pieces)} pieces; {len(cases)} cases")


if __name__ == "__main__":
    main()
