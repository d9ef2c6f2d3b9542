"""Pure-Python restatement of the reference's SentencePiece detokeniser
(crates/stt-wasm/src/tokenizer.rs), the step after the decode path.

TEST INFRASTRUCTURE ONLY: the checker for libsttb200's stt_spm_* calls, imported by tests/ and
by the fixture generator in tests/golden/.  The library never imports it.

Parity is pinned against the `sentencepiece` package (0.2.1 in this image) where the two agree
by construction: the vocabulary of a trained model (id_to_piece) and the text of encoded,
already-normalised input (the reference keeps the leading U+2581 that `sentencepiece` strips).
The remaining rules (skipped ids, dropped invalid byte runs, the u8::from_str_radix form of
byte pieces) follow the reference's code, cited per function.
"""
from __future__ import annotations


def read_varint(buf: bytes, pos: int):
    """tokenizer.rs:98-115: 7-bit groups until a byte without the continuation bit or the end
    of the buffer.  Returns (value, bytes consumed).  Shifts past bit 63 wrap (release build)."""
    value, shift, p = 0, 0, pos
    while p < len(buf):
        b = buf[p]
        p += 1
        value |= ((b & 0x7F) << (shift % 64)) & 0xFFFFFFFFFFFFFFFF
        shift += 7
        if b & 0x80 == 0:
            break
    return value, p - pos


def skip_field(buf: bytes, pos: int, wire_type: int) -> int:
    """tokenizer.rs:117-136."""
    if wire_type == 0:
        p = pos
        while p < len(buf) and buf[p] & 0x80:
            p += 1
        return p + 1
    if wire_type == 1:
        return pos + 8
    if wire_type == 2:
        n, used = read_varint(buf, pos)
        return pos + used + n
    if wire_type == 5:
        return pos + 4
    return pos + 1


def parse_sentence_piece(buf: bytes) -> str:
    """tokenizer.rs:74-96: the last field-1 string of a SentencePiece message, lossily decoded."""
    pos, piece = 0, ""
    while pos < len(buf):
        tag, used = read_varint(buf, pos)
        pos += used
        if tag >> 3 == 1 and tag & 7 == 2:
            n, used = read_varint(buf, pos)
            pos += used
            if pos + n > len(buf):
                raise ValueError("piece length runs past its entry")   # slice panic in the reference
            piece = buf[pos:pos + n].decode("utf-8", "replace")
            pos += n
        else:
            pos = skip_field(buf, pos, tag & 7)
    return piece


def parse_vocab(data: bytes) -> list:
    """tokenizer.rs:44-72: every top-level field-1 message is the next token id's piece."""
    pieces, pos = [], 0
    while pos < len(data):
        tag, used = read_varint(data, pos)
        pos += used
        if tag >> 3 == 1 and tag & 7 == 2:
            n, used = read_varint(data, pos)
            pos += used
            if pos + n > len(data):
                raise ValueError("entry length runs past the model")   # slice panic in the reference
            pieces.append(parse_sentence_piece(data[pos:pos + n]))
            pos += n
        else:
            pos = skip_field(data, pos, tag & 7)
    return pieces


def _u8_from_str_radix16(s: str):
    """Rust's u8::from_str_radix(s, 16): an optional '+', then one or more hex digits, value < 256."""
    if s.startswith("+"):
        s = s[1:]
    if not s or any(c not in "0123456789abcdefABCDEF" for c in s):
        return None
    v = int(s, 16)
    return v if v < 256 else None


def byte_piece_value(piece: str):
    """tokenizer.rs:166-171: "<0xHH>" of six bytes whose characters 3..5 parse as a u8."""
    raw = piece.encode("utf-8")
    if len(raw) != 6 or not piece.startswith("<0x") or not piece.endswith(">"):
        return None
    return _u8_from_str_radix16(raw[3:5].decode("utf-8"))


def decode(vocab: list, ids) -> str:
    """tokenizer.rs:150-192."""
    pieces, run = [], bytearray()

    def flush():
        if run:
            try:
                pieces.append(bytes(run).decode("utf-8"))
            except UnicodeDecodeError:
                pass                     # an invalid byte run is dropped whole
            run.clear()

    for i in ids:
        i = int(i)
        if i == 0 or i == 3 or not 0 <= i < len(vocab):
            continue
        v = byte_piece_value(vocab[i])
        if v is not None:
            run.append(v)
            continue
        flush()
        pieces.append(vocab[i])
    flush()
    return "".join(pieces).replace("▁", " ")
