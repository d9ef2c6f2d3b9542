"""Generates the committed golden fixtures of tests/golden/ from the stt-web reference.

Run where a checkout of the stt-web reference is readable, naming its root either as the first
argument or in the STT_WEB_REFERENCE environment variable:

    python tests/golden/make_golden.py <path of the stt-web checkout>

Fixtures written (all small):
  q4_quantize.npz     inputs and the bytes scripts/quantize.py:quantize_q4_0 produces for them
  tiny_ref.gguf       a tiny checkpoint converted by scripts/quantize.py:load_and_quantize_model
                      (the reference's own safetensors -> Q4_0 GGUF pipeline, Q4_0 embeddings)
  tiny_ref_meta.json  the shapes of that checkpoint
  q4_matmul_kats.npz  the four self-contained cases of crates/stt-wasm/tests/q4_matmul.rs:100-393,
                      restated: formula weights, that test's own quantiser (truncating f32->f16,
                      round half away from zero), its CPU dequantisation and f32 reference product
  f16_gguf.npy        f16_to_f32 of crates/stt-wasm/src/gguf.rs:45-73 for all 65536 inputs
"""
from __future__ import annotations

import json
import os
import struct
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_root() -> str:
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("STT_WEB_REFERENCE")
    if not root or not os.path.isfile(os.path.join(root, "scripts", "quantize.py")):
        sys.exit("usage: make_golden.py <stt-web checkout> (or set STT_WEB_REFERENCE); "
                 "the checkout must hold scripts/quantize.py")
    return root


def ref_quantize_module():
    sys.path.insert(0, os.path.join(reference_root(), "scripts"))
    import quantize  # noqa: E402  (the reference's script, imported unmodified)
    return quantize


def make_q4_quantize(quantize):
    import torch
    rng = np.random.default_rng(20261201)
    parts = []
    for scale in (0.02, 1.0, 1e-3, 1e-5, 50.0):
        parts.append((rng.standard_normal(32 * 64) * scale).astype(np.float32))
    edge = np.zeros((8, 32), np.float32)
    edge[1, :] = 1e-7                      # tiny block: f16 subnormal scale
    edge[2, 5] = 3.5                       # single spike
    edge[3, :] = np.linspace(-7, 7, 32)    # exact multiples of the scale
    edge[4, :] = np.linspace(-1, 1, 32) * 0.5
    edge[4, ::7] = 0.5 * 7 / 7             # values on rounding ties
    edge[5, :] = -2.0                      # negative constant
    edge[6, :] = (np.arange(32) % 15 - 7).astype(np.float32) * 0.1
    edge[7, :] = np.float32(65504.0 * 7)   # scale overflows f16 -> inf
    parts.append(edge.ravel())
    x = np.concatenate(parts)
    blocks = []
    for i in range(x.size // 32):  # quantize per block so a non-finite block stays isolated
        b = x[i * 32:(i + 1) * 32]
        with np.errstate(all="ignore"):
            blocks.append(np.frombuffer(quantize.quantize_q4_0(torch.from_numpy(b.copy())), np.uint8))
    y = np.concatenate(blocks)
    np.savez_compressed(os.path.join(HERE, "q4_quantize.npz"), x=x, q=y)


TINY = dict(num_layers=2, hidden=256, heads=2, ffn=512, vocab=1000, text_vocab=1001, codebooks=4, audio_vocab=300)


def make_tiny_gguf(quantize):
    import torch
    from safetensors.torch import save_file
    t = TINY
    D, F = t["hidden"], t["ffn"]
    g = torch.Generator().manual_seed(1234)
    tensors = {}

    def w(*shape, std=0.02, mean=0.0):
        return (torch.randn(*shape, generator=g) * std + mean).to(torch.bfloat16).to(torch.float32)

    for i in range(t["codebooks"]):
        tensors[f"emb.{i}.weight"] = w(t["audio_vocab"], D)
    tensors["text_emb.weight"] = w(t["text_vocab"], D)
    tensors["text_linear.weight"] = w(t["vocab"], D)
    tensors["out_norm.alpha"] = w(1, 1, D, mean=1.0)
    for l in range(t["num_layers"]):
        p = f"transformer.layers.{l}."
        tensors[p + "norm1.alpha"] = w(1, 1, D, mean=1.0)
        tensors[p + "self_attn.in_proj_weight"] = w(3 * D, D)
        tensors[p + "self_attn.out_proj.weight"] = w(D, D)
        tensors[p + "norm2.alpha"] = w(1, 1, D, mean=1.0)
        tensors[p + "gating.linear_in.weight"] = w(2 * F, D)
        tensors[p + "gating.linear_out.weight"] = w(D, F)
    tensors["extra_heads.0.weight"] = w(6, D)          # skipped by the converter (VAD head)
    tensors["mimi.encoder.conv.weight"] = w(4, 32)      # not an STT tensor: filtered out
    with tempfile.TemporaryDirectory() as d:
        save_file(tensors, os.path.join(d, "model.safetensors"))
        out = os.path.join(d, "tiny.gguf")
        quantize.load_and_quantize_model(__import__("pathlib").Path(d), __import__("pathlib").Path(out), 512)
        data = open(out, "rb").read()
    open(os.path.join(HERE, "tiny_ref.gguf"), "wb").write(data)
    json.dump(t, open(os.path.join(HERE, "tiny_ref_meta.json"), "w"), indent=1)


# ---- crates/stt-wasm/tests/q4_matmul.rs helpers, restated ----------------------------------

def rs_f32_to_f16_bits(val: np.float32) -> int:
    """q4_matmul.rs:41-61: truncating conversion, subnormals flushed to zero."""
    bits = int(np.float32(val).view(np.uint32))
    sign = (bits >> 16) & 0x8000
    exp = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    if exp == 255:
        return sign | 0x7C00 | int(mant != 0)
    new_exp = exp - 127 + 15
    if new_exp >= 31:
        return sign | 0x7C00
    if new_exp <= 0:
        return sign
    return sign | (new_exp << 10) | (mant >> 13)


def rs_quantize_block(values: np.ndarray) -> bytes:
    """q4_matmul.rs:64-82 (f32 arithmetic; Rust f32::round is half away from zero)."""
    v = values.astype(np.float32)
    abs_max = np.float32(0.0)
    for x in v:
        abs_max = max(abs_max, np.float32(abs(x)))
    scale = np.float32(abs_max / np.float32(7.0)) if abs_max > 0 else np.float32(1.0)
    out = bytearray(struct.pack("<H", rs_f32_to_f16_bits(scale)))

    def rnd(x):
        q = np.float32(x / scale)
        r = np.floor(np.abs(q) + np.float32(0.5)) * np.sign(q)
        return int(np.clip(r, -8.0, 7.0))

    for j in range(16):
        lo = (rnd(v[j]) + 8) & 0x0F
        hi = (rnd(v[j + 16]) + 8) & 0x0F
        out.append((hi << 4) | lo)
    return bytes(out)


def rs_quantize_matrix(data: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = bytearray()
    for r in range(rows):
        for b in range(cols // 32):
            out += rs_quantize_block(data[r * cols + b * 32: r * cols + b * 32 + 32])
    return np.frombuffer(bytes(out), np.uint8)


def rs_dequantize(raw: np.ndarray, n: int) -> np.ndarray:
    """q4_matmul.rs:12-34: assumes a normal f16 scale."""
    out = np.zeros(n, np.float32)
    for b in range(n // 32):
        o = b * 18
        bits = int(raw[o]) | (int(raw[o + 1]) << 8)
        sign, exp, mant = (bits >> 15) & 1, (bits >> 10) & 0x1F, bits & 0x3FF
        d = np.uint32((sign << 31) | (((exp - 15 + 127) & 0xFF) << 23) | (mant << 13)).view(np.float32)
        for i in range(16):
            byte = int(raw[o + 2 + i])
            out[b * 32 + i] = np.float32((byte & 0x0F) - 8.0) * d
            out[b * 32 + i + 16] = np.float32(((byte >> 4) & 0x0F) - 8.0) * d
    return out


def rs_cpu_matmul(deq: np.ndarray, n: int, k: int, x: np.ndarray) -> np.ndarray:
    """The f32 loop of q4_matmul.rs:133-138 (expected[row] += input[col] * w[row, col])."""
    out = np.zeros(n, np.float32)
    for row in range(n):
        acc = np.float32(0.0)
        for col in range(k):
            acc = np.float32(acc + np.float32(x[col] * deq[row * k + col]))
        out[row] = acc
    return out


def make_kats():
    cases = {}
    # test_q4_matmul_identity_like (q4_matmul.rs:100-155)
    n = k = 64
    w = np.zeros(n * k, np.float32)
    for i in range(64):
        w[i * k + i] = 7.0
    x = (np.arange(k, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    cases["identity"] = (n, k, w, [x], 0.5)
    # test_q4_matmul_different_inputs (:157-229)
    n = k = 128
    w = np.array([((i * 7 + 13) % 15) - 7.0 for i in range(n * k)], np.float32)
    x1 = np.array([i * 0.1 - 6.4 for i in range(k)], np.float32)
    x2 = np.array([(i * 3 + 5) * 0.05 - 3.2 for i in range(k)], np.float32)
    cases["different_inputs"] = (n, k, w, [x1, x2], 1.0)
    # test_q4_matmul_larger_realistic (:231-307)
    n = k = 256
    w = np.array([(((i * 17 + 31) % 256) / 256.0 - 0.5) * 2.0 for i in range(n * k)], np.float32)
    xs = [np.array([((i * (s * 7 + 3) + s * 11 + 7) % 200) / 100.0 - 1.0 for i in range(k)], np.float32)
          for s in range(3)]
    cases["larger_realistic"] = (n, k, w, xs, 2.0)
    # test_embedding_sum_then_q4_matmul (:309-393): dim 128, 64 outputs, 32 codebooks of 8 rows
    n, k = 64, 128
    w = np.array([((i * 13 + 7) % 15) - 7.0 for i in range(n * k)], np.float32)
    tables = np.array([[[((cb * 10000 + tok * 100 + d) * 7 + 3) % 200 / 100.0 - 1.0 for d in range(k)]
                        for tok in range(8)] for cb in range(32)], np.float32)
    sets = [[0] * 32, [1] * 32, [i % 8 for i in range(32)]]
    xs = []
    for toks in sets:
        acc = np.zeros(k, np.float32)
        for cb, t in enumerate(toks):
            acc = (acc + tables[cb, t]).astype(np.float32)
        xs.append(acc)
    cases["embedding_sum"] = (n, k, w, xs, None)
    arrays = {}
    for name, (n, k, w, xs, tol) in cases.items():
        raw = rs_quantize_matrix(w, n, k)
        deq = rs_dequantize(raw, n * k)
        arrays[f"{name}__shape"] = np.array([n, k])
        arrays[f"{name}__raw"] = raw
        arrays[f"{name}__x"] = np.stack(xs)
        arrays[f"{name}__expected"] = np.stack([rs_cpu_matmul(deq, n, k, x) for x in xs])
        arrays[f"{name}__tol"] = np.array([tol if tol is not None else -1.0], np.float32)
    np.savez_compressed(os.path.join(HERE, "q4_matmul_kats.npz"), **arrays)


def make_f16_gguf():
    """gguf.rs:45-73 restated for every 16-bit pattern."""
    out = np.zeros(65536, np.uint32)
    for bits in range(65536):
        sign, exponent, mantissa = (bits >> 15) & 1, (bits >> 10) & 0x1F, bits & 0x3FF
        if exponent == 0:
            if mantissa == 0:
                out[bits] = sign << 31
            else:
                e, m = 1, mantissa
                while (m & 0x400) == 0:
                    m <<= 1
                    e += 1
                m &= 0x3FF
                f32_exp = (127 - (15 + e - 1)) & 0xFFFFFFFF
                out[bits] = (sign << 31) | (f32_exp << 23) | (m << 13)
        elif exponent == 31:
            out[bits] = (sign << 31) | (0xFF << 23) | (mantissa << 13)
        else:
            out[bits] = (sign << 31) | ((exponent - 15 + 127) << 23) | (mantissa << 13)
    np.save(os.path.join(HERE, "f16_gguf.npy"), out)


def main():
    quantize = ref_quantize_module()
    make_q4_quantize(quantize)
    make_tiny_gguf(quantize)
    make_kats()
    make_f16_gguf()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
