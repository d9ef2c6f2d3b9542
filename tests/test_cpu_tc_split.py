"""The arithmetic behind the tensor-core path's weight operand (csrc/tc_gemm.cu, dequant_words), checked
exhaustively on the CPU over every f16 block scale and every Q4_0 value.

The dequantised weight q * s (q = nibble - 8, s the block's f16 scale; crates/stt-wasm/src/gguf.rs:616-633,
scripts/quantize.py:95-114) is split into two f16 parts with s' = s * 2^10: hi = rn(q * s') and
lo = rn(q * s' - hi), the latter one fused multiply-add.  The claims the kernel relies on:
  - s' is exact in f16 for every scale the loader lets through (|s| <= 4, tc_gemm_scales_ok);
  - the nibble trick gives q exactly: the f16 with bits 0x6400 | n is 1024 + n, minus 1032 is n - 8;
  - hi is finite and lo is exactly q * s' - hi, so hi + lo == q * s' with no error at all.
"""
import numpy as np


def _eligible_scales():
    bits = np.arange(0x10000, dtype=np.uint32)
    ok = (bits & 0x7FFF) <= 0x4400                      # the loader's test: |s| <= 4.0, no inf or nan
    return bits[ok].astype(np.uint16)


def test_eligibility_boundary_is_four():
    s = _eligible_scales().view(np.float16).astype(np.float64)
    assert np.isfinite(s).all() and np.abs(s).max() == 4.0
    above = np.array([0x4401, 0xC401, 0x7C00, 0x7E00], dtype=np.uint16).view(np.float16).astype(np.float64)
    assert not np.any(np.abs(above[np.isfinite(above)]) <= 4.0)


def test_scale_times_1024_is_exact_in_f16():
    s = _eligible_scales().view(np.float16)
    s1024 = s.astype(np.float64) * 1024.0
    assert np.array_equal(s1024.astype(np.float16).astype(np.float64), s1024)


def test_nibble_bias_trick_gives_q_exactly():
    n = np.arange(16, dtype=np.uint16)
    v = (n | 0x6400).view(np.float16).astype(np.float64)
    assert np.array_equal(v, 1024.0 + n)
    assert np.array_equal((v.astype(np.float16) - np.float16(1032)).astype(np.float64), n - 8.0)


def test_hi_lo_split_is_exact_for_every_scale_and_value():
    s1024 = (_eligible_scales().view(np.float16).astype(np.float64) * 1024.0)[:, None]
    q = np.arange(-8, 8, dtype=np.float64)[None, :]
    exact = q * s1024                                  # exact in f64: 4-bit times 11-bit significands
    hi = exact.astype(np.float16)                      # rn to f16, what __hmul2_rn gives
    assert np.isfinite(hi).all()
    rem = exact - hi.astype(np.float64)                # what the fused multiply-add computes before its rounding
    lo = rem.astype(np.float16)
    assert np.array_equal(lo.astype(np.float64), rem)  # the rounding of lo is exact ...
    assert np.array_equal(hi.astype(np.float64) + lo.astype(np.float64), exact)  # ... so hi + lo = q * s'
    # and scaling the accumulated products back by 2^-10 is exact in f32 (a power of two, no underflow)
    w = exact / 1024.0
    assert np.array_equal(w.astype(np.float32).astype(np.float64), w)
