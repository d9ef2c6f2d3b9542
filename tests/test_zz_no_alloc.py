"""The split-K Q4 matmul that requests no device memory (stt_q4_matmul_device_noalloc) against
the allocating entry point stt_q4_matmul_device on the same inputs.

The two sum the reduction in different orders (per split, then across splits in split order), so
they agree to f32 rounding: the bound is 1e-5 of the largest output.  Two calls in a row with the
same inputs must also agree bit for bit with each other; the second call only works if the first
left every tile counter of the fixed scratch at zero."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
import stt_b200
from stt_b200._lib import lib, STT_E_INVALID_ARG

pytestmark = pytest.mark.gpu

REL = 1e-5


def q4(n, k, seed):
    rng = np.random.default_rng(seed)
    return stt_b200.quantize_q4_0((rng.standard_normal(n * k) * 0.02).astype(np.float32))


def existing(t, x, rows, n, in_dtype):
    import torch
    out = torch.empty(rows, n, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib().stt_q4_matmul_device(t._h, x.data_ptr(), in_dtype, rows, out.data_ptr(), s) == 0
    return out


def noalloc(t, x, rows, n, in_dtype, splits, out=None):
    import torch
    if out is None:
        out = torch.full((rows, n), float("nan"), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    rc = lib().stt_q4_matmul_device_noalloc(t._h, x.data_ptr(), in_dtype, rows, splits, out.data_ptr(), s)
    assert rc == 0, lib().stt_last_error().decode()
    return out


@pytest.mark.parametrize("n,k,rows,splits", [(2048, 8448, 1, 8), (2048, 2048, 4, 4), (8001, 2048, 3, 2),
                                             (6144, 2048, 16, 1), (16896, 2048, 1, 16)])
def test_two_calls_in_a_row_match_the_allocating_entry_point(n, k, rows, splits):
    import torch
    raw = q4(n, k, n + k + rows)
    t = stt_b200.Q4Tensor.from_q4_bytes(raw, (n, k))
    x = torch.randn(rows, k, dtype=torch.float32, device="cuda")
    ref = existing(t, x, rows, n, 0)
    a = noalloc(t, x, rows, n, 0, splits)
    b = noalloc(t, x, rows, n, 0, splits)
    torch.cuda.synchronize()
    ref_h, a_h, b_h = ref.cpu().numpy(), a.cpu().numpy(), b.cpu().numpy()
    scale = np.abs(ref_h).max()
    assert np.isfinite(a_h).all()
    assert np.abs(a_h - ref_h).max() <= REL * scale
    assert np.array_equal(a_h.view(np.uint32), b_h.view(np.uint32))
    # and against the oracle on a few rows
    exp = O.q4_matmul(raw, n, k, x[:1].cpu().numpy())
    assert np.abs(a_h[:1] - exp).max() <= REL * np.abs(exp).max()


def test_bf16_input_and_changing_split_counts():
    import torch
    n, k, rows = 2048, 2048, 5
    raw = q4(n, k, 5)
    t = stt_b200.Q4Tensor.from_q4_bytes(raw, (n, k))
    x = torch.randn(rows, k, dtype=torch.float32, device="cuda").to(torch.bfloat16)
    ref = existing(t, x, rows, n, 1).cpu().numpy()
    scale = np.abs(ref).max()
    for splits in (3, 7, 1, 64, 7):
        got = noalloc(t, x, rows, n, 1, splits).cpu().numpy()
        assert np.abs(got - ref).max() <= REL * scale, splits


def test_calls_leave_device_memory_unchanged():
    import torch
    n, k, rows = 2048, 8448, 2
    t = stt_b200.Q4Tensor.from_q4_bytes(q4(n, k, 6), (n, k))
    x = torch.randn(rows, k, dtype=torch.float32, device="cuda")
    out = torch.empty(rows, n, dtype=torch.float32, device="cuda")
    noalloc(t, x, rows, n, 0, 4, out)  # the first call on the device looks the scratch address up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for splits in (4, 8, 16):
        noalloc(t, x, rows, n, 0, splits, out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_sizes_beyond_the_fixed_scratch_are_rejected():
    import torch
    n, k = 16896, 2048
    t = stt_b200.Q4Tensor.from_q4_bytes(q4(n, k, 7), (n, k))
    x = torch.randn(16, k, dtype=torch.float32, device="cuda")
    out = torch.empty(16, n, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    # 4 splits x 16 rows x 16896 outputs x 4 bytes = 4.3 MB > 4 MiB
    rc = lib().stt_q4_matmul_device_noalloc(t._h, x.data_ptr(), 0, 16, 4, out.data_ptr(), s)
    assert rc == STT_E_INVALID_ARG
    msg = lib().stt_last_error().decode()
    assert "fixed scratch holds 4194304" in msg, msg
    for bad in (0, 65, 65536):
        assert lib().stt_q4_matmul_device_noalloc(t._h, x.data_ptr(), 0, 1, bad, out.data_ptr(), s) == STT_E_INVALID_ARG
        assert "splits" in lib().stt_last_error().decode()
    # the f16 tensor-core product needs scratch that grows with the rows: not offered here
    rc = lib().stt_q4_matmul_device_noalloc(t._h, x.data_ptr(), 2, 1, 2, out.data_ptr(), s)
    assert rc == STT_E_INVALID_ARG
    assert "in_dtype 2" in lib().stt_last_error().decode()
    # misaligned input
    rc = lib().stt_q4_matmul_device_noalloc(t._h, C.c_void_p(x.data_ptr() + 4), 0, 1, 2, out.data_ptr(), s)
    assert rc == STT_E_INVALID_ARG
    # the rejected calls launched nothing: a valid call still matches
    ref = existing(t, x[:2], 2, n, 0).cpu().numpy()
    got = noalloc(t, x[:2], 2, n, 0, 3).cpu().numpy()
    assert np.abs(got - ref).max() <= REL * np.abs(ref).max()
