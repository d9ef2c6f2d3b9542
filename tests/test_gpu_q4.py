"""Q4_0 weight store and matmul on the GPU against the oracle: bit-exact dequantisation and the
isolated q4_matmul (gguf.rs:517-578) over the layer shapes of the model."""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import oracle as O
import stt_b200

pytestmark = pytest.mark.gpu

SHAPES = [(6144, 2048), (2048, 2048), (16896, 2048), (2048, 8448), (8001, 2048)]  # (N, K)


def q4_bytes(n, k, seed, std=0.02):
    rng = np.random.default_rng(seed)
    return stt_b200.quantize_q4_0((rng.standard_normal(n * k) * std).astype(np.float32))


@pytest.mark.parametrize("n,k", SHAPES)
def test_dequant_bit_exact(n, k):
    raw = q4_bytes(n, k, n + k)
    t = stt_b200.Q4Tensor.from_q4_bytes(raw, (n, k))
    got = t.dequant()
    ref = O.dequant_q4_0(raw, n, k)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_dequant_subnormal_and_edge_scales():
    z = np.load(os.path.join(GOLDEN, "q4_quantize.npz"))
    raw = z["q"]
    nblk = raw.size // 18
    k = 32 * 8
    n = nblk // 8
    raw = raw[: n * 8 * 18].copy()
    # force a few subnormal, zero and negative scales
    blocks = raw.reshape(-1, 18)
    blocks[0, :2] = [0x01, 0x00]
    blocks[1, :2] = [0xFF, 0x03]
    blocks[2, :2] = [0x00, 0x80]
    blocks[3, :2] = [0x00, 0xBC]
    t = stt_b200.Q4Tensor.from_q4_bytes(raw, (n, k))
    got = t.dequant()
    ref = O.dequant_q4_0(raw, n, k)
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin].view(np.uint32), ref[fin].view(np.uint32))


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", [1, 2, 3, 4, 7, 16])
def test_q4_matmul_matches_oracle(n, k, m):
    """Batches of 1 to 8 rows take one pass of the GEMV (16 rows: two passes of 8, or four of 4
    when K > 4096); 3 and 7 rows leave batch columns of the pass unused."""
    raw = q4_bytes(n, k, 7 * n + k)
    x = np.random.default_rng(m).standard_normal((1, m, k)).astype(np.float32)
    t = stt_b200.Q4Tensor.from_q4_bytes(raw, (n, k))
    got = stt_b200.q4_matmul(x, t)[0]
    ref = O.q4_matmul(raw, n, k, x[0])
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= 2e-6 * scale * np.sqrt(k / 2048), np.abs(got - ref).max() / scale


@pytest.mark.parametrize("case", ["identity", "different_inputs", "larger_realistic", "embedding_sum"])
def test_q4_matmul_reference_cases(case):
    z = np.load(os.path.join(GOLDEN, "q4_matmul_kats.npz"))
    n, k = [int(v) for v in z[f"{case}__shape"]]
    x = z[f"{case}__x"]
    t = stt_b200.Q4Tensor.from_q4_bytes(z[f"{case}__raw"], (n, k))
    out = stt_b200.q4_matmul(x[None], t)[0]
    exp = z[f"{case}__expected"]
    tol = float(z[f"{case}__tol"][0])
    if tol > 0:  # q4_matmul.rs:151, 228, 306
        assert np.abs(out - exp).max() < tol
    assert np.abs(out - exp).max() <= 1e-5 * max(1.0, np.abs(exp).max())
    for i in range(len(x)):
        for j in range(i + 1, len(x)):
            assert np.abs(out[i] - out[j]).sum() > 1.0


def test_q4_matmul_rejects_bad_shapes():
    raw = q4_bytes(64, 64, 1)
    with pytest.raises(stt_b200.SttError, match="byte count mismatch"):
        stt_b200.Q4Tensor.from_q4_bytes(raw[:-1], (64, 64))
    t = stt_b200.Q4Tensor.from_q4_bytes(raw, (64, 64))
    with pytest.raises(stt_b200.SttError, match="K dimension mismatch"):
        stt_b200.q4_matmul(np.zeros((1, 1, 32), np.float32), t)


def test_q4_matmul_bf16_input():
    import torch
    n, k, m = 2048, 2048, 4
    raw = q4_bytes(n, k, 99)
    t = stt_b200.Q4Tensor.from_q4_bytes(raw, (n, k))
    x = torch.randn(m, k, dtype=torch.float32).to(torch.bfloat16)
    dx = x.cuda()
    out = torch.empty(m, n, dtype=torch.float32, device="cuda")
    from stt_b200._lib import lib
    rc = lib().stt_q4_matmul_device(t._h, dx.data_ptr(), 1, m, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    ref = O.q4_matmul(raw, n, k, x.float().numpy())
    assert np.abs(out.cpu().numpy() - ref).max() <= 2e-6 * np.abs(ref).max()


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", [1, 16, 64, 200])
def test_q4_matmul_tensor_cores_f16_input(n, k, m):
    """in_dtype 2: tcgen05 MMAs with each dequantised weight split exactly into two f16 parts
    and f32 accumulation, the input taken as exact f16.  The products are exact, so only the f32
    sums differ from the oracle's; the bound is 1e-4 of the largest output."""
    import torch
    from stt_b200._lib import lib
    raw = q4_bytes(n, k, 3 * n + k + m)
    t = stt_b200.Q4Tensor.from_q4_bytes(raw, (n, k))
    x = torch.from_numpy(np.random.default_rng(m + n).standard_normal((m, k)).astype(np.float32)).to(torch.float16)
    dx = x.cuda()
    out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    rc = lib().stt_q4_matmul_device(t._h, dx.data_ptr(), 2, m, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib().stt_last_error().decode()
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    ref = O.q4_matmul(raw, n, k, x.float().numpy())
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max(), np.abs(got - ref).max() / np.abs(ref).max()


def test_q4_matmul_tensor_cores_rejects_unsupported():
    """in_dtype 2 needs in_features a multiple of 256 and Q4_0 scales of magnitude <= 4."""
    import torch
    from stt_b200._lib import lib
    m = 16
    for n, k, big in [(256, 320, False), (256, 512, True)]:
        raw = bytearray(q4_bytes(n, k, 5))
        if big:
            raw[18 * 7: 18 * 7 + 2] = np.float16(5.0).tobytes()  # one block with scale 5
        t = stt_b200.Q4Tensor.from_q4_bytes(bytes(raw), (n, k))
        dx = torch.zeros((m, k), dtype=torch.float16, device="cuda")
        out = torch.zeros((m, n), dtype=torch.float32, device="cuda")
        rc = lib().stt_q4_matmul_device(t._h, dx.data_ptr(), 2, m, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc != 0
        assert ("256" if not big else "at most 4") in lib().stt_last_error().decode()


def test_mma_gemv_bounded_wait_runs_out_and_the_next_call_recovers():
    """The test hook leaves the integer-MMA GEMV's first weight stage unloaded for one launch: the
    warps waiting for it give up after their limit, the kernel stops through its timeout path, and
    the call reports STT_E_DEVICE_FLAG (nothing faults or hangs).  The next call is exact again."""
    import time
    from stt_b200._lib import STT_E_DEVICE_FLAG, lib
    n, k, m = 2048, 2048, 4
    raw = q4_bytes(n, k, 17)
    x = np.random.default_rng(4).standard_normal((1, m, k)).astype(np.float32)
    t = stt_b200.Q4Tensor.from_q4_bytes(raw, (n, k))
    ref = O.q4_matmul(raw, n, k, x[0])
    assert lib().stt_debug_q4_arm_wait_timeout(t._h) == 0
    t0 = time.perf_counter()
    with pytest.raises(stt_b200.SttError) as err:
        stt_b200.q4_matmul(x, t)
    assert err.value.code == STT_E_DEVICE_FLAG
    print(f"timed out and returned in {time.perf_counter() - t0:.2f} s")
    t.status()  # the flag was cleared by the failed call
    got = stt_b200.q4_matmul(x, t)[0]
    assert np.abs(got - ref).max() <= 2e-6 * np.abs(ref).max()

