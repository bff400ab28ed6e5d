"""The tensor-core GEMM behind large frontend contractions (GPU).

to_gemm_tf32x3 through the C ABI: C[m][n] = sum_k A[m][k] B[n][k] from TF32
hi/lo splits (three TF32 products, fp32 accumulation in TMEM drained in IEEE
fp32).  Against a float64 product of the same fp32 inputs: relative L2 error
<= 1e-5 (the dropped lo*lo term is about 2^-22), for K within one
accumulation chunk, across several chunks and with a ragged last chunk, and
with zero-padded rows / columns.  Grids smaller than the 148 SMs, and the
tiles of a partial last wave, are split in K between two CTAs adding into a
zeroed C; a last wave fuller than half the SMs is not.  Argument errors are
reported, not faulted.
"""
import numpy as np
import pytest

from tensoroperations_b200 import abi

pytestmark = pytest.mark.gpu


def tf32_split(x):
    """hi = x rounded to TF32 (nearest, ties away from zero), lo = x - hi (exact)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    hb = ((b + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).astype(np.uint32)
    hi = hb.view(np.float32)
    return hi, (x.astype(np.float32) - hi).astype(np.float32)


def run(M, N, K, Mp, Np, Kp, seed):
    import torch
    rng = np.random.default_rng(seed)
    A = np.zeros((Mp, Kp), np.float32)
    B = np.zeros((Np, Kp), np.float32)
    A[:M, :K] = rng.standard_normal((M, K)).astype(np.float32)
    B[:N, :K] = rng.standard_normal((N, K)).astype(np.float32)
    ah, al = tf32_split(A)
    bh, bl = tf32_split(B)
    d = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (ah, al, bh, bl)]
    C = torch.full((Mp, Np), float("nan"), dtype=torch.float32, device="cuda")
    abi.gemm_tf32x3(Mp, Np, Kp, *d, C)
    torch.cuda.synchronize()
    abi.check(abi.lib.to_device_status(1), "device status")
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    got = C.cpu().numpy().astype(np.float64)
    return np.linalg.norm(got - ref) / np.linalg.norm(ref), got, ref


@pytest.mark.parametrize("M,N,K,Mp,Np,Kp", [
    (128, 256, 32, 128, 256, 32),        # one tile, one K step
    (300, 500, 200, 384, 512, 224),      # ragged, zero-padded, one chunk
    (256, 256, 1504, 256, 256, 1504),    # 47 K steps: two full chunks and a ragged one
    (1024, 768, 4096, 1024, 768, 4096),  # 128 K steps, 8 chunks
    (1600, 3000, 90, 1664, 3072, 96),    # 156 tiles: one full wave, the last 8 split in K
    (1536, 5120, 64, 1536, 5120, 64),    # 240 tiles: a last wave of 92, not split
])
def test_gemm_matches_float64(M, N, K, Mp, Np, Kp):
    err, got, ref = run(M, N, K, Mp, Np, Kp, seed=M + N + K)
    assert err <= 1e-5, err
    # padded rows and columns come out zero
    assert np.all(got[M:, :] == 0) and np.all(got[:, N:] == 0)


def test_bad_sizes_are_rejected():
    import torch
    x = torch.zeros(128 * 32, device="cuda")
    c = torch.zeros(128 * 256, device="cuda")
    with pytest.raises(abi.ToError):
        abi.gemm_tf32x3(100, 256, 32, x, x, x, x, c)
    with pytest.raises(abi.ToError):
        abi.gemm_tf32x3(128, 256, 30, x, x, x, x, c)
