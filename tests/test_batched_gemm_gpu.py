"""Batched small GEMM with a shared left operand (config 2) on the GPU.

C[b] = A @ B[b] against numpy in float64 on the same inputs (A, B N(0,1)):
relative L2 <= 1e-5 (f32) and <= 1e-12 (f64).  Shapes: the configuration's
(5x5 @ 5x25, batch 65536) and the NGLL-8 one (8x8 @ 8x64), plus a ragged
batch.
"""
import numpy as np
import pytest

from tensoroperations_b200 import abi

pytestmark = pytest.mark.gpu
TOL = {np.float32: 1e-5, np.float64: 1e-12}


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("M,N,batch", [(5, 25, 65536), (8, 64, 1000), (5, 25, 7)])
def test_batched_small_gemm(dtype, M, N, batch):
    import torch
    rng = np.random.default_rng(M * 1000 + batch)
    A = rng.standard_normal((M, M))
    B = rng.standard_normal((batch, M, N)).astype(dtype)
    tdt = torch.float32 if dtype == np.float32 else torch.float64
    dB = torch.from_numpy(B).cuda()
    dC = torch.empty((batch, M, N), dtype=tdt, device="cuda")
    abi.batched_small_gemm(A, dB, dC)
    torch.cuda.synchronize()
    ref = np.einsum("ik,bkj->bij", A.astype(dtype).astype(np.float64), B.astype(np.float64))
    got = dC.cpu().numpy().astype(np.float64)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < TOL[dtype]


def test_rejects_unbuilt_shape():
    import torch
    B = torch.zeros((2, 3, 4), device="cuda")
    C = torch.zeros((2, 3, 4), device="cuda")
    with pytest.raises(abi.ToError) as e:
        abi.batched_small_gemm(np.eye(3), B, C)
    assert e.value.status == abi.TO_ERR_UNSUPPORTED
