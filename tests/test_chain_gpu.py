"""The permuted multilevel contraction chain on the tensor cores (GPU).

T[a,b,c,d] = sum_{e,f} A[a,e,c,f] B[f,b,e,d];  R[a,d] = sum_{b,c} T[a,b,c,d] C[c,b]
against numpy in float64 on the same float32 inputs (N(0,1), seeded).
Tolerance: relative L2 <= 1e-5 (fp32), on T and on R.  The split-TF32
products make the result fp32-accurate; a plain TF32 product would miss this
tolerance by two orders of magnitude.
"""
import numpy as np
import pytest

from tensoroperations_b200 import abi

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _rel(a, b):
    return float(np.linalg.norm((a - b).ravel()) / np.linalg.norm(b.ravel()))


def _inputs(E, seed):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((E,) * 4, dtype=np.float32)
    B = rng.standard_normal((E,) * 4, dtype=np.float32)
    Cm = rng.standard_normal((E, E), dtype=np.float32)
    return A, B, Cm


def _reference(A, B, Cm):
    A64, B64, C64 = (x.astype(np.float64) for x in (A, B, Cm))
    E = A.shape[0]
    # T[a,b,c,d] = sum_{e,f} A[a,e,c,f] B[f,b,e,d]: a GEMM over (e,f)
    Am = A64.transpose(0, 2, 1, 3).reshape(E * E, E * E)          # (a,c) x (e,f)
    Bm = B64.transpose(2, 0, 1, 3).reshape(E * E, E * E)          # (e,f) x (b,d)
    T = (Am @ Bm).reshape(E, E, E, E).transpose(0, 2, 1, 3)       # [a,b,c,d]
    R = np.einsum("abcd,cb->ad", T, C64, optimize=True)
    return T, R


@pytest.mark.parametrize("E,seed", [(32, 1), (64, 2)])
def test_chain_matches_float64(E, seed):
    import torch
    A, B, Cm = _inputs(E, seed)
    Tref, Rref = _reference(A, B, Cm)
    dA, dB, dC = (torch.from_numpy(x).cuda() for x in (A, B, Cm))
    R = torch.full((E, E), float("nan"), device="cuda")
    T = torch.zeros((E,) * 4, device="cuda")
    ws = torch.empty(abi.lib.to_chain_workspace_bytes(E), dtype=torch.uint8, device="cuda")
    abi.chain_f32(E, dA, dB, dC, R, ws, T=T)
    torch.cuda.synchronize()
    abi.check(abi.lib.to_device_status(1), "to_device_status")
    assert _rel(T.cpu().numpy(), Tref) < TOL
    assert _rel(R.cpu().numpy(), Rref) < TOL
    # the fused path (no T) gives the same R
    R2 = torch.zeros((E, E), device="cuda")
    abi.chain_f32(E, dA, dB, dC, R2, ws)
    torch.cuda.synchronize()
    assert _rel(R2.cpu().numpy(), Rref) < TOL


def test_chain_rejects_bad_arguments():
    import torch
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(16, device="cuda")
    with pytest.raises(abi.ToError) as e:
        abi.chain_f32(48, x, x, x, x, ws)
    assert e.value.status == abi.TO_ERR_UNSUPPORTED
    with pytest.raises(abi.ToError) as e:
        abi.chain_f32(32, x, x, x, x, ws)  # workspace too small
    assert e.value.status == abi.TO_ERR_INVALID_ARGUMENT
