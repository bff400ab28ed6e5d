"""Parity of the sm_100a SEM 3D elastic kernel with the CPU oracle (GPU).

Tolerances (relative L2 over all three force components, as BASELINE states):
  f32: <= 1e-5 against the same-precision oracle;  f64: <= 1e-12.
Small meshes use odd, distinct extents so a transposed index cannot pass, and
element counts that leave a partial batch.  The full config-3 mesh (64^3
hexes, NGLL 5, f32, assembled) is checked against the oracle too (seconds on
the host) and through size-independent properties: rigid translation in the
kernel, linearity, symmetry of the assembled operator.
"""
import numpy as np
import pytest

from oracle import sem as osem
from tensoroperations_b200 import abi
from tensoroperations_b200.sem3d import structured_problem, to_device

pytestmark = pytest.mark.gpu

TOL = {np.float32: 1e-5, np.float64: 1e-12}


def _run(prob, accumulate=False, f_init=None):
    import torch
    u, f, arrays, ibool = to_device(prob)
    if f_init is not None:
        for c in range(3):
            f[c].copy_(torch.from_numpy(f_init[c]))
    plan = prob.plan()
    plan.apply(plan.fields(u, f, arrays, ibool), accumulate=accumulate,
               stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return [x.cpu().numpy() for x in f]


def _oracle(prob):
    if prob.assembled:
        return osem.assembled(prob.nelem, prob.ngll, prob.nglob, prob.ibool, prob.u, prob.arrays,
                              prob.H, prob.Hw, prob.w, prob.dtype)
    return osem.local(prob.nelem, prob.ngll, prob.u, prob.arrays, prob.H, prob.Hw, prob.w,
                      prob.dtype)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("assembled", [False, True])
@pytest.mark.parametrize("mesh", [(1, 1, 1), (3, 5, 7), (7, 3, 2), (33, 1, 1)])
def test_small_meshes_match_oracle(dtype, assembled, mesh):
    prob = structured_problem(*mesh, ngll=5, dtype=dtype, assembled=assembled, seed=99)
    got = _run(prob)
    ref = _oracle(prob)
    err = osem.rel_l2(got, ref)
    assert err <= TOL[dtype], err


def test_element_count_not_a_multiple_of_the_batch():
    for E in (1, 31, 33, 65, 1001):
        prob = structured_problem(E, 1, 1, ngll=5, dtype=np.float32, assembled=False, seed=E)
        assert osem.rel_l2(_run(prob), _oracle(prob)) <= 1e-5


def test_accumulate_adds_into_f():
    prob = structured_problem(4, 3, 2, ngll=5, dtype=np.float32, assembled=True, seed=5)
    base = [np.full(prob.nglob, 0.25, dtype=np.float32) * (c + 1) for c in range(3)]
    got = _run(prob, accumulate=True, f_init=base)
    ref = _oracle(prob)
    assert osem.rel_l2([g - b for g, b in zip(got, base)], ref) <= 1e-5


def test_zero_elements_is_a_no_op():
    import torch
    prob = structured_problem(1, 1, 1, ngll=5, dtype=np.float32, assembled=False)
    _, w, H, Hw = abi.gll_operators(5)
    plan = abi.Sem3dPlan(np.float32, 5, 0, H, Hw, w)
    u, f, arrays, _ = to_device(prob)
    f[0].fill_(7.0)
    plan.apply(plan.fields(u, f, arrays))
    torch.cuda.synchronize()
    assert float(f[0][0]) == 7.0


@pytest.fixture(scope="module")
def full():
    """The bench configuration: 64^3 hexes, NGLL 5, f32, assembled."""
    import torch
    prob = structured_problem(64, 64, 64, ngll=5, dtype=np.float32, assembled=True)
    u, f, arrays, ibool = to_device(prob)
    plan = prob.plan()
    stream = torch.cuda.current_stream().cuda_stream

    def apply(uu):
        out = [torch.empty_like(x) for x in uu]
        plan.apply(plan.fields(uu, out, arrays, ibool), stream=stream)
        return out
    return prob, u, apply


def test_full_size_matches_oracle(full):
    import torch
    prob, u, apply = full
    got = [x.cpu().numpy() for x in apply(u)]
    torch.cuda.synchronize()
    ref = _oracle(prob)
    assert osem.rel_l2(got, ref) <= 1e-5


def test_full_size_rigid_translation(full):
    import torch
    prob, u, apply = full
    const = [torch.full_like(u[0], v) for v in (1.0, -2.0, 0.5)]
    f = apply(const)
    fu = apply(u)
    num = max(float(x.abs().max()) for x in f)
    den = max(float(x.abs().max()) for x in fu)
    assert num <= 1e-4 * den


def test_full_size_linearity_and_symmetry(full):
    import torch
    prob, u, apply = full
    g = torch.Generator(device="cuda").manual_seed(11)
    v = [torch.randn(u[0].shape, device="cuda", generator=g) for _ in range(3)]
    Ku, Kv = apply(u), apply(v)
    Kw = apply([2.0 * a - 3.0 * b for a, b in zip(u, v)])
    lin = torch.sqrt(sum(((kw - (2 * ku - 3 * kv)).double() ** 2).sum() for kw, ku, kv in zip(Kw, Ku, Kv)))
    ref = torch.sqrt(sum(((2 * ku - 3 * kv).double() ** 2).sum() for ku, kv in zip(Ku, Kv)))
    assert float(lin / ref) < 1e-5
    vKu = sum(float((a.double() * b.double()).sum()) for a, b in zip(v, Ku))
    uKv = sum(float((a.double() * b.double()).sum()) for a, b in zip(u, Kv))
    scale = sum(float((a.double().abs() * b.double().abs()).sum()) for a, b in zip(v, Ku))
    assert abs(vKu - uKv) <= 1e-5 * scale


def test_unaligned_arrays_take_the_streaming_kernel_and_match():
    """Arrays offset by one value are not 16-byte aligned: the register-streaming
    kernel runs instead of the TMA-staged one and must give the same answer."""
    import torch
    prob = structured_problem(5, 3, 2, ngll=5, dtype=np.float32, assembled=True, seed=17)

    def shifted(x):
        t = torch.empty(x.size + 1, dtype=torch.float32 if x.dtype == np.float32 else torch.int32,
                        device="cuda")
        t[1:].copy_(torch.from_numpy(x))
        return t[1:]
    arrays = {n: shifted(a) for n, a in prob.arrays.items()}
    u = [shifted(x) for x in prob.u]
    f = [torch.zeros(prob.nglob, device="cuda") for _ in range(3)]
    ib = shifted(prob.ibool)
    assert arrays["xix"].data_ptr() % 16 != 0
    plan = prob.plan()
    plan.apply(plan.fields(u, f, arrays, ib), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert osem.rel_l2([x.cpu().numpy() for x in f], _oracle(prob)) <= 1e-5


@pytest.mark.parametrize("variant", ["0", "1", "2", "3", "4", "5", "6", "7"])
def test_every_kernel_variant_matches_oracle(variant):
    """TO_SEM3D_VARIANT selects the f32 kernel (0: point-pair pipelined 8 elements x
    2 CTAs/SM, 1: TMA-staged 8 x 2, 2: register streaming, 3: point-pair 4 x 4,
    4: point-pair 16 x 1); each one is checked in a fresh process on assembled and
    element-local meshes with a partial batch."""
    import os
    import subprocess
    import sys
    code = (
        "import numpy as np, torch\n"
        "from oracle import sem as osem\n"
        "from tensoroperations_b200.sem3d import structured_problem, to_device\n"
        "for asm, mesh in ((True, (7, 5, 3)), (False, (37, 1, 1))):\n"
        "    p = structured_problem(*mesh, ngll=5, dtype=np.float32, assembled=asm, seed=3)\n"
        "    u, f, a, ib = to_device(p)\n"
        "    pl = p.plan(); pl.apply(pl.fields(u, f, a, ib)); torch.cuda.synchronize()\n"
        "    got = [x.cpu().numpy() for x in f]\n"
        "    ref = (osem.assembled(p.nelem, 5, p.nglob, p.ibool, p.u, p.arrays, p.H, p.Hw, p.w, np.float32)\n"
        "           if asm else osem.local(p.nelem, 5, p.u, p.arrays, p.H, p.Hw, p.w, np.float32))\n"
        "    err = osem.rel_l2(got, ref)\n"
        "    assert err <= 1e-5, (asm, err)\n"
        "from tensoroperations_b200 import abi\n"
        "abi.check(abi.lib.to_device_status(0), 'status')\n"
        "print('ok')\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, TO_SEM3D_VARIANT=variant, PYTHONPATH=root)
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


@pytest.mark.parametrize("mesh", [(6, 5, 4), (3, 3, 1)])
def test_interleaved_node_layout(mesh):
    """Assembled u and f interleaved per node (x, y, z, unused): the same result
    as the oracle, with 128-bit gathers and scatter-adds."""
    import torch
    prob = structured_problem(*mesh, ngll=5, dtype=np.float32, assembled=True, seed=12)
    u4 = np.zeros((prob.nglob, 4), dtype=np.float32)
    for c in range(3):
        u4[:, c] = prob.u[c]
    du4 = torch.from_numpy(u4).cuda()
    df4 = torch.full((prob.nglob, 4), float("nan"), device="cuda")
    arrays = {k: torch.from_numpy(v).cuda() for k, v in prob.arrays.items()}
    ibool = torch.from_numpy(prob.ibool).cuda()
    plan = abi.Sem3dPlan(np.float32, 5, prob.nelem, prob.H, prob.Hw, prob.w, nglob=prob.nglob,
                         assembled=True, interleaved=True)
    fl = plan.fields([du4, None, None], [df4, None, None], arrays, ibool)
    plan.apply(fl)
    torch.cuda.synchronize()
    got = df4.cpu().numpy()
    ref = osem.assembled(prob.nelem, 5, prob.nglob, prob.ibool, prob.u, prob.arrays, prob.H,
                         prob.Hw, prob.w, np.float32)
    assert osem.rel_l2([got[:, c].copy() for c in range(3)], ref) < 1e-5
    assert np.all(got[:, 3] == 0.0)


def test_interleaved_layout_is_rejected_where_not_built():
    _, w, H, Hw = abi.gll_operators(5)
    with pytest.raises(abi.ToError) as e:
        abi.Sem3dPlan(np.float64, 5, 4, H, Hw, w, nglob=10, assembled=True, interleaved=True)
    assert e.value.status == abi.TO_ERR_UNSUPPORTED
