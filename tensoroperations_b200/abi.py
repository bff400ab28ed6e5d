"""ctypes binding of include/tensoroperations_b200.h.

This is the Python-side counterpart a maintainer binds against the C ABI; the
C++ frontend under include/ and tensoroperations_b200/include/ is the other.
Every wrapper raises `ToError` with the library's own one-line reason when a
call returns a non-zero status.  The library is loaded from the package
directory (in-tree build); a missing library is an ImportError, never a silent
fallback.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libtensoroperations_b200.so"
HEADER = PKG.parent / "include" / "tensoroperations_b200.h"

TO_OK = 0
TO_ERR_INVALID_ARGUMENT = 1
TO_ERR_UNSUPPORTED = 2
TO_ERR_CUDA = 3
TO_ERR_SCRATCH = 4
TO_ERR_ALIGNMENT = 5
TO_ERR_TIMEOUT = 6
TO_ERR_COMM = 7
TO_ERR_NO_DEVICE = 8
TO_ERR_GRID = 9

TO_F32 = 0
TO_F64 = 1


class ToError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str):
        super().__init__(f"{where}: {status_name(status)}: {detail}")
        self.status = status


def _load():
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
    return C.CDLL(str(LIB_PATH))


lib = _load()


class Sem3dDesc(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("ngll", C.c_int32), ("nelem", C.c_int64),
                ("nglob", C.c_int64), ("assembled", C.c_int32), ("node_layout", C.c_int32),
                ("hprime", C.POINTER(C.c_double)), ("hprimewgll", C.POINTER(C.c_double)),
                ("wgll", C.POINTER(C.c_double))]


POINT_ARRAYS = ("xix", "xiy", "xiz", "etax", "etay", "etaz", "gamx", "gamy", "gamz",
                "jac", "l2m", "mu")


class Sem3dFields(C.Structure):
    _fields_ = [("u", C.c_void_p * 3), ("f", C.c_void_p * 3), ("ibool", C.c_void_p)] + \
        [(n, C.c_void_p) for n in POINT_ARRAYS] + [("u_norm2", C.c_void_p)]

    def copy(self) -> "Sem3dFields":
        out = Sem3dFields()
        C.pointer(out)[0] = self
        return out


class Sem2dFields(C.Structure):
    _fields_ = [("u", C.c_void_p * 2), ("f", C.c_void_p * 2)] + \
        [(n, C.c_void_p) for n in ("xix", "xiz", "gamx", "gamz", "jac", "l2m", "mu")]


SEM2D_ARRAYS = ("xix", "xiz", "gamx", "gamz", "jac", "l2m", "mu")


class Acoustic2dDesc(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("ngll", C.c_int32), ("nelem", C.c_int64),
                ("nglob", C.c_int64), ("hprime", C.c_void_p), ("hprimewgll", C.c_void_p),
                ("wgll", C.c_void_p)]


class Acoustic2dFields(C.Structure):
    _fields_ = [("u", C.c_void_p), ("f", C.c_void_p), ("ibool", C.c_void_p)] + \
        [(n, C.c_void_p) for n in ("xix", "xiz", "gamx", "gamz", "jac", "rho")]


class HostNodes(C.Structure):
    """to_host_nodes: host u / f (one array per component) and device stage arrays."""
    _fields_ = [("u", C.c_void_p * 3), ("f", C.c_void_p * 3), ("stage", C.c_void_p * 3)]


class Slab(C.Structure):
    """to_slab: one rank's z-slab of a structured mesh (see to_sem3d_elastic_mgpu)."""
    _fields_ = [("prev", C.c_int32), ("next", C.c_int32), ("layer_elems", C.c_int64),
                ("plane_nodes", C.c_int64), ("recv", C.c_void_p * 2), ("sync", C.c_void_p),
                ("f_is_zero", C.c_int32)]


NCCL_UNIQUE_ID_BYTES = 128


def _sig(name, restype, argtypes):
    fn = getattr(lib, name)
    fn.restype = restype
    fn.argtypes = argtypes
    return fn


_sig("to_abi_version", C.c_int, [])
_sig("to_status_string", C.c_char_p, [C.c_int])
_sig("to_last_error", C.c_char_p, [])
_sig("to_device_sm_count", C.c_int, [])
_sig("to_device_status", C.c_int, [C.c_int32])
_sig("to_mesh_structured_ibool", C.c_int, [C.c_int32] * 4 + [C.c_void_p])
_sig("to_gll_operators", C.c_int, [C.c_int32] + [C.c_void_p] * 4)
_sig("to_synth_fill", C.c_int, [C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_int32,
                                C.c_double, C.c_double])
_sig("to_synth_fill_at", C.c_int, [C.c_void_p, C.c_int32, C.c_int64, C.c_int64, C.c_uint64,
                                   C.c_int32, C.c_double, C.c_double])
_sig("to_sem3d_apply_elements", C.c_int, [C.c_void_p, C.POINTER(Sem3dFields), C.c_int64,
                                          C.c_int64, C.c_void_p])
_sig("to_sem3d_halo_pack", C.c_int, [C.c_int32, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p,
                                     C.c_void_p])
_sig("to_sem3d_halo_accumulate", C.c_int, [C.c_int32, C.c_void_p, C.c_int64, C.c_int64,
                                           C.c_void_p, C.c_void_p])
_sig("to_sumsq3_workspace_bytes", C.c_size_t, [C.c_int64])
_sig("to_sumsq3", C.c_int, [C.c_int32, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p,
                            C.c_size_t, C.c_void_p])
_sig("to_sumsq3_noalloc", C.c_int, [C.c_int32, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p,
                                    C.c_void_p])
_sig("to_sumsq3_noalloc_max_n", C.c_int64, [])
_sig("to_scale3", C.c_int, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p])
_sig("to_sem2d_elastic_local", C.c_int, [C.c_int32, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.POINTER(Sem2dFields), C.c_void_p])
_sig("to_sem2d_acoustic_apply", C.c_int, [C.POINTER(Acoustic2dDesc), C.POINTER(Acoustic2dFields),
                                          C.c_int32, C.c_void_p])
_sig("to_batched_small_gemm", C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int64,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p])
_sig("to_chain_workspace_bytes", C.c_size_t, [C.c_int32])
_sig("to_chain_f32", C.c_int, [C.c_int32] + [C.c_void_p] * 6 + [C.c_size_t, C.c_void_p])
_sig("to_gemm_tf32x3", C.c_int, [C.c_int64] * 3 + [C.c_void_p] * 6)
_sig("to_chain_flops", C.c_double, [C.c_int32])
_sig("to_synth_fill_device", C.c_int, [C.c_void_p, C.c_int32, C.c_int64, C.c_int64, C.c_uint64,
                                       C.c_int32, C.c_double, C.c_double, C.c_double, C.c_void_p])
_sig("to_axpy2_device", C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int64, C.c_void_p])
_sig("to_mesh_structured_ibool_device", C.c_int, [C.c_int32] * 4 + [C.c_void_p, C.c_void_p])
_sig("to_sem3d_plan_create", C.c_int, [C.POINTER(Sem3dDesc), C.POINTER(C.c_void_p)])
_sig("to_sem3d_plan_destroy", C.c_int, [C.c_void_p])
_sig("to_sem3d_apply", C.c_int, [C.c_void_p, C.POINTER(Sem3dFields), C.c_int32, C.c_void_p])
_sig("to_sem3d_algorithmic_bytes", C.c_double, [C.c_void_p])
_sig("to_sem3d_flops", C.c_double, [C.c_void_p])
_sig("to_nodes_interleave", C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p])
_sig("to_nodes_deinterleave", C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p])
_sig("to_slab_sync_bytes", C.c_size_t, [])
_sig("to_sem3d_elastic_mgpu", C.c_int, [C.c_void_p, C.POINTER(Sem3dFields), C.POINTER(Slab),
                                        C.c_void_p, C.c_void_p, C.c_void_p])
_sig("to_sem3d_elastic_mgpu_host", C.c_int, [C.c_void_p, C.POINTER(Sem3dFields), C.POINTER(Slab),
                                             C.c_void_p, C.POINTER(HostNodes), C.c_void_p,
                                             C.c_void_p])
_sig("to_nccl_unique_id", C.c_int, [C.c_void_p])
_sig("to_nccl_comm_init", C.c_int, [C.c_int32, C.c_int32, C.c_void_p, C.POINTER(C.c_void_p)])
_sig("to_nccl_comm_destroy", C.c_int, [C.c_void_p])
_sig("to_nccl_allreduce_sum_f64", C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p])


def status_name(status: int) -> str:
    return lib.to_status_string(status).decode()


def check(status: int, where: str):
    if status != TO_OK:
        raise ToError(status, where, lib.to_last_error().decode())


def header_functions(header: Path = HEADER):
    """Names of every function the public header declares."""
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(to_[a-z0-9_]+)\s*\(", text)))


def _ptr(a) -> int:
    if a is None:
        return 0
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()  # torch.Tensor


# ---- host utilities ---------------------------------------------------------

def gll_operators(ngll: int):
    """(nodes, weights, hprime H(i,p), hprimewgll Hw(q,i)) as float64 numpy arrays."""
    x = np.zeros(ngll)
    w = np.zeros(ngll)
    H = np.zeros((ngll, ngll))
    Hw = np.zeros((ngll, ngll))
    check(lib.to_gll_operators(ngll, _ptr(x), _ptr(w), _ptr(H), _ptr(Hw)), "to_gll_operators")
    return x, w, H, Hw


def structured_ibool(nex: int, ney: int, nez: int, ngll: int) -> np.ndarray:
    out = np.empty((nex * ney * nez, ngll, ngll, ngll), dtype=np.int32)
    check(lib.to_mesh_structured_ibool(nex, ney, nez, ngll, _ptr(out)), "to_mesh_structured_ibool")
    return out


def synth_fill(n: int, dtype, seed: int, dist: str, a: float, b: float,
               first: int = 0) -> np.ndarray:
    """Seeded fill: dist 'uniform' -> U[a,b), 'normal' -> N(a, b^2); elements
    [first, first + n) of the sequence."""
    dt = np.dtype(dtype)
    code = TO_F32 if dt == np.float32 else TO_F64
    out = np.empty(n, dtype=dt)
    check(lib.to_synth_fill_at(_ptr(out), code, first, n, seed,
                               {"uniform": 0, "normal": 1}[dist], a, b), "to_synth_fill_at")
    return out


def _fptrs(f):
    arr = (C.c_void_p * 3)(*[_ptr(x) for x in f])
    return arr


def halo_pack(dtype, f, offset: int, n: int, buf, stream: int = 0):
    """buf[c*n + i] = f[c][offset + i] on the device (one kernel)."""
    code = TO_F32 if np.dtype(dtype) == np.float32 else TO_F64
    check(lib.to_sem3d_halo_pack(code, _fptrs(f), offset, n, _ptr(buf), stream),
          "to_sem3d_halo_pack")


def halo_accumulate(dtype, f, offset: int, n: int, buf, stream: int = 0):
    """f[c][offset + i] += buf[c*n + i] on the device (one kernel)."""
    code = TO_F32 if np.dtype(dtype) == np.float32 else TO_F64
    check(lib.to_sem3d_halo_accumulate(code, _fptrs(f), offset, n, _ptr(buf), stream),
          "to_sem3d_halo_accumulate")


def _dcode(dtype):
    return TO_F32 if np.dtype(dtype) == np.float32 else TO_F64


def sumsq3_workspace_bytes(n: int) -> int:
    return lib.to_sumsq3_workspace_bytes(n)


def sumsq3(dtype, x, first: int, n: int, result, workspace, stream: int = 0):
    """result[0] (device double) = sum of x[c][first:first+n]^2; workspace is a
    device tensor of at least sumsq3_workspace_bytes(n) bytes."""
    nbytes = workspace.numel() * workspace.element_size()
    check(lib.to_sumsq3(_dcode(dtype), _fptrs(x), first, n, _ptr(result), _ptr(workspace), nbytes,
                        stream), "to_sumsq3")


def sumsq3_noalloc(dtype, x, first: int, n: int, result, stream: int = 0):
    """sumsq3 with the library's fixed scratch instead of a workspace (no
    allocation; calls that overlap on the GPU race on that scratch)."""
    check(lib.to_sumsq3_noalloc(_dcode(dtype), _fptrs(x), first, n, _ptr(result), stream),
          "to_sumsq3_noalloc")


def scale3(dtype, y, x, n: int, sumsq, stream: int = 0):
    """y[c][:n] = x[c][:n] / sqrt(sumsq[0]) on the device."""
    check(lib.to_scale3(_dcode(dtype), _fptrs(y), _fptrs(x), n, _ptr(sumsq), stream), "to_scale3")


def sem2d_elastic_local(ngll: int, nelem: int, H, Hw, w, u, f, arrays, stream: int = 0):
    """f[c] = K u (2D elastic P-SV, element-local) on the device; H, Hw, w host arrays."""
    ops = [np.ascontiguousarray(x, dtype=np.float64) for x in (H, Hw, w)]
    fl = Sem2dFields()
    for c in range(2):
        fl.u[c] = _ptr(u[c])
        fl.f[c] = _ptr(f[c])
    for n in SEM2D_ARRAYS:
        setattr(fl, n, _ptr(arrays[n]))
    check(lib.to_sem2d_elastic_local(ngll, nelem, ops[0].ctypes.data, ops[1].ctypes.data,
                                     ops[2].ctypes.data, C.byref(fl), stream),
          "to_sem2d_elastic_local")


def sem2d_acoustic_apply(ngll, nelem, nglob, H, Hw, w, u, f, ibool, arrays, dtype,
                         accumulate=False, stream: int = 0):
    """f = K u for the 2D acoustic operator (assembled) on the device."""
    ops = [np.ascontiguousarray(x, dtype=np.float64) for x in (H, Hw, w)]
    d = Acoustic2dDesc()
    d.dtype = TO_F64 if np.dtype(dtype) == np.float64 else TO_F32
    d.ngll, d.nelem, d.nglob = ngll, nelem, nglob
    d.hprime, d.hprimewgll, d.wgll = (x.ctypes.data for x in ops)
    fl = Acoustic2dFields()
    fl.u, fl.f, fl.ibool = _ptr(u), _ptr(f), _ptr(ibool)
    for n in ("xix", "xiz", "gamx", "gamz", "jac", "rho"):
        setattr(fl, n, _ptr(arrays[n]))
    check(lib.to_sem2d_acoustic_apply(C.byref(d), C.byref(fl), 1 if accumulate else 0, stream),
          "to_sem2d_acoustic_apply")


def batched_small_gemm(A, B, Cout, stream: int = 0):
    """Cout[b] = A @ B[b] on the device; A is a host (M, K) array, B (batch, K, N)."""
    Ah = np.ascontiguousarray(A, dtype=np.float64)
    M, K = Ah.shape
    batch, K2, N = B.shape
    assert K2 == K and tuple(Cout.shape) == (batch, M, N)
    code = TO_F64 if str(B.dtype).endswith("float64") else TO_F32
    check(lib.to_batched_small_gemm(code, M, K, N, batch, Ah.ctypes.data, _ptr(B), _ptr(Cout), stream),
          "to_batched_small_gemm")


def chain_f32(E: int, A, B, Cm, R, workspace, T=None, stream: int = 0):
    """R[a,d] = sum_{b,c} (sum_{e,f} A[a,e,c,f] B[f,b,e,d]) C[c,b] on the tensor cores."""
    nbytes = workspace.numel() * workspace.element_size()
    check(lib.to_chain_f32(E, _ptr(A), _ptr(B), _ptr(Cm), _ptr(R), _ptr(T), _ptr(workspace), nbytes,
                           stream), "to_chain_f32")


def gemm_tf32x3(Mp: int, Np: int, Kp: int, Ahi, Alo, Bhi, Blo, Cout, stream: int = 0):
    """Cout[m][n] = sum_k (Ahi+Alo)[m][k] (Bhi+Blo)[n][k] on the tensor cores (K-major operands)."""
    check(lib.to_gemm_tf32x3(Mp, Np, Kp, _ptr(Ahi), _ptr(Alo), _ptr(Bhi), _ptr(Blo), _ptr(Cout),
                             stream), "to_gemm_tf32x3")


def nccl_unique_id() -> bytes:
    """A new NCCL unique id (rank 0 makes it; every rank passes it to nccl_comm_init)."""
    buf = C.create_string_buffer(NCCL_UNIQUE_ID_BYTES)
    check(lib.to_nccl_unique_id(buf), "to_nccl_unique_id")
    return buf.raw


def nccl_comm_init(nranks: int, rank: int, uid: bytes) -> int:
    """This rank's NCCL communicator (the current CUDA device is its GPU), as an int handle."""
    if len(uid) != NCCL_UNIQUE_ID_BYTES:
        raise ValueError(f"NCCL unique id of {len(uid)} bytes")
    h = C.c_void_p()
    check(lib.to_nccl_comm_init(nranks, rank, C.c_char_p(uid), C.byref(h)), "to_nccl_comm_init")
    return h.value


def nccl_comm_destroy(comm: int):
    check(lib.to_nccl_comm_destroy(comm), "to_nccl_comm_destroy")


def nccl_allreduce_sum_f64(x, n: int, comm: int, stream: int = 0):
    """x[:n] (device doubles) <- their sum over the communicator's ranks, in place."""
    check(lib.to_nccl_allreduce_sum_f64(_ptr(x), n, comm, stream), "to_nccl_allreduce_sum_f64")


def nodes_interleave(x, out, n: int, stream: int = 0):
    """out ([n][4] f32, device) = (x[0], x[1], x[2], 0) per node."""
    check(lib.to_nodes_interleave(_fptrs(x), _ptr(out), n, stream), "to_nodes_interleave")


def nodes_deinterleave(inp, x, n: int, stream: int = 0):
    """x[c][i] = inp[i][c] for c < 3 (inp [n][4] f32, device)."""
    check(lib.to_nodes_deinterleave(_ptr(inp), _fptrs(x), n, stream), "to_nodes_deinterleave")


def slab_sync_bytes() -> int:
    return lib.to_slab_sync_bytes()


def sem3d_elastic_mgpu(plan, fields, slab: Slab, comm: int, compute_stream: int, comm_stream: int):
    """f = K u on a z-slab rank, shared planes summed across its neighbours (NCCL)."""
    check(lib.to_sem3d_elastic_mgpu(plan._h, C.byref(fields), C.byref(slab), comm or None,
                                    compute_stream, comm_stream), "to_sem3d_elastic_mgpu")


def sem3d_elastic_mgpu_host(plan, fields, slab: Slab, comm: int, host: HostNodes,
                            compute_stream: int, comm_stream: int):
    """to_sem3d_elastic_mgpu with host u / f: copies in, applies, copies out."""
    check(lib.to_sem3d_elastic_mgpu_host(plan._h, C.byref(fields), C.byref(slab), comm or None,
                                         C.byref(host), compute_stream, comm_stream),
          "to_sem3d_elastic_mgpu_host")


def sm_count() -> int:
    n = lib.to_device_sm_count()
    if n < 0:
        check(-n, "to_device_sm_count")
    return n


# ---- SEM 3D elastic operator ------------------------------------------------

class Sem3dPlan:
    """A validated operator description (host) -> launches on any stream."""

    def __init__(self, dtype, ngll: int, nelem: int, H, Hw, w, nglob: int = 0,
                 assembled: bool = False, interleaved: bool = False):
        self.dtype = np.dtype(dtype)
        self._H = np.ascontiguousarray(H, dtype=np.float64)
        self._Hw = np.ascontiguousarray(Hw, dtype=np.float64)
        self._w = np.ascontiguousarray(w, dtype=np.float64)
        d = Sem3dDesc()
        d.dtype = TO_F32 if self.dtype == np.float32 else TO_F64
        d.ngll = ngll
        d.nelem = nelem
        d.nglob = nglob
        d.assembled = 1 if assembled else 0
        d.node_layout = 1 if interleaved else 0
        d.hprime = self._H.ctypes.data_as(C.POINTER(C.c_double))
        d.hprimewgll = self._Hw.ctypes.data_as(C.POINTER(C.c_double))
        d.wgll = self._w.ctypes.data_as(C.POINTER(C.c_double))
        self.desc = d
        self._h = C.c_void_p()
        check(lib.to_sem3d_plan_create(C.byref(d), C.byref(self._h)), "to_sem3d_plan_create")
        self.ngll, self.nelem, self.nglob, self.assembled = ngll, nelem, nglob, assembled
        self.interleaved = interleaved

    def __del__(self):
        h = getattr(self, "_h", None)
        # at interpreter exit the module's globals may already be cleared
        if h is not None and h.value and lib is not None:
            lib.to_sem3d_plan_destroy(h)
            self._h = None

    @staticmethod
    def fields(u, f, arrays, ibool=None) -> Sem3dFields:
        fl = Sem3dFields()
        for c in range(3):
            fl.u[c] = _ptr(u[c])
            fl.f[c] = _ptr(f[c])
        fl.ibool = _ptr(ibool)
        for n in POINT_ARRAYS:
            setattr(fl, n, _ptr(arrays[n]))
        return fl

    def apply(self, fields: Sem3dFields, accumulate: bool = False, stream: int = 0):
        check(lib.to_sem3d_apply(self._h, C.byref(fields), 1 if accumulate else 0, stream),
              "to_sem3d_apply")

    def apply_elements(self, fields: Sem3dFields, first: int, count: int, stream: int = 0):
        """Add the contribution of elements [first, first + count) to f."""
        check(lib.to_sem3d_apply_elements(self._h, C.byref(fields), first, count, stream),
              "to_sem3d_apply_elements")

    def algorithmic_bytes(self) -> float:
        return lib.to_sem3d_algorithmic_bytes(self._h)

    def flops(self) -> float:
        return lib.to_sem3d_flops(self._h)
