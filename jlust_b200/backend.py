"""B200Backend: the plug-in that executes JLUST ops on libjlust_b200.so.

Mirrors the reference's backend boundary (src/backends.jl:3-195):
`supports_backend(backend, op)`, `execute(backend, op, tensors...; alpha,
beta)`, `prepare(backend, OpType, u_A)` returning an AbstractKernelHandle,
`update_values(handle, u_A)`, `validate_storage(u, backend)` and the
`default_backend` policy that routes CUDA-resident tensors here (the
reference's CUDAExt policy, ext/CUDAExt/CUDAExt.jl:232-241, picks
EmitterBackend for SpMV and cuSPARSE for SpMM/SDDMM; this backend takes all
three).  There is no CPU or library fallback: an op the backend cannot run
raises UnsupportedFormat / UnsupportedValueType / DeviceMismatch.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .errors import (DeviceMismatch, IncompatibleExtents, UnsupportedFormat,
                     UnsupportedValueType)
from .formats import TensorFormat
from .ops import Op, OpType
from .tensor import (USTensor, coordinates, csr_tensor, dense_layout, nonzeros, positions,
                     ust)


class AbstractUSTBackend:
    pass


class AbstractKernelHandle:
    pass


class B200Backend(AbstractUSTBackend):
    """Hand-written sm_100a kernels behind a C ABI."""

    def __eq__(self, other):
        return isinstance(other, B200Backend)

    def __hash__(self):
        return hash("B200Backend")

    def __repr__(self):
        return "B200Backend()"


_DTYPE = {torch.float32: _lib.F32, torch.float64: _lib.F64, torch.bfloat16: _lib.BF16}


def _dense_n(f: TensorFormat, n: int) -> bool:
    return f.family == "Dense" and f.ndims() == n


def supports_backend(backend, op: Op) -> bool:
    """Capability by (tag, operand formats), as CUDAExt.jl:253-343 does."""
    if not isinstance(backend, B200Backend):
        return False
    f = op.formats
    if op.tag == "SpMV" and len(f) == 3:
        return (f[0].family in ("CSR", "DCSR", "COO", "CSC", "ShiftedDiag") and _dense_n(f[1], 1)
                and _dense_n(f[2], 1))
    if op.tag == "SpMM" and len(f) == 3:
        return f[0].family in ("CSR", "BSR") and _dense_n(f[1], 2) and _dense_n(f[2], 2)
    if op.tag == "SDDMM" and len(f) == 3:
        return _dense_n(f[0], 2) and _dense_n(f[1], 2) and f[2].family == "CSR"
    if op.tag == "BlockSpMM" and len(f) == 3:
        return f[0].family == "BSR" and _dense_n(f[1], 2) and _dense_n(f[2], 2)
    if op.tag == "SpGEMM" and len(f) in (2, 3):
        return all(x.family == "CSR" for x in f)
    return False


def default_backend(u, op_type) -> AbstractUSTBackend:
    """Every CUDA-resident tensor goes to B200Backend (the drop-in policy)."""
    return B200Backend()


def _stream(device: torch.device):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None and t.numel() > 0 else C.c_void_p(0)


def _same_device(*ts):
    devs = {t.device for t in ts if t is not None}
    if len(devs) != 1:
        raise DeviceMismatch(f"operands live on different devices: {sorted(map(str, devs))}")
    d = next(iter(devs))
    if d.type != "cuda":
        raise DeviceMismatch(f"B200Backend runs on CUDA devices only (operands on {d}); "
                             "there is no CPU fallback")
    return d


def _vec(t: torch.Tensor, what: str) -> torch.Tensor:
    if t.dim() != 1 or (t.numel() > 1 and t.stride(0) != 1):
        raise IncompatibleExtents(f"{what} must be a contiguous vector")
    return t


def _csr_parts(A: USTensor):
    rowptr, colind, val = positions(A, 2), coordinates(A, 2), nonzeros(A)
    m, n = A.extents
    if val.dim() != 1 or not val.is_contiguous():
        raise IncompatibleExtents("CSR values must be a contiguous vector")
    return m, n, rowptr, colind, val


def _value_type(t: torch.Tensor, allowed, what):
    if t.dtype not in allowed:
        raise UnsupportedValueType(f"{what}: value type {t.dtype} not supported by B200Backend")
    return _DTYPE[t.dtype]


def spmv(A: USTensor, x, y, alpha=1.0, beta=0.0, input_fn=None, output_fn=None):
    """y = alpha*A*x + beta*y (KA spmv.jl:371-504 semantics)."""
    if input_fn is not None or output_fn is not None:
        raise UnsupportedFormat("B200Backend: input_fn/output_fn closures cannot cross the C ABI")
    x, y = ust(x).val, ust(y).val
    fam = A.format.family
    if fam == "ShiftedDiag":
        return _shifted_diag_spmv(A, x, y, alpha, beta)
    if fam not in ("CSR", "DCSR", "COO", "CSC"):
        raise UnsupportedFormat(f"B200Backend SpMV: format {A.format.name} is not supported")
    m, n = A.extents
    val = nonzeros(A)
    if val.dim() != 1 or not val.is_contiguous():
        raise IncompatibleExtents("SpMV: values must be a contiguous vector")
    dt = _value_type(val, (torch.float32, torch.float64), "SpMV")
    if x.dtype != val.dtype or y.dtype != val.dtype:
        raise UnsupportedValueType("SpMV: A, x and y must share one value type")
    _vec(x, "x"), _vec(y, "y")
    if x.numel() != n or y.numel() != m:
        raise IncompatibleExtents(f"SpMV: A is {m}x{n}, x has {x.numel()}, y has {y.numel()}")
    base, nnz, a, b = A.origin.offset, val.numel(), float(alpha), float(beta)
    if fam == "CSR":
        rowptr, colind = positions(A, 2), coordinates(A, 2)
        dev = _same_device(rowptr, colind, val, x, y)
        _lib.call("jlb_csr_spmv", _stream(dev), dt, base, m, n, nnz, _ptr(rowptr), _ptr(colind),
                  _ptr(val), _ptr(x), _ptr(y), a, b)
    elif fam == "DCSR":
        # outer level: stored rows (coordinates); inner level: positions + columns
        row_ids, fibptr, colind = coordinates(A, 1), positions(A, 2), coordinates(A, 2)
        dev = _same_device(row_ids, fibptr, colind, val, x, y)
        _lib.call("jlb_dcsr_spmv", _stream(dev), dt, base, m, n, row_ids.numel(), nnz,
                  _ptr(fibptr), _ptr(row_ids), _ptr(colind), _ptr(val), _ptr(x), _ptr(y), a, b)
    elif fam == "COO":
        rows, cols = coordinates(A, 1), coordinates(A, 2)
        dev = _same_device(rows, cols, val, x, y)
        _lib.call("jlb_coo_spmv", _stream(dev), dt, base, m, n, nnz, _ptr(rows), _ptr(cols),
                  _ptr(val), _ptr(x), _ptr(y), a, b)
    else:  # CSC: dense outer level over columns, compressed rows inside
        colptr, rowind = positions(A, 2), coordinates(A, 2)
        dev = _same_device(colptr, rowind, val, x, y)
        _lib.call("jlb_csc_spmv", _stream(dev), dt, base, m, n, nnz, _ptr(colptr), _ptr(rowind),
                  _ptr(val), _ptr(x), _ptr(y), a, b)
    return y


_PATCHES = {}


def _patch_buffers(dev, patches):
    """Device copies of selector patches (first row, last row, column of the
    first row, value), kept per device and patch list."""
    key = (str(dev), tuple(patches))
    buf = _PATCHES.get(key)
    if buf is None:
        if len(_PATCHES) >= 256:      # bounded: distinct selector shapes are few
            _PATCHES.clear()
        rows = torch.tensor([v for p in patches for v in (p[0], p[1])], dtype=torch.int64)
        cols = torch.tensor([p[2] for p in patches], dtype=torch.int64)
        vals = torch.tensor([p[3] for p in patches], dtype=torch.float64)
        buf = _PATCHES[key] = (rows.to(dev), cols.to(dev), vals.to(dev))
    return buf


def _shifted_diag_spmv(A: USTensor, x, y, alpha, beta):
    """y = alpha * S x + beta * y for a ShiftedDiag tensor S: row r gets
    val * x[r + shift] (JLUST's walker with a ShiftedDiag leaf,
    src/backends.jl:223-227), through the patched SpMV kernel with no CSR
    entries and one patch over all rows."""
    m, n = A.extents
    shift, v = A.format.diag
    dt = _value_type(x, (torch.float32, torch.float64), "SpMV")
    if y.dtype != x.dtype or A.val.dtype != x.dtype:
        raise UnsupportedValueType("SpMV: A, x and y must share one value type")
    _vec(x, "x"), _vec(y, "y")
    if x.numel() != n or y.numel() != m:
        raise IncompatibleExtents(f"SpMV: A is {m}x{n}, x has {x.numel()}, y has {y.numel()}")
    if m > 0 and (shift < 0 or m - 1 + shift >= n):
        raise IncompatibleExtents(f"SpMV: ShiftedDiag shift {shift} reaches outside {m}x{n}")
    dev = _same_device(x, y)
    pr, pc, pv = _patch_buffers(dev, [(0, m - 1, shift, v)])
    _lib.call("jlb_csr_patched_spmv", _stream(dev), dt, 0, m, n, 0, None, None, None, 1,
              _ptr(pr), _ptr(pc), _ptr(pv), _ptr(x), _ptr(y), float(alpha), float(beta))
    return y


def spmm(A: USTensor, B, Cm, alpha=1.0, beta=0.0):
    """C = alpha*A*B + beta*C for CSR A (KA spmm.jl:397-423) or BSR A."""
    if A.format.family == "BSR":
        return bsr_spmm(A, B, Cm, alpha, beta)
    B, Cm = ust(B).val, ust(Cm).val
    m, n, rowptr, colind, val = _csr_parts(A)
    dt = _value_type(val, (torch.float32, torch.float64), "SpMM")
    if B.dtype != val.dtype or Cm.dtype != val.dtype:
        raise UnsupportedValueType("SpMM: A, B and C must share one value type")
    if B.dim() != 2 or Cm.dim() != 2 or B.shape[0] != n or Cm.shape[0] != m or B.shape[1] != Cm.shape[1]:
        raise IncompatibleExtents(f"SpMM: A {m}x{n}, B {tuple(B.shape)}, C {tuple(Cm.shape)}")
    lb, lc = dense_layout(B), dense_layout(Cm)
    if lb is None or lc is None:
        raise IncompatibleExtents("SpMM: B and C must be row- or column-major strided")
    dev = _same_device(rowptr, colind, val, B, Cm)
    k = B.shape[1]
    # column-major B and C (JLUST's native layout) go through row-major
    # copies in a workspace
    wsb = _lib.load().jlb_csr_spmm_workspace_size(dt, m, n, k, lb[0], lc[0])
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev) if wsb else None
    _lib.call("jlb_csr_spmm_ws", _stream(dev), dt, A.origin.offset, m, n, val.numel(),
              _ptr(rowptr), _ptr(colind), _ptr(val), k, _ptr(B), lb[1], lb[0], _ptr(Cm), lc[1],
              lc[0], float(alpha), float(beta), _ptr(ws), wsb)
    return Cm


def sddmm(A, B, Cs: USTensor, alpha=1.0, beta=0.0, mode="add", S=None):
    """Sampled product over the pattern of CSR Cs, in place on its values.
    mode="add": nz = alpha*(A*B)_ij + beta*nz  (KA sddmm.jl:23-36);
    mode="mul": nz = alpha*(A*B)_ij * S_ij + beta*nz, S defaulting to the
    current values of Cs (the sampled-product form)."""
    A, B = ust(A).val, ust(B).val
    m, n, rowptr, colind, val = _csr_parts(Cs)
    dt = _value_type(val, (torch.float32, torch.float64), "SDDMM")
    if A.dtype != val.dtype or B.dtype != val.dtype:
        raise UnsupportedValueType("SDDMM: A, B and C must share one value type")
    if A.dim() != 2 or B.dim() != 2 or A.shape[0] != m or B.shape[1] != n or A.shape[1] != B.shape[0]:
        raise IncompatibleExtents(f"SDDMM: A {tuple(A.shape)}, B {tuple(B.shape)}, C {m}x{n}")
    la, lb = dense_layout(A), dense_layout(B)
    if la is None or lb is None:
        raise IncompatibleExtents("SDDMM: A and B must be row- or column-major strided")
    mode_code = {"add": _lib.SDDMM_ADD, "mul": _lib.SDDMM_MUL}[mode]
    if mode == "mul" and S is None:
        S = val
    if S is not None:
        _vec(S, "S")
    dev = _same_device(rowptr, colind, val, A, B)
    K = A.shape[1]
    _lib.call("jlb_sddmm", _stream(dev), dt, Cs.origin.offset, m, n, val.numel(), _ptr(rowptr),
              _ptr(colind), K, _ptr(A), la[1], la[0], _ptr(B), lb[1], lb[0], _ptr(S), _ptr(val),
              mode_code, float(alpha), float(beta))
    return Cs


def bsr_spmm(A: USTensor, B, Cm, alpha=1.0, beta=0.0):
    """C (fp32) = alpha*A*B + beta*C for BSRRight A with bf16 values and bf16 B."""
    B, Cm = ust(B).val, ust(Cm).val
    b1, b2 = A.format.block
    if b1 != b2:
        raise UnsupportedFormat("B200Backend BSR SpMM needs square blocks")
    if A.format.keys[2].dim != "i":
        raise UnsupportedFormat("B200Backend BSR SpMM needs row-major (BSRRight) blocks")
    bs = b1
    m, n = A.extents
    browptr, bcolind, bval = positions(A, 2), coordinates(A, 2), nonzeros(A)
    if bval.dtype != torch.bfloat16 or B.dtype != torch.bfloat16 or Cm.dtype != torch.float32:
        raise UnsupportedValueType("BSR SpMM: values and B must be BFloat16, C Float32")
    mb, nb = -(-m // bs), -(-n // bs)
    N = B.shape[1]
    if B.dim() != 2 or Cm.dim() != 2 or B.shape[0] != nb * bs or Cm.shape[0] != mb * bs or Cm.shape[1] != N:
        raise IncompatibleExtents(f"BSR SpMM: A {m}x{n} (bs {bs}), B {tuple(B.shape)}, C {tuple(Cm.shape)}")
    lb, lc = dense_layout(B), dense_layout(Cm)
    if lb is None or lc is None or lb[0] != 0 or lc[0] != 0:
        raise IncompatibleExtents("BSR SpMM: B and C must be row-major")
    dev = _same_device(browptr, bcolind, bval, B, Cm)
    _lib.call("jlb_bsr_spmm", _stream(dev), A.origin.offset, mb, nb, bcolind.numel(), bs,
              _ptr(browptr), _ptr(bcolind), _ptr(bval), N, _ptr(B), lb[1], _ptr(Cm), lc[1],
              float(alpha), float(beta))
    return Cm


def spgemm(A: USTensor, B: USTensor, C0=None, alpha=1.0, beta=0.0, transa="N", transb="N"):
    """C = alpha*A*B for CSR A and B, a new CSR tensor (execute(SpGEMMOp,
    u_A, u_B, u_C0), KA spgemm.jl:493-506): a plan's symbolic pass, then its
    numeric pass."""
    h = B200SpGEMMHandle(A, B, transa=transa, transb=transb, beta=beta)
    return h.execute(A, B, alpha=alpha, beta=beta)


_EXEC = {"SpMV": spmv, "SpMM": spmm, "SDDMM": sddmm, "BlockSpMM": bsr_spmm, "SpGEMM": spgemm}


def backend_execute(backend, op: Op, *tensors, **kw):
    if not supports_backend(backend, op):
        raise UnsupportedFormat(f"{op} not supported by {backend!r}")
    return _EXEC[op.tag](*tensors, **kw)


def execute(op_or_type, *args, backend=None, **kw):
    """execute(OpType, tensors...; backend, alpha, beta, ...) (src/convenience.jl:15-39),
    execute(backend, op, tensors...) or execute(handle, tensors...)."""
    if isinstance(op_or_type, AbstractKernelHandle):
        return op_or_type.execute(*args, **kw)
    if isinstance(op_or_type, AbstractUSTBackend):
        return backend_execute(op_or_type, args[0], *args[1:], **kw)
    if isinstance(op_or_type, OpType):
        if args and isinstance(args[0], AbstractKernelHandle):
            return args[0].execute(*args[1:], **kw)
        from .block import BlockBandedMatrix, BlockSparseMatrix, bbm_spmv, block_spmm, block_spmv
        if args and isinstance(args[0], BlockBandedMatrix):
            if op_or_type.tag != "BBMSpMV":
                raise UnsupportedFormat(f"{op_or_type} does not take a BlockBandedMatrix")
            return bbm_spmv(args[0], args[1], args[2])
        if args and isinstance(args[0], BlockSparseMatrix):
            if op_or_type.tag == "BlockSpMV":
                return block_spmv(args[0], args[1], args[2], backend=backend)
            if op_or_type.tag == "BlockSpMM":
                return block_spmm(args[0], args[1], args[2], backend=backend)
            raise UnsupportedFormat(f"{op_or_type} does not take a BlockSparseMatrix")
        tensors = [ust(a) for a in args]
        primary = tensors[2] if op_or_type.tag == "SDDMM" else tensors[0]
        be = backend if backend is not None else default_backend(primary, op_or_type)
        op = op_or_type(*(t.format for t in tensors))
        return backend_execute(be, op, *args, **kw)
    raise TypeError(f"execute: unsupported first argument {op_or_type!r}")


def mul(y, A: USTensor, x, alpha=1.0, beta=0.0):
    """LinearAlgebra.mul!(y, A, x[, alpha, beta]) (src/convenience.jl:46-59)."""
    from .ops import SpMMOp, SpMVOp
    op = SpMVOp if ust(x).val.dim() == 1 else SpMMOp
    execute(op, A, x, y, alpha=alpha, beta=beta)
    return y


def validate_storage(u: USTensor, backend=None, op="unknown", require_sorted=False) -> None:
    """Structural checks (src/backends.jl:309-316) run on the device."""
    if u.format.family != "CSR":
        if nonzeros(u).dim() != 1:
            raise IncompatibleExtents("values must be a vector")
        return
    m, n, rowptr, colind, val = _csr_parts(u)
    dev = _same_device(rowptr, colind, val)
    _lib.call("jlb_csr_validate", _stream(dev), u.origin.offset, m, n, val.numel(), _ptr(rowptr),
              _ptr(colind), 1 if require_sorted else 0)


class B200SpMVHandle(AbstractKernelHandle):
    """Prepared SpMV (the reference's EmitterSpMVHandle / CUSPARSESpMVHandle)."""

    def __init__(self, A: USTensor):
        m, n, rowptr, colind, val = _csr_parts(A)
        self.dtype = _value_type(val, (torch.float32, torch.float64), "SpMV")
        self.A = A
        self.m, self.n = m, n
        self.device = _same_device(rowptr, colind, val)
        plan = C.c_void_p()
        _lib.call("jlb_spmv_plan_create", C.byref(plan), _stream(self.device), self.dtype,
                  A.origin.offset, m, n, val.numel(), _ptr(rowptr), _ptr(colind))
        self._plan = plan
        self._val = val

    def info(self):
        mx, mean, var = C.c_int64(), C.c_double(), C.c_int()
        _lib.call("jlb_spmv_plan_info", self._plan, C.byref(mx), C.byref(mean), C.byref(var))
        return {"max_row": mx.value, "mean_row": mean.value, "variant": var.value}

    def set_variant(self, variant: int):
        """Force the kernel variant: 0 (a thread per row, bit-exact for rows of
        up to 32 entries), 1 (the same sums with x staged in shared memory per
        block of rows, for banded structure) or W in 2, 4, 8, 16, 32 (groups of
        W lanes per row)."""
        _lib.call("jlb_spmv_plan_set_variant", self._plan, int(variant))
        return self

    def execute(self, *args, alpha=1.0, beta=0.0):
        # execute(h, x, y) or execute(h, A, x, y) (KA spmv.jl:533-544)
        if len(args) == 3:
            _, x, y = args
        else:
            x, y = args
        x, y = ust(x).val, ust(y).val
        if x.dtype != self._val.dtype or y.dtype != self._val.dtype:
            raise UnsupportedValueType("SpMV handle: x and y must match the matrix value type")
        _vec(x, "x"), _vec(y, "y")
        if x.numel() != self.n or y.numel() != self.m:
            raise IncompatibleExtents("SpMV handle: x or y length does not match the matrix")
        _same_device(self._val, x, y)
        _lib.call("jlb_spmv_plan_execute", self._plan, _stream(self.device), _ptr(self._val),
                  _ptr(x), _ptr(y), float(alpha), float(beta))
        return y

    def update_values(self, A: USTensor):
        val = nonzeros(A)
        if val.numel() != self._val.numel() or val.dtype != self._val.dtype:
            raise IncompatibleExtents("update_values!: structure or value type changed")
        self._val = val
        self.A = A
        return self

    def __del__(self):
        try:
            if getattr(self, "_plan", None) and self._plan.value:
                _lib.load().jlb_spmv_plan_destroy(self._plan)
                self._plan = C.c_void_p()
        except Exception:
            pass


class B200SpGEMMHandle(AbstractKernelHandle):
    """Prepared SpGEMM (the reference's EmitterSpGEMMHandle, KA
    spgemm.jl:298-438): the plan keeps C's structure and the sorted product
    list; execute(h, u_A, u_B; alpha) recomputes C's values for new values of
    the same structures without sorting or allocating on the device."""

    def __init__(self, A: USTensor, B: USTensor, transa="N", transb="N", beta=0.0, **_):
        if transa != "N" or transb != "N":
            raise UnsupportedFormat("SpGEMM: transposed operands are not supported")
        if beta != 0:
            raise UnsupportedFormat("SpGEMM: beta != 0 is not supported")
        if A.format.family != "CSR" or B.format.family != "CSR":
            raise UnsupportedFormat("SpGEMM: only CSR x CSR is supported")
        m, k, a_rp, a_ci, a_v = _csr_parts(A)
        k2, n, b_rp, b_ci, b_v = _csr_parts(B)
        if k != k2:
            raise IncompatibleExtents(f"SpGEMM: A is {m}x{k}, B is {k2}x{n}")
        if A.origin.offset != B.origin.offset:
            from .errors import IndexOriginMismatch
            raise IndexOriginMismatch("SpGEMM: A and B have different index origins")
        self.dtype = _value_type(a_v, (torch.float32, torch.float64), "SpGEMM")
        if b_v.dtype != a_v.dtype:
            raise UnsupportedValueType("SpGEMM: A and B must share one value type")
        self.device = _same_device(a_rp, a_ci, a_v, b_rp, b_ci, b_v)
        self.m, self.k, self.n = m, k, n
        self.origin = A.origin
        self.vdtype = a_v.dtype
        self.nnz_a, self.nnz_b = a_v.numel(), b_v.numel()
        plan, nnz_c, prods = C.c_void_p(), C.c_int64(), C.c_int64()
        _lib.call("jlb_spgemm_plan_create", C.byref(plan), _stream(self.device), self.dtype,
                  A.origin.offset, m, k, n, self.nnz_a, _ptr(a_rp), _ptr(a_ci), self.nnz_b,
                  _ptr(b_rp), _ptr(b_ci), C.byref(nnz_c), C.byref(prods))
        self._plan = plan
        self.nnz_c, self.products = nnz_c.value, prods.value
        self.c_rowptr = torch.empty(m + 1, dtype=torch.int32, device=self.device)
        self.c_colind = torch.empty(self.nnz_c, dtype=torch.int32, device=self.device)
        _lib.call("jlb_spgemm_plan_structure", self._plan, _stream(self.device),
                  _ptr(self.c_rowptr), _ptr(self.c_colind))

    def execute(self, A: USTensor, B: USTensor, alpha=1.0, beta=0.0, out=None):
        if beta != 0:
            raise UnsupportedFormat("SpGEMM: beta != 0 is not supported")
        a_v, b_v = nonzeros(A), nonzeros(B)
        if a_v.numel() != self.nnz_a or b_v.numel() != self.nnz_b:
            raise IncompatibleExtents("SpGEMM handle: A or B does not have the planned structure")
        if a_v.dtype != self.vdtype or b_v.dtype != self.vdtype:
            raise UnsupportedValueType("SpGEMM handle: value type differs from the plan's")
        c_v = out if out is not None else torch.empty(self.nnz_c, dtype=self.vdtype,
                                                      device=self.device)
        _same_device(a_v, b_v, c_v)
        _lib.call("jlb_spgemm_plan_execute", self._plan, _stream(self.device), _ptr(a_v),
                  _ptr(b_v), _ptr(c_v), float(alpha))
        return csr_tensor(self.c_rowptr, self.c_colind, c_v, (self.m, self.n), origin=self.origin)

    def __del__(self):
        try:
            if getattr(self, "_plan", None) and self._plan.value:
                _lib.load().jlb_spgemm_plan_destroy(self._plan)
                self._plan = C.c_void_p()
        except Exception:
            pass


def prepare(backend, op_type: OpType, A: USTensor, *more, **kw) -> AbstractKernelHandle:
    """prepare(backend, OpType, u_A[, u_B]) (src/ops.jl:187-202)."""
    if not isinstance(backend, B200Backend):
        raise UnsupportedFormat(f"prepare: {backend!r} is not B200Backend")
    if op_type.tag == "SpMV":
        return B200SpMVHandle(A)
    if op_type.tag == "SpGEMM":
        return B200SpGEMMHandle(A, *more, **kw)
    raise UnsupportedFormat(f"prepare: {op_type!r} has no prepared form on B200Backend")


def update_values(handle: AbstractKernelHandle, A: USTensor):
    """update_values!(handle, u_A) (src/ops.jl:204-211)."""
    return handle.update_values(A)
