"""jlust_b200 -- B200 (sm_100a) sparse-kernel backend for JLUST.

The public surface mirrors JLUST's Julia API for the sparse hot path
(src/JLUST.jl exports): tensors (USTensor, csr_tensor, coo_tensor,
bsr_tensor, ust), formats (Formats.CSR/COO/BSRRight/DensedRight), op tags
(SpMVOp, SpMMOp, SDDMMOp, BlockSpMMOp), the backend boundary
(B200Backend, supports_backend, execute, prepare, update_values,
validate_storage, default_backend), convert_format and the reference's error
types.  Every op runs on libjlust_b200.so (hand-written CUDA for sm_100a);
there is no CPU fallback.
"""
from . import errors, synth  # noqa: F401
from .backend import (AbstractKernelHandle, AbstractUSTBackend, B200Backend,  # noqa: F401
                      B200SpMVHandle, default_backend, execute, mul, prepare,
                      supports_backend, update_values, validate_storage)
from .convert import convert_format, exclusive_scan  # noqa: F401
from .block import BlockBandedMatrix, BlockSparseMatrix, mul, update_block_values  # noqa: F401
from .errors import (DeviceMismatch, DeviceTimeout, IncompatibleExtents,  # noqa: F401
                     IndexOriginMismatch, InvalidLevelAccess, NonCanonicalStorage,
                     UnsupportedFormat, UnsupportedIndexType, UnsupportedValueType)
from .formats import Formats, TensorFormat, dim2lvl, format_family, lvl2dim  # noqa: F401
from .ops import (BBMSpMVOp, BlockSpMMOp, BlockSpMVOp, Op, SDDMMOp, SpGEMMOp, SpMMOp,  # noqa: F401
                  SpMVOp, SpSMOp, SpSVOp, SparseToDenseOp)
from .tensor import (OneBased, USTensor, ZeroBased, bsr_tensor, coo_tensor, shifted_diag_tensor,  # noqa: F401
                     coordinates, csr_tensor, extents, has_coordinates, has_positions,
                     index_origin, nnz, nonzeros, positions, ust)

__version__ = "0.1.0"


def device_status(device=None) -> None:
    """Synchronise the current stream and raise if a kernel reported a bounded
    wait that gave up or a failed bounds check (jlb_device_status)."""
    import ctypes as C

    import torch

    from . import _lib
    s = torch.cuda.current_stream(device).cuda_stream
    _lib.call("jlb_device_status", C.c_void_p(s))


def l2_persist(base, nbytes: int, device=None) -> int:
    """Keep [base, base + nbytes) in L2 across the kernels launched afterwards
    on the current stream (jlb_l2_persist): base is a device pointer or a
    tensor.  Returns the bytes the persisting set-aside covers.  nbytes == 0
    clears the window and returns the set-aside."""
    import ctypes as C

    import torch

    from . import _lib
    ptr = base.data_ptr() if hasattr(base, "data_ptr") else int(base)
    s = torch.cuda.current_stream(device).cuda_stream
    out = C.c_size_t(0)
    _lib.call("jlb_l2_persist", C.c_void_p(s), C.c_void_p(ptr), C.c_size_t(int(nbytes)),
              C.byref(out))
    return out.value
