"""Exception types of the reference (src/errors.jl:1-9) plus the backend's own.

Status codes returned by libjlust_b200.so map one to one onto these classes
(include/jlust_b200.h, enum jlb_status_code).
"""


class JLUSTError(Exception):
    """Base class of every error raised by jlust_b200."""


class InvalidTensorFormat(JLUSTError):       # errors.jl:1
    pass


class InvalidLevelAccess(JLUSTError):        # errors.jl:2
    pass


class UnsupportedFormat(JLUSTError):         # errors.jl:3
    pass


class UnsupportedIndexType(JLUSTError):      # errors.jl:4
    pass


class UnsupportedValueType(JLUSTError):      # errors.jl:5
    pass


class IndexOriginMismatch(JLUSTError):       # errors.jl:6
    pass


class DeviceMismatch(JLUSTError):            # errors.jl:7
    pass


class IncompatibleExtents(JLUSTError):       # errors.jl:8
    pass


class NonCanonicalStorage(JLUSTError):       # errors.jl:9
    pass


class InvalidArgument(JLUSTError):
    pass


class CudaError(JLUSTError):
    pass


class DeviceTimeout(JLUSTError):
    pass


class WorkspaceTooSmall(JLUSTError):
    pass


_BY_STATUS = {
    1: UnsupportedFormat,
    2: UnsupportedIndexType,
    3: UnsupportedValueType,
    4: IndexOriginMismatch,
    5: DeviceMismatch,
    6: IncompatibleExtents,
    7: NonCanonicalStorage,
    8: InvalidArgument,
    9: CudaError,
    10: DeviceTimeout,
    11: WorkspaceTooSmall,
}


def from_status(status: int, msg: str) -> JLUSTError:
    return _BY_STATUS.get(status, JLUSTError)(msg)
