"""Exception types with the reference's names and hierarchy (include/matrix_pro/core/errors.hpp:8-42)."""


class MatrixProError(RuntimeError):
    """Base of every library error (errors.hpp:8)."""


class InvalidArgumentError(MatrixProError):
    """Bad argument: alias, option, int32 overflow, wrong thread/device/stream (errors.hpp:13)."""


class ShapeMismatchError(MatrixProError):
    """Operand shapes disagree (errors.hpp:18)."""


class CudaError(MatrixProError):
    """A CUDA call failed (errors.hpp:28)."""


class DeviceTimeoutError(CudaError):
    """A bounded device-side wait gave up (MFB_ETIMEOUT); the context stays usable."""
