"""Exceptions raised by the Python binding, one per C-ABI status code.

They mirror the exception classes the reference's AexisOps throws for the same
conditions (ArgumentNullException, ArgumentOutOfRangeException,
ArgumentException, NotSupportedException, InvalidOperationException; e.g.
Packages/com.aexis/Runtime/Execution/Graph/AexisOps.cs:3651-3657, 706-709).
"""


class AexisError(RuntimeError):
    status = -1


class ArgumentNullError(AexisError, ValueError):
    status = 1


class ArgumentOutOfRangeError(AexisError, ValueError):
    status = 2


class ArgumentError(AexisError, ValueError):
    status = 3


class NotSupportedError(AexisError, NotImplementedError):
    status = 4


class InvalidOperationError(AexisError):
    status = 5


class CudaError(AexisError):
    status = 6


class DeviceTimeoutError(AexisError, TimeoutError):
    status = 7


BY_STATUS = {c.status: c for c in (ArgumentNullError, ArgumentOutOfRangeError, ArgumentError, NotSupportedError,
                                   InvalidOperationError, CudaError, DeviceTimeoutError)}
