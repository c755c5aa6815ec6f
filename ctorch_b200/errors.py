"""ctorch's exception tree (include/ctorch/errors.h:26-58), raised by the ctorch_b200 ops."""


class Error(RuntimeError):
    """Base of every ctorch error (ctorch::Error)."""


class ShapeError(Error):
    """Incompatible shapes, bad axis, out-of-range index (ctorch::ShapeError)."""


class DTypeError(Error):
    """Unsupported or unpromotable dtype (ctorch::DTypeError)."""


class DeviceError(Error):
    """Operands on the wrong / different devices, or a CUDA failure (ctorch::DeviceError)."""


class AliasError(Error):
    """In-place destination aliases a non-trivial view of an input (ctorch::AliasError)."""


class CommTimeoutError(DeviceError):
    """A rank of a cross-GPU exchange did not arrive within the wait's time limit (the C ABI's
    bounded waits; no ctorch counterpart, ctorch has no multi-GPU layer)."""
