"""Native sm_100a kernels and their Python entry points. Importing the package
registers the ``torch.ops.dmb`` custom ops."""

from . import library  # noqa: F401
