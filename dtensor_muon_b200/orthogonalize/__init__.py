"""Orthogonalisation entry points and loops; the same exports as the
reference's ``src/muonium/orthogonalize/__init__.py:1-15``."""

from .newton_schulz import ns_loop
from .orthogonalize import (
    OrthogonalizationStrategy,
    foreach_zeropower,
    foreach_zeropower_3d_fsdp,
    get_dtensor_metadata,
    is_fsdp_3d_sharded,
    orthogonalize_local,
    zeropower,
)
from .polar_express import POLAR_EXPRESS_COEFFS, pe_loop

__all__ = [
    "OrthogonalizationStrategy",
    "POLAR_EXPRESS_COEFFS",
    "foreach_zeropower",
    "foreach_zeropower_3d_fsdp",
    "get_dtensor_metadata",
    "is_fsdp_3d_sharded",
    "ns_loop",
    "orthogonalize_local",
    "pe_loop",
    "zeropower",
]
