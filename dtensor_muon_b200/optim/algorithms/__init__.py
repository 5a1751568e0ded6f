"""Pluggable Muon algorithm variants, selected per param group by
``{"params": ..., "algorithm": "<name>"}``. Subclass :class:`MuonAlgorithm` and
decorate with :func:`register_muon_algorithm` to add one."""

from .base import (
    BufferSpec,
    MuonAlgorithm,
    get_algorithm,
    orthogonalize_batch,
    orthogonalize_single,
    register_muon_algorithm,
    registered_algorithms,
    split_lr_scales,
)
from .muon import MuonBaseline  # noqa: E402  (registers "muon")
from .normuon import NorMuon  # noqa: E402  (registers "normuon")

__all__ = [
    "BufferSpec",
    "MuonAlgorithm",
    "MuonBaseline",
    "NorMuon",
    "get_algorithm",
    "orthogonalize_batch",
    "orthogonalize_single",
    "register_muon_algorithm",
    "registered_algorithms",
    "split_lr_scales",
]
