"""Optimizers and the algorithm registry; the same exports as the reference's
``src/muonium/optim/__init__.py:1-26``."""

from .algorithms import (
    BufferSpec,
    MuonAlgorithm,
    get_algorithm,
    register_muon_algorithm,
    registered_algorithms,
)
from .optim import Muon
from .optim_lp import Muon4bit, Muon8bit, MuonFp8, MuonLP, QuantizedState

__all__ = [
    "BufferSpec",
    "Muon",
    "Muon4bit",
    "Muon8bit",
    "MuonAlgorithm",
    "MuonFp8",
    "MuonLP",
    "QuantizedState",
    "get_algorithm",
    "register_muon_algorithm",
    "registered_algorithms",
]
