"""dtensor_muon_b200: a B200-native distributed Muon optimizer and training stack.

Same public surface as ``muonium`` (tonyf/dtensor-muon): ``Muon``, ``MuonLP``
(+ ``Muon8bit`` / ``Muon4bit`` / ``MuonFp8``), ``MuonAlgorithm``,
``BufferSpec``, ``OrthogonalizationStrategy`` and the algorithm registry
(reference: ``src/muonium/__init__.py:1-28``; ``MuonLP`` needs no torchao here).
Hot paths run hand-written sm_100a kernels from the in-tree extension
``dtensor_muon_b200._C``.
"""

from .optim import (
    BufferSpec,
    Muon,
    Muon4bit,
    Muon8bit,
    MuonAlgorithm,
    MuonFp8,
    MuonLP,
    QuantizedState,
    get_algorithm,
    register_muon_algorithm,
    registered_algorithms,
)
from .orthogonalize import OrthogonalizationStrategy

__all__ = [
    "BufferSpec",
    "Muon",
    "Muon4bit",
    "Muon8bit",
    "MuonAlgorithm",
    "MuonFp8",
    "MuonLP",
    "OrthogonalizationStrategy",
    "QuantizedState",
    "get_algorithm",
    "register_muon_algorithm",
    "registered_algorithms",
]
__version__ = "0.1.0"
