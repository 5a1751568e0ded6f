from .distributed import run_distributed

__all__ = ["run_distributed"]
