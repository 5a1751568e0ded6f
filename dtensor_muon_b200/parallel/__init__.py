"""Distributed execution: symmetric-memory workspaces, the fused owner-compute
Muon path for FSDP-sharded matrices, and expert-parallel token exchange."""
