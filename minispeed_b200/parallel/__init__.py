"""Multi-GPU communication: collective strategies and the NVLink peer runtime."""

from .collectives import LibraryCollectives, LocalCollectives

__all__ = ["LibraryCollectives", "LocalCollectives"]
