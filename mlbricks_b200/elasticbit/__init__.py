"""ElasticBit adaptive threshold-driven weight compression on B200."""

from .core import BackendInfo, BitAnalysis, BitCandidate, ElasticBit, RuntimeMatrix

__all__ = ["ElasticBit", "RuntimeMatrix", "BitAnalysis", "BitCandidate", "BackendInfo"]
