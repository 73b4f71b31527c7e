"""mlbricks_b200 -- B200-native ElasticBit compressed-linear runtime.

Drop-in for the ElasticBit path of MLBricks: ``import mlbricks_b200 as mlb``
then ``mlb.ElasticBit.compress(model, calibrationData=..., threshold=...)``.
"""

from .elasticbit import BackendInfo, BitAnalysis, BitCandidate, ElasticBit, RuntimeMatrix

__version__ = "0.1.0"

__all__ = ["ElasticBit", "RuntimeMatrix", "BitAnalysis", "BitCandidate", "BackendInfo"]
