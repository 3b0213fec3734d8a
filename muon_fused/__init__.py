"""B200-native (sm_100a) Newton-Schulz engine for the Muon optimizer.

Drop-in for StarrickLiu/fused-muon's public surface (muon_fused/__init__.py:1-4):
``FusedMuon``, ``fused_newton_schulz`` and ``__version__``.
"""

from muon_fused.optimizer import FusedMuon
from muon_fused.ns_step import fused_newton_schulz, workspace_size

__version__ = "0.1.0"
__all__ = ["FusedMuon", "fused_newton_schulz", "workspace_size"]
