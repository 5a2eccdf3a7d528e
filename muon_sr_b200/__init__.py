"""muon_sr_b200 -- a B200 (sm_100a) optimizer-step engine with the Python API of
bab2min/muon_sr 0.1.2 (muon_sr/__init__.py:3-14).

The optimizers below keep the reference's names, arguments, param-group keys, state keys
and seed rules; their numeric work runs in hand-written CUDA kernels (tcgen05 Newton-Schulz
GEMM chains, fused SR elementwise kernels, single-pass 8-bit AdamW) in the in-tree C-ABI
library ``libmuon_sr_b200.so``. There is no CPU fallback.
"""
from ._version import __version__
from .adamw import SRAccumulator, TritonAdamW, TritonSRAccumulator
from .adamw8bit import TritonAdamW8bit, create_dynamic_map
from .muon import MuonSR, MuonSRWithAuxAdam, TritonMuonSR, TritonMuonSRWithAuxAdam
from .kernels import set_sr_noise
from .sharding import Sharder
from .staging import HostStaging
from .graph import StepGraph

__all__ = [
    "SRAccumulator",
    "TritonAdamW8bit",
    "TritonAdamW", "TritonSRAccumulator",
    "MuonSR", "MuonSRWithAuxAdam",
    "TritonMuonSR", "TritonMuonSRWithAuxAdam",
    "Sharder", "HostStaging", "StepGraph", "create_dynamic_map", "set_sr_noise",
]
