"""nablatensor_b200 -- B200-native replay engine for NablaTensor valuation tapes.

A recorded tape (``tape.AadRecorder``) is lowered to a loop-aware sm_100a
kernel, compiled with NVRTC, and replayed one scenario per thread as a fused
Monte-Carlo forward + adjoint sweep (``engine.CudaAadEngine``, engine name
"cuda").  The compute path is libnabla_b200.so; this package is the host-side
mirror of the reference's recording and engine SPI.
"""
from .tape import AadOpEnum, AadRecorder, AadTape, ADouble
from .engine import (AadEngine, AadEngines, AadExecutable, AadOptions, AadResult, B200AadExecutable, CudaAadEngine,
                     PrecisionEnum)

__all__ = ["AadOpEnum", "AadRecorder", "AadTape", "ADouble", "AadEngine", "AadEngines", "AadExecutable",
           "AadOptions", "AadResult", "B200AadExecutable", "CudaAadEngine", "PrecisionEnum"]
