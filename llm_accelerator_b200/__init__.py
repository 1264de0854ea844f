"""B200 execution engine for taccel programs (SayatAbdikul/LLM_accelerator).

The golden simulator's per-instruction NumPy loop is replaced by a C++
compiler that plans each straight-line instruction stream once and a CUDA
engine (sm_100a) that runs the plan for a batch of sequences.  The public
classes keep the reference interfaces:

* ``B200Simulator``  - drop-in for ``taccel.golden_model.simulator.Simulator``
* ``HostRunner``     - drop-in for ``taccel.runtime.host_runner.HostRunner``
* ``BatchedRunner``  - many sequences per GPU, greedy decode on device
* ``ProgramBundle``  - the reference bundle format, with file I/O
* ``gemm``           - stand-alone INT8 GEMM kernels with requant epilogues
"""
from .bundle import ProgramBundle, RelocationSite, RuntimeConfigAttnSite, RuntimePatchSite  # noqa: F401
from .errors import (ConfigError, DRAMAccessError, EngineError, IllegalBufferError,  # noqa: F401
                     IllegalOpcodeError, SimulatorError, SRAMAccessError)


_LAZY = {"B200Simulator": "simulator", "B200State": "simulator", "HostRunner": "runner",
         "BatchedRunner": "runner", "Engine": "engine", "compile_program": "engine"}


def __getattr__(name):
    # CUDA-backed classes load libtaccel_b200.so on first use.
    import importlib
    if name in _LAZY:
        return getattr(importlib.import_module(f".{_LAZY[name]}", __name__), name)
    if name == "gemm":
        return importlib.import_module(".gemm", __name__)
    raise AttributeError(name)
