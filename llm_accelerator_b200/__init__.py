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


def __getattr__(name):
    # CUDA-backed classes load libtaccel_b200.so on first use.
    if name in ("B200Simulator", "B200State"):
        from . import simulator
        return getattr(simulator, name)
    if name in ("HostRunner", "BatchedRunner"):
        from . import runner
        return getattr(runner, name)
    if name in ("Engine", "compile_program"):
        from . import engine
        return getattr(engine, name)
    if name == "gemm":
        from . import gemm
        return gemm
    raise AttributeError(name)
