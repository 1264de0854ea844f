"""ctypes binding of libtaccel_b200.so (declarations in include/taccel_b200.h).

Importing this module loads the CUDA library; if it has not been built the
import fails with a message saying how to build it.  There is no CPU path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

from . import errors as E

LIB_PATH = Path(__file__).resolve().parent / "libtaccel_b200.so"

# status codes (enum tac_status)
OK = 0
E_SIMULATOR, E_ILLEGAL_OPCODE, E_ILLEGAL_BUFFER, E_CONFIG = 1, 2, 3, 4
E_SRAM_ACCESS, E_DRAM_ACCESS, E_VALUE = 5, 6, 7
E_ARGUMENT, E_UNSUPPORTED, E_SHARED_WRITE, E_CUDA, E_DEVICE, E_RECOMPILE = 16, 17, 18, 19, 20, 21


class Fault(C.Structure):
    _fields_ = [("status", C.c_int32), ("buf_id", C.c_int32), ("pc", C.c_uint64), ("raw_word", C.c_uint64),
                ("addr", C.c_uint64), ("offset", C.c_int64), ("limit", C.c_int64), ("message", C.c_char * 320)]


class Regs(C.Structure):
    _fields_ = [("addr_regs", C.c_uint64 * 4), ("tile_valid", C.c_int32), ("tile", C.c_uint32 * 3),
                ("attn_valid", C.c_int32), ("attn_qrb", C.c_uint32), ("attn_vkl", C.c_uint32),
                ("attn_mode", C.c_uint32)]


class VarSite(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("addr_reg", C.c_uint32), ("lo_pc", C.c_uint64), ("hi_pc", C.c_uint64),
                ("range_lo", C.c_uint64), ("range_hi", C.c_uint64)]


class BundleView(C.Structure):
    _fields_ = [("prefill", C.c_void_p), ("prefill_len", C.c_uint64), ("decode", C.c_void_p),
                ("decode_len", C.c_uint64), ("shared", C.c_void_p), ("shared_len", C.c_uint64),
                ("meta_json", C.c_void_p), ("meta_len", C.c_uint64)]


class ExecInfo(C.Structure):
    _fields_ = [("executed", C.c_uint64), ("final_pc", C.c_uint64), ("halted", C.c_int32),
                ("faulted", C.c_int32), ("cycles", C.c_uint64), ("n_ops", C.c_uint64),
                ("n_levels", C.c_uint64), ("n_tasks", C.c_uint64), ("n_segments", C.c_uint64),
                ("arena_bytes", C.c_uint64), ("n_slots", C.c_uint64), ("n_var_words", C.c_uint64),
                ("final_regs", Regs)]


COMPILE_NO_PACK = 1   # TAC_COMPILE_NO_PACK


class CompileOpts(C.Structure):
    _fields_ = [("n_live", C.c_uint32), ("sram_live", C.c_int32), ("sregs_live", C.c_int32),
                ("flags", C.c_int32), ("live", C.c_void_p)]


_P = C.c_void_p
_U64 = C.c_uint64
_I = C.c_int

# name -> (restype, argtypes); every symbol include/taccel_b200.h declares
SIGNATURES = {
    "tac_engine_create": (_I, [_I, _I, _U64, _U64, C.POINTER(_P)]),
    "tac_engine_destroy": (_I, [_P]),
    "tac_engine_batch": (_I, [_P]),
    "tac_dram_write": (_I, [_P, _I, _U64, _P, _U64]),
    "tac_dram_read": (_I, [_P, _I, _U64, _P, _U64]),
    "tac_sram_write": (_I, [_P, _I, _I, _U64, _P, _U64]),
    "tac_sram_read": (_I, [_P, _I, _I, _U64, _P, _U64]),
    "tac_sregs_write": (_I, [_P, _I, _P]),
    "tac_sregs_read": (_I, [_P, _I, _P]),
    "tac_compile": (_I, [_I, _U64, _U64, _P, _U64, _U64, _U64, C.POINTER(Regs), _I, C.POINTER(VarSite), _I,
                         C.POINTER(_P), C.POINTER(ExecInfo), C.POINTER(Fault)]),
    "tac_compile_ex": (_I, [_I, _U64, _U64, _P, _U64, _U64, _U64, C.POINTER(Regs), _I, C.POINTER(VarSite), _I,
                            C.POINTER(CompileOpts), C.POINTER(_P), C.POINTER(ExecInfo), C.POINTER(Fault)]),
    "tac_program_home_reads": (_I, [_P, _P, C.c_uint32, _P, _P, _P]),
    "tac_program_destroy": (_I, [_P]),
    "tac_program_info": (_I, [_P, C.POINTER(ExecInfo), C.POINTER(Fault)]),
    "tac_program_record_size": (_U64, [_I]),
    "tac_program_dump": (_I, [_P, _P, _P, _P, _P]),
    "tac_run_async": (_I, [_P, _P, _P, _P, C.POINTER(Fault)]),
    "tac_run": (_I, [_P, _P, _P, C.POINTER(Fault)]),
    "tac_check_device_status": (_I, [_P, C.POINTER(Fault)]),
    "tac_program_param_count": (_U64, [_P]),
    "tac_program_attn_key_cols": (C.c_uint32, [_P]),
    "tac_encode_params": (_I, [_P, _I, _P, _P, C.POINTER(Fault)]),
    "tac_run_async_params": (_I, [_P, _P, _P, _P, C.POINTER(Fault)]),
    "tac_program_set_var_formula": (_I, [_P, C.c_uint32, _P, _P, _P, _P]),
    "tac_encode_params_tp": (_I, [_P, _I, _P, _P, _P, C.POINTER(Fault)]),
    "tac_run_async_tp": (_I, [_P, _P, _P, _P, _P, C.POINTER(Fault)]),
    "tac_argmax_f16": (_I, [_P, _U64, _U64, _P, _P]),
    "tac_set_profiling": (_I, [_P, _I]),
    "tac_read_profile": (_I, [_P, _P, C.c_uint32, _P]),
    "tac_read_task_profile": (_I, [_P, _P, _U64, _P]),
    "tac_engine_layout": (_I, [_P, C.POINTER(_P), C.POINTER(_U64), C.POINTER(_P)]),
    "tac_engine_grid": (_I, [_P]),
    "tac_gemm_i8_requant_pc": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "tac_gemm_i8_requant_shift": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "tac_gemm_i8_i32": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "tac_gemm_status": (_I, [_P]),
    "tac_gemm_i8_requant_pc_bt": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "tac_gemm_i8_i32_bt": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "tac_gemv_i8_requant_pc_static": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "tac_gemm_wo_f16_i8": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "tac_fwht_f16": (_I, [_P, _P, _I, _I, _I, _P]),
    "tac_quarot_workspace_bytes": (_U64, [_I, _I]),
    "tac_quarot_w8a16": (_I, [_P, _P, _P, _P, _P, _P, _U64, _I, _I, _I, _I, _P]),
    "tac_quantize_weight_i8": (_I, [_P, _I, _I, _I, _P, _P, _P, _P]),
    "tac_bundle_open": (_I, [C.c_char_p, C.POINTER(BundleView), C.POINTER(_P)]),
    "tac_bundle_close": (_I, [_P]),
}


def _load():
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH.name} is not built; run `python -m llm_accelerator_b200.build` "
                          "(nvcc, sm_100a) first")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def fault_to_exception(f: Fault, status: int | None = None) -> Exception:
    """Maps a fault record to the exception the golden simulator raises."""
    s = f.status if status is None else status
    msg = f.message.decode(errors="replace")
    if s == E_SIMULATOR:
        return E.SimulatorError(msg)
    if s == E_ILLEGAL_OPCODE:
        return E.IllegalOpcodeError(int(f.pc), int(f.raw_word).to_bytes(8, "big"))
    if s == E_ILLEGAL_BUFFER:
        return E.IllegalBufferError(int(f.buf_id))
    if s == E_CONFIG:
        return E.ConfigError(msg)
    if s == E_SRAM_ACCESS:
        return E.SRAMAccessError(int(f.buf_id), int(f.offset), int(f.limit))
    if s == E_DRAM_ACCESS:
        return E.DRAMAccessError(int(f.addr))
    if s == E_VALUE:
        return ValueError(msg)
    return E.EngineError(f"taccel_b200 status {s}: {msg}")


def check(status: int, what: str = "") -> None:
    if status != OK:
        raise E.EngineError(f"{what or 'taccel_b200 call'} failed with status {status}")
