// Epilogues of the stand-alone INT8 GEMMs (shared by the GEMM kernels and
// the layers that call them).
#pragma once

namespace tac {

enum GemmEpilogue : int {
  EPI_I32 = 0,              // int32 out
  EPI_REQUANT_PC = 1,       // int8 = sat(rint(f32(acc) * f32(scale[n])))
  EPI_REQUANT_SHIFT = 2,    // int8 = sat((acc * mult[n] + 2^(shift-1)) >> shift)
  EPI_DEQUANT_SCALED = 3,   // fp16 = (f32(acc) * f32(scale[n])) * f32(act) [+ f32(bias[n])]
};

}  // namespace tac
