// all_kernels.cu -- the library's device code as one translation unit.
//
// Compiled without relocatable device code (-rdc): ptxas ignores setmaxnreg in relocatable
// code ("to maintain compatibility across compilation units"), and the warp-specialised
// kernels rely on it to give their math warps more registers than their data-movement warps.
// One unit also lets the status word and the wait limit (sm100.cuh) be plain definitions.
#include "status.cu"
#include "layer_norm.cu"
#include "attention_fwd.cu"
#include "attention_bwd.cu"
#include "gdp.cu"
#include "gate.cu"
#include "linear.cu"
#include "peer.cu"
