// Single translation unit of libwgb_b200.so: the level-wise engine and the
// binning / prediction / reference-compatible entry points share kernels.
#include "wgb_engine.cu"
#include "wgb_ops.cu"
#include "wgb_io.cu"
#include "wgb_quantile.cu"
#include "wgb_noalloc.cu"
#include "wgb_comm.cu"
#include "wgb_decode.cu"
