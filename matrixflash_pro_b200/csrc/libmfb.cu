// Single translation unit of libmfb.so: the device status word (mfb::g_status) is
// defined once and named directly by every kernel without relocatable device code.
#include "mfb_abi.cu"
#include "gemm_tc.cu"
#include "gemv.cu"
#include "conv.cu"
#include "noalloc.cu"
#include "stats.cu"
#include "peak_probe.cu"
#include "collectives.cu"
#include "host_gemm.cu"
#include "multi_gemm.cu"
#include "plugin.cu"
