// gplk_unity.cu - the single translation unit of libgplk.so. Kernels share
// the device status word in gplk_core.cu, so they are compiled together.
#include "gplk_core.cu"
#include "gplk_memstream.cu"
#include "gplk_sgemm.cu"
#include "gplk_gemm_pair.cu"
#include "gplk_gemm_tc.cu"
#include "gplk_powervirus.cu"
#include "gplk_powervirus_noalloc.cu"
#include "gplk_gemm_lt.cu"
#include "gplk_fabric.cu"
