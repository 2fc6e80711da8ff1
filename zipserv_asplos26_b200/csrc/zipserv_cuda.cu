// The library's device code as one translation unit: the kernels share the
// device-side failure flag without relocatable device code.
#include "zipgemm.cu"
#include "decompress.cu"
#include "capi_cuda.cu"
#include "noalloc.cu"
#include "gpu_packer.cu"
