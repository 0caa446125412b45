// Single translation unit of libkf_sm100.so: the kernels share the device
// status word and the host helpers without relocatable device code.
#include "kf_runtime.cu"
#include "ln_sm100.cu"
#include "gemm_sm100.cu"
#include "flash_sm100.cu"
#include "flash_persist_sm100.cu"
#include "noalloc_sm100.cu"
