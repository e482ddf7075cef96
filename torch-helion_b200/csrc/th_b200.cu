// Unity translation unit of libth_b200.so: one TU so the device error word
// is shared by every kernel without relocatable device code.
#include "common.cu"
#include "norm.cu"
#include "gemm.cu"
#include "attention.cu"
#include "ssd.cu"
#include "selftest.cu"
#include "allreduce.cu"
