// libaudio8_b200.so: the whole library as one translation unit (its kernels share the device error record).
#include "gemm.cu"
#include "attention.cu"
#include "rowops.cu"
#include "sample.cu"
#include "conv.cu"
#include "codec.cu"
#include "vocoder.cu"
#include "engine.cu"
