// Unity build of libanima_b200.so: one translation unit, so the device error word and the kernels
// share a module without relocatable device code.
#include "runtime.cu"
#include "rowops.cu"
#include "gemm_i8.cu"
#include "attention.cu"
#include "peer.cu"
#include "vae.cu"
