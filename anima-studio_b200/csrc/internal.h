// Host-side internals shared by the .cu files of libanima_b200.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/anima_b200.h"

struct anima_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  bool profile = false;
  void* prof = nullptr;  // ProfileState* (runtime.cu)
  float* attn_ws = nullptr;         // stream-K attention partials (attention.cu)
  unsigned* attn_flags = nullptr;   // their ready flags, zero between launches
  int attn_split = -1;              // anima_ctx_set_attention_split mode
  void* attn_static_ws = nullptr;   // static workspace of anima_attention_noalloc (flags first)
  int8_t* w4_ws = nullptr;          // int8 grid of the W4 weight anima_linear is running (gemm_i8.cu)
  size_t w4_ws_bytes = 0;
  void* vae_ws = nullptr;           // bf16 hi/lo planes of the VAE convolution's input (vae.cu)
  size_t vae_ws_bytes = 0;
  void* mat_ws = nullptr;           // scores, probability and operand planes of attention_planes (vae.cu)
  size_t mat_ws_bytes = 0;
};

namespace anima {

int set_error(int status, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
int check_launch(const char* what);

// Encode a tiled tensor map (driver entry point fetched at run time, no -lcuda needed).
// dims/strides: dims[0] is the contiguous dimension; strides are in bytes for dims 1..rank-1.
int make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// Makes the context's device current for the length of one entry point and puts the caller's
// device back afterwards, so one host thread can drive contexts on several GPUs in turn (kernel
// launches, symbol reads and allocations all act on the current device).
struct DeviceScope {
  int prev = -1;
  int status = ANIMA_OK;
  explicit DeviceScope(const anima_ctx* ctx);
  ~DeviceScope();
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;
};

// cudaFuncAttributeMaxDynamicSharedMemorySize = bytes for kernel fn on the current device. The
// attribute belongs to the device, so it is set once per (kernel, device) pair, under a lock.
int set_max_dynamic_smem(const void* fn, int bytes);

// Single-head attention with a wide head (the VAE's d = 384 over every latent pixel) on the tensor
// cores, with the scores materialised (vae.cu); attention_planes_ok says whether it takes `a`.
bool attention_planes_ok(const anima_attention_args* a);
int attention_planes(anima_ctx* ctx, const anima_attention_args* a);

// C (+)= A B^T + bias for fp32 A [M, K] (rows lda apart) and bf16 (f16: fp16) B [N, K] on the tensor
// cores (A as two planes of B's type), C [M, N] dense (vae.cu). Returns ANIMA_ERR_UNSUPPORTED, with nothing launched,
// when the shape or alignment does not suit it or its plane buffer would have to grow inside
// stream capture; the caller then takes the CUDA-core GEMM.
int matmul_planes(anima_ctx* ctx, int M, int N, int K, const float* A, int lda, const void* B, const float* bias,
                  float* C, int ldc, int accumulate, bool f16);

// Decode 4-bit weights to their int8 grid values (rowops.cu; the arithmetic of anima_unpack_w4):
// out int8 [N, K] from packed nibbles [N, K/2] and fp8 group scales [N, K/16].
int launch_w4_decode(anima_ctx* ctx, const uint8_t* packed, const uint8_t* s_rel, const float* codebook, int N, int K,
                     int8_t* out);

// Profiling scope: records CUDA events around a launch when ANIMA_PROFILE=1.
struct ProfScope {
  anima_ctx* ctx;
  const char* name;
  double flops, bytes;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  ProfScope(anima_ctx* c, const char* n, double f = 0, double b = 0);
  ~ProfScope();
};

}  // namespace anima

#define ANIMA_REQUIRE(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) return ::anima::set_error(ANIMA_ERR_ARG, __VA_ARGS__); \
  } while (0)

#define ANIMA_CUDA(call)                                           \
  do {                                                             \
    int _st = ::anima::check_cuda((call), #call);                  \
    if (_st) return _st;                                           \
  } while (0)

// First statement after an entry point's NULL check of ctx: run the rest on ctx->device.
#define ANIMA_ON_DEVICE(ctx)                                       \
  ::anima::DeviceScope _anima_device_scope(ctx);                   \
  if (_anima_device_scope.status) return _anima_device_scope.status
