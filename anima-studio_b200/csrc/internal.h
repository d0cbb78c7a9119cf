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
};

namespace anima {

int set_error(int status, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
int check_launch(const char* what);

// Encode a tiled tensor map (driver entry point fetched at run time, no -lcuda needed).
// dims/strides: dims[0] is the contiguous dimension; strides are in bytes for dims 1..rank-1.
int make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

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
