// Context, errors, memory, tensor maps and the per-op profiler of libanima_b200
// (the role of the reference's GPU class, app/gpu/device.js:59-232).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "internal.h"
#include "sm100.cuh"

namespace anima {

static thread_local std::string t_last_error;

int set_error(int status, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return status;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ANIMA_OK;
  return set_error(ANIMA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return ANIMA_OK;
  return set_error(ANIMA_ERR_CUDA, "launch of %s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(ANIMA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(ANIMA_ERR_ARG, "TMA base address %p is not 16-byte aligned", base);
  for (int i = 1; i < rank; ++i)
    if (strides_bytes[i - 1] % 16 != 0)
      return set_error(ANIMA_ERR_ARG, "TMA stride %llu bytes is not a multiple of 16",
                       (unsigned long long)strides_bytes[i - 1]);
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
  CUresult r = fn(map, dtype, rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ANIMA_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return ANIMA_OK;
}

// ------------------------------------------------------------------ devices

DeviceScope::DeviceScope(const anima_ctx* ctx) {
  int cur = 0;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) {
    status = check_cuda(e, "cudaGetDevice");
    return;
  }
  if (cur == ctx->device) return;
  e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) {
    status = check_cuda(e, "cudaSetDevice (the context's device)");
    return;
  }
  prev = cur;
}

DeviceScope::~DeviceScope() {
  if (prev >= 0) cudaSetDevice(prev);
}

int set_max_dynamic_smem(const void* fn, int bytes) {
  int dev = 0;
  ANIMA_CUDA(cudaGetDevice(&dev));
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({fn, dev})) return ANIMA_OK;
  ANIMA_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert({fn, dev});
  return ANIMA_OK;
}

// ------------------------------------------------------------------ profiler

struct ProfEntry {
  double ms = 0, flops = 0, bytes = 0;
  long calls = 0;
};
struct PendingEvent {
  std::string name;
  double flops, bytes;
  cudaEvent_t e0, e1;
};
struct ProfileState {
  std::map<std::string, ProfEntry> table;
  std::vector<PendingEvent> pending;
};

static void prof_collect(anima_ctx* ctx) {
  auto* st = static_cast<ProfileState*>(ctx->prof);
  if (!st) return;
  for (auto& p : st->pending) {
    float ms = 0;
    cudaEventSynchronize(p.e1);
    cudaEventElapsedTime(&ms, p.e0, p.e1);
    auto& e = st->table[p.name];
    e.ms += ms;
    e.flops += p.flops;
    e.bytes += p.bytes;
    e.calls += 1;
    cudaEventDestroy(p.e0);
    cudaEventDestroy(p.e1);
  }
  st->pending.clear();
}

ProfScope::ProfScope(anima_ctx* c, const char* n, double f, double b) : ctx(c), name(n), flops(f), bytes(b) {
  if (!ctx || !ctx->profile) return;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, ctx->stream);
}

ProfScope::~ProfScope() {
  if (!e0) return;
  cudaEventRecord(e1, ctx->stream);
  static_cast<ProfileState*>(ctx->prof)->pending.push_back({name, flops, bytes, e0, e1});
}

}  // namespace anima

using namespace anima;

extern "C" {

int anima_version(void) { return 1; }

const char* anima_last_error(void) { return t_last_error.c_str(); }

int anima_ctx_create(int device, anima_ctx** out) {
  ANIMA_REQUIRE(out != nullptr, "anima_ctx_create: out is NULL");
  int n = 0;
  ANIMA_CUDA(cudaGetDeviceCount(&n));
  ANIMA_REQUIRE(device >= 0 && device < n, "anima_ctx_create: device %d out of range (%d devices)", device, n);
  anima_ctx probe;
  probe.device = device;
  ANIMA_ON_DEVICE(&probe);  // the caller's current device is left as it was
  cudaDeviceProp prop;
  ANIMA_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return set_error(ANIMA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device,
                     prop.major, prop.minor);
  auto* c = new anima_ctx();
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  const char* split = getenv("ANIMA_ATTN_STREAMK");
  if (split && split[0]) c->attn_split = atoi(split) != 0 ? 1 : 0;
  const char* p = getenv("ANIMA_PROFILE");
  c->profile = p && p[0] == '1';
  if (c->profile) c->prof = new ProfileState();
  *out = c;
  return ANIMA_OK;
}

int anima_ctx_destroy(anima_ctx* ctx) {
  if (!ctx) return ANIMA_OK;
  ANIMA_ON_DEVICE(ctx);
  if (ctx->prof) {
    prof_collect(ctx);
    delete static_cast<ProfileState*>(ctx->prof);
  }
  if (ctx->attn_ws) cudaFree(ctx->attn_ws);
  if (ctx->attn_flags) cudaFree(ctx->attn_flags);
  if (ctx->w4_ws) cudaFree(ctx->w4_ws);
  if (ctx->vae_ws) cudaFree(ctx->vae_ws);
  if (ctx->mat_ws) cudaFree(ctx->mat_ws);
  delete ctx;
  return ANIMA_OK;
}

int anima_ctx_set_stream(anima_ctx* ctx, void* stream) {
  ANIMA_REQUIRE(ctx, "anima_ctx_set_stream: ctx is NULL");
  ctx->stream = static_cast<cudaStream_t>(stream);
  return ANIMA_OK;
}

int anima_ctx_set_attention_split(anima_ctx* ctx, int mode) {
  ANIMA_REQUIRE(ctx, "anima_ctx_set_attention_split: ctx is NULL");
  ANIMA_REQUIRE(mode >= -1 && mode <= 1, "anima_ctx_set_attention_split: mode %d (-1, 0 or 1)", mode);
  ctx->attn_split = mode;
  return ANIMA_OK;
}

int anima_sync(anima_ctx* ctx) {
  ANIMA_REQUIRE(ctx, "anima_sync: ctx is NULL");
  ANIMA_ON_DEVICE(ctx);  // the error word and the flags below are this device's
  ANIMA_CUDA(cudaStreamSynchronize(ctx->stream));
  unsigned err = 0, zero = 0;
  ANIMA_CUDA(cudaMemcpyFromSymbol(&err, g_device_error, sizeof(err)));
  if (err) {
    ANIMA_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
    // an aborted stream-K attention can leave a partial's ready flag raised
    if (ctx->attn_flags)
      ANIMA_CUDA(cudaMemset(ctx->attn_flags, 0, static_cast<size_t>(ctx->num_sms) * 16 * sizeof(unsigned)));
    if (ctx->attn_static_ws)
      ANIMA_CUDA(cudaMemset(ctx->attn_static_ws, 0, static_cast<size_t>(ctx->num_sms) * 16 * sizeof(unsigned)));
    return set_error(ANIMA_ERR_DEVICE, "device error flags 0x%x (%s%s%s%s%s%s)", err,
                     (err & kErrTimeoutFull) ? "data wait timed out; " : "",
                     (err & kErrTimeoutEmpty) ? "stage wait timed out; " : "",
                     (err & kErrTimeoutAcc) ? "accumulator wait timed out; " : "",
                     (err & kErrTimeoutDrain) ? "drain after abort timed out; " : "",
                     (err & kErrBadArgs) ? "kernel rejected its arguments; " : "",
                     (err & kErrPeerWait) ? "cross-GPU barrier timed out waiting for another rank; " : "");
  }
  if (ctx->profile) prof_collect(ctx);
  return ANIMA_OK;
}

// Failure-path self test: one warp waits, with the pipelines' bounded wait, on an mbarrier phase
// that nothing completes. After timeout_ns the wait raises kErrTimeoutFull in the device error
// word and the CTA abort flag and returns; out = {wait succeeded, abort flag}.
__global__ void selftest_wait_kernel(unsigned long long timeout_ns, int* out) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncwarp();
  int ok = 1;
  if (threadIdx.x == 0) ok = mbar_wait_for(&bar, 0, &abort_flag, kErrTimeoutFull, timeout_ns) ? 1 : 0;
  __syncwarp();
  if (threadIdx.x == 0) {
    out[0] = ok;
    out[1] = abort_flag;
  }
}

int anima_selftest_wait_timeout(anima_ctx* ctx, unsigned timeout_us, int* result) {
  ANIMA_REQUIRE(ctx && result && timeout_us > 0 && timeout_us <= 2000000u,
                "anima_selftest_wait_timeout: bad argument (timeout 1 us .. 2 s)");
  ANIMA_ON_DEVICE(ctx);
  int* d = nullptr;
  ANIMA_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&d), 2 * sizeof(int), ctx->stream));
  selftest_wait_kernel<<<1, 32, 0, ctx->stream>>>(1000ull * timeout_us, d);
  int st = check_launch("selftest_wait_kernel");
  if (!st) st = check_cuda(cudaMemcpyAsync(result, d, 2 * sizeof(int), cudaMemcpyDeviceToHost, ctx->stream),
                           "anima_selftest_wait_timeout: copy");
  cudaFreeAsync(d, ctx->stream);
  if (!st) st = check_cuda(cudaStreamSynchronize(ctx->stream), "anima_selftest_wait_timeout: synchronize");
  return st;
}

int anima_alloc(anima_ctx* ctx, size_t bytes, void** out) {
  ANIMA_REQUIRE(ctx && out, "anima_alloc: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_CUDA(cudaMallocAsync(out, bytes ? bytes : 16, ctx->stream));
  return ANIMA_OK;
}

int anima_free(anima_ctx* ctx, void* ptr) {
  ANIMA_REQUIRE(ctx, "anima_free: ctx is NULL");
  ANIMA_ON_DEVICE(ctx);
  if (ptr) ANIMA_CUDA(cudaFreeAsync(ptr, ctx->stream));
  return ANIMA_OK;
}

int anima_upload(anima_ctx* ctx, void* dst, const void* src, size_t bytes) {
  ANIMA_REQUIRE(ctx && dst && src, "anima_upload: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return ANIMA_OK;
}

int anima_download(anima_ctx* ctx, void* dst, const void* src, size_t bytes) {
  ANIMA_REQUIRE(ctx && dst && src, "anima_download: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return ANIMA_OK;
}

int anima_zero(anima_ctx* ctx, void* p, size_t bytes) {
  ANIMA_REQUIRE(ctx && p, "anima_zero: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_CUDA(cudaMemsetAsync(p, 0, bytes, ctx->stream));
  return ANIMA_OK;
}

int anima_profile_report(anima_ctx* ctx, char* buf, size_t cap) {
  ANIMA_REQUIRE(ctx && buf && cap > 0, "anima_profile_report: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  std::string s;
  if (!ctx->profile) {
    s = "profiling disabled (set ANIMA_PROFILE=1 before creating the context)\n";
  } else {
    ANIMA_CUDA(cudaStreamSynchronize(ctx->stream));
    prof_collect(ctx);
    auto* st = static_cast<ProfileState*>(ctx->prof);
    char line[256];
    snprintf(line, sizeof(line), "%-28s %8s %12s %12s %10s\n", "op", "calls", "total ms", "TFLOP/s", "GB/s");
    s += line;
    for (auto& kv : st->table) {
      const ProfEntry& e = kv.second;
      double sec = e.ms * 1e-3;
      snprintf(line, sizeof(line), "%-28s %8ld %12.3f %12.1f %10.1f\n", kv.first.c_str(), e.calls, e.ms,
               sec > 0 ? e.flops / sec * 1e-12 : 0.0, sec > 0 ? e.bytes / sec * 1e-9 : 0.0);
      s += line;
    }
  }
  size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
  memcpy(buf, s.data(), n);
  buf[n] = 0;
  return ANIMA_OK;
}

}  // extern "C"
