// Peer memory of the sequence-parallel mode: CUDA IPC buffers and the cross-GPU barrier.
//
// The ranks of one node (one process per GPU) split an image's token rows; the qkv GEMM of each
// rank stores its k|v tiles straight into every rank's gathered k|v buffer over NVLink (TMA
// stores through tensor maps on the IPC mappings, gemm_i8.cu), and anima_peer_barrier then
// orders those writes before any rank's attention reads its buffer.
#include <cuda_runtime.h>

#include <cstring>

#include "internal.h"
#include "sm100.cuh"

namespace anima {
namespace peer {

__device__ __forceinline__ void st_release_sys(unsigned* q, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(q), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* q) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(q) : "memory");
  return v;
}

// One warp. Lane r (< world) tells rank r that this rank reached `epoch`, then waits until rank r
// told this rank the same. Epochs only grow, so "arrived" is (flag - epoch) read as signed >= 0.
__global__ void barrier_kernel(anima_peer_group g, unsigned long long timeout_ns) {
  __shared__ unsigned epoch;
  if (threadIdx.x == 0) {
    epoch = *g.counter + 1u;
    *g.counter = epoch;
    // writes of this rank's earlier kernels (k|v tiles in peer memory) before the flags
    __threadfence_system();
  }
  __syncwarp();
  const int r = threadIdx.x;
  if (r < g.world) st_release_sys(g.flags[r] + g.rank, epoch);
  if (r < g.world) {
    const unsigned* mine = g.flags[g.rank] + r;
    const unsigned long long t0 = globaltimer();
    while (static_cast<int>(ld_acquire_sys(mine) - epoch) < 0) {
      if (globaltimer() - t0 > timeout_ns) {
        flag_error(kErrPeerWait);
        break;
      }
    }
  }
  __syncwarp();
}

}  // namespace peer
}  // namespace anima

using namespace anima;

extern "C" {

int anima_ipc_alloc(anima_ctx* ctx, size_t bytes, void** ptr, unsigned char handle[64]) {
  ANIMA_REQUIRE(ctx && ptr && handle && bytes > 0, "anima_ipc_alloc: bad argument");
  ANIMA_ON_DEVICE(ctx);
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
  void* p = nullptr;
  ANIMA_CUDA(cudaMalloc(&p, bytes));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return check_cuda(e, "anima_ipc_alloc");
  }
  memcpy(handle, &h, 64);
  *ptr = p;
  return ANIMA_OK;
}

int anima_ipc_open(anima_ctx* ctx, const unsigned char handle[64], void** ptr) {
  ANIMA_REQUIRE(ctx && handle && ptr, "anima_ipc_open: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, 64);
  ANIMA_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return ANIMA_OK;
}

int anima_ipc_close(anima_ctx* ctx, void* ptr) {
  ANIMA_REQUIRE(ctx && ptr, "anima_ipc_close: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_CUDA(cudaIpcCloseMemHandle(ptr));
  return ANIMA_OK;
}

int anima_ipc_free(anima_ctx* ctx, void* ptr) {
  ANIMA_REQUIRE(ctx && ptr, "anima_ipc_free: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_CUDA(cudaFree(ptr));
  return ANIMA_OK;
}

int anima_peer_barrier(anima_ctx* ctx, const anima_peer_group* g) {
  ANIMA_REQUIRE(ctx && g, "anima_peer_barrier: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_REQUIRE(g->world >= 1 && g->world <= 8 && g->rank >= 0 && g->rank < g->world && g->counter,
                "anima_peer_barrier: rank %d of world %d (at most 8)", g->rank, g->world);
  for (int r = 0; r < g->world; ++r)
    ANIMA_REQUIRE(g->flags[r] != nullptr, "anima_peer_barrier: no flags for rank %d", r);
  ANIMA_REQUIRE(g->timeout_us <= 2000000u, "anima_peer_barrier: timeout above 2 s");
  const unsigned long long t = g->timeout_us ? 1000ull * g->timeout_us : kWaitTimeoutNs;
  peer::barrier_kernel<<<1, 32, 0, ctx->stream>>>(*g, t);
  return check_launch("peer barrier_kernel");
}

}  // extern "C"
