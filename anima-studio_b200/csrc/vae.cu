// Wan-2.1 VAE decoder operators (app/models/vae.js; math of tools/reference.py:254-295): the NHWC
// 3x3 convolution as a tensor-core implicit GEMM (the nearest 2x upsample of Resample applied when
// the input is split into its bf16 planes), the same GEMM for bf16 matmuls and for the decoder's
// wide single-head attention, and the channel RMS norm with the SiLU that follows it. Activations
// stay fp32 between kernels; the weights are bf16 (OHWI, as the reference's asset builder stores
// them).
#include "internal.h"
#include "sm100.cuh"

namespace anima {
namespace vae {

// ------------------------------------------------------------------ tcgen05 implicit GEMM
// out[p, o] (+)= bias[o] + sum_{tap, c} in[p + tap offset, c] * w[o, tap, c] with the input given
// as two bf16 planes, in = hi + lo (hi = bf16(x), lo = bf16(x - hi): about 16 significant bits),
// both multiplied by the bf16 weights on the tensor core (kind::f16, fp32 accumulation in tensor
// memory). A tile is 128 output pixels, a run of tile_w columns by tile_h rows of the image, by BN
// output channels. Its K loop walks the taps and, per tap, the input channels in chunks of 64: the
// A tile of a (tap, chunk) is one TMA box of the plane, {64 channels, tile_w, tile_h} at the
// tap-shifted pixel origin, so the zero padding of the border and the channels past cin come from
// the TMA's out-of-bounds fill (a chunk's weights past its tap multiply zeros); the B tile is the
// weights' [BN rows x 64] box at K offset tap * cin + chunk * 64 (rows past cout are zeros too).
// Persistent CTAs, 320 threads: warps 0-3 and 6-9 two epilogue warpgroups (thread = pixel row of the
// accumulator; with BN >= 128 each takes half of every tile's channels, which halves the
// latency-bound epilogue of short-K GEMMs), warp 4 TMA producer, warp 5 TMEM allocator and
// single-thread MMA issuer; three pipeline stages and two accumulator buffers in tensor memory, so
// a tile's epilogue overlaps the next tile's MMAs.
namespace tc {

constexpr int BM = 128;
constexpr int CK = 64;                      // input channels per k-block: one 128-byte row of bf16
constexpr int A_BYTES = BM * CK * 2;        // one plane's tile
constexpr int MAX_BN = 256;
constexpr int STAGES = 3;
constexpr int STAGE_BYTES = 2 * A_BYTES + MAX_BN * CK * 2;
constexpr int THREADS = 320;
constexpr int SMEM = STAGES * STAGE_BYTES + 256 + 1024;

struct Params {
  int H, W, cin, cout, taps;       // taps: 9 (3x3, pad 1) or 1
  int f16;                         // operands fp16 instead of bf16
  int tile_w, tile_h, tiles_x, n_tiles, num_tiles, BN, nchunks;
  const float* bias;
  float* out;
  int accumulate;
};

template <bool DUMMY = false>
__global__ void __launch_bounds__(THREADS, 1) conv_tc_kernel(const __grid_constant__ CUtensorMap tm_hi,
                                                             const __grid_constant__ CUtensorMap tm_lo,
                                                             const __grid_constant__ CUtensorMap tm_w, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nkb = p.taps * p.nchunks;

  if (warp == 4) {  // producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int armed[STAGES];
      for (int s = 0; s < STAGES; ++s) armed[s] = -1;
      const uint32_t tx = 2 * A_BYTES + p.BN * CK * 2;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        const int nt = t % p.n_tiles, pt = t / p.n_tiles;
        const int x0 = (pt % p.tiles_x) * p.tile_w, y0 = (pt / p.tiles_x) * p.tile_h;
        for (int kb = 0; kb < nkb; ++kb) {
          const int tap = kb / p.nchunks, ch = kb % p.nchunks;
          const int dx = p.taps == 9 ? tap % 3 - 1 : 0, dy = p.taps == 9 ? tap / 3 - 1 : 0;
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, kErrTimeoutEmpty)) goto producer_done;
          uint8_t* sa = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], tx);
          tma_load_3d(sa, &tm_hi, &full[stage], ch * CK, x0 + dx, y0 + dy);
          tma_load_3d(sa + A_BYTES, &tm_lo, &full[stage], ch * CK, x0 + dx, y0 + dy);
          tma_load_2d(sa + 2 * A_BYTES, &tm_w, &full[stage], tap * p.cin + ch * CK, nt * p.BN);
          armed[stage] = static_cast<int>(phase);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:
      if (*abort_flag) {  // copies in flight land before the CTA exits
        for (int s = 0; s < STAGES; ++s) {
          if (armed[s] < 0) continue;
          const unsigned long long t0 = globaltimer();
          while (!mbar_test(smem_u32(&full[s]), static_cast<uint32_t>(armed[s]))) {
            if (globaltimer() - t0 > kWaitTimeoutNs) {
              flag_error(kErrTimeoutDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 5) {  // MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BM, p.BN, !p.f16, false);
      int stage = 0;
      uint32_t phase = 0;
      int i = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (!mbar_wait(&acc_empty[buf], ((i >> 1) & 1) ^ 1, abort_flag, kErrTimeoutAcc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + buf * MAX_BN;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + 2 * A_BYTES;
#pragma unroll
          for (int k = 0; k < CK / 16; ++k) {  // K = 16 bf16 = 32 bytes per MMA
            const uint64_t bd = sdesc_sw128(sb + 32 * k, 16, 1024);
            umma_f16(d, sdesc_sw128(sa + 32 * k, 16, 1024), bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            umma_f16(d, sdesc_sw128(sa + A_BYTES + 32 * k, 16, 1024), bd, idesc, 1u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
      if (*abort_flag) {  // MMAs already issued complete before TMEM is released
        umma_commit(drain);
        const unsigned long long t0 = globaltimer();
        while (!mbar_test(smem_u32(drain), 0)) {
          if (globaltimer() - t0 > kWaitTimeoutNs) {
            flag_error(kErrTimeoutDrain);
            break;
          }
        }
      }
    }
  } else {  // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (pixel rows of the tile)
    const int quad = warp & 3;
    const int g = warp >= 6 ? 1 : 0;
    const int row = quad * 32 + lane;
    const bool vec = (p.cout & 3) == 0;
    // this warpgroup's channels of a tile: halves when BN >= 128 (multiples of 32 columns)
    const bool halves = p.BN >= 128;
    const int cb = halves ? g * (p.BN / 2) : 0;
    const int ce = halves ? cb + p.BN / 2 : (g == 0 ? p.BN : 0);
    int i = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++i) {
      const int buf = i & 1;
      if (!mbar_wait(&acc_full[buf], (i >> 1) & 1, abort_flag, kErrTimeoutAcc)) break;
      tc_fence_after();
      const int nt = t % p.n_tiles, pt = t / p.n_tiles;
      const int x = (pt % p.tiles_x) * p.tile_w + row % p.tile_w;
      const int y = (pt / p.tiles_x) * p.tile_h + row / p.tile_w;
      const bool in = x < p.W && y < p.H;
      const int n0 = nt * p.BN;
      float* o = p.out + (static_cast<long long>(in ? y : 0) * p.W + (in ? x : 0)) * p.cout;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * MAX_BN;
      // 32 columns at a time, the next group's TMEM load in flight while this one is stored
      auto store32 = [&](const uint32_t (&r)[32], int c0) {
        if (!in) return;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const int n = n0 + c0 + j;
          if (n >= p.cout) break;
          float v[4];
          if (vec && p.bias) {
            const float4 b4 = __ldg(reinterpret_cast<const float4*>(p.bias + n));
            v[0] = __uint_as_float(r[j]) + b4.x;
            v[1] = __uint_as_float(r[j + 1]) + b4.y;
            v[2] = __uint_as_float(r[j + 2]) + b4.z;
            v[3] = __uint_as_float(r[j + 3]) + b4.w;
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              v[q] = __uint_as_float(r[j + q]) + (p.bias && n + q < p.cout ? p.bias[n + q] : 0.f);
          }
          if (vec) {
            float4* d4 = reinterpret_cast<float4*>(o + n);
            float4 cur = p.accumulate ? *d4 : make_float4(0.f, 0.f, 0.f, 0.f);
            *d4 = make_float4(cur.x + v[0], cur.y + v[1], cur.z + v[2], cur.w + v[3]);
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (n + q < p.cout) o[n + q] = (p.accumulate ? o[n + q] : 0.f) + v[q];
          }
        }
      };
      uint32_t r0[32], r1[32];
      if (cb < ce) {
        tmem_ld32(taddr + cb, r0);
        tmem_ld_wait(r0);
      }
      for (int c0 = cb; c0 < ce; c0 += 64) {  // r0 holds columns c0 .. c0 + 31
        const bool more1 = c0 + 32 < ce, more2 = c0 + 64 < ce;
        if (more1) tmem_ld32(taddr + c0 + 32, r1);
        store32(r0, c0);
        if (!more1) break;
        tmem_ld_wait(r1);
        if (more2) tmem_ld32(taddr + c0 + 64, r0);
        store32(r1, c0 + 32);
        if (more2) tmem_ld_wait(r0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// Input planes for the tensor-core convolution: hi = T(x), lo = T(x - hi) per element (T bf16, or
// fp16 for the LoRA up-projection's small-range operands), with
// the nearest 2x upsample applied on the way when up != 0; x rows (pixels) ldx floats apart. One
// thread per 8 channels of a pixel.
template <typename T>
__global__ void split_planes_kernel(const float* __restrict__ x, int h, int w, int c, long long ldx, int up,
                                    T* __restrict__ hi, T* __restrict__ lo, long long n8) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const int c8 = c / 8;
  const long long pix = i / c8;
  const int cc = static_cast<int>(i % c8) * 8;
  const int W = up ? 2 * w : w;
  const int yy = static_cast<int>(pix / W), xx = static_cast<int>(pix % W);
  const float* src = x + (static_cast<long long>(up ? yy / 2 : yy) * w + (up ? xx / 2 : xx)) * ldx + cc;
  const float4 a = *reinterpret_cast<const float4*>(src), b = *reinterpret_cast<const float4*>(src + 4);
  const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t hw[4], lw[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if constexpr (std::is_same<T, __half>::value) {
      const __half2 h2 = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
      const float2 hf = __half22float2(h2);
      const __half2 l2 = __floats2half2_rn(v[2 * k] - hf.x, v[2 * k + 1] - hf.y);
      hw[k] = *reinterpret_cast<const uint32_t*>(&h2);
      lw[k] = *reinterpret_cast<const uint32_t*>(&l2);
    } else {
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
      const float2 hf = __bfloat1622float2(h2);
      const __nv_bfloat162 l2 = __floats2bfloat162_rn(v[2 * k] - hf.x, v[2 * k + 1] - hf.y);
      hw[k] = *reinterpret_cast<const uint32_t*>(&h2);
      lw[k] = *reinterpret_cast<const uint32_t*>(&l2);
    }
  }
  reinterpret_cast<uint4*>(hi)[i] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  reinterpret_cast<uint4*>(lo)[i] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

// Rows of S (Lk scores each) to probabilities P = exp(scale (s - max)) / sum, written as bf16 hi/lo
// planes. One CTA per row: a pass for the running maximum and sum (each thread online over its
// columns, then merged across the CTA), a pass that writes P.
__global__ void __launch_bounds__(256) softmax_planes_kernel(const float* __restrict__ S, int Lk, float scale_log2,
                                                             __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
  __shared__ float sm[8], ss[8];
  const float* row = S + static_cast<long long>(blockIdx.x) * Lk;
  float m = -INFINITY, l = 0.f;
  for (int c = threadIdx.x * 4; c < Lk; c += 1024) {
    const float4 v = *reinterpret_cast<const float4*>(row + c);
    const float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)) * scale_log2;
    const float mn = fmaxf(m, mx);
    l = l * exp2f(m - mn) + exp2f(v.x * scale_log2 - mn) + exp2f(v.y * scale_log2 - mn) + exp2f(v.z * scale_log2 - mn) +
        exp2f(v.w * scale_log2 - mn);
    m = mn;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, o), lo_ = __shfl_xor_sync(0xffffffffu, l, o);
    const float mn = fmaxf(m, mo);
    l = (m == -INFINITY ? 0.f : l * exp2f(m - mn)) + (mo == -INFINITY ? 0.f : lo_ * exp2f(mo - mn));
    m = mn;
  }
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = l;
  }
  __syncthreads();
  float M = sm[0];
  for (int i = 1; i < 8; ++i) M = fmaxf(M, sm[i]);
  float L = 0.f;
  for (int i = 0; i < 8; ++i) L += sm[i] == -INFINITY ? 0.f : ss[i] * exp2f(sm[i] - M);
  const float inv = 1.0f / L;
  __nv_bfloat16* hr = hi + static_cast<long long>(blockIdx.x) * Lk;
  __nv_bfloat16* lr = lo + static_cast<long long>(blockIdx.x) * Lk;
  for (int c = threadIdx.x * 4; c < Lk; c += 1024) {
    const float4 v = *reinterpret_cast<const float4*>(row + c);
    const float p[4] = {exp2f(v.x * scale_log2 - M) * inv, exp2f(v.y * scale_log2 - M) * inv,
                        exp2f(v.z * scale_log2 - M) * inv, exp2f(v.w * scale_log2 - M) * inv};
    uint32_t hw[2], lw[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(p[2 * k], p[2 * k + 1]);
      const float2 hf = __bfloat1622float2(h2);
      const __nv_bfloat162 l2 = __floats2bfloat162_rn(p[2 * k] - hf.x, p[2 * k + 1] - hf.y);
      hw[k] = *reinterpret_cast<const uint32_t*>(&h2);
      lw[k] = *reinterpret_cast<const uint32_t*>(&l2);
    }
    *reinterpret_cast<uint2*>(hr + c) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(lr + c) = make_uint2(lw[0], lw[1]);
  }
}

// V [L rows, d] (rows ldv floats apart) to the planes of V^T [d, L]: 32 x 32 tiles through shared
// memory, so both the reads and the writes are coalesced.
__global__ void __launch_bounds__(256) transpose_split_kernel(const float* __restrict__ v, long long ldv, int L, int d,
                                                              __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
  __shared__ float t[32][33];
  const int l0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int r = ty; r < 32; r += 8) {
    const int l = l0 + r, c = d0 + tx;
    t[r][tx] = (l < L && c < d) ? v[static_cast<long long>(l) * ldv + c] : 0.f;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int c = d0 + r, l = l0 + tx;
    if (c < d && l < L) {
      const float x = t[tx][r];
      const __nv_bfloat16 h = __float2bfloat16_rn(x);
      hi[static_cast<long long>(c) * L + l] = h;
      lo[static_cast<long long>(c) * L + l] = __float2bfloat16_rn(x - __bfloat162float(h));
    }
  }
}

}  // namespace tc

// y = x / max(||x||_2, 1e-12) * sqrt(C) * gamma over each row's C channels (F.normalize over the
// channel dim, tools/reference.py:264-265), then SiLU when silu != 0. One warp per row.
__global__ void channel_norm_kernel(const float* __restrict__ x, long long rows, int C, const float* __restrict__ gamma,
                                    int silu, float* __restrict__ y) {
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + row * C;
  float ss = 0.f;
  for (int c = lane; c < C; c += 32) ss = fmaf(xr[c], xr[c], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float s = sqrtf(static_cast<float>(C)) / fmaxf(sqrtf(ss), 1e-12f);
  float* yr = y + row * C;
  for (int c = lane; c < C; c += 32) {
    const float v = xr[c] * s * gamma[c];
    yr[c] = silu ? v / (1.0f + expf(-v)) : v;
  }
}

// Grow a context-owned device buffer outside stream capture (kernels of earlier calls may still
// read the old one, so its stream is drained first).
static int grow_ws(anima_ctx* ctx, void** buf, size_t* have, size_t want, const char* who) {
  if (*have >= want) return ANIMA_OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  ANIMA_CUDA(cudaStreamIsCapturing(ctx->stream, &cap));
  ANIMA_REQUIRE(cap == cudaStreamCaptureStatusNone, "%s: its workspace would grow to %zu bytes inside stream capture",
                who, want);
  if (*buf) {
    ANIMA_CUDA(cudaStreamSynchronize(ctx->stream));
    ANIMA_CUDA(cudaFree(*buf));
    *buf = nullptr;
    *have = 0;
  }
  ANIMA_CUDA(cudaMalloc(buf, want));
  *have = want;
  return ANIMA_OK;
}

// out[p, n] (+)= bias[n] + sum_{tap, c} (hi + lo)[p + tap offset, c] * w[n, tap, c] on the tensor
// cores: planes [H, W, cin] bf16, w bf16 [N, taps * cin] K-major, out fp32 [H W, N].
static int tc_gemm(anima_ctx* ctx, const void* hi, const void* lo, int H, int W, int cin, int taps,
                   const void* wdata, int N, const float* bias, float* out, int accumulate, bool f16 = false) {
  tc::Params p{};
  p.f16 = f16 ? 1 : 0;
  const CUtensorMapDataType dt = f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  p.H = H;
  p.W = W;
  p.cin = cin;
  p.cout = N;
  p.taps = taps;
  p.tile_w = 1;
  while (p.tile_w * 2 <= W && p.tile_w * 2 <= tc::BM) p.tile_w *= 2;  // 128 pixels: tile_w x tile_h
  p.tile_h = tc::BM / p.tile_w;
  p.tiles_x = (W + p.tile_w - 1) / p.tile_w;
  const int tiles_y = (H + p.tile_h - 1) / p.tile_h;
  const int n16 = (N + 15) / 16 * 16;
  p.BN = n16 <= tc::MAX_BN ? n16 : n16 % 256 == 0 ? 256 : n16 % 192 == 0 ? 192 : 128;
  p.n_tiles = (N + p.BN - 1) / p.BN;
  const long long tiles = static_cast<long long>(p.tiles_x) * tiles_y * p.n_tiles;
  ANIMA_REQUIRE(tiles < (1ll << 31), "tensor-core convolution: %lld tiles", tiles);
  p.num_tiles = static_cast<int>(tiles);
  p.nchunks = (cin + tc::CK - 1) / tc::CK;
  p.bias = bias;
  p.out = out;
  p.accumulate = accumulate;
  CUtensorMap tm_hi, tm_lo, tm_w;
  const uint64_t adims[3] = {static_cast<uint64_t>(cin), static_cast<uint64_t>(W), static_cast<uint64_t>(H)};
  const uint64_t astr[2] = {static_cast<uint64_t>(cin) * 2, static_cast<uint64_t>(W) * cin * 2};
  const uint32_t abox[3] = {static_cast<uint32_t>(tc::CK), static_cast<uint32_t>(p.tile_w), static_cast<uint32_t>(p.tile_h)};
  int st = make_tmap(&tm_hi, dt, 3, hi, adims, astr, abox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!st) st = make_tmap(&tm_lo, dt, 3, lo, adims, astr, abox, CU_TENSOR_MAP_SWIZZLE_128B);
  const uint64_t wdims[2] = {static_cast<uint64_t>(taps) * cin, static_cast<uint64_t>(N)};
  const uint64_t wstr[1] = {static_cast<uint64_t>(taps) * cin * 2};
  const uint32_t wbox[2] = {static_cast<uint32_t>(tc::CK), static_cast<uint32_t>(p.BN)};
  if (!st) st = make_tmap(&tm_w, dt, 2, wdata, wdims, wstr, wbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  st = set_max_dynamic_smem(reinterpret_cast<const void*>(&tc::conv_tc_kernel<false>), tc::SMEM);
  if (st) return st;
  const int grid = p.num_tiles < ctx->num_sms ? p.num_tiles : ctx->num_sms;
  tc::conv_tc_kernel<false><<<grid, tc::THREADS, tc::SMEM, ctx->stream>>>(tm_hi, tm_lo, tm_w, p);
  return check_launch("conv_tc_kernel");
}

template <typename T>
static int split_planes(anima_ctx* ctx, const float* x, int h, int w, int c, long long ldx, int up, T* hi, T* lo) {
  const long long n8 = static_cast<long long>(up ? 4 : 1) * h * w * (c / 8);
  tc::split_planes_kernel<T><<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, ctx->stream>>>(x, h, w, c, ldx, up, hi,
                                                                                            lo, n8);
  return check_launch("split_planes_kernel");
}

}  // namespace vae

// The VAE's single attention (one head, d = 384, every latent pixel a token: 16384 at 1024^2) on
// the tensor cores: S = Q K^T and O = P V as bf16 two-plane GEMMs (each operand split into hi +
// lo; the B side by two calls, the second accumulating), with the fp32 scores materialised and a
// row softmax between them that writes P as planes. Taken for fp32 q/k/v and output, one head,
// no mask, batch 1, d a multiple of 64, and at least 2^20 scores (smaller ones stay on the
// CUDA-core kernel, as the text models' do).
int matmul_planes(anima_ctx* ctx, int M, int N, int K, const float* A, int lda, const void* B, const float* bias,
                  float* C, int ldc, int accumulate, bool f16) {
  if (M < 256 || K % 8 != 0 || lda % 8 != 0 || ldc != N || (reinterpret_cast<uintptr_t>(A) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(B) & 15) != 0 || (reinterpret_cast<uintptr_t>(C) & 15) != 0)
    return ANIMA_ERR_UNSUPPORTED;
  const size_t plane = static_cast<size_t>(M) * K;
  if (ctx->vae_ws_bytes < 2 * plane * sizeof(__nv_bfloat16)) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    ANIMA_CUDA(cudaStreamIsCapturing(ctx->stream, &cap));
    if (cap != cudaStreamCaptureStatusNone) return ANIMA_ERR_UNSUPPORTED;
  }
  int st = vae::grow_ws(ctx, &ctx->vae_ws, &ctx->vae_ws_bytes, 2 * plane * sizeof(__nv_bfloat16), "anima_matmul");
  if (st) return st;
  if (f16) {
    auto* hi = static_cast<__half*>(ctx->vae_ws);
    st = vae::split_planes(ctx, A, 1, M, K, lda, 0, hi, hi + plane);
  } else {
    auto* hi = static_cast<__nv_bfloat16*>(ctx->vae_ws);
    st = vae::split_planes(ctx, A, 1, M, K, lda, 0, hi, hi + plane);
  }
  if (st) return st;
  auto* hi = static_cast<uint16_t*>(ctx->vae_ws);
  return vae::tc_gemm(ctx, hi, hi + plane, 1, M, K, 1, B, N, bias, C, accumulate, f16);
}

bool attention_planes_ok(const anima_attention_args* a) {
  return a->dtype == ANIMA_F32 && a->out_dtype == ANIMA_F32 && a->heads == 1 && a->batch == 1 && a->group <= 1 &&
         !a->causal && !a->key_len && a->head_dim % 64 == 0 && a->head_dim <= 1024 &&
         static_cast<long long>(a->Lq) * a->Lk >= (1ll << 20) && a->Lk % 8 == 0 && a->ldo == a->head_dim &&
         a->ldq % 8 == 0 && a->ldk % 8 == 0 && a->ldv % 8 == 0 && a->q_off % 8 == 0 && a->k_off % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(a->q) & 15) == 0 && (reinterpret_cast<uintptr_t>(a->k) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a->out) & 15) == 0;
}

int attention_planes(anima_ctx* ctx, const anima_attention_args* a) {
  using bf = __nv_bfloat16;
  const int Lq = a->Lq, Lk = a->Lk, d = a->head_dim;
  const size_t s_bytes = static_cast<size_t>(Lq) * Lk * 4;
  const size_t p_bytes = static_cast<size_t>(Lq) * Lk * 2;  // per plane
  const size_t q_elems = static_cast<size_t>(Lq) * d, k_elems = static_cast<size_t>(Lk) * d;
  const size_t want = s_bytes + 2 * p_bytes + 2 * (q_elems + 2 * k_elems) * sizeof(bf);
  int st = vae::grow_ws(ctx, &ctx->mat_ws, &ctx->mat_ws_bytes, want, "anima_attention (wide single head)");
  if (st) return st;
  ProfScope prof(ctx, "attention.planes", 4.0 * Lq * Lk * d, 0);
  float* S = static_cast<float*>(ctx->mat_ws);
  bf* p_hi = reinterpret_cast<bf*>(reinterpret_cast<char*>(ctx->mat_ws) + s_bytes);
  bf* p_lo = p_hi + static_cast<size_t>(Lq) * Lk;
  bf* q_hi = p_lo + static_cast<size_t>(Lq) * Lk;
  bf* q_lo = q_hi + q_elems;
  bf* k_hi = q_lo + q_elems;
  bf* k_lo = k_hi + k_elems;
  bf* v_hi = k_lo + k_elems;  // V^T [d, Lk]
  bf* v_lo = v_hi + k_elems;
  const float* q = static_cast<const float*>(a->q) + a->q_off;
  const float* k = static_cast<const float*>(a->k) + a->k_off;
  const float* v = static_cast<const float*>(a->v) + a->v_off;
  st = vae::split_planes(ctx, q, 1, Lq, d, a->ldq, 0, q_hi, q_lo);
  if (!st) st = vae::split_planes(ctx, k, 1, Lk, d, a->ldk, 0, k_hi, k_lo);
  if (st) return st;
  vae::tc::transpose_split_kernel<<<dim3((Lk + 31) / 32, (d + 31) / 32), 256, 0, ctx->stream>>>(v, a->ldv, Lk, d, v_hi, v_lo);
  st = check_launch("transpose_split_kernel");
  // S = Q K^T: the queries as an image of 1 x Lq pixels with d channels, the keys as the weights
  if (!st) st = vae::tc_gemm(ctx, q_hi, q_lo, 1, Lq, d, 1, k_hi, Lk, nullptr, S, 0);
  if (!st) st = vae::tc_gemm(ctx, q_hi, q_lo, 1, Lq, d, 1, k_lo, Lk, nullptr, S, 1);
  if (st) return st;
  const float scale = a->scale > 0.f ? a->scale : 1.0f / sqrtf(static_cast<float>(d));
  vae::tc::softmax_planes_kernel<<<Lq, 256, 0, ctx->stream>>>(S, Lk, scale * 1.4426950408889634f, p_hi, p_lo);
  st = check_launch("softmax_planes_kernel");
  // O = P V: P as an image of 1 x Lq pixels with Lk channels, V^T as the weights
  float* out = static_cast<float*>(a->out);
  if (!st) st = vae::tc_gemm(ctx, p_hi, p_lo, 1, Lq, Lk, 1, v_hi, d, nullptr, out, 0);
  if (!st) st = vae::tc_gemm(ctx, p_hi, p_lo, 1, Lq, Lk, 1, v_lo, d, nullptr, out, 1);
  return st;
}

}  // namespace anima

using namespace anima;

extern "C" {

int anima_conv3x3(anima_ctx* ctx, const float* x, int h, int w, int cin, const anima_weight* W, int up, float* out,
                  int accumulate) {
  ANIMA_REQUIRE(ctx && x && W && W->data && out, "anima_conv3x3: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_REQUIRE(W->kind == ANIMA_W_BF16 && W->K == 9 * cin && W->N > 0, "anima_conv3x3: W must be bf16 [N, 9 * cin]");
  ANIMA_REQUIRE(h > 0 && w > 0 && cin > 0 && cin % 8 == 0, "anima_conv3x3: cin %d must be a positive multiple of 8", cin);
  ANIMA_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(W->data) & 15) == 0,
                "anima_conv3x3: x and W must be 16-byte aligned");
  const int H = up ? 2 * h : h, Wd = up ? 2 * w : w;
  const long long M = static_cast<long long>(H) * Wd;
  ProfScope prof(ctx, up ? "vae.conv3x3+up" : "vae.conv3x3", 2.0 * M * W->N * W->K, 0);

  // the input as two bf16 planes (upsampled here when up), in a buffer the context keeps
  const size_t plane = static_cast<size_t>(M) * cin;
  int st = vae::grow_ws(ctx, &ctx->vae_ws, &ctx->vae_ws_bytes, 2 * plane * sizeof(__nv_bfloat16), "anima_conv3x3");
  if (st) return st;
  auto* hi = static_cast<__nv_bfloat16*>(ctx->vae_ws);
  auto* lo = hi + plane;
  st = vae::split_planes(ctx, x, h, w, cin, cin, up, hi, lo);
  if (st) return st;
  return vae::tc_gemm(ctx, hi, lo, H, Wd, cin, 9, W->data, W->N, W->bias, out, accumulate);
}

int anima_channel_norm(anima_ctx* ctx, const float* x, long long rows, int C, const float* gamma, int silu, float* y) {
  ANIMA_REQUIRE(ctx && x && gamma && y && rows > 0 && C > 0, "anima_channel_norm: bad argument");
  ANIMA_ON_DEVICE(ctx);
  ProfScope prof(ctx, silu ? "vae.channel_norm+silu" : "vae.channel_norm", 0, 8.0 * rows * C);
  vae::channel_norm_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, ctx->stream>>>(x, rows, C, gamma, silu, y);
  return check_launch("channel_norm_kernel");
}

}  // extern "C"
