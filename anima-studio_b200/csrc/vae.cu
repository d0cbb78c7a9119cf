// Wan-2.1 VAE decoder operators (app/models/vae.js; math of tools/reference.py:254-295):
// NHWC 3x3 convolution as an implicit GEMM with the nearest 2x upsample of Resample fused into its
// loads, and the decoder's channel RMS norm with the SiLU that follows it.
//
// The VAE runs once per image (after the denoising loop), so these are CUDA-core kernels: fp32
// activations, bf16 weights (OHWI, as the reference's asset builder stores them), fp32 sums.
#include "internal.h"
#include "sm100.cuh"

namespace anima {
namespace vae {

constexpr int BM = 64;   // output pixels per tile
constexpr int BN = 64;   // output channels per tile
constexpr int BK = 32;   // input channels per k-step (one filter tap at a time)

// out[p, o] (+)= bias[o] + sum_{ky, kx, c} in[p + (ky - 1, kx - 1), c] * w[o, ky, kx, c], pad 1;
// with UP the input is first upsampled 2x (nearest): in_up[y, x] = in[y / 2, x / 2].
// A 256-thread CTA computes a 64-pixel x 64-channel tile, 4 x 4 per thread, from k-major tiles
// of the gathered inputs and the weights in shared memory.
template <bool UP>
__global__ void __launch_bounds__(256) conv3x3_kernel(const float* __restrict__ x, int h, int w, int cin,
                                                      const __nv_bfloat16* __restrict__ wt,
                                                      const float* __restrict__ bias, int cout, float* out,
                                                      int accumulate) {
  __shared__ __align__(16) float As[BK][BM];
  __shared__ __align__(16) float Bs[BK][BN];
  const int Ho = UP ? 2 * h : h, Wo = UP ? 2 * w : w;
  const long long M = static_cast<long long>(Ho) * Wo;
  const long long p0 = static_cast<long long>(blockIdx.x) * BM;
  const int o0 = blockIdx.y * BN;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  // the pixel this thread gathers for the A tile, and its output coordinates
  const int ap = tid & 63;
  const long long gp = p0 + ap;
  const int oy = gp < M ? static_cast<int>(gp / Wo) : 0, ox = gp < M ? static_cast<int>(gp % Wo) : 0;
  const int K = 9 * cin;
  float acc[4][4] = {};
  for (int tap = 0; tap < 9; ++tap) {
    const int iy = oy + tap / 3 - 1, ix = ox + tap % 3 - 1;  // in the (upsampled) input
    const bool inside = gp < M && iy >= 0 && iy < Ho && ix >= 0 && ix < Wo;
    const float* src = inside ? x + (static_cast<long long>(UP ? iy / 2 : iy) * w + (UP ? ix / 2 : ix)) * cin : x;
    for (int c0 = 0; c0 < cin; c0 += BK) {
      __syncthreads();
      // A: 64 pixels x 32 channels, 4 channels per load, two loads per thread
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int cc = ((tid >> 6) + 4 * r) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (inside && c0 + cc < cin) v = *reinterpret_cast<const float4*>(src + c0 + cc);
        As[cc][ap] = v.x;
        As[cc + 1][ap] = v.y;
        As[cc + 2][ap] = v.z;
        As[cc + 3][ap] = v.w;
      }
      // B: 64 output channels x 32 inputs of this tap, 8 bf16 per load
      {
        const int o = tid >> 2, j = (tid & 3) * 8;
        float bv[8] = {};
        if (o0 + o < cout && c0 + j < cin) {
          const uint4 u = *reinterpret_cast<const uint4*>(wt + static_cast<long long>(o0 + o) * K + tap * cin + c0 + j);
          const __nv_bfloat16* hv = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
          for (int i = 0; i < 8; ++i) bv[i] = __bfloat162float(hv[i]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) Bs[j + i][o] = bv[i];
      }
      __syncthreads();
#pragma unroll 8
      for (int k = 0; k < BK; ++k) {
        const float4 a = *reinterpret_cast<const float4*>(&As[k][ty * 4]);
        const float4 b = *reinterpret_cast<const float4*>(&Bs[k][tx * 4]);
        const float av[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bw[j], acc[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const long long p = p0 + ty * 4 + i;
    if (p >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int o = o0 + tx * 4 + j;
      if (o >= cout) continue;
      const float v = acc[i][j] + (bias ? bias[o] : 0.f);
      float* d = out + p * cout + o;
      *d = accumulate ? *d + v : v;
    }
  }
}

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

}  // namespace vae
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
  const long long M = static_cast<long long>(up ? 2 * h : h) * (up ? 2 * w : w);
  const dim3 grid(static_cast<unsigned>((M + vae::BM - 1) / vae::BM), (W->N + vae::BN - 1) / vae::BN);
  ProfScope prof(ctx, up ? "vae.conv3x3+up" : "vae.conv3x3", 2.0 * M * W->N * W->K, 0);
  const auto* wt = static_cast<const __nv_bfloat16*>(W->data);
  if (up)
    vae::conv3x3_kernel<true><<<grid, 256, 0, ctx->stream>>>(x, h, w, cin, wt, W->bias, W->N, out, accumulate);
  else
    vae::conv3x3_kernel<false><<<grid, 256, 0, ctx->stream>>>(x, h, w, cin, wt, W->bias, W->N, out, accumulate);
  return check_launch("conv3x3_kernel");
}

int anima_channel_norm(anima_ctx* ctx, const float* x, long long rows, int C, const float* gamma, int silu, float* y) {
  ANIMA_REQUIRE(ctx && x && gamma && y && rows > 0 && C > 0, "anima_channel_norm: bad argument");
  ANIMA_ON_DEVICE(ctx);
  ProfScope prof(ctx, silu ? "vae.channel_norm+silu" : "vae.channel_norm", 0, 8.0 * rows * C);
  vae::channel_norm_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, ctx->stream>>>(x, rows, C, gamma, silu, y);
  return check_launch("channel_norm_kernel");
}

}  // extern "C"
