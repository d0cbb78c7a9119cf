// HBM-bound row kernels: adaLN-modulated LayerNorm, the 256-point ConvRot Hadamard, per-token
// activation quantization, RMSNorm, q/k norm + RoPE, RoPE, elementwise ops, W4 decode, and the
// model glue (patchify, timestep embedding, Euler step). The reference's counterparts are the
// WGSL kernels of app/gpu/kernels.js; these are written for coalesced 16-byte accesses with warp
// shuffles instead of workgroup-memory reductions.

#include "internal.h"
#include "sm100.cuh"

namespace anima {
namespace rowops {

// ------------------------------------------------------------------ dtype helpers

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// 8 consecutive elements <-> registers (16- or 32-byte vector access).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&x)[8]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = to_f<T>(h[j]);
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&x)[8]) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(x[4], x[5], x[6], x[7]);
  } else {
    uint4 u;
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = from_f<T>(x[j]);
    *reinterpret_cast<uint4*>(p) = u;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 256-point ConvRot Hadamard of the group held by one warp, lane l holding elements 8l..8l+7:
// y = x H, H = kron(H4, H4, H4, H4) / 16 with the regular H4 = [[1,1,1,-1],[1,1,-1,1],
// [1,-1,1,1],[-1,1,1,1]] (tools/quant.py:30-38). Index i = d0 + 4 d1 + 16 d2 + 64 d3; each
// base-4 digit gets one 4-point transform, y[d] = (x0 + x1 + x2 + x3) - 2 x[3 - d].
// d0 and the low bit of d1 are within the thread; the rest of d1 is lane bit 0, d2 lane bits
// 1-2 and d3 lane bits 3-4, reached with xor shuffles.
__device__ __forceinline__ void fwht256_warp(float (&x)[8]) {
  const int lane = threadIdx.x & 31;
  // digit 0: elements j, j+1, j+2, j+3 of each half
#pragma unroll
  for (int h = 0; h < 8; h += 4) {
    const float s = x[h] + x[h + 1] + x[h + 2] + x[h + 3];
    const float a0 = x[h], a1 = x[h + 1], a2 = x[h + 2], a3 = x[h + 3];
    x[h] = s - 2.f * a3;
    x[h + 1] = s - 2.f * a2;
    x[h + 2] = s - 2.f * a1;
    x[h + 3] = s - 2.f * a0;
  }
  // digit 1: e = (j >> 2) + 2 (lane & 1); partner lane ^ 1 holds the other two values
  {
    float p[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) p[j] = __shfl_xor_sync(0xffffffffu, x[j], 1);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float s = x[j] + x[j + 4] + p[j] + p[j + 4];
      // own d = 2b + t; x[3 - d] lives in the partner at t' = 1 - t
      const float y0 = s - 2.f * p[j + 4];
      const float y1 = s - 2.f * p[j];
      x[j] = y0;
      x[j + 4] = y1;
    }
    (void)lane;
  }
  // digit 2: lanes differing in bits 1-2; x[3 - d] sits at lane ^ 6
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float a = x[j] + __shfl_xor_sync(0xffffffffu, x[j], 2);
    const float s = a + __shfl_xor_sync(0xffffffffu, a, 4);
    x[j] = s - 2.f * __shfl_xor_sync(0xffffffffu, x[j], 6);
  }
  // digit 3: lanes differing in bits 3-4; x[3 - d] sits at lane ^ 24
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float a = x[j] + __shfl_xor_sync(0xffffffffu, x[j], 8);
    const float s = a + __shfl_xor_sync(0xffffffffu, a, 16);
    x[j] = s - 2.f * __shfl_xor_sync(0xffffffffu, x[j], 24);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] *= 0.0625f;
}

// ------------------------------------------------------------------ row kernel: LN + adaLN, ConvRot, quant
// One row per warp for rows up to 1024 wide (WPR = 1), WPR = cols / 1024 warps per row beyond;
// 8 warps per CTA. Lane l holds, for each of the warp's G groups of 256 columns, the 8 consecutive
// elements 8l..8l+7 of that group, so every warp access is a contiguous 256-element segment and
// every ConvRot group lives in one warp (fwht256_warp). Reductions are warp shuffles, plus one
// shared-memory step across the WPR warps of a row.
//   LN      y = LN(x) * (1 + mod[scale_off + c]) + mod[shift_off + c]  (fp32 two-pass mean/var,
//           biased variance, eps: tools/reference.py:190-191, kernels.js:95-145)
//   act     y <- GELU(y) (the MLP's activation, applied here when the layer1 GEMM stored its
//           pre-activation)
//   rotate  y <- y H per 256 group (tools/quant.py:30-45)
//   quant   s = amax / 127; a = y * (127 / amax); hi = rne(a); lo = rne((a - hi) * 254)
//           (|a| <= 127 and |a - hi| <= 1/2, so neither needs clamping)
template <int WPR>
__device__ __forceinline__ float row_reduce(float v, float* red, bool is_max) {
  v = is_max ? warp_max(v) : warp_sum(v);
  if constexpr (WPR == 1) {
    return v;
  } else {
    const int warp = threadIdx.x >> 5;
    const int base = (warp / WPR) * WPR;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float t = red[base];
#pragma unroll
    for (int i = 1; i < WPR; ++i) t = is_max ? fmaxf(t, red[base + i]) : t + red[base + i];
    __syncthreads();
    return t;
  }
}

template <int COLS, typename TIn, typename TOut, bool LN>
__global__ void __launch_bounds__(256) rows_kernel(const TIn* __restrict__ x, int rows, int ldx,
                                                   const float* __restrict__ mod, int shift_off, int scale_off,
                                                   float eps, int rotate, TOut* y, int8_t* qhi, int8_t* qlo,
                                                   float* qscale, int qld, int act) {
  constexpr int WPR = COLS > 1024 ? COLS / 1024 : 1;  // warps per row: at most 4 groups of 256 per warp
  constexpr int G = COLS / 256 / WPR;
  constexpr int RPC = 8 / WPR;
  static_assert(G >= 1 && G <= 8 && COLS % 256 == 0, "unsupported row width");
  __shared__ float red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * RPC + warp / WPR;
  const int wr = warp % WPR;
  const bool valid = row < rows;
  const size_t r = valid ? static_cast<size_t>(row) : 0;
  float v[G][8];
  int col[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    col[g] = (wr * G + g) * 256 + 8 * lane;
    if (valid) {
      load8(x + r * ldx + col[g], v[g]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[g][j] = 0.f;
    }
  }
  if constexpr (LN) {
    float sum = 0.f;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[g][j];
    const float mean = row_reduce<WPR>(sum, red, false) / static_cast<float>(COLS);
    float sq = 0.f;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[g][j] - mean;
        sq += d * d;
      }
    const float var = row_reduce<WPR>(sq, red, false) / static_cast<float>(COLS);
    const float rstd = 1.0f / sqrtf(var + eps);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float sc[8], sh[8];
      load8(mod + scale_off + col[g], sc);
      load8(mod + shift_off + col[g], sh);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[g][j] = (v[g][j] - mean) * rstd * (1.0f + sc[j]) + sh[j];
    }
  }
  if (act == ANIMA_ACT_GELU) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < 8; ++j) v[g][j] = gelu_erf(v[g][j]);
  }
  if (rotate) {
#pragma unroll
    for (int g = 0; g < G; ++g) fwht256_warp(v[g]);
  }
  if (qhi) {
    float amax = 0.f;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[g][j]));
    amax = row_reduce<WPR>(amax, red, true);
    if (!valid) return;
    const float inv = amax > 0.f ? 127.0f / amax : 0.f;
    if (wr == 0 && lane == 0) qscale[r] = amax > 0.f ? amax / 127.0f : 1.0f;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      uint32_t h2[2], l2[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        // round to nearest even through the 1.5 * 2^23 magic number (|a| <= 127, |lo| <= 127):
        // integer values come straight out of the float's mantissa, no conversion unit needed
        int hv[4], lv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = v[g][4 * half + j] * inv;
          const float t = a + 12582912.0f;
          hv[j] = __float_as_int(t) - 0x4B400000;
          const float rem = a - (t - 12582912.0f);
          lv[j] = __float_as_int(fmaf(rem, 254.0f, 12582912.0f)) - 0x4B400000;
        }
        h2[half] = __byte_perm(__byte_perm(hv[0], hv[1], 0x0040), __byte_perm(hv[2], hv[3], 0x0040), 0x5410);
        l2[half] = __byte_perm(__byte_perm(lv[0], lv[1], 0x0040), __byte_perm(lv[2], lv[3], 0x0040), 0x5410);
      }
      *reinterpret_cast<uint2*>(qhi + r * qld + col[g]) = make_uint2(h2[0], h2[1]);
      if (qlo) *reinterpret_cast<uint2*>(qlo + r * qld + col[g]) = make_uint2(l2[0], l2[1]);
    }
  } else if (valid) {
#pragma unroll
    for (int g = 0; g < G; ++g) store8(y + r * COLS + col[g], v[g]);
  }
}

// ------------------------------------------------------------------ RMSNorm (warp per row)
template <typename TIn, typename TOut>
__global__ void rmsnorm_kernel(const TIn* __restrict__ x, int rows, int cols, const float* __restrict__ w, float eps,
                               TOut* y) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const TIn* xr = x + static_cast<size_t>(row) * cols;
  float ss = 0.f;
  for (int c = lane; c < cols; c += 32) {
    const float t = to_f<TIn>(xr[c]);
    ss += t * t;
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
  TOut* yr = y + static_cast<size_t>(row) * cols;
  for (int c = lane; c < cols; c += 32) yr[c] = from_f<TOut>(to_f<TIn>(xr[c]) * r * w[c]);
}

// ------------------------------------------------------------------ q/k RMSNorm + RoPE, RoPE
// One warp per (token, q-or-k head) of a fused qkv row; lane holds dims lane, lane+32, lane+64,
// lane+96, so both RoPE pairs (i, i+64) are in-thread (kernels.js:301-334 semantics).
template <typename T>
__global__ void qk_norm_rope_kernel(T* qkv, int L, int H, int D, int ld, const float* __restrict__ qn,
                                    const float* __restrict__ kn, const float* __restrict__ rope, int rope_rows,
                                    float eps) {
  const int warps = blockDim.x >> 5;
  const long long id = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (id >= static_cast<long long>(L) * 2 * H) return;
  const int l = static_cast<int>(id / (2 * H));
  const int h = static_cast<int>(id % (2 * H));
  T* p = qkv + static_cast<size_t>(l) * ld + static_cast<size_t>(h) * D;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = to_f<T>(p[lane + 32 * i]);
  float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
  const float* w = h < H ? qn : kn;
  const int tok = l % rope_rows;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int d = lane + 32 * i;
    const float y1 = v[i] * r * w[d];
    const float y2 = v[i + 2] * r * w[d + 64];
    const float c = rope[static_cast<size_t>(tok) * 64 + d];
    const float s = rope[static_cast<size_t>(rope_rows) * 64 + static_cast<size_t>(tok) * 64 + d];
    p[d] = from_f<T>(y1 * c - y2 * s);
    p[d + 64] = from_f<T>(y2 * c + y1 * s);
  }
}

template <typename T>
__global__ void rope_kernel(T* x, int L, int H, int D, int row_stride, int col_off, const float* __restrict__ rope,
                            int rope_rows) {
  const int half = D / 2;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(L) * H * half) return;
  const int i = static_cast<int>(idx % half);
  const int h = static_cast<int>((idx / half) % H);
  const int l = static_cast<int>(idx / (static_cast<long long>(half) * H));
  T* p = x + static_cast<size_t>(l) * row_stride + col_off + static_cast<size_t>(h) * D;
  const int tok = l % rope_rows;
  const float c = rope[static_cast<size_t>(tok) * half + i];
  const float s = rope[static_cast<size_t>(rope_rows) * half + static_cast<size_t>(tok) * half + i];
  const float x1 = to_f<T>(p[i]), x2 = to_f<T>(p[i + half]);
  p[i] = from_f<T>(x1 * c - x2 * s);
  p[i + half] = from_f<T>(x2 * c + x1 * s);
}

// ------------------------------------------------------------------ elementwise
__global__ void elementwise_kernel(int op, const float* __restrict__ a, const float* __restrict__ b, float* y,
                                   long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = a[i];
  float r;
  switch (op) {
    case 0: r = x; break;
    case 1: r = x + b[i]; break;
    case 2: r = silu_f(x); break;
    default: r = silu_f(x) * b[i]; break;
  }
  y[i] = r;
}

// ------------------------------------------------------------------ W4 decode (bit-exact)
// fp8 e4m3fn -> fp32 exactly (sign, 4-bit exponent bias 7, 3-bit mantissa, subnormals, NaN at
// 0x7f/0xff as torch decodes them).
__device__ __forceinline__ float fp8_e4m3fn(uint32_t b) {
  const uint32_t e = (b >> 3) & 15u, m = b & 7u;
  float v;
  if (e == 0)
    v = static_cast<float>(m) * 0.001953125f;
  else if (e == 15 && m == 7)
    v = __int_as_float(0x7fc00000);
  else
    v = __int_as_float(static_cast<int>(((e + 120u) << 23) | (m << 20)));
  return (b & 128u) ? -v : v;
}

// One thread per packed byte (two codes). grid value = clamp(rne(cb[code] * fp8(s_rel)), +-127).
__global__ void unpack_w4_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ s_rel,
                                 const float* __restrict__ cb, long long n_bytes, int K, int8_t* out) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_bytes) return;
  const uint32_t b = packed[i];
  const long long k0 = 2 * i;  // flat index of the even code
  const long long row = k0 / K;
  const long long kk = k0 % K;
  const float s = fp8_e4m3fn(s_rel[row * (K / 16) + kk / 16]);
  const float p0 = __fmul_rn(cb[b & 15u], s);
  const float p1 = __fmul_rn(cb[(b >> 4) & 15u], s);
  out[k0] = static_cast<int8_t>(fminf(fmaxf(rintf(p0), -127.f), 127.f));
  out[k0 + 1] = static_cast<int8_t>(fminf(fmaxf(rintf(p1), -127.f), 127.f));
}

// ------------------------------------------------------------------ model glue
__global__ void patchify_kernel(const float* __restrict__ lat, int B, int h, int w, float* patches) {
  const int Hp = h / 2, Wp = w / 2;
  const long long n = static_cast<long long>(B) * Hp * Wp * 68;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int f = static_cast<int>(i % 68);
  const long long t = i / 68;
  const int x = static_cast<int>(t % Wp), y = static_cast<int>((t / Wp) % Hp);
  const int b = static_cast<int>(t / (static_cast<long long>(Wp) * Hp));
  const int c = f / 4, mm = (f / 2) % 2, nn = f % 2;
  patches[i] = c < 16 ? lat[(static_cast<size_t>(b) * 16 + c) * h * w + static_cast<size_t>(2 * y + mm) * w + 2 * x + nn]
                      : 0.0f;
}

__global__ void unpatchify_kernel(const float* __restrict__ o, int B, int h, int w, float* lat) {
  const long long n = static_cast<long long>(B) * 16 * h * w;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int xx = static_cast<int>(i % w), yy = static_cast<int>((i / w) % h);
  const int c = static_cast<int>((i / (static_cast<long long>(w) * h)) % 16);
  const int b = static_cast<int>(i / (16LL * w * h));
  const int Wp = w / 2, Hp = h / 2;
  const int p1 = yy % 2, p2 = xx % 2;
  const size_t tok = static_cast<size_t>(b) * Hp * Wp + static_cast<size_t>(yy / 2) * Wp + xx / 2;
  lat[i] = o[tok * 64 + p1 * 32 + p2 * 16 + c];
}

// temb[b] = cat(cos(sigma f), sin(sigma f)), f_i = exp(-ln(1e4) i / 1024), all in fp32.
__global__ void timestep_embedding_kernel(const float* __restrict__ sigmas, int B, float* temb) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * 1024) return;
  const int b = i / 1024, k = i % 1024;
  const float f = expf(__fmul_rn(-9.210340371976184f, static_cast<float>(k) / 1024.0f));
  const float a = __fmul_rn(sigmas[b], f);
  temb[static_cast<size_t>(b) * 2048 + k] = cosf(a);
  temb[static_cast<size_t>(b) * 2048 + 1024 + k] = sinf(a);
}

__global__ void euler_kernel(float* x, const float* __restrict__ v, const float* __restrict__ vu, float cfg, float sigma,
                             float sigma_next, long long n, float* den_out) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float vel = v[i];
  if (vu) vel = vu[i] + (vel - vu[i]) * cfg;
  const float xi = x[i];
  const float den = xi - vel * sigma;
  if (den_out) den_out[i] = den;
  x[i] = sigma_next == 0.0f ? den : xi + (xi - den) / sigma * (sigma_next - sigma);
}

// ------------------------------------------------------------------ SIMT GEMM for bf16 / f32 weights
// C[m, n] = act(alpha * sum_k A[m, k] B[n, k] (+ bias[n])), stored or accumulated (C += gate * y).
// 64 x 64 tiles, 256 threads, 4 x 4 outputs per thread, K tiles of 16 through shared memory.
// QA: A is given as quantized rows, A[m, k] = qs[m] * (qhi[m, k] + qlo[m, k] / 254).
template <typename TB, bool QA = false>
__global__ void __launch_bounds__(256) simt_gemm_kernel(int M, int N, int K, float alpha, const float* __restrict__ A,
                                                        int lda, const TB* __restrict__ B, int ldb,
                                                        const float* __restrict__ bias, int act, float* C, int ldc,
                                                        int accumulate, const float* __restrict__ gate, int gate_off,
                                                        const int8_t* __restrict__ qhi = nullptr,
                                                        const int8_t* __restrict__ qlo = nullptr,
                                                        const float* __restrict__ qs = nullptr) {
  __shared__ float As[16][65];
  __shared__ float Bs[16][65];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int r = i / 16, kk = i % 16;
      const int m = m0 + r, n = n0 + r, k = k0 + kk;
      if constexpr (QA) {
        float a = 0.f;
        if (m < M && k < K) {
          const size_t idx = static_cast<size_t>(m) * lda + k;
          a = static_cast<float>(qhi[idx]);
          if (qlo) a += static_cast<float>(qlo[idx]) * (1.0f / 254.0f);
          a *= qs[m];
        }
        As[kk][r] = a;
      } else {
        As[kk][r] = (m < M && k < K) ? A[static_cast<size_t>(m) * lda + k] : 0.f;
      }
      Bs[kk][r] = (n < N && k < K) ? to_f<TB>(B[static_cast<size_t>(n) * ldb + k]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[kk][ty * 4 + i];
        b[i] = Bs[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float r = acc[i][j] * alpha;
      if (bias) r += bias[n];
      if (act == ANIMA_ACT_GELU) r = gelu_erf(r);
      if (act == ANIMA_ACT_SILU) r = silu_f(r);
      float* c = C + static_cast<size_t>(m) * ldc + n;
      if (accumulate)
        *c += (gate ? gate[gate_off + n] : 1.0f) * r;
      else
        *c = r;
    }
  }
}

template <typename TIn, typename TOut, bool LN>
int launch_rows(anima_ctx* ctx, const TIn* x, int rows, int cols, int ldx, const float* mod, int so, int sco,
                float eps, int rotate, TOut* y, const anima_qact* q, int act = ANIMA_ACT_NONE) {
  int8_t* hi = q ? q->hi : nullptr;
  int8_t* lo = q ? q->lo : nullptr;
  float* sc = q ? q->scale : nullptr;
  const int qld = q ? q->ld : 0;
#define ROWS_CASE(C)                                                                                             \
  case C: {                                                                                                      \
    constexpr int rpc = 8 / (C > 1024 ? C / 1024 : 1);                                                          \
    rows_kernel<C, TIn, TOut, LN><<<(rows + rpc - 1) / rpc, 256, 0, ctx->stream>>>(x, rows, ldx, mod, so, sco,   \
                                                                                  eps, rotate, y, hi, lo, sc, qld, act); \
    break;                                                                                                       \
  }
  switch (cols) {
    ROWS_CASE(256)
    ROWS_CASE(512)
    ROWS_CASE(1024)
    ROWS_CASE(2048)
    ROWS_CASE(4096)
    ROWS_CASE(8192)
    default:
      return set_error(ANIMA_ERR_UNSUPPORTED, "row kernel: cols=%d (supported: 256, 512, 1024, 2048, 4096, 8192)", cols);
  }
#undef ROWS_CASE
  return check_launch("rows_kernel");
}

template <typename TOut>
int launch_ln(anima_ctx* ctx, const float* x, int rows, int cols, const float* mod, int so, int sco, float eps,
              int rotate, TOut* y, const anima_qact* q) {
  return launch_rows<float, TOut, true>(ctx, x, rows, cols, cols, mod, so, sco, eps, rotate, y, q);
}

template <typename TIn, typename TOut>
int launch_rot(anima_ctx* ctx, const TIn* x, int rows, int cols, int ldx, int rotate, TOut* y, const anima_qact* q,
               int act = ANIMA_ACT_NONE) {
  return launch_rows<TIn, TOut, false>(ctx, x, rows, cols, ldx, nullptr, 0, 0, 0.f, rotate, y, q, act);
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace rowops
}  // namespace anima

using namespace anima;
using namespace anima::rowops;

static int grid1(long long n, int block) { return static_cast<int>((n + block - 1) / block); }

static int check_qact(const anima_qact* q, int rows, int cols, const char* who) {
  ANIMA_REQUIRE(q && q->hi && q->scale, "%s: output activation is incomplete", who);
  ANIMA_REQUIRE(q->rows == rows && q->cols == cols, "%s: output activation is [%d, %d], expected [%d, %d]", who,
                q->rows, q->cols, rows, cols);
  ANIMA_REQUIRE(q->ld >= cols && q->ld % 16 == 0 && al16(q->hi) && (!q->lo || al16(q->lo)),
                "%s: output activation ld/alignment invalid", who);
  return ANIMA_OK;
}

extern "C" {

int anima_layernorm_mod(anima_ctx* ctx, const float* x, int rows, int cols, const float* mod, int shift_off,
                        int scale_off, float eps, int rotate, void* out, int out_dtype) {
  ANIMA_REQUIRE(ctx && x && mod && out, "anima_layernorm_mod: NULL argument");
  ANIMA_REQUIRE(rows > 0, "anima_layernorm_mod: rows=%d", rows);
  ANIMA_REQUIRE(al16(x) && al16(out) && shift_off % 4 == 0 && scale_off % 4 == 0 && al16(mod),
                "anima_layernorm_mod: pointers/offsets must be 16-byte aligned");
  ProfScope prof(ctx, rotate ? "layernorm_mod+rot" : "layernorm_mod", 0, rows * (double)cols * 8);
  switch (out_dtype) {
    case ANIMA_F32: return launch_ln<float>(ctx, x, rows, cols, mod, shift_off, scale_off, eps, rotate, (float*)out, nullptr);
    case ANIMA_BF16: return launch_ln<__nv_bfloat16>(ctx, x, rows, cols, mod, shift_off, scale_off, eps, rotate, (__nv_bfloat16*)out, nullptr);
    case ANIMA_F16: return launch_ln<__half>(ctx, x, rows, cols, mod, shift_off, scale_off, eps, rotate, (__half*)out, nullptr);
  }
  return set_error(ANIMA_ERR_ARG, "anima_layernorm_mod: out_dtype %d", out_dtype);
}

int anima_layernorm_mod_quant(anima_ctx* ctx, const float* x, int rows, int cols, const float* mod, int shift_off,
                              int scale_off, float eps, const anima_qact* out) {
  ANIMA_REQUIRE(ctx && x && mod, "anima_layernorm_mod_quant: NULL argument");
  ANIMA_REQUIRE(rows > 0, "anima_layernorm_mod_quant: rows=%d", rows);
  int st = check_qact(out, rows, cols, "anima_layernorm_mod_quant");
  if (st) return st;
  ANIMA_REQUIRE(al16(x) && shift_off % 4 == 0 && scale_off % 4 == 0 && al16(mod),
                "anima_layernorm_mod_quant: pointers/offsets must be 16-byte aligned");
  ProfScope prof(ctx, "layernorm_mod+rot+quant", 0, rows * (double)cols * (4 + (out->lo ? 2 : 1)));
  return launch_ln<float>(ctx, x, rows, cols, mod, shift_off, scale_off, eps, 1, nullptr, out);
}

int anima_rotate(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, int ldx, void* y, int out_dtype) {
  ANIMA_REQUIRE(ctx && x && y, "anima_rotate: NULL argument");
  ANIMA_REQUIRE(rows > 0 && ldx >= cols && al16(x) && al16(y), "anima_rotate: bad shape or alignment");
  ANIMA_REQUIRE(in_dtype == ANIMA_F32 && out_dtype == ANIMA_F32, "anima_rotate: only fp32 in/out (use anima_rotate_quant)");
  ProfScope prof(ctx, "hadamard", 0, rows * (double)cols * 8);
  return launch_rot<float, float>(ctx, (const float*)x, rows, cols, ldx, 1, (float*)y, nullptr);
}

static int rot_quant(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, int ldx, const anima_qact* out,
                     int rotate, const char* who, int act = ANIMA_ACT_NONE) {
  ANIMA_REQUIRE(ctx && x, "%s: NULL argument", who);
  ANIMA_REQUIRE(rows > 0 && ldx >= cols && al16(x), "%s: bad shape or alignment", who);
  int st = check_qact(out, rows, cols, who);
  if (st) return st;
  const int esz = in_dtype == ANIMA_F32 ? 4 : 2;
  ANIMA_REQUIRE((static_cast<long long>(ldx) * esz) % 16 == 0, "%s: ldx must give 16-byte aligned rows", who);
  ANIMA_REQUIRE(act == ANIMA_ACT_NONE || act == ANIMA_ACT_GELU, "%s: act %d (none or gelu)", who, act);
  ProfScope prof(ctx, act ? "gelu+hadamard+quant" : rotate ? "hadamard+quant" : "quant", 0,
                 rows * (double)cols * (esz + (out->lo ? 2 : 1)));
  switch (in_dtype) {
    case ANIMA_F32: return launch_rot<float, float>(ctx, (const float*)x, rows, cols, ldx, rotate, nullptr, out, act);
    case ANIMA_BF16: return launch_rot<__nv_bfloat16, float>(ctx, (const __nv_bfloat16*)x, rows, cols, ldx, rotate, nullptr, out, act);
    case ANIMA_F16: return launch_rot<__half, float>(ctx, (const __half*)x, rows, cols, ldx, rotate, nullptr, out, act);
  }
  return set_error(ANIMA_ERR_ARG, "%s: in_dtype %d", who, in_dtype);
}

int anima_rotate_quant(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, int ldx, const anima_qact* out) {
  return rot_quant(ctx, x, in_dtype, rows, cols, ldx, out, 1, "anima_rotate_quant");
}

int anima_act_rotate_quant(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, int ldx, int act,
                           const anima_qact* out) {
  return rot_quant(ctx, x, in_dtype, rows, cols, ldx, out, 1, "anima_act_rotate_quant", act);
}

int anima_quant_rows(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, int ldx, const anima_qact* out) {
  return rot_quant(ctx, x, in_dtype, rows, cols, ldx, out, 0, "anima_quant_rows");
}

int anima_rmsnorm(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, const float* w, float eps, void* y,
                  int out_dtype) {
  ANIMA_REQUIRE(ctx && x && w && y && rows > 0 && cols > 0, "anima_rmsnorm: bad argument");
  ProfScope prof(ctx, "rmsnorm", 0, 8.0 * rows * cols);
  const int grid = grid1(rows, 8);
#define RMS(TI, TO) rmsnorm_kernel<TI, TO><<<grid, 256, 0, ctx->stream>>>((const TI*)x, rows, cols, w, eps, (TO*)y)
  if (in_dtype == ANIMA_F32 && out_dtype == ANIMA_F32) RMS(float, float);
  else if (in_dtype == ANIMA_F32 && out_dtype == ANIMA_BF16) RMS(float, __nv_bfloat16);
  else if (in_dtype == ANIMA_F32 && out_dtype == ANIMA_F16) RMS(float, __half);
  else if (in_dtype == ANIMA_BF16 && out_dtype == ANIMA_BF16) RMS(__nv_bfloat16, __nv_bfloat16);
  else if (in_dtype == ANIMA_F16 && out_dtype == ANIMA_F16) RMS(__half, __half);
  else return set_error(ANIMA_ERR_UNSUPPORTED, "anima_rmsnorm: dtype pair %d -> %d", in_dtype, out_dtype);
#undef RMS
  return check_launch("rmsnorm_kernel");
}

int anima_qk_norm_rope(anima_ctx* ctx, void* qkv, int dtype, int L, int H, int D, int ld, const float* qn,
                       const float* kn, const float* rope, int rope_rows, float eps) {
  ANIMA_REQUIRE(ctx && qkv && qn && kn && rope && L > 0 && H > 0 && rope_rows > 0, "anima_qk_norm_rope: bad argument");
  ANIMA_REQUIRE(D == 128, "anima_qk_norm_rope: head dim %d (only 128)", D);
  ProfScope prof(ctx, "qk_norm_rope", 0, 2.0 * L * 2 * H * D * (dtype == ANIMA_F32 ? 4 : 2));
  const long long n = static_cast<long long>(L) * 2 * H;
  const int grid = grid1(n, 8);
  if (dtype == ANIMA_F32) qk_norm_rope_kernel<float><<<grid, 256, 0, ctx->stream>>>((float*)qkv, L, H, D, ld, qn, kn, rope, rope_rows, eps);
  else if (dtype == ANIMA_BF16) qk_norm_rope_kernel<__nv_bfloat16><<<grid, 256, 0, ctx->stream>>>((__nv_bfloat16*)qkv, L, H, D, ld, qn, kn, rope, rope_rows, eps);
  else if (dtype == ANIMA_F16) qk_norm_rope_kernel<__half><<<grid, 256, 0, ctx->stream>>>((__half*)qkv, L, H, D, ld, qn, kn, rope, rope_rows, eps);
  else return set_error(ANIMA_ERR_ARG, "anima_qk_norm_rope: dtype %d", dtype);
  return check_launch("qk_norm_rope_kernel");
}

int anima_rope(anima_ctx* ctx, void* x, int dtype, int L, int H, int D, int row_stride, int col_off, const float* rope,
               int rope_rows) {
  ANIMA_REQUIRE(ctx && x && rope && L > 0 && H > 0 && D > 0 && D % 2 == 0 && rope_rows > 0, "anima_rope: bad argument");
  const long long n = static_cast<long long>(L) * H * (D / 2);
  ProfScope prof(ctx, "rope", 0, 2.0 * n * 2 * (dtype == ANIMA_F32 ? 4 : 2));
  if (dtype == ANIMA_F32) rope_kernel<float><<<grid1(n, 256), 256, 0, ctx->stream>>>((float*)x, L, H, D, row_stride, col_off, rope, rope_rows);
  else if (dtype == ANIMA_BF16) rope_kernel<__nv_bfloat16><<<grid1(n, 256), 256, 0, ctx->stream>>>((__nv_bfloat16*)x, L, H, D, row_stride, col_off, rope, rope_rows);
  else if (dtype == ANIMA_F16) rope_kernel<__half><<<grid1(n, 256), 256, 0, ctx->stream>>>((__half*)x, L, H, D, row_stride, col_off, rope, rope_rows);
  else return set_error(ANIMA_ERR_ARG, "anima_rope: dtype %d", dtype);
  return check_launch("rope_kernel");
}

int anima_elementwise(anima_ctx* ctx, int op, const float* a, const float* b, float* y, long long n) {
  ANIMA_REQUIRE(ctx && a && y && n >= 0 && op >= 0 && op <= 3, "anima_elementwise: bad argument");
  ANIMA_REQUIRE(!(op == 1 || op == 3) || b, "anima_elementwise: binary op needs b");
  if (n == 0) return ANIMA_OK;
  elementwise_kernel<<<grid1(n, 256), 256, 0, ctx->stream>>>(op, a, b, y, n);
  return check_launch("elementwise_kernel");
}

int anima_unpack_w4(anima_ctx* ctx, const uint8_t* packed, const uint8_t* s_rel, const float* codebook, int N, int K,
                    int8_t* out) {
  ANIMA_REQUIRE(ctx && packed && s_rel && codebook && out, "anima_unpack_w4: NULL argument");
  ANIMA_REQUIRE(N > 0 && K > 0 && K % 16 == 0, "anima_unpack_w4: K=%d must be a positive multiple of 16", K);
  const long long nb = static_cast<long long>(N) * K / 2;
  ProfScope prof(ctx, "unpack_w4", 0, nb * 3.0);
  unpack_w4_kernel<<<grid1(nb, 256), 256, 0, ctx->stream>>>(packed, s_rel, codebook, nb, K, out);
  return check_launch("unpack_w4_kernel");
}

int anima_matmul(anima_ctx* ctx, int M, int N, int K, float alpha, const float* A, int lda, const anima_weight* B,
                 int act, float* C, int ldc, int accumulate, const float* gate, int gate_off) {
  ANIMA_REQUIRE(ctx && A && B && B->data && C, "anima_matmul: NULL argument");
  ANIMA_REQUIRE(M > 0 && N > 0 && K > 0 && lda >= K && ldc >= N, "anima_matmul: bad shape");
  ANIMA_REQUIRE(B->kind == ANIMA_W_BF16 || B->kind == ANIMA_W_F32, "anima_matmul: weight kind %d (bf16 or f32 only)",
                B->kind);
  ProfScope prof(ctx, B->kind == ANIMA_W_BF16 ? "gemm.bf16" : "gemm.f32", 2.0 * M * N * K, 0);
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  if (B->kind == ANIMA_W_BF16)
    simt_gemm_kernel<__nv_bfloat16><<<grid, 256, 0, ctx->stream>>>(M, N, K, alpha, A, lda,
                                                                   (const __nv_bfloat16*)B->data, K, B->bias, act, C,
                                                                   ldc, accumulate, gate, gate_off);
  else
    simt_gemm_kernel<float><<<grid, 256, 0, ctx->stream>>>(M, N, K, alpha, A, lda, (const float*)B->data, K, B->bias,
                                                           act, C, ldc, accumulate, gate, gate_off);
  return check_launch("simt_gemm_kernel");
}

int anima_lora_down(anima_ctx* ctx, const anima_qact* x, const float* A, int r, float* T, int ldt) {
  ANIMA_REQUIRE(ctx && x && x->hi && x->scale && A && T && r > 0 && ldt >= r, "anima_lora_down: bad argument");
  ProfScope prof(ctx, "lora.down", 2.0 * x->rows * r * x->cols, 0);
  dim3 grid((r + 63) / 64, (x->rows + 63) / 64);
  simt_gemm_kernel<float, true><<<grid, 256, 0, ctx->stream>>>(x->rows, r, x->cols, 1.0f, nullptr, x->ld, A, x->cols,
                                                                nullptr, 0, T, ldt, 0, nullptr, 0, x->hi, x->lo,
                                                                x->scale);
  return check_launch("simt_gemm_kernel<lora_down>");
}

int anima_patchify(anima_ctx* ctx, const float* latent, int B, int h, int w, float* patches) {
  ANIMA_REQUIRE(ctx && latent && patches && B > 0 && h > 0 && w > 0 && h % 2 == 0 && w % 2 == 0, "anima_patchify: bad argument");
  const long long n = static_cast<long long>(B) * (h / 2) * (w / 2) * 68;
  patchify_kernel<<<grid1(n, 256), 256, 0, ctx->stream>>>(latent, B, h, w, patches);
  return check_launch("patchify_kernel");
}

int anima_unpatchify(anima_ctx* ctx, const float* o, int B, int h, int w, float* latent) {
  ANIMA_REQUIRE(ctx && o && latent && B > 0 && h > 0 && w > 0 && h % 2 == 0 && w % 2 == 0, "anima_unpatchify: bad argument");
  const long long n = static_cast<long long>(B) * 16 * h * w;
  unpatchify_kernel<<<grid1(n, 256), 256, 0, ctx->stream>>>(o, B, h, w, latent);
  return check_launch("unpatchify_kernel");
}

int anima_timestep_embedding(anima_ctx* ctx, const float* sigmas, int B, float* temb) {
  ANIMA_REQUIRE(ctx && sigmas && temb && B > 0, "anima_timestep_embedding: bad argument");
  timestep_embedding_kernel<<<grid1(B * 1024LL, 256), 256, 0, ctx->stream>>>(sigmas, B, temb);
  return check_launch("timestep_embedding_kernel");
}

int anima_euler_step(anima_ctx* ctx, float* x, const float* v, const float* v_uncond, float cfg, float sigma,
                     float sigma_next, long long n, float* den_out) {
  ANIMA_REQUIRE(ctx && x && v && n > 0 && sigma > 0.f, "anima_euler_step: bad argument");
  euler_kernel<<<grid1(n, 256), 256, 0, ctx->stream>>>(x, v, v_uncond, cfg, sigma, sigma_next, n, den_out);
  return check_launch("euler_kernel");
}

}  // extern "C"
