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

// ------------------------------------------------------------------ packed fp32 pairs
// The row kernels keep their data as float2 pairs of neighbouring elements so the bulk of the
// arithmetic uses the paired fp32 instructions (f2 helpers in sm100.cuh).
//
// Lane order: a half-warp holds one group of 256 elements, lane t (0..15) the 16 elements
// 4t + 64k + e (k, e = 0..3) as register a = e + 4k, i.e. pairs P[2k] = (e 0, 1), P[2k+1] =
// (e 2, 3). Each k is one 16-byte (fp32) or 8-byte (16-bit) access, and the 16 lanes of a
// half-warp read 256 (fp32) or 128 (16-bit) contiguous bytes per access, so every sector an
// access touches is fully used. p points at element 4t of the lane's group.

template <typename T>
__device__ __forceinline__ f2 to_f2(uint32_t w) {
  if constexpr (std::is_same<T, __half>::value)
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  else
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

template <typename T>
__device__ __forceinline__ uint32_t from_f2(f2 v) {
  if constexpr (std::is_same<T, __half>::value) {
    const __half2 h = __floats2half2_rn(v.x, v.y);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

template <typename T>
__device__ __forceinline__ void load_lane16(const T* p, f2 (&x)[8]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if constexpr (sizeof(T) == 4) {
      const float4 a = *reinterpret_cast<const float4*>(p + 64 * k);
      x[2 * k] = make_float2(a.x, a.y);
      x[2 * k + 1] = make_float2(a.z, a.w);
    } else {
      const uint2 u = *reinterpret_cast<const uint2*>(p + 64 * k);
      x[2 * k] = to_f2<T>(u.x);
      x[2 * k + 1] = to_f2<T>(u.y);
    }
  }
}

template <typename T>
__device__ __forceinline__ void store_lane16(T* p, const f2 (&x)[8]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if constexpr (sizeof(T) == 4)
      *reinterpret_cast<float4*>(p + 64 * k) = make_float4(x[2 * k].x, x[2 * k].y, x[2 * k + 1].x, x[2 * k + 1].y);
    else
      *reinterpret_cast<uint2*>(p + 64 * k) = make_uint2(from_f2<T>(x[2 * k]), from_f2<T>(x[2 * k + 1]));
  }
}

// ------------------------------------------------------------------ ConvRot Hadamard (256-point)
// y = x H per group of 256, H = kron(H4, H4, H4, H4) / 16 with the regular
// H4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]] (tools/quant.py:30-38). Within a group,
// element i = d0 + 4 d1 + 16 d2 + 64 d3 (base-4 digits, d3 the outermost kron factor).
//
// With D = diag(1,1,1,-1), D H4 D is the Sylvester (Walsh) matrix with rows 1 and 2 swapped, so
// H4 = D W4 P D per digit and, for the whole group,
//     y[j] = sigma(j) * WHT(sigma * x)[swap(j)] / 16
// where sigma(i) = (-1)^(number of digits equal to 3), WHT is the natural-order Walsh-Hadamard
// transform over the 8 index bits (radix-2 butterflies) and swap() exchanges the two bits of
// every digit. sigma on the input is folded into the first butterfly stage, swap() into the
// shared-memory addressing, sigma on the output into the caller's per-element multiplier.
//
// In the lane order of load_lane16, register a = e + 4k of lane t holds element (a & 3) + 4t +
// 64 (a >> 2): the register index is the digit pair (d0, d3) and the lane the pair (d1, d2), so
// sigma and swap() split into a register part and a lane part (sgn4 and swap4 below). The
// transform runs the register bits (d0, d3) first, transposes the 16 x 16 tile through shared
// memory (lane c then holds register index c of lanes b = 0..15, pairs (b, b+1)), runs the lane
// bits (d1, d2), and transposes back with swap() applied, leaving every lane with the output
// positions of its input positions, up to sigma and 1/16.

// sigma over a 4-bit index (two base-4 digits)
__host__ __device__ constexpr float sgn4(int a) { return ((a & 3) == 3) != ((a >> 2) == 3) ? -1.f : 1.f; }
__host__ __device__ constexpr int swap4(int a) { return ((a & 5) << 1) | ((a >> 1) & 5); }

// natural-order WHT over 4 bits held as 8 pairs, with sigma applied to the input
__device__ __forceinline__ void wht16(f2 (&P)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // bit 0, within the pair
    const float p = sgn4(2 * j) < 0 ? -P[j].x : P[j].x;
    const float q = sgn4(2 * j + 1) < 0 ? -P[j].y : P[j].y;
    P[j] = make_float2(p + q, p - q);
  }
#pragma unroll
  for (int m = 1; m < 8; m <<= 1)  // bits 1-3, across pairs
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (!(j & m)) {
        const f2 a = P[j], b = P[j | m];
        P[j] = add2(a, b);
        P[j | m] = sub2(a, b);
      }
}

// One 16 x 16 fp32 tile per half-warp, row stride 20 words. The second half-warp's tile starts 336
// words (16 mod 32) after the first, so a column access by the whole warp touches each bank once;
// the 16-byte row accesses are conflict-free because 20 t mod 32 differs for any 8 consecutive t.
constexpr int kTileStride = 20;
constexpr int kTileHalf = 336;
constexpr int kTileWords = kTileHalf + 16 * kTileStride;  // per warp

// V[p]: lane t's 16 elements of a group (lane order of load_lane16). Transforms V[p0 .. p0 + NP - 1]
// in place (unscaled, without the output sigma; lane t keeps the same 16 positions), NP groups per
// half-warp at once in NP tiles kTileWords apart (tb: the first), so the shared-memory round trips
// of the NP transposes overlap.
template <int NP, int NV>
__device__ __forceinline__ void hadamard256_n(float* tb, int t, f2 (&V)[NV][8], int p0) {
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    f2 (&P)[8] = V[p0 + i];
    float* b = tb + i * kTileWords;
    wht16(P);  // register bits (d0, d3)
#pragma unroll
    for (int k = 0; k < 4; ++k)
      *reinterpret_cast<float4*>(b + t * kTileStride + 4 * k) = make_float4(P[2 * k].x, P[2 * k].y, P[2 * k + 1].x, P[2 * k + 1].y);
  }
  __syncwarp();
  const int ct = swap4(t);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    f2 (&P)[8] = V[p0 + i];
    const float* b = tb + i * kTileWords;
#pragma unroll
    for (int j = 0; j < 8; ++j) P[j] = make_float2(b[(2 * j) * kTileStride + t], b[(2 * j + 1) * kTileStride + t]);
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    f2 (&P)[8] = V[p0 + i];
    float* b = tb + i * kTileWords;
    wht16(P);  // lane bits (d1, d2); P[j] = register t of lanes 2j, 2j + 1
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      b[swap4(2 * j) * kTileStride + ct] = P[j].x;
      b[swap4(2 * j + 1) * kTileStride + ct] = P[j].y;
    }
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    f2 (&P)[8] = V[p0 + i];
    const float* b = tb + i * kTileWords;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 q = *reinterpret_cast<const float4*>(b + t * kTileStride + 4 * k);
      P[2 * k] = make_float2(q.x, q.y);
      P[2 * k + 1] = make_float2(q.z, q.w);
    }
  }
  __syncwarp();
}

// Per-pair multipliers that apply the output sigma: sigma of register a of lane t is
// sgn4(t) sgn4(a), and over the pair (a, a + 1) = (2j, 2j + 1) sgn4 takes the patterns (+,+),
// (+,-), (-,-), (-,+).
struct PairScale {
  f2 pp, pm, mm, mp;
  __device__ __forceinline__ PairScale(float w, bool signed_out) {
    pp = dup2(w);
    pm = signed_out ? make_float2(w, -w) : pp;
    mm = signed_out ? dup2(-w) : pp;
    mp = signed_out ? make_float2(-w, w) : pp;
  }
  __device__ __forceinline__ f2 of(int j) const {
    const bool lo = sgn4(2 * j) > 0, hi = sgn4(2 * j + 1) > 0;
    return lo ? (hi ? pp : pm) : (hi ? mp : mm);
  }
};

// ------------------------------------------------------------------ per-lane pieces of the row kernels
//   LN      y = LN(x) * (1 + mod[scale_off + c]) + mod[shift_off + c]  (fp32 two-pass mean/var,
//           biased variance, eps: tools/reference.py:190-191, kernels.js:95-145)
//   act     y <- GELU(y) (the MLP's activation, applied here when the layer1 GEMM stored its
//           pre-activation)
//   rotate  y <- y H per 256 group (tools/quant.py:30-45)
//   quant   s = amax / 127; a = y * (127 / amax); hi = rne(a); lo = rne((a - hi) * 254)
//           (|a| <= 127 and |a - hi| <= 1/2, so neither needs clamping)

// c * (rstd * (1 + scale)) + shift on lane t's 16 centred values c = x - mean; sc/sh point at the
// lane's first column of the scale and shift vectors (lane order).
__device__ __forceinline__ void ln_apply16(f2 (&v)[8], f2 rs, const float* sc, const float* sh) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float4 c = *reinterpret_cast<const float4*>(sc + 64 * k);
    const float4 d = *reinterpret_cast<const float4*>(sh + 64 * k);
    v[2 * k] = fma2(v[2 * k], fma2(rs, make_float2(c.x, c.y), rs), make_float2(d.x, d.y));
    v[2 * k + 1] = fma2(v[2 * k + 1], fma2(rs, make_float2(c.z, c.w), rs), make_float2(d.z, d.w));
  }
}

// Quantize lane t's 16 values, a = v * ps (ps carries 127 / amax and the Hadamard's output sigma),
// into the two int8 planes: register a = e + 4k goes to byte e of the 32-bit word at hi / lo + 64 k.
// hi = rne(a) through the 1.5 * 2^23 magic number, with the product kept exact inside the fma:
// the float's low byte is then the two's-complement int8 of hi (|a| <= 127). lo = rne((a - hi) *
// 254) the same way, a - hi again from the exact product (|a - hi| <= 1/2, so |lo| <= 127).
__device__ __forceinline__ void quant_store16(const f2 (&v)[8], const PairScale& ps, int8_t* hi, int8_t* lo) {
  const f2 magic = dup2(12582912.0f), c254 = dup2(254.0f), m1 = dup2(-1.0f);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t hb[4], lb[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int j = 2 * k + i;
      const f2 m = fma2(v[j], ps.of(j), magic);        // magic + hi
      const f2 rem = fma2(v[j], ps.of(j), fma2(m, m1, magic));  // a - hi
      const f2 l = fma2(rem, c254, magic);
      hb[2 * i] = __float_as_uint(m.x);
      hb[2 * i + 1] = __float_as_uint(m.y);
      lb[2 * i] = __float_as_uint(l.x);
      lb[2 * i + 1] = __float_as_uint(l.y);
    }
    reinterpret_cast<uint32_t*>(hi)[16 * k] = __byte_perm(__byte_perm(hb[0], hb[1], 0x0040), __byte_perm(hb[2], hb[3], 0x0040), 0x5410);
    if (lo) reinterpret_cast<uint32_t*>(lo)[16 * k] = __byte_perm(__byte_perm(lb[0], lb[1], 0x0040), __byte_perm(lb[2], lb[3], 0x0040), 0x5410);
  }
}

__device__ __forceinline__ float amax16(const f2 (&v)[8], float m) {
#pragma unroll
  for (int j = 0; j < 8; ++j) m = fmax3(m, fabsf(v[j].x), fabsf(v[j].y));
  return m;
}

// ------------------------------------------------------------------ row kernel: LN + adaLN, ConvRot, quant
// Geometry: a warp pass covers two groups of 256 columns, one per half-warp; a warp makes G2
// passes and WPR warps share a row. Rows of a single group are handled by one half-warp each.
template <int COLS>
struct RowGeom {
  static constexpr int NG = COLS / 256;
  static constexpr bool HALF = NG == 1;
  static constexpr int G2 = NG % 3 == 0 ? 3 : (NG >= 4 ? 2 : 1);  // 3072 (Qwen3's MLP): 3 passes, 2 warps
  static constexpr int WPR = HALF ? 1 : NG / (2 * G2);
  static constexpr int RPC = HALF ? 16 : 8 / WPR;  // rows per 256-thread CTA
  static_assert(COLS % 256 == 0 && NG <= 64 && (HALF || NG % (2 * G2) == 0) && WPR <= 8, "unsupported row width");
};

// Sum or max over the row: (half-)warp shuffles, then one shared-memory step across the WPR warps.
template <int COLS, bool MAX>
__device__ __forceinline__ float row_reduce(float v, float* red) {
  using Gm = RowGeom<COLS>;
#pragma unroll
  for (int o = Gm::HALF ? 8 : 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, w) : v + w;
  }
  if constexpr (Gm::WPR == 1) {
    return v;
  } else {
    const int warp = threadIdx.x >> 5;
    const int base = (warp / Gm::WPR) * Gm::WPR;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float s = red[base];
#pragma unroll
    for (int i = 1; i < Gm::WPR; ++i) s = MAX ? fmaxf(s, red[base + i]) : s + red[base + i];
    __syncthreads();
    return s;
  }
}

// The general row kernel (every supported width and output), rows straight from global memory.
template <int COLS, typename TIn, typename TOut, bool LN>
__global__ void __launch_bounds__(256, 4) rows_kernel(const TIn* __restrict__ x, int rows, int ldx,
                                                   const float* __restrict__ mod, int shift_off, int scale_off,
                                                   float eps, int rotate, TOut* y, int8_t* qhi, int8_t* qlo,
                                                   float* qscale, int qld, int act) {
  using Gm = RowGeom<COLS>;
  constexpr int G2 = Gm::G2;
  __shared__ float red[8];
  __shared__ __align__(16) float tiles[8 * kTileWords];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, t = lane & 15;
  const int row = Gm::HALF ? blockIdx.x * 16 + warp * 2 + half : blockIdx.x * Gm::RPC + warp / Gm::WPR;
  const int wr = Gm::HALF ? 0 : warp % Gm::WPR;
  const bool valid = row < rows;
  const size_t r = valid ? static_cast<size_t>(row) : 0;
  float* tb = tiles + warp * kTileWords + half * kTileHalf;
  f2 v[G2][8];
  int col[G2];  // the lane's first column in each pass
#pragma unroll
  for (int p = 0; p < G2; ++p) {
    col[p] = (Gm::HALF ? 0 : ((wr * G2 + p) * 2 + half) * 256) + 4 * t;
    if (valid) {
      load_lane16(x + r * ldx + col[p], v[p]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[p][j] = dup2(0.f);
    }
  }
  if constexpr (LN) {
    f2 s2 = dup2(0.f);
#pragma unroll
    for (int p = 0; p < G2; ++p)
#pragma unroll
      for (int j = 0; j < 8; ++j) s2 = add2(s2, v[p][j]);
    const float mean = row_reduce<COLS, false>(s2.x + s2.y, red) / static_cast<float>(COLS);
    const f2 nm = dup2(-mean);
    f2 q2 = dup2(0.f);
#pragma unroll
    for (int p = 0; p < G2; ++p)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[p][j] = add2(v[p][j], nm);
        q2 = fma2(v[p][j], v[p][j], q2);
      }
    const float var = row_reduce<COLS, false>(q2.x + q2.y, red) / static_cast<float>(COLS);
    const f2 rs = dup2(1.0f / sqrtf(var + eps));
#pragma unroll
    for (int p = 0; p < G2; ++p) ln_apply16(v[p], rs, mod + scale_off + col[p], mod + shift_off + col[p]);
  }
  if (act == ANIMA_ACT_GELU) {
#pragma unroll
    for (int p = 0; p < G2; ++p)
#pragma unroll
      for (int j = 0; j < 8; ++j) v[p][j] = gelu2(v[p][j]);
  }
  if (rotate) {
#pragma unroll
    for (int p = 0; p < G2; ++p) hadamard256_n<1>(tb, t, v, p);
  }
  // the lane part of the Hadamard's output sigma
  const float lane_sign = rotate ? sgn4(t) : 1.0f;
  if (qhi) {
    float amax = 0.f;
#pragma unroll
    for (int p = 0; p < G2; ++p) amax = amax16(v[p], amax);
    amax = row_reduce<COLS, true>(amax, red);
    if (!valid) return;
    // a = (y / 16) * 127 / (amax / 16) = y * (127 / amax) for the unscaled y: the 1/16 is a power of
    // two, so this is the same fp32 value as quantizing the scaled y
    const float post = rotate ? 0.0625f : 1.0f;
    const float inv = amax > 0.f ? 127.0f / amax : 0.f;
    if (wr == 0 && (Gm::HALF ? t : lane) == 0) qscale[r] = amax > 0.f ? (amax * post) / 127.0f : 1.0f;
    const PairScale ps(inv * lane_sign, rotate != 0);
#pragma unroll
    for (int p = 0; p < G2; ++p) quant_store16(v[p], ps, qhi + r * qld + col[p], qlo ? qlo + r * qld + col[p] : nullptr);
  } else if (valid) {
    const PairScale ps((rotate ? 0.0625f : 1.0f) * lane_sign, rotate != 0);
#pragma unroll
    for (int p = 0; p < G2; ++p) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[p][j] = mul2(v[p][j], ps.of(j));
      store_lane16(y + r * COLS + col[p], v[p]);
    }
  }
}

// ------------------------------------------------------------------ persistent ring row kernel
// The block's hot rows (2048 and 8192 columns, int8 outputs): LN+adaLN+ConvRot+quant of the
// residual stream and ConvRot+quant of the attention output and of the MLP's hidden layer. One CTA
// per SM runs until its rows are done. A producer lane streams whole rows into a ring of
// shared-memory stages with 1D bulk copies (cp.async.bulk, mbarrier completion), so the loads in
// flight hold no registers and overlap the arithmetic of earlier rows. Teams of WPR consumer
// warps take one row each at a time, every warp PASSES x 512 columns of it (two groups per pass,
// one per half-warp); the row's sums and maximum go across the team through shared memory. Rows
// are split so that the 27-28 rows an SM gets divide evenly over the teams (at 2048 columns 7
// teams of 2 warps take 4 rows each; at 8192, 3 teams of 8 warps 9-10 rows each), with enough
// columns per warp that the per-row work (waits, reductions, the scale) is spread thin. CTA b takes rows b, b + grid, b + 2 grid, ... and
// team m of it the CTA's m-th, (m + TEAMS)-th, ... row.
namespace ring {

constexpr int kSmemLimit = 232448;  // 227 KB of opt-in dynamic shared memory per CTA
constexpr int kMaxStages = 32;

template <int COLS, typename TIn, bool LN>
struct Geom {
  static constexpr int PASSES = 2;                   // passes (512 columns each) per warp
  static constexpr int WPR = COLS / (512 * PASSES);  // warps per row: 2 at 2048, 8 at 8192
  static constexpr int CW = COLS == 2048 ? 14 : 24;  // consumer warps (+ 1 producer: 15 / 25)
  static constexpr int TEAMS = CW / WPR;             // rows in work at once: 7 / 3
  static constexpr int THREADS = 32 * (CW + 1);
  static constexpr int ROWB = COLS * static_cast<int>(sizeof(TIn));
  // shared memory: ring [STAGES][ROWB] | Hadamard tiles [CW] | scale, shift [2][COLS] (LN) |
  // reduction slots [2][CW] | full, empty mbarriers [STAGES] | modulation mbarrier | abort flag
  static constexpr int FIXED = CW * kTileWords * 4 + (LN ? 8 * COLS : 0) + 8 * CW + 8 + 16;
  static constexpr int FIT = (kSmemLimit - FIXED) / (ROWB + 16);
  static constexpr int STAGES = FIT < kMaxStages ? FIT : kMaxStages;
  static constexpr int SMEM = STAGES * (ROWB + 16) + FIXED;
  static_assert(COLS == 512 * PASSES * WPR && CW % WPR == 0 && THREADS <= 1024 && STAGES >= 4 &&
                SMEM <= kSmemLimit, "ring geometry");
};

struct Args {
  const void* x;
  long long rows, ldx;
  const float* mod;
  int shift_off, scale_off;
  float eps;
  int rotate, act;
  int8_t* qhi;
  int8_t* qlo;
  float* qscale;
  long long qld;
};

// Wait for a copy in flight to land, bounded, ignoring the abort flag (used when leaving).
__device__ __forceinline__ bool drain_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t b = smem_u32(bar);
  const unsigned long long t0 = globaltimer();
  while (!mbar_test_sleep(b, parity)) {
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      flag_error(kErrTimeoutDrain);
      return false;
    }
  }
  return true;
}

// Named barrier of team m (ids 2..; 0 is __syncthreads): the WPR warps
// of the team, every thread taking part. bar.red.and also returns whether every thread's pred was
// true.
__device__ __forceinline__ void team_bar(int m, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(2 + m), "r"(threads) : "memory");
}
__device__ __forceinline__ bool team_all(int m, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(2 + m), "r"(threads)
      : "memory");
  return r != 0;
}

// Sum (MAX false) or max of v over the team's row: warp shuffles, then for WPR > 1 one exchange
// through the slots red[phase & 1][team's warps] around the team's barrier. A slot buffer is
// written again two reductions later, after every warp of the team has passed the barrier of
// the reduction in between and so has read it.
template <int WPR, int CW, bool MAX>
__device__ __forceinline__ float team_reduce(float v, float* tred, int team, int& phase) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, w) : v + w;
  }
  if constexpr (WPR == 1) {
    return v;
  } else {
    float* buf = tred + (phase & 1) * CW;
    ++phase;
    if ((threadIdx.x & 31) == 0) buf[(threadIdx.x >> 5) % WPR] = v;
    team_bar(team, 32 * WPR);
    float r = buf[0];
#pragma unroll
    for (int i = 1; i < WPR; ++i) r = MAX ? fmaxf(r, buf[i]) : r + buf[i];
    return r;
  }
}

template <int COLS, typename TIn, bool LN>
__global__ void __launch_bounds__(Geom<COLS, TIn, LN>::THREADS, 1) rows_ring_kernel(const Args a) {
  using G = Geom<COLS, TIn, LN>;
  constexpr int S = G::STAGES;
  extern __shared__ __align__(128) uint8_t smem[];
  TIn* ring = reinterpret_cast<TIn*>(smem);
  float* tiles = reinterpret_cast<float*>(smem + S * G::ROWB);
  float* modv = tiles + G::CW * kTileWords;
  float* red = modv + (LN ? 2 * COLS : 0);
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * G::CW);
  uint64_t* empty = full + S;
  uint64_t* modbar = empty + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(modbar + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == G::CW && lane == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], G::WPR);
    }
    mbar_init(modbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const long long grid = gridDim.x;

  if (warp == G::CW) {  // producer
    if (lane == 0) {
      const TIn* x = static_cast<const TIn*>(a.x);
      if constexpr (LN) {  // the scale and shift vectors, once per CTA, ahead of the first row
        mbar_arrive_expect_tx(modbar, 8 * COLS);
        bulk_load_1d(modv, a.mod + a.scale_off, 4 * COLS, modbar);
        bulk_load_1d(modv + COLS, a.mod + a.shift_off, 4 * COLS, modbar);
      }
      long long issued = 0;
      for (long long u = 0;; ++u) {
        const long long row = blockIdx.x + u * grid;
        if (row >= a.rows) break;
        const int s = static_cast<int>(u % S);
        const uint32_t n = static_cast<uint32_t>(u / S);
        if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, abort_flag, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&full[s], G::ROWB);
        bulk_load_1d(ring + static_cast<size_t>(s) * COLS, x + row * a.ldx, G::ROWB, &full[s]);
        issued = u + 1;
      }
      // the copies of the last S rows may still be in flight after an abort: they land before the
      // CTA's shared memory is released (on the normal path these waits return at once)
      for (long long u = issued > S ? issued - S : 0; u < issued; ++u)
        if (!drain_wait(&full[u % S], static_cast<uint32_t>(u / S) & 1)) break;
      if constexpr (LN) drain_wait(modbar, 0);
    }
    return;
  }

  const int team = warp / G::WPR, wr = warp % G::WPR;
  const int half = lane >> 4, t = lane & 15;
  float* tb = tiles + warp * kTileWords + half * kTileHalf;
  float* tred = red + team * G::WPR;
  int phase = 0;
  const float lane_sign = a.rotate ? sgn4(t) : 1.0f;  // the lane part of the Hadamard's output sigma
  const float post = a.rotate ? 0.0625f : 1.0f;
  const int col0 = wr * (512 * G::PASSES) + half * 256 + 4 * t;  // pass p adds 512
  for (long long u = team;; u += G::TEAMS) {
    const long long row = blockIdx.x + u * grid;
    if (row >= a.rows) break;
    const int s = static_cast<int>(u % S);
    // a wait that gave up (bounded; the abort is raised) ends the whole team together, so no warp
    // is left at a team barrier
    bool ok = true;
    if (LN && u == team) ok = mbar_wait(modbar, 0, abort_flag, kErrTimeoutFull);  // before the first row
    ok = ok && mbar_wait(&full[s], static_cast<uint32_t>(u / S) & 1, abort_flag, kErrTimeoutFull);
    if constexpr (G::WPR == 1) {
      if (!ok) return;
    } else {
      if (!team_all(team, 32 * G::WPR, ok)) return;
    }
    f2 v[G::PASSES][8];
    const TIn* src = ring + static_cast<size_t>(s) * COLS + col0;
#pragma unroll
    for (int p = 0; p < G::PASSES; ++p) load_lane16(src + 512 * p, v[p]);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // the stage may be refilled
    if constexpr (LN) {
      f2 s2 = dup2(0.f);
#pragma unroll
      for (int p = 0; p < G::PASSES; ++p)
#pragma unroll
        for (int j = 0; j < 8; ++j) s2 = add2(s2, v[p][j]);
      const float sum = team_reduce<G::WPR, G::CW, false>(s2.x + s2.y, tred, team, phase);
      const f2 nm = dup2(-sum / static_cast<float>(COLS));
      f2 q2 = dup2(0.f);
#pragma unroll
      for (int p = 0; p < G::PASSES; ++p)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[p][j] = add2(v[p][j], nm);
          q2 = fma2(v[p][j], v[p][j], q2);
        }
      const float ss = team_reduce<G::WPR, G::CW, false>(q2.x + q2.y, tred, team, phase);
      const f2 rs = dup2(1.0f / sqrtf(ss / static_cast<float>(COLS) + a.eps));
#pragma unroll
      for (int p = 0; p < G::PASSES; ++p) ln_apply16(v[p], rs, modv + col0 + 512 * p, modv + COLS + col0 + 512 * p);
    }
    if (a.act == ANIMA_ACT_GELU) {
#pragma unroll
      for (int p = 0; p < G::PASSES; ++p)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[p][j] = gelu2(v[p][j]);
    }
    if (a.rotate) {
#pragma unroll
      for (int p = 0; p < G::PASSES; ++p) hadamard256_n<1>(tb, t, v, p);
    }
    float amax = 0.f;
#pragma unroll
    for (int p = 0; p < G::PASSES; ++p) amax = amax16(v[p], amax);
    amax = team_reduce<G::WPR, G::CW, true>(amax, tred, team, phase);
    // quantizing the unscaled Hadamard output with 127 / amax gives the same fp32 values as
    // quantizing y / 16 (the 1/16 is a power of two)
    const float inv = amax > 0.f ? __fdividef(127.0f, amax) : 0.f;
    if (wr == 0 && lane == 0) a.qscale[row] = amax > 0.f ? (amax * post) / 127.0f : 1.0f;
    const PairScale ps(inv * lane_sign, a.rotate != 0);
    int8_t* hi = a.qhi + row * a.qld + col0;
    int8_t* lo = a.qlo ? a.qlo + row * a.qld + col0 : nullptr;
#pragma unroll
    for (int p = 0; p < G::PASSES; ++p) quant_store16(v[p], ps, hi + 512 * p, lo ? lo + 512 * p : nullptr);
  }
}

}  // namespace ring

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
// y = c0 x0 + c1 x1 + c2 x2 + c3 x3 (NULL terms dropped), 4 elements per thread when aligned.
__global__ void lincomb_kernel(float* y, long long n, const float* x0, const float* x1, const float* x2,
                               const float* x3, float c0, float c1, float c2, float c3) {
  const long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i >= n) return;
  const float* xs[4] = {x0, x1, x2, x3};
  const float cs[4] = {c0, c1, c2, c3};
  if (i + 4 <= n) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (!xs[k]) continue;
      const float4 v = *reinterpret_cast<const float4*>(xs[k] + i);
      acc.x = fmaf(cs[k], v.x, acc.x);
      acc.y = fmaf(cs[k], v.y, acc.y);
      acc.z = fmaf(cs[k], v.z, acc.z);
      acc.w = fmaf(cs[k], v.w, acc.w);
    }
    *reinterpret_cast<float4*>(y + i) = acc;
  } else {
    for (long long e = i; e < n; ++e) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (xs[k]) acc = fmaf(cs[k], xs[k][e], acc);
      y[e] = acc;
    }
  }
}

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

// 32 codes per thread (16 packed bytes = two fp8 groups), the arithmetic of unpack_w4_kernel,
// written as two 16-byte stores. Nibble e of packed word j holds code 8j + e (the low nibble of a
// byte is the even k). The codebook sits in shared memory: 16 distinct words in 16 banks, so the
// data-dependent lookups never conflict.
__global__ void __launch_bounds__(256) w4_decode_kernel(const uint8_t* __restrict__ packed,
                                                        const uint8_t* __restrict__ s_rel, const float* __restrict__ cb,
                                                        long long n_chunks, int K, int8_t* __restrict__ out) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = cb[threadIdx.x];
  __syncthreads();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_chunks) return;
  const long long k0 = 32 * i;  // flat index of the chunk's first code
  const long long row = k0 / K;
  const int kk = static_cast<int>(k0 - row * K);
  const uint4 p = __ldg(reinterpret_cast<const uint4*>(packed) + i);
  const uint8_t* sr = s_rel + row * (K / 16) + kk / 16;
  const float sg[2] = {fp8_e4m3fn(__ldg(sr)), fp8_e4m3fn(__ldg(sr + 1))};
  const uint32_t w[4] = {p.x, p.y, p.z, p.w};
  uint32_t o[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float s = sg[j >> 1];
    uint32_t half[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float v = fminf(fmaxf(rintf(__fmul_rn(lut[(w[j] >> (4 * e)) & 15u], s)), -127.f), 127.f);
      half[e >> 2] |= (static_cast<uint32_t>(static_cast<int>(v)) & 0xFFu) << (8 * (e & 3));
    }
    o[2 * j] = half[0];
    o[2 * j + 1] = half[1];
  }
  uint4* dst = reinterpret_cast<uint4*>(out + k0);
  dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
  dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
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
// 256 threads compute a BM x 64 tile (BM = 64, 32 or 16, the tallest that still gives two CTAs
// per SM). The threads form KS = 64 / BM K-slices of 4 BM threads; a slice walks every KS-th K
// tile of 32, each thread accumulating a 4 x 4 block from two 16-byte shared-memory reads per k,
// and the slices' partial tiles are summed through shared memory at the end. The next tile's
// global loads are issued before the current tile's FMAs.
// QA: A is given as quantized rows, A[m, k] = qs[m] * (qhi[m, k] + qlo[m, k] / 254).
// VEC: A (fp32) and B are read as 16-byte vectors (4 fp32 or 8 16-bit values along k; needs K,
// lda and ldb multiples of 8 and 16-byte aligned rows), else element by element.
template <typename TB, bool QA, int BM, bool VEC>
__global__ void __launch_bounds__(256, 2) simt_gemm_kernel(int M, int N, int K, float alpha, const float* __restrict__ A,
                                                        int lda, const TB* __restrict__ B, int ldb,
                                                        const float* __restrict__ bias, int act, float* C, int ldc,
                                                        int accumulate, const float* __restrict__ gate, int gate_off,
                                                        const int8_t* __restrict__ qhi = nullptr,
                                                        const int8_t* __restrict__ qlo = nullptr,
                                                        const float* __restrict__ qs = nullptr) {
  constexpr int BN = 64, BK = 32, KS = 64 / BM, ST = 4 * BM;
  constexpr int AE = BM * BK / ST, BE = BN * BK / ST;
  constexpr int AS = BM + 4, BS = BN + 4;            // padded rows, 16-byte aligned
  constexpr int SLICE = BK * AS + BK * BS;           // floats per slice
  static_assert(KS * SLICE >= KS * BM * BN, "reduction buffer");
  __shared__ __align__(16) float smem[KS * SLICE];
  const int sl = threadIdx.x / ST, lt = threadIdx.x % ST;
  const int tx = lt % 16, ty = lt / 16;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float* As = smem + sl * SLICE;
  float* Bs = As + BK * AS;
  float ra[AE], rb[BE];
  // element e of this thread's share of the A (B) tile: row i / BK, column i % BK of the tile, with
  // i = lt + e * ST element by element, or, for 16-byte vectors of V elements, i = V * (lt + (e / V)
  // * ST) + e % V (a vector's elements are consecutive along k)
  auto a_idx = [&](int e) {
    return VEC && !QA ? 4 * (lt + (e / 4) * ST) + e % 4 : lt + e * ST;
  };
  constexpr int VB = 16 / static_cast<int>(sizeof(TB));
  auto b_idx = [&](int e) { return VEC ? VB * (lt + (e / VB) * ST) + e % VB : lt + e * ST; };
  auto fetch = [&](int k0) {
    if constexpr (VEC && !QA) {
#pragma unroll
      for (int e = 0; e < AE; e += 4) {
        const int i = a_idx(e), r = i / BK, k = k0 + i % BK, m = m0 + r;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        if (m < M && k < K) a = *reinterpret_cast<const float4*>(A + static_cast<size_t>(m) * lda + k);
        ra[e] = a.x; ra[e + 1] = a.y; ra[e + 2] = a.z; ra[e + 3] = a.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < AE; ++e) {
        const int i = a_idx(e), r = i / BK, k = k0 + i % BK, m = m0 + r;
        float a = 0.f;
        if (m < M && k < K) {
          const size_t idx = static_cast<size_t>(m) * lda + k;
          if constexpr (QA) {
            a = static_cast<float>(qhi[idx]);
            if (qlo) a += static_cast<float>(qlo[idx]) * (1.0f / 254.0f);
            a *= qs[m];
          } else {
            a = A[idx];
          }
        }
        ra[e] = a;
      }
    }
    if constexpr (VEC) {
#pragma unroll
      for (int e = 0; e < BE; e += VB) {
        const int i = b_idx(e), r = i / BK, k = k0 + i % BK, n = n0 + r;
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (n < N && k < K) u = *reinterpret_cast<const uint4*>(B + static_cast<size_t>(n) * ldb + k);
        const TB* h = reinterpret_cast<const TB*>(&u);
#pragma unroll
        for (int j = 0; j < VB; ++j) rb[e + j] = to_f<TB>(h[j]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < BE; ++e) {
        const int i = b_idx(e), r = i / BK, k = k0 + i % BK, n = n0 + r;
        rb[e] = (n < N && k < K) ? to_f<TB>(B[static_cast<size_t>(n) * ldb + k]) : 0.f;
      }
    }
  };
  float acc[4][4] = {};
  const int nk = (K + BK - 1) / BK;
  const int steps = (nk + KS - 1) / KS;  // the same for every slice: all threads meet every barrier
  fetch(sl * BK);
  for (int t = 0; t < steps; ++t) {
#pragma unroll
    for (int e = 0; e < AE; ++e) {
      const int i = a_idx(e);
      As[(i % BK) * AS + i / BK] = ra[e];
    }
#pragma unroll
    for (int e = 0; e < BE; ++e) {
      const int i = b_idx(e);
      Bs[(i % BK) * BS + i / BK] = rb[e];
    }
    __syncthreads();
    if (t + 1 < steps) fetch(((t + 1) * KS + sl) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(As + kk * AS + 4 * ty);
      const float4 b = *reinterpret_cast<const float4*>(Bs + kk * BS + 4 * tx);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  if constexpr (KS > 1) {
    float* red = smem + sl * BM * BN;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<float4*>(red + (4 * ty + i) * BN + 4 * tx) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    __syncthreads();
    if (sl != 0) return;
#pragma unroll
    for (int q = 1; q < KS; ++q)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 v = *reinterpret_cast<const float4*>(smem + q * BM * BN + (4 * ty + i) * BN + 4 * tx);
        acc[i][0] += v.x; acc[i][1] += v.y; acc[i][2] += v.z; acc[i][3] += v.w;
      }
  }
  // the thread's 4 columns go out as one 16-byte store when the row allows it
  const int nb = n0 + 4 * tx;
  const bool vec = !accumulate && nb + 4 <= N && ((reinterpret_cast<uintptr_t>(C) | (static_cast<uintptr_t>(ldc) * 4)) & 15) == 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + 4 * ty + i;
    if (m >= M) continue;
    float r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      r[j] = acc[i][j] * alpha;
      if (bias && nb + j < N) r[j] += bias[nb + j];
      if (act == ANIMA_ACT_GELU) r[j] = gelu_erf(r[j]);
      if (act == ANIMA_ACT_SILU) r[j] = silu_f(r[j]);
    }
    float* c = C + static_cast<size_t>(m) * ldc + nb;
    if (vec) {
      *reinterpret_cast<float4*>(c) = make_float4(r[0], r[1], r[2], r[3]);
      continue;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (nb + j >= N) continue;
      if (accumulate)
        c[j] += (gate ? gate[gate_off + nb + j] : 1.0f) * r[j];
      else
        c[j] = r[j];
    }
  }
}

// Tile height for the SIMT GEMM: the tallest tile that still gives two CTAs per SM.
inline int simt_bm(int M, int N, int sms) {
  const long long nt = (N + 63) / 64;
  for (int bm : {64, 32}) {
    if (nt * ((M + bm - 1) / bm) >= 2LL * sms) return bm;
  }
  return 16;
}

template <typename TB, bool QA>
void launch_simt(cudaStream_t st, int sms, int M, int N, int K, float alpha, const float* A, int lda, const TB* B,
                 int ldb, const float* bias, int act, float* C, int ldc, int accumulate, const float* gate,
                 int gate_off, const int8_t* qhi = nullptr, const int8_t* qlo = nullptr, const float* qs = nullptr) {
  const int bm = simt_bm(M, N, sms);
  const dim3 grid((N + 63) / 64, (M + bm - 1) / bm);
  const bool vec = K % 8 == 0 && ldb % 8 == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0 &&
                   (QA || (lda % 8 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0));
#define SIMT(BMV, V)                                                                                             \
  simt_gemm_kernel<TB, QA, BMV, V><<<grid, 256, 0, st>>>(M, N, K, alpha, A, lda, B, ldb, bias, act, C, ldc, accumulate, \
                                                         gate, gate_off, qhi, qlo, qs)
  if (vec) {
    if (bm == 64) SIMT(64, true);
    else if (bm == 32) SIMT(32, true);
    else SIMT(16, true);
  } else {
    if (bm == 64) SIMT(64, false);
    else if (bm == 32) SIMT(32, false);
    else SIMT(16, false);
  }
#undef SIMT
}

template <int COLS, typename TIn, bool LN>
int launch_ring(anima_ctx* ctx, const ring::Args& a) {
  using G = ring::Geom<COLS, TIn, LN>;
  const void* fn = reinterpret_cast<const void*>(&ring::rows_ring_kernel<COLS, TIn, LN>);
  int st = set_max_dynamic_smem(fn, G::SMEM);
  if (st) return st;
  const long long need = (a.rows + G::TEAMS - 1) / G::TEAMS;
  const int grid = static_cast<int>(need < ctx->num_sms ? need : ctx->num_sms);
  ring::rows_ring_kernel<COLS, TIn, LN><<<grid, G::THREADS, G::SMEM, ctx->stream>>>(a);
  return check_launch("rows_ring_kernel");
}

// The ring kernel takes the int8-output cases of 2048 and 8192 columns (rows read with 1D bulk
// copies: 16-byte aligned row starts); everything else runs on rows_kernel.
template <typename TIn, bool LN>
bool ring_case(int cols, const TIn* x, int ldx, const anima_qact* q) {
  return q && q->hi && (cols == 2048 || cols == 8192) && (!LN || cols == 2048) &&
         (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (static_cast<long long>(ldx) * sizeof(TIn)) % 16 == 0;
}

template <typename TIn, typename TOut, bool LN>
int launch_rows(anima_ctx* ctx, const TIn* x, int rows, int cols, int ldx, const float* mod, int so, int sco,
                float eps, int rotate, TOut* y, const anima_qact* q, int act = ANIMA_ACT_NONE) {
  if (ring_case<TIn, LN>(cols, x, ldx, q)) {
    const ring::Args a{x, rows, ldx, mod, so, sco, eps, rotate, act, q->hi, q->lo, q->scale, q->ld};
    if constexpr (LN) {
      return launch_ring<2048, TIn, true>(ctx, a);
    } else {
      return cols == 2048 ? launch_ring<2048, TIn, false>(ctx, a) : launch_ring<8192, TIn, false>(ctx, a);
    }
  }
  int8_t* hi = q ? q->hi : nullptr;
  int8_t* lo = q ? q->lo : nullptr;
  float* sc = q ? q->scale : nullptr;
  const int qld = q ? q->ld : 0;
#define ROWS_CASE(C)                                                                                             \
  case C: {                                                                                                      \
    constexpr int rpc = RowGeom<C>::RPC;                                                                         \
    rows_kernel<C, TIn, TOut, LN><<<(rows + rpc - 1) / rpc, 256, 0, ctx->stream>>>(x, rows, ldx, mod, so, sco,   \
                                                                                  eps, rotate, y, hi, lo, sc, qld, act); \
    break;                                                                                                       \
  }
  switch (cols) {
    ROWS_CASE(256)
    ROWS_CASE(512)
    ROWS_CASE(1024)
    ROWS_CASE(2048)
    ROWS_CASE(3072)
    ROWS_CASE(4096)
    ROWS_CASE(8192)
    default:
      return set_error(ANIMA_ERR_UNSUPPORTED, "row kernel: cols=%d (supported: 256, 512, 1024, 2048, 3072, 4096, 8192)", cols);
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

int launch_w4_decode(anima_ctx* ctx, const uint8_t* packed, const uint8_t* s_rel, const float* codebook, int N, int K,
                     int8_t* out) {
  if (K % 32 != 0 || !rowops::al16(packed) || !rowops::al16(out))
    return set_error(ANIMA_ERR_ARG, "W4 decode: K=%d must be a multiple of 32, packed/out 16-byte aligned", K);
  const long long chunks = static_cast<long long>(N) * K / 32;
  ProfScope prof(ctx, "w4.decode", 0, static_cast<double>(N) * K * 1.5 + static_cast<double>(N) * K / 16);
  rowops::w4_decode_kernel<<<static_cast<int>((chunks + 255) / 256), 256, 0, ctx->stream>>>(packed, s_rel, codebook,
                                                                                            chunks, K, out);
  return check_launch("w4_decode_kernel");
}

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
  ANIMA_ON_DEVICE(ctx);
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
  ANIMA_ON_DEVICE(ctx);
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
  ANIMA_ON_DEVICE(ctx);
  ANIMA_REQUIRE(rows > 0 && ldx >= cols && al16(x) && al16(y), "anima_rotate: bad shape or alignment");
  ANIMA_REQUIRE(in_dtype == ANIMA_F32 && out_dtype == ANIMA_F32, "anima_rotate: only fp32 in/out (use anima_rotate_quant)");
  ProfScope prof(ctx, "hadamard", 0, rows * (double)cols * 8);
  return launch_rot<float, float>(ctx, (const float*)x, rows, cols, ldx, 1, (float*)y, nullptr);
}

static int rot_quant(anima_ctx* ctx, const void* x, int in_dtype, int rows, int cols, int ldx, const anima_qact* out,
                     int rotate, const char* who, int act = ANIMA_ACT_NONE) {
  ANIMA_REQUIRE(ctx && x, "%s: NULL argument", who);
  ANIMA_ON_DEVICE(ctx);
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
  ANIMA_ON_DEVICE(ctx);
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
  ANIMA_ON_DEVICE(ctx);
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
  ANIMA_ON_DEVICE(ctx);
  const long long n = static_cast<long long>(L) * H * (D / 2);
  ProfScope prof(ctx, "rope", 0, 2.0 * n * 2 * (dtype == ANIMA_F32 ? 4 : 2));
  if (dtype == ANIMA_F32) rope_kernel<float><<<grid1(n, 256), 256, 0, ctx->stream>>>((float*)x, L, H, D, row_stride, col_off, rope, rope_rows);
  else if (dtype == ANIMA_BF16) rope_kernel<__nv_bfloat16><<<grid1(n, 256), 256, 0, ctx->stream>>>((__nv_bfloat16*)x, L, H, D, row_stride, col_off, rope, rope_rows);
  else if (dtype == ANIMA_F16) rope_kernel<__half><<<grid1(n, 256), 256, 0, ctx->stream>>>((__half*)x, L, H, D, row_stride, col_off, rope, rope_rows);
  else return set_error(ANIMA_ERR_ARG, "anima_rope: dtype %d", dtype);
  return check_launch("rope_kernel");
}

int anima_lincomb(anima_ctx* ctx, float* y, long long n, const float* x0, const float* x1, const float* x2,
                  const float* x3, const float* c) {
  ANIMA_REQUIRE(ctx && y && c && n > 0, "anima_lincomb: bad argument");
  ANIMA_ON_DEVICE(ctx);
  const float* xs[4] = {x0, x1, x2, x3};
  ANIMA_REQUIRE(al16(y), "anima_lincomb: y must be 16-byte aligned");
  for (int k = 0; k < 4; ++k) ANIMA_REQUIRE(!xs[k] || al16(xs[k]), "anima_lincomb: x%d must be 16-byte aligned", k);
  lincomb_kernel<<<static_cast<int>((n + 1023) / 1024), 256, 0, ctx->stream>>>(y, n, x0, x1, x2, x3, c[0], c[1], c[2],
                                                                              c[3]);
  return check_launch("lincomb_kernel");
}

int anima_elementwise(anima_ctx* ctx, int op, const float* a, const float* b, float* y, long long n) {
  ANIMA_REQUIRE(ctx && a && y && n >= 0 && op >= 0 && op <= 3, "anima_elementwise: bad argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_REQUIRE(!(op == 1 || op == 3) || b, "anima_elementwise: binary op needs b");
  if (n == 0) return ANIMA_OK;
  elementwise_kernel<<<grid1(n, 256), 256, 0, ctx->stream>>>(op, a, b, y, n);
  return check_launch("elementwise_kernel");
}

int anima_unpack_w4(anima_ctx* ctx, const uint8_t* packed, const uint8_t* s_rel, const float* codebook, int N, int K,
                    int8_t* out) {
  ANIMA_REQUIRE(ctx && packed && s_rel && codebook && out, "anima_unpack_w4: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_REQUIRE(N > 0 && K > 0 && K % 16 == 0, "anima_unpack_w4: K=%d must be a positive multiple of 16", K);
  if (K % 32 == 0 && al16(packed) && al16(out)) return launch_w4_decode(ctx, packed, s_rel, codebook, N, K, out);
  const long long nb = static_cast<long long>(N) * K / 2;
  ProfScope prof(ctx, "unpack_w4", 0, nb * 3.0);
  unpack_w4_kernel<<<grid1(nb, 256), 256, 0, ctx->stream>>>(packed, s_rel, codebook, nb, K, out);
  return check_launch("unpack_w4_kernel");
}

int anima_matmul(anima_ctx* ctx, int M, int N, int K, float alpha, const float* A, int lda, const anima_weight* B,
                 int act, float* C, int ldc, int accumulate, const float* gate, int gate_off) {
  ANIMA_REQUIRE(ctx && A && B && B->data && C, "anima_matmul: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_REQUIRE(M > 0 && N > 0 && K > 0 && lda >= K && ldc >= N, "anima_matmul: bad shape");
  ANIMA_REQUIRE(B->kind == ANIMA_W_BF16 || B->kind == ANIMA_W_F32 || B->kind == ANIMA_W_F16,
                "anima_matmul: weight kind %d (bf16, f32 or f16 only)", B->kind);
  ProfScope prof(ctx, B->kind == ANIMA_W_F32 ? "gemm.f32" : "gemm.16bit", 2.0 * M * N * K, 0);
  // 16-bit weights, no scale, activation or gate: the tensor-core GEMM on two planes of A when the
  // shape suits it, else the CUDA-core kernel below
  if (B->kind != ANIMA_W_F32 && alpha == 1.0f && act == ANIMA_ACT_NONE && !gate) {
    const int st = matmul_planes(ctx, M, N, K, A, lda, B->data, B->bias, C, ldc, accumulate, B->kind == ANIMA_W_F16);
    if (st != ANIMA_ERR_UNSUPPORTED) return st;
  }
  if (B->kind == ANIMA_W_F16)
    launch_simt<__half, false>(ctx->stream, ctx->num_sms, M, N, K, alpha, A, lda, (const __half*)B->data, K, B->bias,
                               act, C, ldc, accumulate, gate, gate_off);
  else if (B->kind == ANIMA_W_BF16)
    launch_simt<__nv_bfloat16, false>(ctx->stream, ctx->num_sms, M, N, K, alpha, A, lda, (const __nv_bfloat16*)B->data, K,
                                      B->bias, act, C, ldc, accumulate, gate, gate_off);
  else
    launch_simt<float, false>(ctx->stream, ctx->num_sms, M, N, K, alpha, A, lda, (const float*)B->data, K, B->bias, act,
                              C, ldc, accumulate, gate, gate_off);
  return check_launch("simt_gemm_kernel");
}

int anima_lora_down(anima_ctx* ctx, const anima_qact* x, const float* A, int r, float* T, int ldt) {
  ANIMA_REQUIRE(ctx && x && x->hi && x->scale && A && T && r > 0 && ldt >= r, "anima_lora_down: bad argument");
  ANIMA_ON_DEVICE(ctx);
  ProfScope prof(ctx, "lora.down", 2.0 * x->rows * r * x->cols, 0);
  launch_simt<float, true>(ctx->stream, ctx->num_sms, x->rows, r, x->cols, 1.0f, nullptr, x->ld, A, x->cols, nullptr, 0, T,
                           ldt, 0, nullptr, 0, x->hi, x->lo, x->scale);
  return check_launch("simt_gemm_kernel<lora_down>");
}

int anima_patchify(anima_ctx* ctx, const float* latent, int B, int h, int w, float* patches) {
  ANIMA_REQUIRE(ctx && latent && patches && B > 0 && h > 0 && w > 0 && h % 2 == 0 && w % 2 == 0, "anima_patchify: bad argument");
  ANIMA_ON_DEVICE(ctx);
  const long long n = static_cast<long long>(B) * (h / 2) * (w / 2) * 68;
  patchify_kernel<<<grid1(n, 256), 256, 0, ctx->stream>>>(latent, B, h, w, patches);
  return check_launch("patchify_kernel");
}

int anima_unpatchify(anima_ctx* ctx, const float* o, int B, int h, int w, float* latent) {
  ANIMA_REQUIRE(ctx && o && latent && B > 0 && h > 0 && w > 0 && h % 2 == 0 && w % 2 == 0, "anima_unpatchify: bad argument");
  ANIMA_ON_DEVICE(ctx);
  const long long n = static_cast<long long>(B) * 16 * h * w;
  unpatchify_kernel<<<grid1(n, 256), 256, 0, ctx->stream>>>(o, B, h, w, latent);
  return check_launch("unpatchify_kernel");
}

int anima_timestep_embedding(anima_ctx* ctx, const float* sigmas, int B, float* temb) {
  ANIMA_REQUIRE(ctx && sigmas && temb && B > 0, "anima_timestep_embedding: bad argument");
  ANIMA_ON_DEVICE(ctx);
  timestep_embedding_kernel<<<grid1(B * 1024LL, 256), 256, 0, ctx->stream>>>(sigmas, B, temb);
  return check_launch("timestep_embedding_kernel");
}

int anima_euler_step(anima_ctx* ctx, float* x, const float* v, const float* v_uncond, float cfg, float sigma,
                     float sigma_next, long long n, float* den_out) {
  ANIMA_REQUIRE(ctx && x && v && n > 0 && sigma > 0.f, "anima_euler_step: bad argument");
  ANIMA_ON_DEVICE(ctx);
  euler_kernel<<<grid1(n, 256), 256, 0, ctx->stream>>>(x, v, v_uncond, cfg, sigma, sigma_next, n, den_out);
  return check_launch("euler_kernel");
}

}  // extern "C"
