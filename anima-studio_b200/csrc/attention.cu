// Non-causal multi-head attention on tcgen05 (kind::f16), head_dim 128: the DiT's self-attention
// (Lq = Lk = 4096 at 1024^2) and cross-attention against cached text keys (Lk = 256..512). The
// reference's counterpart is the fp32 WGSL flash kernel of app/gpu/kernels.js:147-299; this one
// keeps S = QK^T and O_j = P_j V_j in TMEM and does the online softmax in fp32 registers.
//
// One CTA = one (batch, head, 128-query tile); 192 threads:
//   warp 0      TMA producer: Q once, then K_j / V_j tiles (128 keys) into two stages each
//   warp 1      TMEM allocator + single-thread UMMA issuer:
//                 S_j = Q K_j^T (M=128, N=128, K=16 x 8)   into S[j % 2]   (TMEM cols 0 / 128)
//                 O_j = P_j V_j (M=128, N=128, K=16 x 8)   into O[j % 2]   (TMEM cols 256 / 384)
//               issued as S_0, S_1, PV_0, S_2, PV_1, ... so QK^T of block j+1 overlaps softmax j.
//   warps 2..5  softmax, one query row per thread: row max and exp2 of S_j, P_j (16-bit) into
//               shared memory in the SWIZZLE_128B K-major layout, running sum l; O accumulated in
//               registers one block behind (O = O * 2^(m_{j-1} - m_j) + O_j), normalised by l.
// Keys >= key_len[b] (and >= Lk) get probability 0; key blocks entirely past key_len are skipped.

#include "internal.h"
#include "sm100.cuh"

namespace anima {
namespace attn {

constexpr int TILE = 128;     // query rows per CTA and keys per block
constexpr int HD = 128;       // head dim
constexpr int THREADS = 192;
constexpr int ATOM = 16384;   // one SWIZZLE_128B atom column: 128 rows x 128 bytes
constexpr int TILE_BYTES = 2 * ATOM;
// shared memory: Q | K[2] | V[2] | P[2] | barriers
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE_BYTES;
constexpr int OFF_V = OFF_K + 2 * TILE_BYTES;
constexpr int OFF_P = OFF_V + 2 * TILE_BYTES;
constexpr int OFF_BAR = OFF_P + 2 * TILE_BYTES;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;

struct Params {
  int Lq, Lk, heads, q_tiles;
  int q_col, k_col, v_col;  // column offsets of head 0
  void* out;
  long long ldo, o_bstride;
  int out_dtype;
  const int* key_len;
  int kv_bcast;      // one K/V (and key_len) shared by every batch item
  float scale_log2;  // softmax scale * log2(e)
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned err) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, err) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_empty = bars + 11; // [2]
  uint64_t* p_full = bars + 13;  // [2]
  uint64_t* o_full = bars + 15;  // [2]
  uint64_t* o_empty = bars + 17; // [2]
  uint64_t* drain = bars + 19;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x % p.q_tiles;
  const int bh = blockIdx.x / p.q_tiles;
  const int h = bh % p.heads;
  const int b = bh / p.heads;
  const int q0 = qt * TILE;
  int kv_len = p.Lk;
  const int kvb = p.kv_bcast ? 0 : b;
  if (p.key_len) kv_len = min(kv_len, p.key_len[kvb]);
  const int nblk = (kv_len + TILE - 1) / TILE;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const int qc = p.q_col + h * HD, kc = p.k_col + h * HD, vc = p.v_col + h * HD;
      int armed[5] = {-1, -1, -1, -1, -1};  // parity of the last arm: q, k0, k1, v0, v1
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_3d(smem + OFF_Q, &tm_q, q_full, qc, q0, b);
      tma_load_3d(smem + OFF_Q + ATOM, &tm_q, q_full, qc + 64, q0, b);
      armed[0] = 0;
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_empty[st], ph ^ 1, abort_flag, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
        tma_load_3d(smem + OFF_K + st * TILE_BYTES, &tm_k, &k_full[st], kc, j * TILE, kvb);
        tma_load_3d(smem + OFF_K + st * TILE_BYTES + ATOM, &tm_k, &k_full[st], kc + 64, j * TILE, kvb);
        armed[1 + st] = static_cast<int>(ph);
        if (!mbar_wait(&v_empty[st], ph ^ 1, abort_flag, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
        tma_load_3d(smem + OFF_V + st * TILE_BYTES, &tm_v, &v_full[st], vc, j * TILE, kvb);
        tma_load_3d(smem + OFF_V + st * TILE_BYTES + ATOM, &tm_v, &v_full[st], vc + 64, j * TILE, kvb);
        armed[3 + st] = static_cast<int>(ph);
      }
      if (*abort_flag) {
        uint64_t* fb[5] = {q_full, &k_full[0], &k_full[1], &v_full[0], &v_full[1]};
        for (int i = 0; i < 5; ++i) {
          if (armed[i] < 0) continue;
          const unsigned long long t0 = globaltimer();
          while (!mbar_test(smem_u32(fb[i]), static_cast<uint32_t>(armed[i]))) {
            if (globaltimer() - t0 > kWaitTimeoutNs) {
              flag_error(kErrTimeoutDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(TILE, TILE, BF16, false);
      const uint32_t id_pv = idesc_f16(TILE, HD, BF16, true);
      const uint32_t sq = smem_u32(smem + OFF_Q);
      bool ok = mbar_wait(q_full, 0, abort_flag, kErrTimeoutFull);
      auto issue_pv = [&](int i) -> bool {
        const int st = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(&p_full[st], ph, abort_flag, kErrTimeoutFull)) return false;
        if (!mbar_wait(&v_full[st], ph, abort_flag, kErrTimeoutFull)) return false;
        if (!mbar_wait(&o_empty[st], ph ^ 1, abort_flag, kErrTimeoutAcc)) return false;
        tc_fence_after();
        const uint32_t sp = smem_u32(smem + OFF_P + st * TILE_BYTES);
        const uint32_t sv = smem_u32(smem + OFF_V + st * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < TILE / 16; ++k) {
          const uint64_t ad = sdesc_sw128(sp + (k >> 2) * ATOM + (k & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(sv + k * 16 * 128, ATOM, 1024);
          umma_f16(tmem + 256 + st * 128, ad, bd, id_pv, k > 0 ? 1u : 0u);
        }
        umma_commit(&v_empty[st]);
        umma_commit(&o_full[st]);
        return true;
      };
      for (int j = 0; ok && j < nblk; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_full[st], ph, abort_flag, kErrTimeoutFull)) { ok = false; break; }
        if (!mbar_wait(&s_empty[st], ph ^ 1, abort_flag, kErrTimeoutAcc)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + OFF_K + st * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * ATOM + (k & 3) * 32;
          umma_f16(tmem + st * 128, sdesc_sw128(sq + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), id_qk,
                   k > 0 ? 1u : 0u);
        }
        umma_commit(&k_empty[st]);
        umma_commit(&s_full[st]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && nblk > 0) ok = issue_pv(nblk - 1);
      if (*abort_flag) {
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
  } else {
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    float o[HD];
#pragma unroll
    for (int c = 0; c < HD; ++c) o[c] = 0.f;
    float m_prev = -INFINITY;  // running max (log2 domain) after the previous block
    float m_lag = -INFINITY;   // max of the block whose O_j is accumulated next
    float m_acc = -INFINITY;   // max the register O is currently relative to
    float l = 0.f;
    bool ok = true;

    auto accumulate = [&](int i, float m_i) -> bool {
      const int st = i & 1;
      const uint32_t ph = (i >> 1) & 1;
      if (!warp_wait(&o_full[st], ph, abort_flag, kErrTimeoutAcc)) return false;
      tc_fence_after();
      const float alpha = (m_acc == -INFINITY) ? 0.f : ex2(m_acc - m_i);
#pragma unroll
      for (int c = 0; c < HD; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_addr + 256 + st * 128 + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) o[c + t] = fmaf(o[c + t], alpha, __uint_as_float(r[t]));
      }
      m_acc = m_i;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[st]);
      return true;
    };

    uint8_t* prow_base = smem + OFF_P + row * 128;
    for (int j = 0; j < nblk; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!warp_wait(&s_full[st], ph, abort_flag, kErrTimeoutFull)) { ok = false; break; }
      tc_fence_after();
      const uint32_t s_addr = tmem + lane_addr + st * 128;
      const int kbase = j * TILE;
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < TILE; c += 32) {
        uint32_t r[32];
        tmem_ld32(s_addr + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const float s = (kbase + c + t < kv_len) ? __uint_as_float(r[t]) * p.scale_log2 : -INFINITY;
          mx = fmaxf(mx, s);
        }
      }
      const float m_new = fmaxf(m_prev, mx);
      // pass 2: probabilities -> shared memory (16-bit, SWIZZLE_128B K-major), row sum
      float rs = 0.f;
      uint8_t* prow = prow_base + st * TILE_BYTES;
#pragma unroll
      for (int c = 0; c < TILE; c += 32) {
        uint32_t r[32];
        tmem_ld32(s_addr + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const bool valid = kbase + c + t < kv_len;
          const float e = valid ? ex2(fmaf(__uint_as_float(r[t]), p.scale_log2, -m_new)) : 0.f;
          rs += e;
          r[t] = __float_as_uint(e);
        }
        // 32 keys = 4 chunks of 8; chunk index within the 64-key atom: (c % 64) / 8 + q
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int key0 = c + 8 * q;
          const int atom = key0 >> 6;
          const int chunk = (key0 & 63) >> 3;
          uint4 u;
          u.x = pack2<BF16>(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
          u.y = pack2<BF16>(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
          u.z = pack2<BF16>(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
          u.w = pack2<BF16>(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
          *reinterpret_cast<uint4*>(prow + atom * ATOM + ((chunk ^ (row & 7)) << 4)) = u;
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_empty[st]);
        mbar_arrive(&p_full[st]);
      }
      l = (m_prev == -INFINITY ? 0.f : l * ex2(m_prev - m_new)) + rs;
      if (j >= 1 && !accumulate(j - 1, m_lag)) { ok = false; break; }
      m_lag = m_new;
      m_prev = m_new;
    }
    if (ok && nblk > 0) ok = accumulate(nblk - 1, m_lag);
    // normalised output row
    const int qrow = q0 + row;
    if (ok && qrow < p.Lq) {
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      const size_t base = static_cast<size_t>(b) * p.o_bstride + static_cast<size_t>(qrow) * p.ldo + static_cast<size_t>(h) * HD;
      if (p.out_dtype == ANIMA_F32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + base);
#pragma unroll
        for (int c = 0; c < HD / 4; ++c)
          dst[c] = make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv, o[4 * c + 3] * inv);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + base);
        const bool obf = p.out_dtype == ANIMA_BF16;
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) {
          uint4 u;
          if (obf) {
            u.x = pack2<true>(o[8 * c] * inv, o[8 * c + 1] * inv);
            u.y = pack2<true>(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
            u.z = pack2<true>(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
            u.w = pack2<true>(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          } else {
            u.x = pack2<false>(o[8 * c] * inv, o[8 * c + 1] * inv);
            u.y = pack2<false>(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
            u.z = pack2<false>(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
            u.w = pack2<false>(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          }
          dst[c] = u;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn
}  // namespace anima

using namespace anima;

extern "C" int anima_attention(anima_ctx* ctx, const anima_attention_args* a) {
  ANIMA_REQUIRE(ctx && a, "anima_attention: NULL argument");
  ANIMA_REQUIRE(a->head_dim == attn::HD, "anima_attention: head_dim %d (only 128)", a->head_dim);
  ANIMA_REQUIRE(a->dtype == ANIMA_BF16 || a->dtype == ANIMA_F16, "anima_attention: q/k/v dtype must be bf16 or f16");
  ANIMA_REQUIRE(a->out_dtype == ANIMA_F32 || a->out_dtype == ANIMA_BF16 || a->out_dtype == ANIMA_F16,
                "anima_attention: out_dtype %d", a->out_dtype);
  ANIMA_REQUIRE(a->batch > 0 && a->heads > 0 && a->Lq > 0 && a->Lk > 0, "anima_attention: empty problem");
  ANIMA_REQUIRE(a->q && a->k && a->v && a->out, "anima_attention: NULL data pointer");
  const long long cols_q = a->q_off + static_cast<long long>(a->heads) * a->head_dim;
  const long long cols_k = a->k_off + static_cast<long long>(a->heads) * a->head_dim;
  const long long cols_v = a->v_off + static_cast<long long>(a->heads) * a->head_dim;
  ANIMA_REQUIRE(a->ldq >= cols_q && a->ldk >= cols_k && a->ldv >= cols_v, "anima_attention: row stride too small");
  ANIMA_REQUIRE(a->q_off % 8 == 0 && a->k_off % 8 == 0 && a->v_off % 8 == 0 && a->ldq % 8 == 0 && a->ldk % 8 == 0 &&
                    a->ldv % 8 == 0,
                "anima_attention: offsets and strides must be multiples of 8 elements (16 bytes)");
  ANIMA_REQUIRE(a->batch == 1 || (a->q_bstride % 8 == 0 && a->k_bstride % 8 == 0 && a->v_bstride % 8 == 0),
                "anima_attention: batch strides must be multiples of 8 elements");
  // k_bstride == v_bstride == 0 with batch > 1: one K/V (and key_len[0]) shared by all items
  const bool kv_bcast = a->batch > 1 && a->k_bstride == 0 && a->v_bstride == 0;
  ANIMA_REQUIRE(a->batch == 1 || kv_bcast || (a->k_bstride > 0 && a->v_bstride > 0),
                "anima_attention: k and v batch strides must both be zero (shared) or both positive");
  const int kv_batch = kv_bcast ? 1 : a->batch;
  ANIMA_REQUIRE(a->ldo >= static_cast<long long>(a->heads) * a->head_dim && a->ldo % 8 == 0,
                "anima_attention: bad output stride");

  // 3D maps (cols, rows, batch) over each operand; the box is 64 columns x 128 rows.
  CUtensorMap tq, tk, tv;
  const CUtensorMapDataType dt = a->dtype == ANIMA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  uint32_t box[3] = {64, attn::TILE, 1};
  {
    uint64_t dims[3] = {static_cast<uint64_t>(a->ldq), static_cast<uint64_t>(a->Lq), static_cast<uint64_t>(a->batch)};
    uint64_t str[2] = {static_cast<uint64_t>(a->ldq) * 2,
                       static_cast<uint64_t>(a->batch > 1 ? a->q_bstride : a->ldq * a->Lq) * 2};
    int st = make_tmap(&tq, dt, 3, a->q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  {
    uint64_t dims[3] = {static_cast<uint64_t>(a->ldk), static_cast<uint64_t>(a->Lk), static_cast<uint64_t>(kv_batch)};
    uint64_t str[2] = {static_cast<uint64_t>(a->ldk) * 2,
                       static_cast<uint64_t>(kv_batch > 1 ? a->k_bstride : a->ldk * a->Lk) * 2};
    int st = make_tmap(&tk, dt, 3, a->k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  {
    uint64_t dims[3] = {static_cast<uint64_t>(a->ldv), static_cast<uint64_t>(a->Lk), static_cast<uint64_t>(kv_batch)};
    uint64_t str[2] = {static_cast<uint64_t>(a->ldv) * 2,
                       static_cast<uint64_t>(kv_batch > 1 ? a->v_bstride : a->ldv * a->Lk) * 2};
    int st = make_tmap(&tv, dt, 3, a->v, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  attn::Params p{};
  p.Lq = a->Lq;
  p.Lk = a->Lk;
  p.heads = a->heads;
  p.q_tiles = (a->Lq + attn::TILE - 1) / attn::TILE;
  p.q_col = a->q_off;
  p.k_col = a->k_off;
  p.v_col = a->v_off;
  p.out = a->out;
  p.ldo = a->ldo;
  p.o_bstride = a->batch > 1 ? a->o_bstride : 0;
  p.out_dtype = a->out_dtype;
  p.key_len = a->key_len;
  p.kv_bcast = kv_bcast ? 1 : 0;
  const float scale = a->scale > 0.f ? a->scale : 1.0f / sqrtf(static_cast<float>(a->head_dim));
  p.scale_log2 = scale * 1.4426950408889634f;

  const long long grid = static_cast<long long>(p.q_tiles) * a->heads * a->batch;
  ANIMA_REQUIRE(grid < (1LL << 31), "anima_attention: problem too large");
  ProfScope prof(ctx, "attn.flash", 4.0 * a->batch * a->heads * static_cast<double>(a->Lq) * a->Lk * a->head_dim, 0);
  if (a->dtype == ANIMA_BF16) {
    static bool set = false;
    if (!set) {
      ANIMA_CUDA(cudaFuncSetAttribute(attn::attention_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      attn::SMEM_BYTES));
      set = true;
    }
    attn::attention_kernel<true><<<static_cast<int>(grid), attn::THREADS, attn::SMEM_BYTES, ctx->stream>>>(tq, tk, tv, p);
  } else {
    static bool set = false;
    if (!set) {
      ANIMA_CUDA(cudaFuncSetAttribute(attn::attention_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      attn::SMEM_BYTES));
      set = true;
    }
    attn::attention_kernel<false><<<static_cast<int>(grid), attn::THREADS, attn::SMEM_BYTES, ctx->stream>>>(tq, tk, tv, p);
  }
  return check_launch("attention_kernel");
}
