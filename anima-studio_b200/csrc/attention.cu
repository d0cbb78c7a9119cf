// Non-causal multi-head attention on tcgen05 (kind::f16), head_dim 128: the DiT's self-attention
// (Lq = Lk = 4096 at 1024^2) and cross-attention against cached text keys (Lk = 256..512). The
// reference's counterpart is the fp32 WGSL flash kernel of app/gpu/kernels.js:147-299.
//
// One CTA = one (batch, head) and two 128-query tiles A and B; 576 threads:
//   warps 0-7   softmax for tile A, warps 8-15 for tile B. Warp w serves the 32 query rows of
//               lane quadrant w % 4 (the tensor-memory lanes it may access) and the key columns
//               [64 h, 64 h + 64) with h = (w / 4) % 2, so two warps on the same SM sub-partition
//               share each row; they exchange the row maximum through shared memory.
//   warp 16     TMA producer: Q_A, Q_B once, then K_j / V_j (128 keys) into two stages each
//   warp 17     TMEM allocator + single-thread UMMA issuer
// Tensor memory (512 columns): S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512).
// Per key block j the tensor core runs S_X = Q_X K_j^T (smem x smem), the softmax threads read S_X,
// write P_X = 2^(s - m) as 16-bit values back over the first 64 columns of S_X, and the tensor core
// accumulates O_X += P_X V_j with P_X read from tensor memory. Issue order:
//   S_A(0) S_B(0) | PV_A(j) PV_B(j) [wait PV_A(j)] S_A(j+1) [wait PV_B(j)] S_B(j+1) | ...
// so S_X(j+1) never overwrites P_X(j) before PV_X(j) has read it, and while one tile's softmax
// runs the tensor core works on the other tile. O stays in tensor memory; the running max is only
// moved (and O rescaled in place) when it grows by more than 2^8, so P stays <= 256 in between
// (lazy rescaling), and l is kept consistent with the max actually used. Keys >= key_len[b] (and
// >= Lk) get probability 0; key blocks entirely past key_len are skipped.

#include "internal.h"
#include "sm100.cuh"

namespace anima {
namespace attn {

constexpr int TILE = 128;     // query rows per tile and keys per block
constexpr int HD = 128;       // head dim
constexpr int THREADS = 576;
constexpr int SOFTMAX_WARPS = 16;
constexpr int ATOM = 16384;   // one SWIZZLE_128B atom column: 128 rows x 128 bytes
constexpr int TILE_BYTES = 2 * ATOM;
// shared memory: Q_A | Q_B | K[2] | V[2] | barriers
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + 2 * TILE_BYTES;
constexpr int OFF_V = OFF_K + 2 * TILE_BYTES;
constexpr int OFF_BAR = OFF_V + 2 * TILE_BYTES;
constexpr int OFF_RED = OFF_BAR + 256;                 // row max exchange [2 parity][2 tiles][2 halves][128]
constexpr int OFF_RED_L = OFF_RED + 2 * 2 * 2 * 128 * 4;  // row sum exchange [2 tiles][2 halves][128]
constexpr int SMEM_BYTES = OFF_RED_L + 2 * 2 * 128 * 4 + 1024;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when the max grows by > 2^8

struct Params {
  int Lq, Lk, heads, q_pairs;
  int q_col, k_col, v_col;  // column offsets of head 0
  void* out;
  long long ldo, o_bstride;
  int out_dtype;
  const int* key_len;
  int kv_bcast;      // one K/V (and key_len) shared by every batch item
  float scale_log2;  // softmax scale * log2(e)
  int pv_wait;       // issue S_x(j+1) only after PV_x(j) has completed
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

// 18 warps are allocated registers as 20: 96 x 32 x 20 = 61440 of the SM's 65536
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
  uint64_t* s_full = bars + 9;   // [2] per tile: S_X(j) complete
  uint64_t* p_full = bars + 11;  // [2] per tile: P_X(j) written (8 warp arrivals)
  uint64_t* o_done = bars + 13;  // [2] per tile: PV_X(j) complete
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qp = blockIdx.x % p.q_pairs;
  const int bh = blockIdx.x / p.q_pairs;
  const int h = bh % p.heads;
  const int b = bh / p.heads;
  const int q0 = qp * 2 * TILE;
  const int kvb = p.kv_bcast ? 0 : b;
  int kv_len = p.Lk;
  if (p.key_len) kv_len = min(kv_len, p.key_len[kvb]);
  const int nblk = kv_len > 0 ? (kv_len + TILE - 1) / TILE : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], SOFTMAX_WARPS / 2);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  constexpr int kProducerWarp = SOFTMAX_WARPS, kMmaWarp = SOFTMAX_WARPS + 1;
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    if (lane == 0 && nblk > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const int qc = p.q_col + h * HD, kc = p.k_col + h * HD, vc = p.v_col + h * HD;
      int armed[5] = {-1, -1, -1, -1, -1};  // parity of the last arm: q, k0, k1, v0, v1
      mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
      tma_load_3d(smem + OFF_Q, &tm_q, q_full, qc, q0, b);
      tma_load_3d(smem + OFF_Q + ATOM, &tm_q, q_full, qc + 64, q0, b);
      tma_load_3d(smem + OFF_Q + TILE_BYTES, &tm_q, q_full, qc, q0 + TILE, b);
      tma_load_3d(smem + OFF_Q + TILE_BYTES + ATOM, &tm_q, q_full, qc + 64, q0 + TILE, b);
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
  } else if (warp == kMmaWarp) {
    if (lane == 0 && nblk > 0) {
      const uint32_t id_qk = idesc_f16(TILE, TILE, BF16, false);
      const uint32_t id_pv = idesc_f16(TILE, HD, BF16, true);
      const uint32_t sq = smem_u32(smem + OFF_Q);
      auto issue_s = [&](int x, int j) {  // S_x(j) = Q_x K_j^T
        const uint32_t sk = smem_u32(smem + OFF_K + (j & 1) * TILE_BYTES);
        const uint32_t qx = sq + x * TILE_BYTES;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * ATOM + (k & 3) * 32;
          umma_f16(tmem + x * 128, sdesc_sw128(qx + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), id_qk,
                   k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[x]);
      };
      auto issue_pv = [&](int x, int j) {  // O_x (+)= P_x(j) V_j, P from tensor memory
        const uint32_t sv = smem_u32(smem + OFF_V + (j & 1) * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < TILE / 16; ++k) {
          const uint64_t bd = sdesc_sw128(sv + k * 16 * 128, ATOM, 1024);
          umma_f16_ts(tmem + 256 + x * 128, tmem + x * 128 + k * 8, bd, id_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[x]);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, kErrTimeoutFull) &&
                mbar_wait(&k_full[0], 0, abort_flag, kErrTimeoutFull);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&k_empty[0]);
      }
      // Per tile: PV_x(j) as soon as P_x(j) is written, then (once PV_x(j) has read P_x(j), which
      // lives in S_x's columns) S_x(j+1). The two tiles are serviced alternately, so one tile's
      // softmax runs while the tensor core works on the other tile.
      for (int j = 0; ok && j < nblk; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const uint32_t jp = j & 1;
        if (!mbar_wait(&v_full[st], ph, abort_flag, kErrTimeoutFull)) { ok = false; break; }
        const bool more = j + 1 < nblk;
        const int st1 = (j + 1) & 1;
        for (int x = 0; x < 2; ++x) {
          if (!mbar_wait(&p_full[x], jp, abort_flag, kErrTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          issue_pv(x, j);
          if (x == 1) umma_commit(&v_empty[st]);
          if (more) {
            if (x == 0 && !mbar_wait(&k_full[st1], ((j + 1) >> 1) & 1, abort_flag, kErrTimeoutFull)) {
              ok = false;
              break;
            }
            // S_x(j+1) overwrites P_x(j): the tensor core runs this thread's MMAs in issue order,
            // so PV_x(j) has read P_x(j) by then (pv_wait: wait for PV_x(j) explicitly instead)
            if (p.pv_wait) {
              if (!mbar_wait(&o_done[x], jp, abort_flag, kErrTimeoutAcc)) { ok = false; break; }
              tc_fence_after();
            }
            issue_s(x, j + 1);
            if (x == 1) umma_commit(&k_empty[st1]);
          }
        }
      }
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
    // softmax: tile x, lane quadrant `quad` (rows quad * 32 + lane), key-column half hf
    const int x = warp >> 3;
    const int hf = (warp >> 2) & 1;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_addr + x * 128 + 64 * hf;  // fp32 scores of this half
    const uint32_t p_addr = tmem + lane_addr + x * 128 + 32 * hf;  // its 64 probabilities, 2 per column
    const uint32_t o_addr = tmem + lane_addr + 256 + x * 128 + 64 * hf;
    float* red = reinterpret_cast<float*>(smem + OFF_RED);  // [parity][tile][half][row]
    const int bar_id = 1 + x * 4 + quad;                      // named barrier of the two warps of a row
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory"); };
    float m_used = -INFINITY;  // max the probabilities (and O, l) are relative to
    float l = 0.f;             // this half's share of the row sum
    bool ok = true;
    // Every iteration meets pair_sync exactly once, also after a failed wait (the warp then skips
    // the work), so the two warps of a row always agree on the barrier count.
    for (int j = 0; j < nblk; ++j) {
      const uint32_t jp = j & 1;
      if (ok && !warp_wait(&s_full[x], jp, abort_flag, kErrTimeoutFull)) ok = false;
      if (!ok) {
        pair_sync();
        continue;
      }
      tc_fence_after();
      uint32_t sr[2][32];
#pragma unroll
      for (int c = 0; c < 2; ++c) tmem_ld32(s_addr + 32 * c, sr[c]);
#pragma unroll
      for (int c = 0; c < 2; ++c) tmem_ld_wait(sr[c]);
      const int kbase = j * TILE + 64 * hf;
      const bool masked = j * TILE + TILE > kv_len;  // only the last block can hold keys past kv_len
      if (masked) {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int t = 0; t < 32; ++t)
            if (kbase + 32 * c + t >= kv_len) sr[c][t] = __float_as_uint(-INFINITY);
      }
      float mx;
      {  // four independent partial maxima, two new values per max
        float pm[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pm[i] = -INFINITY;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int t = 0; t < 32; t += 2)
            pm[(t >> 1) & 3] = fmax3(pm[(t >> 1) & 3], __uint_as_float(sr[c][t]), __uint_as_float(sr[c][t + 1]));
        mx = fmax3(fmaxf(pm[0], pm[1]), pm[2], pm[3]);
      }
      // the row maximum over both halves (double-buffered by block parity: the partner reads this
      // block's value before it can reach the next block's barrier). The barrier also orders both
      // warps' reads of S before either overwrites S's first 64 columns with P.
      red[((jp * 2 + x) * 2 + hf) * 128 + row] = mx;
      tc_fence_before();
      pair_sync();
      tc_fence_after();
      mx = fmaxf(mx, red[((jp * 2 + x) * 2 + (hf ^ 1)) * 128 + row]) * p.scale_log2;
      // lazy rescale: keep the old max unless the new one is more than 2^8 larger (both halves
      // see the same maximum and take the same decision)
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_used + kRescaleThreshold) {
        rescale = j > 0;
        alpha = (m_used == -INFINITY) ? 0.f : ex2(m_used - mx);
        m_used = mx;
      }
      f2 rsp[2] = {dup2(0.f), dup2(0.f)};  // partial row sums
      const f2 sc2 = dup2(p.scale_log2), nm2 = dup2(-m_used);
      // P over the first 64 columns of S (two 16-bit probabilities per column), 32 keys at a time
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const f2 a = fma2(make_float2(__uint_as_float(sr[c][t]), __uint_as_float(sr[c][t + 1])), sc2, nm2);
          float e0 = ex2(a.x), e1 = ex2(a.y);
          if (masked) {  // -inf scores: exactly zero probability
            if (kbase + 32 * c + t >= kv_len) e0 = 0.f;
            if (kbase + 32 * c + t + 1 >= kv_len) e1 = 0.f;
          }
          rsp[(t >> 1) & 1] = add2(rsp[(t >> 1) & 1], make_float2(e0, e1));
          pk[t / 2] = pack2<BF16>(e0, e1);
        }
        tmem_st16(p_addr + 16 * c, pk);
      }
      l = l * alpha + ((rsp[0].x + rsp[0].y) + (rsp[1].x + rsp[1].y));
      if (rescale) {
        // O holds sum_{i<j} P_i V_i relative to the old max: wait for PV(j-1), then scale in place
        if (!warp_wait(&o_done[x], jp ^ 1, abort_flag, kErrTimeoutAcc)) {
          ok = false;
          continue;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t orr[32];
          tmem_ld32(o_addr + 32 * c, orr);
          tmem_ld_wait(orr);
#pragma unroll
          for (int t = 0; t < 32; ++t) orr[t] = __float_as_uint(__uint_as_float(orr[t]) * alpha);
          tmem_st32(o_addr + 32 * c, orr);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    // the row sum over both halves; a warp that failed still takes part so its partner is released
    float* red_l = reinterpret_cast<float*>(smem + OFF_RED_L);
    red_l[(x * 2 + hf) * 128 + row] = l;
    pair_sync();
    const float l_row = l + red_l[(x * 2 + (hf ^ 1)) * 128 + row];
    // normalised output (this half's 64 columns) once the last PV has landed
    if (ok && nblk > 0 && warp_wait(&o_done[x], (nblk - 1) & 1, abort_flag, kErrTimeoutAcc)) {
      tc_fence_after();
      const int qrow = q0 + x * TILE + row;
      const float inv = l_row > 0.f ? 1.0f / l_row : 0.f;
      const size_t base = static_cast<size_t>(b) * p.o_bstride + static_cast<size_t>(qrow) * p.ldo +
                          static_cast<size_t>(h) * HD + 64 * hf;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t orr[32];
        tmem_ld32(o_addr + 32 * c, orr);
        tmem_ld_wait(orr);
        if (qrow < p.Lq) {
          if (p.out_dtype == ANIMA_F32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + base + 32 * c);
#pragma unroll
            for (int t = 0; t < 8; ++t)
              dst[t] = make_float4(__uint_as_float(orr[4 * t]) * inv, __uint_as_float(orr[4 * t + 1]) * inv,
                                   __uint_as_float(orr[4 * t + 2]) * inv, __uint_as_float(orr[4 * t + 3]) * inv);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + base + 32 * c);
            const bool obf = p.out_dtype == ANIMA_BF16;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(orr[8 * t + e]) * inv;
              uint4 u;
              if (obf) {
                u.x = pack2<true>(v[0], v[1]);
                u.y = pack2<true>(v[2], v[3]);
                u.z = pack2<true>(v[4], v[5]);
                u.w = pack2<true>(v[6], v[7]);
              } else {
                u.x = pack2<false>(v[0], v[1]);
                u.y = pack2<false>(v[2], v[3]);
                u.z = pack2<false>(v[4], v[5]);
                u.w = pack2<false>(v[6], v[7]);
              }
              dst[t] = u;
            }
          }
        }
      }
    } else if (nblk == 0) {
      // no keys: zero rows (the softmax of an empty set is taken as 0)
      const int qrow = q0 + x * TILE + row;
      if (qrow < p.Lq) {
        const size_t base = static_cast<size_t>(b) * p.o_bstride + static_cast<size_t>(qrow) * p.ldo +
                            static_cast<size_t>(h) * HD + 64 * hf;
        const int esz = p.out_dtype == ANIMA_F32 ? 4 : 2;
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + base * esz);
        for (int t = 0; t < 64 * esz / 16; ++t) dst[t] = make_uint4(0, 0, 0, 0);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
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
  p.q_pairs = (a->Lq + 2 * attn::TILE - 1) / (2 * attn::TILE);
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
  static const int pv_wait = [] {
    const char* e = getenv("ANIMA_ATTN_PV_WAIT");
    return e && atoi(e) != 0 ? 1 : 0;
  }();
  p.pv_wait = pv_wait;

  const long long grid = static_cast<long long>(p.q_pairs) * a->heads * a->batch;
  ANIMA_REQUIRE(grid < (1LL << 31), "anima_attention: problem too large");
  ProfScope prof(ctx, "attn.flash", 4.0 * a->batch * a->heads * static_cast<double>(a->Lq) * a->Lk * a->head_dim, 0);
  using Kfn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const attn::Params);
  const int kind = a->dtype == ANIMA_BF16 ? 1 : 0;
  const Kfn fns[2] = {attn::attention_kernel<false>, attn::attention_kernel<true>};
  static bool set[2] = {};
  const Kfn fn = fns[kind];
  if (!set[kind]) {
    ANIMA_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, attn::SMEM_BYTES));
    set[kind] = true;
  }
  fn<<<static_cast<int>(grid), attn::THREADS, attn::SMEM_BYTES, ctx->stream>>>(tq, tk, tv, p);
  return check_launch("attention_kernel");
}
