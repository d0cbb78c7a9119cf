// Multi-head attention on tcgen05 (kind::f16), head_dim 128: the DiT's self-attention (Lq = Lk =
// 4096 at 1024^2), cross-attention against cached text keys (Lk = 256..512), and the Qwen3 text
// encoder's causal attention with 16 q heads over 8 k/v heads (k/v head = h / group; a causal unit
// stops at the key block of its last query and masks each row's later keys). The reference's
// counterpart is the fp32 WGSL flash kernel of app/gpu/kernels.js:147-299.
//
// A unit = one (batch, head) and two 128-query tiles A and B. A CTA runs one unit; with more than
// one wave of units, every grid-th unit (one CTA per SM); or, under stream-K (below), an equal
// share of all units' key blocks. 576 threads:
//   warps 0-7   softmax for tile A, warps 8-15 for tile B. Warp w serves the 32 query rows of
//               lane quadrant w % 4 (the tensor-memory lanes it may access) and the key columns
//               [64 h, 64 h + 64) with h = (w / 4) % 2, so two warps on the same SM sub-partition
//               share each row; they exchange the row maximum through shared memory.
//   warp 16     TMA producer: Q_A, Q_B per unit, then K_j / V_j (128 keys) into two stages each
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

#include <mutex>

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
constexpr int OFF_SEG = OFF_RED_L + 2 * 2 * 128 * 4;   // this CTA's segments (int4 each)
constexpr int MAX_SEGS = 64;
constexpr int SMEM_BYTES = OFF_SEG + MAX_SEGS * 16 + 1024;
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
  // stream-K: the units' key blocks split evenly over the CTAs (no key mask; every unit has ublk)
  int stream_k, units, ublk;
  int persist;       // whole units, CTA c taking units c, c + grid, ... (grid = SM count)
  int group;         // q heads per k/v head (k/v head = h / group)
  int causal;        // key j visible to query i only when j <= i
  float* ws;         // [units][PART_FLOATS] partial softmax states of split units
  unsigned* flags;   // [units] tail part written (cleared by the head part)
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

// One arrival for the warp, from one elected lane (predicated, no branch).
__device__ __forceinline__ void arrive_one_lane(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "@p mbarrier.arrive.shared::cta.b64 _, [%0];\n\t}\n" ::"r"(smem_u32(bar))
      : "memory");
}

// Warp-wide bounded wait: every lane polls, so the common case (phase already complete) has no
// divergent branch; the result is the AND over the lanes.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned err) {
  const uint32_t a = smem_u32(bar);
  if (__all_sync(0xffffffffu, mbar_test(a, parity))) return true;
  // spin without the suspend hint: the wait is on the critical path
  bool ok = true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_test(a, parity)) {
    if (*abort_flag) {
      ok = false;
      break;
    }
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      flag_error(err);
      *abort_flag = 1;
      ok = false;
      break;
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// A CTA's work is a list of segments: (unit, first key block, end key block), a unit being one
// (batch, head, pair of query tiles). Without stream-K each CTA runs whole units (one, or every
// grid-th on a persistent grid). With stream-K
// (long self-attention without a key mask) the units' key blocks are laid end to end and cut into
// one equal range per CTA, so every SM gets the same number of key blocks instead of whole units
// in ceil(units / SMs) waves. The range of CTA c reads: [tail of unit u] whole units... [head of
// unit u']. A cut unit has exactly two parts (a range is at least one unit long): CTA c runs its
// head part and writes the unnormalised O, running max and row sum to workspace slot c, then
// raises one flag per softmax warp; CTA c + 1 runs the tail part LAST in its own range, waits for
// those flags (CTA c, dispatched earlier, has finished its head part by then), merges the two
// softmax states and writes the output. The roles of a CTA pass from one segment to the next
// without a block-wide barrier: the producer reloads Q once the last QK^T of the previous segment
// has completed (q_empty), and the first PV of a segment, issued after its P, finds O already read.
struct Seg {
  int unit, kb0, kb1, kind;
};
constexpr int kWhole = 0, kHeadPart = 1, kTailPart = 2;
// workspace slot: O of both tiles as float4 [tile][half][16 column quads][128 rows], then the max
// and the row sum [tile][half][128 rows] each
constexpr int PART_FLOATS = 2 * TILE * HD + 2 * 2 * 2 * TILE;
constexpr int PART_M = 2 * TILE * HD;
constexpr int PART_L = PART_M + 2 * 2 * TILE;

__device__ __forceinline__ Seg segment_at(const Params& p, long long g, long long end) {
  Seg s;
  s.unit = static_cast<int>(g / p.ublk);
  const long long u0 = static_cast<long long>(s.unit) * p.ublk;
  s.kb0 = static_cast<int>(g - u0);
  s.kb1 = static_cast<int>((end < u0 + p.ublk ? end : u0 + p.ublk) - u0);
  s.kind = s.kb0 > 0 ? kTailPart : (s.kb1 < p.ublk ? kHeadPart : kWhole);
  return s;
}

// The segments of this CTA in the order it runs them (a leading tail part moved to the end),
// written to shared memory by one thread; returns their count (at most MAX_SEGS, which the host
// guarantees for stream-K launches). A whole unit's key blocks end at key_len (blocks entirely past
// it are skipped).
__device__ __forceinline__ int build_segments(const Params& p, int4* out) {
  if (!p.stream_k) {
    // whole units: this CTA's one unit, or (persistent grid) every grid-th unit, so a CTA's next
    // unit loads its Q and starts its first QK^T while the previous unit's output is written
    const int step = p.persist ? static_cast<int>(gridDim.x) : p.units;
    int n = 0;
    for (int unit = blockIdx.x; unit < p.units && n < MAX_SEGS; unit += step) {
      const int b = unit / p.q_pairs / p.heads;
      const int kv_len = p.key_len ? min(p.Lk, p.key_len[p.kv_bcast ? 0 : b]) : p.Lk;
      int nblk = kv_len > 0 ? (kv_len + TILE - 1) / TILE : 0;
      if (p.causal) nblk = min(nblk, 2 * (unit % p.q_pairs) + 2);  // keys up to the pair's last query
      out[n++] = make_int4(unit, 0, nblk, kWhole);
    }
    return n;
  }
  const long long total = static_cast<long long>(p.units) * p.ublk;
  long long g = total * blockIdx.x / gridDim.x;
  const long long end = total * (blockIdx.x + 1) / gridDim.x;
  int n = 0;
  const Seg first = segment_at(p, g, end);
  const bool defer = first.kind == kTailPart;
  if (defer) g = static_cast<long long>(first.unit) * p.ublk + first.kb1;
  while (g < end && n < MAX_SEGS - 1) {
    const Seg sg = segment_at(p, g, end);
    out[n++] = make_int4(sg.unit, sg.kb0, sg.kb1, sg.kind);
    g = static_cast<long long>(sg.unit) * p.ublk + sg.kb1;
  }
  if (g < end) flag_error(kErrBadArgs);  // more segments than MAX_SEGS: the host prevents this
  if (defer) out[n++] = make_int4(first.unit, first.kb0, first.kb1, first.kind);
  return n;
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* q) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(q) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u32(unsigned* q, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(q), "r"(v) : "memory");
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
  uint64_t* q_empty = bars + 16;  // the segment's last QK^T has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* nseg_slot = reinterpret_cast<int*>(tmem_slot + 2);
  int4* segs = reinterpret_cast<int4*>(smem + OFF_SEG);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
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
    *nseg_slot = build_segments(p, segs);
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
  const int nseg = *nseg_slot;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      // the last arm of q_full, k_full[0], k_full[1], v_full[0], v_full[1]: 2 bits each (armed, parity)
      uint32_t armed = 0;
      auto arm = [&](int i, uint32_t ph) { armed = (armed & ~(3u << (2 * i))) | ((2u | ph) << (2 * i)); };
      int gb = 0, qn = 0;                   // key blocks and Q loads so far
      for (int si = 0; si < nseg && !*abort_flag; ++si) {
        const int4 sg = segs[si];  // unit, kb0, kb1, kind
        const int qp = sg.x % p.q_pairs, bh = sg.x / p.q_pairs;
        const int h = bh % p.heads, b = bh / p.heads;
        const int kvb = p.kv_bcast ? 0 : b;
        const int nb = sg.z - sg.y;
        if (nb <= 0) continue;
        const int q0 = qp * 2 * TILE;
        const int qc = p.q_col + h * HD, kc = p.k_col + (h / p.group) * HD, vc = p.v_col + (h / p.group) * HD;
        if (qn > 0 && !mbar_wait(q_empty, (qn - 1) & 1, abort_flag, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
        tma_load_3d(smem + OFF_Q, &tm_q, q_full, qc, q0, b);
        tma_load_3d(smem + OFF_Q + ATOM, &tm_q, q_full, qc + 64, q0, b);
        tma_load_3d(smem + OFF_Q + TILE_BYTES, &tm_q, q_full, qc, q0 + TILE, b);
        tma_load_3d(smem + OFF_Q + TILE_BYTES + ATOM, &tm_q, q_full, qc + 64, q0 + TILE, b);
        arm(0, qn & 1);
        ++qn;
        for (int j = 0; j < nb; ++j) {
          const int G = gb + j, kb = sg.y + j;
          const int st = G & 1;
          const uint32_t ph = (G >> 1) & 1;
          if (!mbar_wait(&k_empty[st], ph ^ 1, abort_flag, kErrTimeoutEmpty)) break;
          mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
          tma_load_3d(smem + OFF_K + st * TILE_BYTES, &tm_k, &k_full[st], kc, kb * TILE, kvb);
          tma_load_3d(smem + OFF_K + st * TILE_BYTES + ATOM, &tm_k, &k_full[st], kc + 64, kb * TILE, kvb);
          arm(1 + st, ph);
          if (!mbar_wait(&v_empty[st], ph ^ 1, abort_flag, kErrTimeoutEmpty)) break;
          mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
          tma_load_3d(smem + OFF_V + st * TILE_BYTES, &tm_v, &v_full[st], vc, kb * TILE, kvb);
          tma_load_3d(smem + OFF_V + st * TILE_BYTES + ATOM, &tm_v, &v_full[st], vc + 64, kb * TILE, kvb);
          arm(3 + st, ph);
        }
        gb += nb;
      }
      if (*abort_flag) {
        // let every copy this thread started land before the CTA exits
        for (int i = 0; i < 5; ++i) {
          const uint32_t a = (armed >> (2 * i)) & 3u;
          if (!(a & 2u)) continue;
          uint64_t* fb = bars + (i < 3 ? i : i + 2);  // q_full, k_full[0..1], v_full[0..1]
          const unsigned long long t0 = globaltimer();
          while (!mbar_test(smem_u32(fb), a & 1u)) {
            if (globaltimer() - t0 > kWaitTimeoutNs) {
              flag_error(kErrTimeoutDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(TILE, TILE, BF16, false);
      const uint32_t id_pv = idesc_f16(TILE, HD, BF16, true);
      const uint32_t sq = smem_u32(smem + OFF_Q);
      auto issue_s = [&](int x, int G) {  // S_x = Q_x K^T for the block in stage G & 1
        const uint32_t sk = smem_u32(smem + OFF_K + (G & 1) * TILE_BYTES);
        const uint32_t qx = sq + x * TILE_BYTES;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * ATOM + (k & 3) * 32;
          umma_f16(tmem + x * 128, sdesc_sw128(qx + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), id_qk,
                   k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[x]);
      };
      auto issue_pv = [&](int x, int G, bool first) {  // O_x (+)= P_x V, P from tensor memory
        const uint32_t sv = smem_u32(smem + OFF_V + (G & 1) * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < TILE / 16; ++k) {
          const uint64_t bd = sdesc_sw128(sv + k * 16 * 128, ATOM, 1024);
          umma_f16_ts(tmem + 256 + x * 128, tmem + x * 128 + k * 8, bd, id_pv, (!first || k > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[x]);
      };
      int gb = 0, qn = 0;
      bool ok = true;
      for (int si = 0; ok && si < nseg; ++si) {
        const int nb = segs[si].z - segs[si].y;
        if (nb <= 0) continue;
        ok = mbar_wait(q_full, qn & 1, abort_flag, kErrTimeoutFull) &&
             mbar_wait(&k_full[gb & 1], (gb >> 1) & 1, abort_flag, kErrTimeoutFull);
        if (!ok) break;
        ++qn;
        // S(0) of this segment queues behind the previous segment's last PV on the tensor core
        tc_fence_after();
        issue_s(0, gb);
        issue_s(1, gb);
        umma_commit(&k_empty[gb & 1]);
        if (nb == 1) umma_commit(q_empty);
        // Per tile: PV_x(j) as soon as P_x(j) is written, then S_x(j+1) into the same columns (the
        // tensor core runs this thread's MMAs in issue order, so PV_x(j) has read P_x(j) first).
        // The two tiles are serviced alternately: one tile's softmax overlaps the other's MMAs.
        // P_x(0) is written after the softmax warps have read the previous segment's O_x, so the
        // first PV (which overwrites O_x) comes after that read.
        for (int j = 0; ok && j < nb; ++j) {
          const int G = gb + j;
          const int st = G & 1;
          const uint32_t ph = (G >> 1) & 1;
          const uint32_t jp = G & 1;
          if (!mbar_wait(&v_full[st], ph, abort_flag, kErrTimeoutFull)) { ok = false; break; }
          const bool more = j + 1 < nb;
          const int st1 = (G + 1) & 1;
          for (int x = 0; x < 2; ++x) {
            if (!mbar_wait(&p_full[x], jp, abort_flag, kErrTimeoutFull)) { ok = false; break; }
            tc_fence_after();
            issue_pv(x, G, j == 0);
            if (x == 1) umma_commit(&v_empty[st]);
            if (more) {
              if (x == 0 && !mbar_wait(&k_full[st1], ((G + 1) >> 1) & 1, abort_flag, kErrTimeoutFull)) {
                ok = false;
                break;
              }
              issue_s(x, G + 1);
              if (x == 1) {
                umma_commit(&k_empty[st1]);
                if (j + 2 == nb) umma_commit(q_empty);
              }
            }
          }
        }
        gb += nb;
      }
      if (!ok) {
        // every MMA this thread issued completes before the CTA frees tensor memory
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
    float* red = reinterpret_cast<float*>(smem + OFF_RED);      // [parity][tile][half][row]
    float* red_l = reinterpret_cast<float*>(smem + OFF_RED_L);  // [tile][half][row]
    const int bar_id = 1 + x * 4 + quad;                        // named barrier of the two warps of a row
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory"); };
    bool ok = true;
    int gb = 0;
    for (int si = 0; si < nseg; ++si) {
      const int kb0 = segs[si].y;
      const int nb = segs[si].z - kb0;
      // keys past kv_len get probability 0; only the last block of a unit can hold such keys
      int kv_len = p.Lk;
      if (p.key_len) kv_len = min(kv_len, p.key_len[p.kv_bcast ? 0 : segs[si].x / p.q_pairs / p.heads]);
      // causal: this thread's row sees keys up to its own index
      if (p.causal) kv_len = min(kv_len, (segs[si].x % p.q_pairs) * 2 * TILE + x * TILE + row + 1);
      // where this warp's output rows go (read again from shared memory after the key loop)
      auto out_base = [&](int& qrow) {
        const int unit = segs[si].x;
        const int qp = unit % p.q_pairs, bh = unit / p.q_pairs;
        const int h = bh % p.heads, b = bh / p.heads;
        qrow = qp * 2 * TILE + x * TILE + row;
        return static_cast<size_t>(b) * p.o_bstride + static_cast<size_t>(qrow) * p.ldo + static_cast<size_t>(h) * HD +
               64 * hf;
      };
      if (nb <= 0) {
        int qrow;
        const size_t obase = out_base(qrow);
        // no keys: zero rows (the softmax of an empty set is taken as 0)
        if (qrow < p.Lq) {
          const int esz = p.out_dtype == ANIMA_F32 ? 4 : 2;
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + obase * esz);
          for (int t = 0; t < 64 * esz / 16; ++t) dst[t] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      float m_used = -INFINITY;  // max the probabilities (and O, l) are relative to
      float l = 0.f;             // this half's share of the row sum
      // Every iteration meets pair_sync exactly once, also after a failed wait (the warp then skips
      // the work), so the two warps of a row always agree on the barrier count.
      for (int j = 0; j < nb; ++j) {
        const int G = gb + j;
        const uint32_t jp = G & 1;
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
        const int kbase = (kb0 + j) * TILE + 64 * hf;
        const bool masked = (kb0 + j) * TILE + TILE > kv_len;
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
        // lazy rescale: keep the old max unless the new one is more than 2^8 larger for some row of
        // the warp; then every row of the warp moves to its larger maximum (a warp-uniform decision,
        // identical in the two warps of a row, which see the same maxima)
        float alpha = 1.f;
        bool rescale = false;
        if (__any_sync(0xffffffffu, mx > m_used + kRescaleThreshold)) {
          const float m_new = fmaxf(m_used, mx);
          rescale = j > 0;
          alpha = (m_used == -INFINITY) ? 0.f : ex2(m_used - m_new);
          m_used = m_new;
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
        arrive_one_lane(&p_full[x]);
      }
      gb += nb;
      // the row sum over both halves (a warp that failed still takes part, releasing its partner).
      // red_l is reused by the next segment only after both warps passed that segment's first
      // pair_sync, which each reaches after reading red_l here.
      red_l[(x * 2 + hf) * 128 + row] = l;
      pair_sync();
      const float l_row = l + red_l[(x * 2 + (hf ^ 1)) * 128 + row];
      // the finished O (this half's 64 columns) once the last PV has landed
      if (!ok || !warp_wait(&o_done[x], (gb - 1) & 1, abort_flag, kErrTimeoutAcc)) {
        ok = false;
        continue;
      }
      tc_fence_after();
      const int kind = segs[si].w;
      if (kind == kHeadPart) {
        // unnormalised partial for the CTA that runs the unit's tail part
        float* slot = p.ws + static_cast<size_t>(blockIdx.x) * PART_FLOATS;
        float4* po = reinterpret_cast<float4*>(slot) + (x * 2 + hf) * 16 * TILE + row;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t orr[32];
          tmem_ld32(o_addr + 32 * c, orr);
          tmem_ld_wait(orr);
#pragma unroll
          for (int t = 0; t < 8; ++t)
            __stcg(po + (c * 8 + t) * TILE, make_float4(__uint_as_float(orr[4 * t]), __uint_as_float(orr[4 * t + 1]),
                                                       __uint_as_float(orr[4 * t + 2]), __uint_as_float(orr[4 * t + 3])));
        }
        __stcg(slot + PART_M + (x * 2 + hf) * TILE + row, m_used);
        __stcg(slot + PART_L + (x * 2 + hf) * TILE + row, l_row);
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_u32(p.flags + blockIdx.x * SOFTMAX_WARPS + warp, 1u);
        continue;
      }
      float fa = 1.f, fb = 0.f, inv = l_row > 0.f ? 1.0f / l_row : 0.f;
      const float4* pb = nullptr;
      if (kind == kTailPart) {
        // wait (bounded) for the head part's partial from the previous CTA, then merge
        const float* slot = p.ws + static_cast<size_t>(blockIdx.x - 1) * PART_FLOATS;
        unsigned* flag = p.flags + (blockIdx.x - 1) * SOFTMAX_WARPS + warp;
        int got = 1;
        if (lane == 0) {
          const unsigned long long t0 = globaltimer();
          while (ld_acquire_u32(flag) != 1u) {
            if (*abort_flag) {
              got = 0;
              break;
            }
            if (globaltimer() - t0 > kWaitTimeoutNs) {
              flag_error(kErrTimeoutAcc);
              *abort_flag = 1;
              got = 0;
              break;
            }
            __nanosleep(256);
          }
          if (got) *reinterpret_cast<volatile unsigned*>(flag) = 0u;  // consumed: clear for the next launch
        }
        __syncwarp();
        if (!__shfl_sync(0xffffffffu, got, 0)) {
          ok = false;
          continue;
        }
        const float mb = __ldcg(slot + PART_M + (x * 2 + hf) * TILE + row);
        const float lb = __ldcg(slot + PART_L + (x * 2 + hf) * TILE + row);
        const float m = fmaxf(m_used, mb);
        fa = ex2(m_used - m);
        fb = ex2(mb - m);
        const float lt = l_row * fa + lb * fb;
        inv = lt > 0.f ? 1.0f / lt : 0.f;
        pb = reinterpret_cast<const float4*>(slot) + (x * 2 + hf) * 16 * TILE + row;
      }
      int qrow;
      const size_t obase = out_base(qrow);
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t orr[32];
        tmem_ld32(o_addr + 32 * c, orr);
        tmem_ld_wait(orr);
        if (qrow >= p.Lq) continue;
        float v[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) v[t] = __uint_as_float(orr[t]) * fa;
        if (pb) {
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float4 o = __ldcg(pb + (c * 8 + t) * TILE);
            v[4 * t] = fmaf(o.x, fb, v[4 * t]);
            v[4 * t + 1] = fmaf(o.y, fb, v[4 * t + 1]);
            v[4 * t + 2] = fmaf(o.z, fb, v[4 * t + 2]);
            v[4 * t + 3] = fmaf(o.w, fb, v[4 * t + 3]);
          }
        }
        if (p.out_dtype == ANIMA_F32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + obase + 32 * c);
#pragma unroll
          for (int t = 0; t < 8; ++t)
            dst[t] = make_float4(v[4 * t] * inv, v[4 * t + 1] * inv, v[4 * t + 2] * inv, v[4 * t + 3] * inv);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + obase + 32 * c);
          const bool obf = p.out_dtype == ANIMA_BF16;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = obf ? pack2<true>(v[8 * t + 2 * e] * inv, v[8 * t + 2 * e + 1] * inv)
                         : pack2<false>(v[8 * t + 2 * e] * inv, v[8 * t + 2 * e + 1] * inv);
            dst[t] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
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


// Stream-K pays when whole units leave the last wave of CTAs far from full. Legal without a key
// mask or causality (every unit has the same key blocks) and with at least one unit per SM (a unit is then cut
// into two parts at most); chosen (mode -1) when the last wave would leave more than 5% of the
// SMs idle and units are long enough (>= 16 key blocks) to hide the cost of a cut: each segment
// reloads Q and refills the pipeline, and a cut unit writes and reads back a 130 KB partial.
// (Cross-attention over 512 keys, 4 blocks per unit, measured slower with it.)
bool use_stream_k(const anima_ctx* ctx, const anima_attention_args* a, long long units, int ublk) {
  const int mode = ctx->attn_split;
  const int sms = ctx->num_sms;
  // a CTA then runs at most units / sms + 3 segments
  if (mode == 0 || a->key_len || a->causal || units < sms || units > static_cast<long long>(MAX_SEGS - 4) * sms ||
      ublk < 1)
    return false;
  if (mode == 1) return true;
  const long long waves = (units + sms - 1) / sms;
  return ublk >= 16 && units % sms != 0 && static_cast<double>(units) / static_cast<double>(waves * sms) < 0.95;
}

// One workspace slot per CTA (a CTA writes at most one partial) and one flag per softmax warp of
// each slot, allocated once per context (its size depends only on the SM count) and zeroed; the
// kernel leaves every flag at zero again. Allocation happens outside stream capture only: a graph
// captured later keeps these pointers, which live as long as the context.
int stream_k_scratch(anima_ctx* ctx) {
  if (ctx->attn_ws) return ANIMA_OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  ANIMA_CUDA(cudaStreamIsCapturing(ctx->stream, &cap));
  ANIMA_REQUIRE(cap == cudaStreamCaptureStatusNone,
                "anima_attention: first stream-K call inside stream capture (run once before capturing)");
  const size_t ws_bytes = static_cast<size_t>(ctx->num_sms) * PART_FLOATS * sizeof(float);
  const size_t flag_bytes = static_cast<size_t>(ctx->num_sms) * SOFTMAX_WARPS * sizeof(unsigned);
  ANIMA_CUDA(cudaMalloc(&ctx->attn_ws, ws_bytes));
  ANIMA_CUDA(cudaMalloc(&ctx->attn_flags, flag_bytes));
  ANIMA_CUDA(cudaMemset(ctx->attn_flags, 0, flag_bytes));
  return ANIMA_OK;
}

// Static workspace of anima_attention_noalloc: the flags of up to kStaticMaxSms CTAs, then one
// partial slot per CTA (21.6 MB in the module's device data). Calls that use it must not overlap
// (same device, any context or stream): they would share flags and slots.
constexpr int kStaticMaxSms = 160;
constexpr size_t kStaticFlagBytes = static_cast<size_t>(kStaticMaxSms) * SOFTMAX_WARPS * sizeof(unsigned);
constexpr size_t kStaticScratchBytes =
    kStaticFlagBytes + static_cast<size_t>(kStaticMaxSms) * PART_FLOATS * sizeof(float);
static_assert(kStaticFlagBytes % 256 == 0, "partial slots stay 256-byte aligned");
static __device__ __align__(256) unsigned char g_attn_static_ws[kStaticScratchBytes];

// The static workspace's device address. In host code g_attn_static_ws names a host-side stand-in,
// not device memory, so the address comes from cudaGetSymbolAddress: once per device, with that
// device made current, on the first call that needs the workspace there. That first call also
// clears the flags, which must start at zero, with a memset on the context's stream (nothing is
// allocated); every launch leaves them at zero again, and anima_sync clears them after a device
// error. The first call on a device should therefore come before any stream capture.
constexpr int kStaticMaxDevices = 64;
int static_scratch(anima_ctx* ctx) {
  ANIMA_REQUIRE(ctx->num_sms <= kStaticMaxSms,
                "anima_attention_noalloc: stream-K needs %d workspace slots (one per SM), the static workspace "
                "holds %d",
                ctx->num_sms, kStaticMaxSms);
  ANIMA_REQUIRE(ctx->device >= 0 && ctx->device < kStaticMaxDevices, "anima_attention_noalloc: device %d",
                ctx->device);
  // the entry point has made ctx->device current (ANIMA_ON_DEVICE), so the symbol resolves there
  static std::mutex mu;
  static void* addr[kStaticMaxDevices] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[ctx->device]) {
    void* base = nullptr;
    ANIMA_CUDA(cudaGetSymbolAddress(&base, g_attn_static_ws));
    ANIMA_CUDA(cudaMemsetAsync(base, 0, kStaticFlagBytes, ctx->stream));
    ANIMA_REQUIRE(base != nullptr, "anima_attention_noalloc: no device address for the static workspace");
    addr[ctx->device] = base;
  }
  ctx->attn_static_ws = addr[ctx->device];  // also lets anima_sync clear the flags after an error
  return ANIMA_OK;
}

}  // namespace attn
}  // namespace anima

// ------------------------------------------------------------------ text-model attention
// The Qwen3 text encoder (causal, 16 q heads over 8 k/v heads, d = 128) and the LLM adapter
// (d = 64, self and cross) attend over a few hundred tokens once per prompt; the reference runs
// them through the same flashAttentionShader with `group` and `causal` (kernels.js:147-299).
// Here a CUDA-core kernel: a CTA takes 16 queries of one head (4 per warp), streams the keys and
// values in 32-key tiles through shared memory (fp32), each lane scores one key of the tile for
// the warp's 4 queries, and the online softmax (running max and sum, exp2 domain) accumulates
// D / 32 output dimensions per lane.
namespace tattn {

constexpr int KT = 32;
constexpr int QPW = 4;
constexpr int WARPS = 4;
constexpr int QPC = QPW * WARPS;

struct Args {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  long long ldq, ldk, ldv, ldo, q_bs, k_bs, v_bs, o_bs;
  int q_off, k_off, v_off;
  int Lq, Lk, group, causal, kv_bcast;
  const int* key_len;
  float scale_log2;
};

__device__ __forceinline__ float cvt_in(float v) { return v; }
__device__ __forceinline__ float cvt_in(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float cvt_in(__half v) { return __half2float(v); }
template <typename T>
__device__ __forceinline__ T cvt_out(float v);
template <>
__device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half cvt_out<__half>(float v) { return __float2half_rn(v); }

// Shared memory: K tile [KT][D + 1] (+1: lane j reads row j, so the column walk is conflict-free),
// V tile [KT][D], the CTA's queries [QPC][D]; fp32. 41 KB at D = 128, 123 KB at D = 384.
template <int D>
constexpr int smem_bytes() {
  return (KT * (D + 1) + KT * D + QPC * D) * 4;
}

template <typename TI, typename TO, int D>
__global__ void __launch_bounds__(WARPS * 32) text_attention_kernel(const Args a) {
  extern __shared__ float sm[];
  float(*ks)[D + 1] = reinterpret_cast<float(*)[D + 1]>(sm);
  float(*vs)[D] = reinterpret_cast<float(*)[D]>(sm + KT * (D + 1));
  float(*qs)[D] = reinterpret_cast<float(*)[D]>(sm + KT * (D + 1) + KT * D);
  constexpr int DPL = D / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * QPC;
  const int hk = h / a.group;
  const int kb = a.kv_bcast ? 0 : b;
  const TI* Q = static_cast<const TI*>(a.q) + b * a.q_bs + a.q_off + static_cast<long long>(h) * D;
  const TI* K = static_cast<const TI*>(a.k) + kb * a.k_bs + a.k_off + static_cast<long long>(hk) * D;
  const TI* V = static_cast<const TI*>(a.v) + kb * a.v_bs + a.v_off + static_cast<long long>(hk) * D;
  int kend = a.Lk;
  if (a.key_len) kend = min(kend, a.key_len[kb]);
  if (a.causal) kend = min(kend, min(q0 + QPC, a.Lq));  // keys past the CTA's last query stay hidden
  for (int i = threadIdx.x; i < QPC * D; i += WARPS * 32) {
    const int r = i / D, c = i % D, qi = q0 + r;
    qs[r][c] = qi < a.Lq ? cvt_in(Q[qi * a.ldq + c]) * a.scale_log2 : 0.f;
  }
  float m[QPW], l[QPW], o[QPW][DPL];
#pragma unroll
  for (int u = 0; u < QPW; ++u) {
    m[u] = -INFINITY;
    l[u] = 0.f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) o[u][d] = 0.f;
  }
  for (int k0 = 0; k0 < kend; k0 += KT) {
    __syncthreads();  // the previous tile is consumed (and the queries are in place)
    for (int i = threadIdx.x; i < KT * D; i += WARPS * 32) {
      const int r = i / D, c = i % D, kj = k0 + r;
      const bool in = kj < kend;
      ks[r][c] = in ? cvt_in(K[kj * a.ldk + c]) : 0.f;
      vs[r][c] = in ? cvt_in(V[kj * a.ldv + c]) : 0.f;
    }
    __syncthreads();
    const int kj = k0 + lane;
    float sc[QPW];
#pragma unroll
    for (int u = 0; u < QPW; ++u) sc[u] = 0.f;
#pragma unroll 8
    for (int c = 0; c < D; ++c) {
      const float kc = ks[lane][c];
#pragma unroll
      for (int u = 0; u < QPW; ++u) sc[u] = fmaf(qs[warp * QPW + u][c], kc, sc[u]);
    }
#pragma unroll
    for (int u = 0; u < QPW; ++u) {
      const int qi = q0 + warp * QPW + u;
      const bool ok = kj < kend && (!a.causal || kj <= qi);
      float mx = ok ? sc[u] : -INFINITY;
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
      const float mnew = fmaxf(m[u], mx);
      if (mnew == -INFINITY) continue;  // nothing visible to this query yet (warp-uniform)
      const float corr = exp2f(m[u] - mnew);  // 0 on the first visible tile (m = -inf)
      const float p = ok ? exp2f(sc[u] - mnew) : 0.f;
      float ps = p;
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, s);
      l[u] = l[u] * corr + ps;
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[u][d] *= corr;
#pragma unroll 8
      for (int j = 0; j < KT; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
#pragma unroll
        for (int d = 0; d < DPL; ++d) o[u][d] = fmaf(pj, vs[j][lane + 32 * d], o[u][d]);
      }
      m[u] = mnew;
    }
  }
  TO* out = static_cast<TO*>(a.out) + b * a.o_bs + static_cast<long long>(h) * D;
#pragma unroll
  for (int u = 0; u < QPW; ++u) {
    const int qi = q0 + warp * QPW + u;
    if (qi >= a.Lq) continue;
    const float inv = l[u] > 0.f ? 1.0f / l[u] : 0.f;  // no visible key (key_len 0): zeros
#pragma unroll
    for (int d = 0; d < DPL; ++d) out[qi * a.ldo + lane + 32 * d] = cvt_out<TO>(o[u][d] * inv);
  }
}

template <typename TI, typename TO, int D>
int launch_typed(const Args& a, dim3 grid, cudaStream_t st) {
  const auto fn = text_attention_kernel<TI, TO, D>;
  if (smem_bytes<D>() > 48 * 1024) {
    const int e = anima::set_max_dynamic_smem(reinterpret_cast<const void*>(fn), smem_bytes<D>());
    if (e) return e;
  }
  fn<<<grid, WARPS * 32, smem_bytes<D>(), st>>>(a);
  return ANIMA_OK;
}

template <typename TI, int D>
int launch_out(const Args& a, int out_dtype, dim3 grid, cudaStream_t st) {
  if (out_dtype == ANIMA_F32) return launch_typed<TI, float, D>(a, grid, st);
  if (out_dtype == ANIMA_BF16) return launch_typed<TI, __nv_bfloat16, D>(a, grid, st);
  return launch_typed<TI, __half, D>(a, grid, st);
}

template <int D>
int launch_in(const Args& a, int in_dtype, int out_dtype, dim3 grid, cudaStream_t st) {
  if (in_dtype == ANIMA_F32) return launch_out<float, D>(a, out_dtype, grid, st);
  if (in_dtype == ANIMA_BF16) return launch_out<__nv_bfloat16, D>(a, out_dtype, grid, st);
  return launch_out<__half, D>(a, out_dtype, grid, st);
}

}  // namespace tattn

using namespace anima;

namespace {

int text_attention(anima_ctx* ctx, const anima_attention_args* a, int group) {
  ANIMA_REQUIRE(a->head_dim == 64 || a->head_dim == 128 || a->head_dim == 384,
                "anima_attention: head_dim %d (64, 128 or 384)", a->head_dim);
  ANIMA_REQUIRE(a->heads % group == 0, "anima_attention: %d heads do not form groups of %d", a->heads, group);
  const long long hd = a->head_dim;
  const long long kv_cols = static_cast<long long>(a->heads / group) * hd;
  ANIMA_REQUIRE(a->ldq >= a->q_off + a->heads * hd && a->ldk >= a->k_off + kv_cols && a->ldv >= a->v_off + kv_cols &&
                    a->ldo >= a->heads * hd && a->q_off >= 0 && a->k_off >= 0 && a->v_off >= 0,
                "anima_attention: row strides too small for %d heads (%lld k/v columns)", a->heads, kv_cols);
  const bool kv_bcast = a->batch > 1 && a->k_bstride == 0 && a->v_bstride == 0;
  tattn::Args t{};
  t.q = a->q;
  t.k = a->k;
  t.v = a->v;
  t.out = a->out;
  t.ldq = a->ldq;
  t.ldk = a->ldk;
  t.ldv = a->ldv;
  t.ldo = a->ldo;
  t.q_bs = a->batch > 1 ? a->q_bstride : 0;
  t.k_bs = a->batch > 1 ? a->k_bstride : 0;
  t.v_bs = a->batch > 1 ? a->v_bstride : 0;
  t.o_bs = a->batch > 1 ? a->o_bstride : 0;
  t.q_off = a->q_off;
  t.k_off = a->k_off;
  t.v_off = a->v_off;
  t.Lq = a->Lq;
  t.Lk = a->Lk;
  t.group = group;
  t.causal = a->causal ? 1 : 0;
  t.kv_bcast = kv_bcast ? 1 : 0;
  t.key_len = a->key_len;
  const float scale = a->scale > 0.f ? a->scale : 1.0f / sqrtf(static_cast<float>(a->head_dim));
  t.scale_log2 = scale * 1.4426950408889634f;
  const dim3 grid((a->Lq + tattn::QPC - 1) / tattn::QPC, a->heads, a->batch);
  ANIMA_REQUIRE(grid.y <= 65535 && grid.z <= 65535, "anima_attention: too many heads or batch items");
  ProfScope prof(ctx, "attn.text", 4.0 * a->batch * a->heads * static_cast<double>(a->Lq) * a->Lk * a->head_dim, 0);
  int st = a->head_dim == 128   ? tattn::launch_in<128>(t, a->dtype, a->out_dtype, grid, ctx->stream)
           : a->head_dim == 384 ? tattn::launch_in<384>(t, a->dtype, a->out_dtype, grid, ctx->stream)
                                : tattn::launch_in<64>(t, a->dtype, a->out_dtype, grid, ctx->stream);
  if (st) return st;
  return check_launch("text_attention_kernel");
}

// static_ws: the stream-K workspace comes from the module's static device array (no allocation)
// instead of the context's lazily allocated one.
int attention_launch(anima_ctx* ctx, const anima_attention_args* a, bool static_ws) {
  ANIMA_REQUIRE(ctx && a, "anima_attention: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_REQUIRE(a->out_dtype == ANIMA_F32 || a->out_dtype == ANIMA_BF16 || a->out_dtype == ANIMA_F16,
                "anima_attention: out_dtype %d", a->out_dtype);
  ANIMA_REQUIRE(a->batch > 0 && a->heads > 0 && a->Lq > 0 && a->Lk > 0, "anima_attention: empty problem");
  ANIMA_REQUIRE(a->q && a->k && a->v && a->out, "anima_attention: NULL data pointer");
  const int group = a->group > 1 ? a->group : 1;
  if (attention_planes_ok(a)) return attention_planes(ctx, a);  // the VAE's wide single head
  if (a->head_dim != attn::HD || a->dtype == ANIMA_F32 || a->heads % group != 0) {
    ANIMA_REQUIRE(a->dtype == ANIMA_F32 || a->dtype == ANIMA_BF16 || a->dtype == ANIMA_F16,
                  "anima_attention: q/k/v dtype %d", a->dtype);
    return text_attention(ctx, a, group);  // no workspace either way
  }
  ANIMA_REQUIRE(a->dtype == ANIMA_BF16 || a->dtype == ANIMA_F16, "anima_attention: q/k/v dtype must be bf16 or f16");
  const long long cols_q = a->q_off + static_cast<long long>(a->heads) * a->head_dim;
  const long long cols_k = a->k_off + static_cast<long long>(a->heads / group) * a->head_dim;
  const long long cols_v = a->v_off + static_cast<long long>(a->heads / group) * a->head_dim;
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
  p.group = group;
  p.causal = a->causal ? 1 : 0;
  const float scale = a->scale > 0.f ? a->scale : 1.0f / sqrtf(static_cast<float>(a->head_dim));
  p.scale_log2 = scale * 1.4426950408889634f;

  const long long units = static_cast<long long>(p.q_pairs) * a->heads * a->batch;
  ANIMA_REQUIRE(units < (1LL << 31), "anima_attention: problem too large");
  p.units = static_cast<int>(units);
  p.ublk = (a->Lk + attn::TILE - 1) / attn::TILE;
  long long grid = units;
  if (attn::use_stream_k(ctx, a, units, p.ublk)) {
    if (static_ws) {
      int st = attn::static_scratch(ctx);
      if (st) return st;
      p.flags = static_cast<unsigned*>(ctx->attn_static_ws);
      p.ws = reinterpret_cast<float*>(static_cast<unsigned char*>(ctx->attn_static_ws) + attn::kStaticFlagBytes);
    } else {
      int st = attn::stream_k_scratch(ctx);
      if (st) return st;
      p.ws = ctx->attn_ws;
      p.flags = ctx->attn_flags;
    }
    p.stream_k = 1;
    grid = ctx->num_sms;
  } else if (units > ctx->num_sms && (units + ctx->num_sms - 1) / ctx->num_sms <= attn::MAX_SEGS) {
    // more than one wave of whole units: a persistent grid, one CTA per SM
    p.persist = 1;
    grid = ctx->num_sms;
  }
  // (profiling events are created only on the allocating entry point)
  ProfScope prof(static_ws ? nullptr : ctx, "attn.flash",
                 4.0 * a->batch * a->heads * static_cast<double>(a->Lq) * a->Lk * a->head_dim, 0);
  using Kfn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const attn::Params);
  const int kind = a->dtype == ANIMA_BF16 ? 1 : 0;
  const Kfn fns[2] = {attn::attention_kernel<false>, attn::attention_kernel<true>};
  const Kfn fn = fns[kind];
  {
    int st = set_max_dynamic_smem(reinterpret_cast<const void*>(fn), attn::SMEM_BYTES);
    if (st) return st;
  }
  fn<<<static_cast<int>(grid), attn::THREADS, attn::SMEM_BYTES, ctx->stream>>>(tq, tk, tv, p);
  return check_launch("attention_kernel");
}

}  // namespace

extern "C" int anima_attention(anima_ctx* ctx, const anima_attention_args* a) {
  return attention_launch(ctx, a, false);
}

extern "C" int anima_attention_noalloc(anima_ctx* ctx, const anima_attention_args* a) {
  return attention_launch(ctx, a, true);
}
