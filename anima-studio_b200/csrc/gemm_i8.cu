// tcgen05 kind::i8 GEMM with fused epilogues: the ConvRot-quantized block linears of the DiT
// (the reference runs them as fp32 WGSL tiles that decode int8 in the loader, app/gpu/gemm.js:129-140).
//
//   C[m, n] = epi( a_scale[m] * w_scale[n] * (acc_hi[m, n] + acc_lo[m, n] / 254) )
//   acc_hi = sum_k hi[m, k] * W[n, k]     acc_lo = sum_k lo[m, k] * W[n, k]     (s32 in TMEM)
//
// Activations are per-token int8 planes of the rotated input (x ~= s * (hi + lo / 254)); with one
// plane (lo == NULL) this is plain W8A8. Weights are int8 [N, K] K-major, i.e. the comfy_quant
// `weight` tensor as stored.
//
// Structure: persistent CTAs (one per SM), 320 threads:
//   WG0, WG1    epilogue: tcgen05.ld of the accumulator rows (thread = row), fused epilogue, stores;
//               WG0 takes the CTA's even tiles, WG1 the odd ones (two warps per scheduler)
//   warp 8      TMA producer: A tile(s) 128 x 128 B and W tile BN x 128 B per stage (SWIZZLE_128B)
//   warp 9      TMEM allocator + single-thread UMMA issuer of the hi plane (M = 128, N = BN, K = 32)
//   warp 10     single-thread UMMA issuer of the lo plane (two planes only): the planes have their
//               own accumulators, so two wait -> issue -> commit chains feed the tensor core at once
//               (one thread issuing both planes was the kernel's critical path)
// The accumulators are double-buffered in TMEM (2 x NPLANES x BN = 512 columns), one buffer per
// epilogue warpgroup, so the epilogues of two tiles overlap the MMAs of the next.

#include <cstring>

#include "internal.h"
#include "sm100.cuh"

namespace anima {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 128;      // bytes of K per stage (one SWIZZLE_128B row)
constexpr int UMMA_K = 32;   // K per kind::i8 instruction
constexpr int THREADS = 352;  // 8 epilogue warps + producer warp + one MMA warp per activation plane

struct Params {
  int M, N, K;
  const float* a_scale;
  const float* w_scale;
  const float* bias;
  const float* add;
  int ld_add;
  int act;
  int out_mode;
  int out_dtype;
  void* out;
  int ldo;
  const float* gate;
  int gate_off;
  const float* norm_q;
  const float* norm_k;
  const float* rope;
  int rope_rows;
  int n_q;
  float eps;
  // LoRA side paths (see anima_linear_opts)
  const float* lora_t;
  int ld_t;
  int lora_t_lo;
  const float* lora_bt;
  int ld_bt;
  int lora_count;
  int lora_off[4], lora_n[4], lora_r0[4], lora_r[4];
  // sequence-parallel k|v exchange (see anima_linear_opts): k|v pieces go to the peer maps
  int peer_count, peer_row0, peer_rows;
  int num_m_blocks, num_n_blocks, num_k_blocks, num_tiles;
  int group_m;
};

// Tensor maps over every rank's gathered k|v buffer (3D: columns, rows of an image, image), as
// mapped in this process; only peer_count of them are encoded.
struct PeerMaps {
  CUtensorMap m[8];
};

// Tile order: groups of group_m m-blocks, n-blocks outermost within a group, so the CTAs in flight
// share a few A row-blocks and sweep the weights (keeps A resident in L2 across the n sweep).
__device__ __forceinline__ void tile_coords(const Params& p, int tile, int& mb, int& nb) {
  const int per_group = p.group_m * p.num_n_blocks;
  const int group = tile / per_group;
  const int first_m = group * p.group_m;
  const int gm = min(p.group_m, p.num_m_blocks - first_m);
  const int within = tile - group * per_group;
  mb = first_m + within % gm;
  nb = within / gm;
}

constexpr int LORA_R = 32;  // rank held per tile by the fused LoRA epilogue

template <int BN, int NPLANES, bool LORA = false>
struct Cfg {
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = NPLANES * A_BYTES + B_BYTES;
  static constexpr int STAGING_BYTES = 8 * 2 * 32 * 128;  // 8 epilogue warps x 2 x 4 KB
  // LoRA: one [LORA_R, BN] fp16 slice of scale * B^T per epilogue warpgroup (fp16 keeps three
  // pipeline stages within the 227 KB a CTA may hold)
  static constexpr int LORA_BYTES = LORA ? 2 * LORA_R * BN * 2 : 0;
  // the tile's per-column vectors (weight scale, bias, gate) per epilogue warpgroup, loaded before
  // the accumulator wait (the LoRA build reads them from global memory: no room for a third stage)
  static constexpr int VEC_BYTES = LORA ? 0 : 2 * 3 * BN * 4;
  static constexpr int STAGES = ((LORA ? 224 : 216) * 1024 - STAGING_BYTES - LORA_BYTES - VEC_BYTES) / STAGE_BYTES;
  static constexpr int ACC_COLS = NPLANES * BN;
  // one accumulator buffer per epilogue warpgroup when two fit in TMEM, else one (the second
  // epilogue warpgroup then idles and the epilogue of a tile delays the next tile's MMAs)
  static constexpr int ACC_BUFS = (2 * ACC_COLS <= 512) ? 2 : 1;
  static_assert(ACC_BUFS * ACC_COLS <= 512, "accumulators exceed TMEM");
  static constexpr int TMEM_COLS = 512;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + LORA_BYTES + VEC_BYTES + BAR_BYTES + 1024;
  static_assert(STAGES >= 2, "need at least two pipeline stages");
  static_assert(SMEM_BYTES <= 232448, "shared memory exceeds the 227 KB a CTA may hold");
};

// ------------------------------------------------------------------ epilogue helpers

__device__ __forceinline__ float act_fn(float v, int act) {
  if (act == ANIMA_ACT_GELU) return gelu_erf(v);
  if (act == ANIMA_ACT_SILU) return silu_f(v);
  return v;
}

// CH consecutive fp32 values through the read-only path as 16-byte loads (p 16-byte aligned).
template <int CH>
__device__ __forceinline__ void ldv(const float* p, float (&v)[CH]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int j = 0; j < CH / 4; ++j) {
    const float4 t = __ldg(q + j);
    v[4 * j] = t.x;
    v[4 * j + 1] = t.y;
    v[4 * j + 2] = t.z;
    v[4 * j + 3] = t.w;
  }
}
__device__ __forceinline__ void ld32(const float* p, float (&v)[32]) { ldv<32>(p, v); }

// CH consecutive fp32 values from shared or global memory (generic 16-byte loads).
template <int CH>
__device__ __forceinline__ void ldg_any(const float* p, float (&v)[CH]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int j = 0; j < CH / 4; ++j) {
    const float4 t = q[j];
    v[4 * j] = t.x;
    v[4 * j + 1] = t.y;
    v[4 * j + 2] = t.z;
    v[4 * j + 3] = t.w;
  }
}

// A tile's row and column constants for the epilogue: this row's activation scale, and the
// weight scale, bias and gate of the tile's columns (indexed by the column within the tile; in
// shared memory, or in global memory for the LoRA build).
struct EpiVec {
  float as;
  const float* ws;
  const float* bias;
  const float* gate;  // residual mode: the gate; per-head norm modes: the norm weight of the column's head
};

template <int CH>
__device__ __forceinline__ void tmem_ldc(uint32_t taddr, uint32_t (&r)[CH]) {
  if constexpr (CH == 32) tmem_ld32(taddr, r); else tmem_ld16(taddr, r);
}

// Issue the TMEM loads of CH accumulator columns (hi plane, and lo plane at +BN) of this row.
template <int BN, int NPLANES, int CH>
__device__ __forceinline__ void issue_cols(uint32_t taddr, int col, uint32_t (&rh)[CH], uint32_t (&rl)[CH]) {
  tmem_ldc<CH>(taddr + col, rh);
  if constexpr (NPLANES == 2) tmem_ldc<CH>(taddr + BN + col, rl);
}

// LoRA: v[j] += sum_i t[i] * bt[i, col + j]. The tile's slice of scale * B^T sits in shared memory
// as fp16 (bt_s [r][BN], read as 16-byte broadcasts: every lane of the warp works on the same
// columns of a different row) and converts to fp32 for paired fp32 FMAs; t = row m of x_r A^T (the
// two partial products summed) is loaded once per tile and held in registers as fp16 pairs. The
// side path's products thus carry fp16 operands (relative rounding 2^-11) with fp32 sums; the
// LoRA delta is a small part of the output, so this adds ~1e-4 of it at most.
struct LoraTile {
  const __half* bt_s;  // nullptr: no LoRA entry covers this tile
  __half2 t[LORA_R / 2];
  int r;
};

template <int BN, int CH>
__device__ __forceinline__ void lora_cols(const LoraTile& lt, int col, float (&v)[CH]) {
  f2 acc[CH / 2];
#pragma unroll
  for (int j = 0; j < CH / 2; ++j) acc[j] = dup2(0.f);
#pragma unroll
  for (int i4 = 0; i4 < LORA_R; i4 += 4) {
    if (i4 < lt.r) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint4* row = reinterpret_cast<const uint4*>(lt.bt_s + (i4 + u) * BN + col);
        const float2 tp = __half22float2(lt.t[(i4 + u) / 2]);
        const f2 tt = dup2((u & 1) ? tp.y : tp.x);
#pragma unroll
        for (int q = 0; q < CH / 8; ++q) {
          const uint4 b = row[q];
          const uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 bf = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
            acc[4 * q + e] = fma2(tt, bf, acc[4 * q + e]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < CH / 2; ++j) {
    v[2 * j] += acc[j].x;
    v[2 * j + 1] += acc[j].y;
  }
}

// After the loads landed: y = a_scale[m] w_scale[n] (hi + lo / 254) (+ bias) (+ add) (+ LoRA) (act).
// av: this piece's ADD values when already loaded (else nullptr: loaded here).
template <int BN, int NPLANES, int CH, bool LORA>
__device__ __forceinline__ void finish_cols(const Params& p, const EpiVec& ev, int m, int n, bool row_ok,
                                            const uint32_t (&rh)[CH], const uint32_t (&rl)[CH], float (&v)[CH],
                                            bool apply_act, const LoraTile& lt, int col, const float* av = nullptr) {
  const float as = ev.as;
  float ws[CH];
  ldg_any<CH>(ev.ws + col, ws);
  if constexpr (NPLANES == 2) {
    const float as_lo = as * (1.0f / 254.0f);
#pragma unroll
    for (int j = 0; j < CH; ++j)
      v[j] = fmaf(static_cast<float>(static_cast<int>(rl[j])), as_lo, static_cast<float>(static_cast<int>(rh[j])) * as) *
             ws[j];
  } else {
#pragma unroll
    for (int j = 0; j < CH; ++j) v[j] = static_cast<float>(static_cast<int>(rh[j])) * as * ws[j];
  }
  if (p.bias) {
    float bv[CH];
    ldg_any<CH>(ev.bias + col, bv);
#pragma unroll
    for (int j = 0; j < CH; ++j) v[j] += bv[j];
  }
  if (p.add && row_ok) {
    if (av) {
#pragma unroll
      for (int j = 0; j < CH; ++j) v[j] += av[j];
    } else {
      float ad[CH];
      ldv<CH>(p.add + static_cast<size_t>(m) * p.ld_add + n, ad);
#pragma unroll
      for (int j = 0; j < CH; ++j) v[j] += ad[j];
    }
  }
  if constexpr (LORA) {
    if (lt.bt_s && row_ok) lora_cols<BN, CH>(lt, col, v);
  }
  if (apply_act && p.act == ANIMA_ACT_GELU) {
#pragma unroll
    for (int j = 0; j < CH; j += 2) {
      const f2 g = gelu2(make_float2(v[j], v[j + 1]));
      v[j] = g.x;
      v[j + 1] = g.y;
    }
  } else if (apply_act && p.act != ANIMA_ACT_NONE) {
#pragma unroll
    for (int j = 0; j < CH; ++j) v[j] = act_fn(v[j], p.act);
  }
}

// Load CH accumulator columns and finish them (no overlap; used by the per-head epilogues).
template <int BN, int NPLANES, bool LORA, int CH = 16>
__device__ __forceinline__ void load_cols(const Params& p, const EpiVec& ev, uint32_t taddr, int col, int m, int n,
                                          bool row_ok, float (&v)[CH], bool apply_act, const LoraTile& lt) {
  uint32_t rh[CH], rl[CH];
  issue_cols<BN, NPLANES, CH>(taddr, col, rh, rl);
  tmem_ld_wait(rh);
  if constexpr (NPLANES == 2) tmem_ld_wait(rl);
  finish_cols<BN, NPLANES, CH, LORA>(p, ev, m, n, row_ok, rh, rl, v, apply_act, lt, col);
}

// ------------------------------------------------------------------ staged stores
// Each epilogue warp owns two 4 KB staging buffers: 32 rows (its TMEM lane quadrant) x 128 bytes,
// in the SWIZZLE_128B layout (16-byte chunk j of row r at r * 128 + ((j ^ (r & 7)) << 4)), so the
// row-per-lane writes are bank-conflict free. A full buffer is written to global memory by one
// TMA tile store (or, for the fp32 residual, a TMA reduce-add), so no lane touches global memory
// row by row. A 128-byte staging row holds CHC = 32 fp32 or 64 16-bit columns.
constexpr int STAGE_BUF = 32 * 128;

// Write a 16-column piece (position q within the 128-byte chunk) of this lane's row.
__device__ __forceinline__ void stage_piece(uint8_t* buf, int lane, int dtype, int q, const float (&v)[16]) {
  uint8_t* row = buf + lane * 128;
  if (dtype == ANIMA_F32) {  // 64 bytes: chunks 4q .. 4q+3
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int chunk = 4 * q + j;
      *reinterpret_cast<float4*>(row + ((chunk ^ (lane & 7)) << 4)) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
  } else {  // 32 bytes: chunks 2q, 2q+1
    const bool bf = dtype == ANIMA_BF16;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float a = v[8 * j + 2 * e], b = v[8 * j + 2 * e + 1];
        if (bf) {
          __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
          w[e] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(a, b);
          w[e] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      const int chunk = 2 * q + j;
      *reinterpret_cast<uint4*>(row + ((chunk ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Hand a filled staging buffer to the TMA unit: box (CHC columns x 32 rows) at (x, y).
__device__ __forceinline__ void stage_flush(const CUtensorMap* tm, const uint8_t* buf, int x, int y, bool reduce) {
  fence_proxy_async_smem();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    if (reduce)
      tma_reduce_add_2d(tm, buf, x, y);
    else
      tma_store_2d(tm, buf, x, y);
    bulk_commit();
  }
  __syncwarp();
}

// Sequence-parallel qkv: a full staging buffer of k|v columns (x >= n_q) goes to every rank's
// gathered k|v buffer at this rank's rows instead of to the local output (one bulk group).
__device__ __forceinline__ void stage_flush_peers(const Params& p, const PeerMaps* pm, const uint8_t* buf, int x,
                                                  int y) {
  fence_proxy_async_smem();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    const int item = y / p.peer_rows;
    const int row = p.peer_row0 + (y - item * p.peer_rows);
    for (int r = 0; r < p.peer_count; ++r) tma_store_3d(&pm->m[r], buf, x - p.n_q, row, item);
    bulk_commit();
  }
  __syncwarp();
}

// Before rewriting a staging buffer: at most N of this warp's stores may still be reading.
template <int N>
__device__ __forceinline__ void stage_acquire() {
  if ((threadIdx.x & 31) == 0) bulk_wait_read<N>();
  __syncwarp();
}

// The store / residual epilogue of NCOL columns [cb, cb + NCOL) of a tile for this warp's 32 rows.
// t: this warp's running tile count; the two staging buffers alternate over the warp's chunks in
// order, across tiles too, so a buffer is rewritten only after the store before the last has read it.
template <int BN, int NPLANES, bool LORA, int NCOL>
__device__ __forceinline__ void store_cols(const Params& p, const EpiVec& ev, const CUtensorMap* tm_out, uint8_t* stage,
                                           uint32_t taddr, int m, int y0, int n0, const LoraTile& lt, int cb, int t) {
  const bool row_ok = m < p.M;
  const int lane = threadIdx.x & 31;
  const int esz = p.out_dtype == ANIMA_F32 ? 4 : 2;
  const int chc = 128 / esz;      // columns per staging chunk
  const int ppc = chc / 16;       // 16-column pieces per chunk
  constexpr int CH = 16;
  static_assert(NCOL % 64 == 0, "whole staging chunks");
  // software pipeline over 16-column pieces: the TMEM loads (and this row's ADD values) of piece
  // c+1 are in flight while piece c is finished and staged
  const bool resid = p.out_mode == ANIMA_OUT_RESID;
  const bool add = !LORA && p.add && row_ok;  // (the LoRA build has no registers to spare for it)
  const float* arow = add ? p.add + static_cast<size_t>(m) * p.ld_add + n0 : nullptr;
  constexpr int PIPE = 2;
  uint32_t rh[PIPE][CH], rl[PIPE][CH];
  float av[PIPE][CH];
  issue_cols<BN, NPLANES, CH>(taddr, cb, rh[0], rl[0]);
  if (add) ldv<CH>(arow + cb, av[0]);
  tmem_ld_wait(rh[0]);
  if constexpr (NPLANES == 2) tmem_ld_wait(rl[0]);
#pragma unroll
  for (int c = 0; c < NCOL / CH; ++c) {
    const int cur = PIPE == 2 ? (c & 1) : 0;
    if (PIPE == 2 && c + 1 < NCOL / CH) {
      issue_cols<BN, NPLANES, CH>(taddr, cb + CH * (c + 1), rh[(cur + 1) % PIPE], rl[(cur + 1) % PIPE]);
      if (add) ldv<CH>(arow + cb + CH * (c + 1), av[(cur + 1) % PIPE]);
    }
    const int col = cb + CH * c;
    const int chunk = col / chc, q = (col % chc) / CH;
    uint8_t* buf = stage + ((t * (NCOL / chc) + (col - cb) / chc) & 1) * STAGE_BUF;
    if (q == 0) stage_acquire<1>();
    float v[CH];
    finish_cols<BN, NPLANES, CH, LORA>(p, ev, m, n0 + col, row_ok, rh[cur], rl[cur], v, true, lt, col,
                                       add ? av[cur] : nullptr);
    if (resid) {
      float g[CH];
      if (p.gate) {
        ldg_any<CH>(ev.gate + col, g);
#pragma unroll
        for (int j = 0; j < CH; ++j) v[j] *= g[j];
      }
    }
    stage_piece(buf, lane, p.out_dtype, q, v);
    if (q == ppc - 1) stage_flush(tm_out, buf, n0 + chunk * chc, y0, resid);
    if (PIPE == 2 && c + 1 < NCOL / CH) {
      tmem_ld_wait(rh[(cur + 1) % PIPE]);
      if constexpr (NPLANES == 2) tmem_ld_wait(rl[(cur + 1) % PIPE]);
    }
  }
}

// One tile's epilogue for this warp's 32 rows (m = row of this lane) over BN columns from n0.
// stage: this warp's two staging buffers; y0: first row of the warp's quadrant.
template <int BN, int NPLANES, bool LORA>
__device__ __forceinline__ void epilogue_tile(const Params& p, const EpiVec& ev, const CUtensorMap* tm_out,
                                              const PeerMaps* pm, uint8_t* stage, uint32_t taddr, int m, int y0,
                                              int n0, const LoraTile& lt) {
  const bool row_ok = m < p.M;
  const int lane = threadIdx.x & 31;
  const int esz = p.out_dtype == ANIMA_F32 ? 4 : 2;
  const int chc = 128 / esz;      // columns per staging chunk
  const int ppc = chc / 16;       // 16-column pieces per chunk
  constexpr int CH = 16;
  if (p.out_mode == ANIMA_OUT_STORE || p.out_mode == ANIMA_OUT_RESID) {
    store_cols<BN, NPLANES, LORA, BN>(p, ev, tm_out, stage, taddr, m, y0, n0, lt, 0, 0);
    return;
  }
  // Per-head RMSNorm (+ split-half RoPE for q/k heads of a fused qkv projection): a head is 128
  // consecutive columns and never straddles a tile (BN is a multiple of 128). Two passes over the
  // accumulator: sum of squares, then normalise (+ rotate) 16-column pieces.
#pragma unroll 1
  for (int h0 = 0; h0 < BN; h0 += 128) {
    const int nh = n0 + h0;
    const bool qkv = p.out_mode == ANIMA_OUT_QKV_NORM_ROPE;
    const bool is_q = !qkv || nh < p.n_q;
    const bool is_k = qkv && !is_q && nh < 2 * p.n_q;
    if (qkv && !is_q && !is_k) {  // v heads: plain store
#pragma unroll 1
      for (int col = 0; col < 128; col += CH) {
        const int chunk = col / chc, q = (col % chc) / CH;
        uint8_t* buf = stage + (chunk & 1) * STAGE_BUF;
        if (q == 0) stage_acquire<1>();
        float v[CH];
        load_cols<BN, NPLANES, LORA, CH>(p, ev, taddr, h0 + col, m, nh + col, row_ok, v, true, lt);
        stage_piece(buf, lane, p.out_dtype, q, v);
        if (q == ppc - 1) {
          if (p.peer_count)
            stage_flush_peers(p, pm, buf, nh + chunk * chc, y0);
          else
            stage_flush(tm_out, buf, nh + chunk * chc, y0, false);
        }
      }
      continue;
    }
    const int tok = (qkv && row_ok) ? (m % p.rope_rows) : 0;
    const float* cs = qkv ? p.rope + static_cast<size_t>(tok) * 64 : nullptr;
    const float* sn = qkv ? p.rope + static_cast<size_t>(p.rope_rows) * 64 + static_cast<size_t>(tok) * 64 : nullptr;
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < 128; c += CH) {
      float v[CH];
      load_cols<BN, NPLANES, LORA, CH>(p, ev, taddr, h0 + c, m, nh + c, row_ok, v, true, lt);
#pragma unroll
      for (int j = 0; j < CH; ++j) ss += v[j] * v[j];
    }
    const float rs = 1.0f / sqrtf(ss * (1.0f / 128.0f) + p.eps);
    // the head's norm weights: in shared memory with the tile's other column constants (global
    // memory in the LoRA build)
    const float* w = LORA ? (is_k ? p.norm_k : p.norm_q) : ev.gate + h0;
    if (qkv) {
      // pieces arrive in pairs (c, 64 + c): the two halves of the head fill buffers 0 and 1
#pragma unroll 1
      for (int c = 0; c < 64; c += CH) {
        const int q = (c % chc) / CH;
        if (q == 0) stage_acquire<0>();
        float v1[CH], v2[CH];
        load_cols<BN, NPLANES, LORA, CH>(p, ev, taddr, h0 + c, m, nh + c, row_ok, v1, true, lt);
        load_cols<BN, NPLANES, LORA, CH>(p, ev, taddr, h0 + 64 + c, m, nh + 64 + c, row_ok, v2, true, lt);
        float a[CH], b[CH];
        ldg_any<CH>(w + c, a);
        ldg_any<CH>(w + 64 + c, b);
#pragma unroll
        for (int j = 0; j < CH; ++j) {
          v1[j] *= rs * a[j];
          v2[j] *= rs * b[j];
        }
        ldv<CH>(cs + c, a);  // cos
        ldv<CH>(sn + c, b);  // sin
#pragma unroll
        for (int j = 0; j < CH; ++j) {
          const float y1 = v1[j], y2 = v2[j];
          v1[j] = y1 * a[j] - y2 * b[j];
          v2[j] = y2 * a[j] + y1 * b[j];
        }
        stage_piece(stage, lane, p.out_dtype, q, v1);
        stage_piece(stage + STAGE_BUF, lane, p.out_dtype, q, v2);
        if (q == ppc - 1) {
          const int x0 = nh + (c / chc) * chc;
          if (is_k && p.peer_count) {
            stage_flush_peers(p, pm, stage, x0, y0);
            stage_flush_peers(p, pm, stage + STAGE_BUF, x0 + 64, y0);
          } else {
            stage_flush(tm_out, stage, x0, y0, false);
            stage_flush(tm_out, stage + STAGE_BUF, x0 + 64, y0, false);
          }
        }
      }
    } else {
#pragma unroll 1
      for (int col = 0; col < 128; col += CH) {
        const int chunk = col / chc, q = (col % chc) / CH;
        uint8_t* buf = stage + (chunk & 1) * STAGE_BUF;
        if (q == 0) stage_acquire<1>();
        float v[CH];
        load_cols<BN, NPLANES, LORA, CH>(p, ev, taddr, h0 + col, m, nh + col, row_ok, v, true, lt);
        float wv[CH];
        ldg_any<CH>(w + col, wv);
#pragma unroll
        for (int j = 0; j < CH; ++j) v[j] = v[j] * rs * wv[j];
        stage_piece(buf, lane, p.out_dtype, q, v);
        if (q == ppc - 1) stage_flush(tm_out, buf, nh + chunk * chc, y0, false);
      }
    }
  }
}

// Warp-uniform bounded wait: lane 0 polls, the result is broadcast.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned err) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, err) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
}

// LORA: the build with the LoRA side path in the epilogue (kept separate so the plain build's
// register allocation does not carry it).
// Barrier of one epilogue warpgroup (named barrier 1 + g, 128 threads) that also returns the AND of
// `ok` over its threads, so the four warps take the same branch after a failed wait.
__device__ __forceinline__ bool wg_sync_and(int g, bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(ok ? 1u : 0u), "r"(1 + g)
      : "memory");
  return r != 0;
}

template <int BN, int NPLANES, bool LORA>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tm_hi, const __grid_constant__ CUtensorMap tm_lo,
                   const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_out,
                   const Params p, const __grid_constant__ PeerMaps pm) {
  using C = Cfg<BN, NPLANES, LORA>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + C::STAGES * C::STAGE_BYTES;  // 1024-aligned (stage sizes are)
  __half* lora_smem = reinterpret_cast<__half*>(staging + C::STAGING_BYTES);
  float* epi_vec = reinterpret_cast<float*>(staging + C::STAGING_BYTES + C::LORA_BYTES);  // [2][3][BN]
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::STAGING_BYTES + C::LORA_BYTES + C::VEC_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;  // one per MMA warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Store and residual epilogues split every tile's columns between the two epilogue warpgroups
  // (each takes BN / 2 columns of every tile): a tile's epilogue is latency-bound per warp, so this
  // halves it, and with it the last tile's epilogue that no MMA overlaps. The per-head norms need
  // a head's 128 columns in one thread and keep one warpgroup per tile, alternating.
  const bool split = !LORA && C::ACC_BUFS == 2 && (p.out_mode == ANIMA_OUT_STORE || p.out_mode == ANIMA_OUT_RESID);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NPLANES);  // a commit from each MMA warp
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], NPLANES);
      mbar_init(&acc_empty[b], split ? 8 : 4);  // one arrival per epilogue warp that reads it
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  constexpr int kProducerWarp = 8, kMmaWarp = 9;
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tm_hi);
    if (NPLANES == 2) tma_prefetch_desc(&tm_lo);
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int armed_parity[C::STAGES];
      for (int s = 0; s < C::STAGES; ++s) armed_parity[s] = -1;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(p, tile, mb, nb);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, kErrTimeoutEmpty)) goto producer_done;
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sa, &tm_hi, &full[stage], kb * BK, mb * BM);
          if (NPLANES == 2) tma_load_2d(sa + C::A_BYTES, &tm_lo, &full[stage], kb * BK, mb * BM);
          tma_load_2d(sa + NPLANES * C::A_BYTES, &tm_w, &full[stage], kb * BK, nb * BN);
          armed_parity[stage] = static_cast<int>(phase);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:
      if (*abort_flag) {
        // Loads still in flight write shared memory: wait (bounded) until every armed stage landed.
        for (int s = 0; s < C::STAGES; ++s) {
          if (armed_parity[s] < 0) continue;
          const unsigned long long t0 = globaltimer();
          while (!mbar_test(smem_u32(&full[s]), static_cast<uint32_t>(armed_parity[s]))) {
            if (globaltimer() - t0 > kWaitTimeoutNs) {
              flag_error(kErrTimeoutDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == kMmaWarp || (NPLANES == 2 && warp == kMmaWarp + 1)) {
    const int plane = warp - kMmaWarp;
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++t) {
        const int buf = t % C::ACC_BUFS;
        const uint32_t acc_phase = (t / C::ACC_BUFS) & 1;
        if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1, abort_flag, kErrTimeoutAcc)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + buf * C::ACC_COLS + plane * BN;  // this plane's accumulator
        bool aborted = false;
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, kErrTimeoutFull)) {
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint32_t s0 = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sa = s0 + plane * C::A_BYTES;
          const uint32_t sb = s0 + NPLANES * C::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
            umma_i8(d, sdesc_sw128(sa + k * UMMA_K, 16, 1024), sdesc_sw128(sb + k * UMMA_K, 16, 1024), idesc, acc);
          }
          umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (aborted) break;
        umma_commit(&acc_full[buf]);
      }
      if (*abort_flag) {
        // MMAs already issued complete before TMEM is released.
        umma_commit(&drain[plane]);
        const unsigned long long t0 = globaltimer();
        while (!mbar_test(smem_u32(&drain[plane]), 0)) {
          if (globaltimer() - t0 > kWaitTimeoutNs) {
            flag_error(kErrTimeoutDrain);
            break;
          }
        }
      }
    }
  } else if (warp < 4 * C::ACC_BUFS) {
    // epilogue warpgroup g = warp / 4
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int g = warp >> 2;
    const int row = quad * 32 + lane;
    // the CTA's local tiles t this warpgroup serves: all of them (split), else t % ACC_BUFS == g
    const int step = split ? 1 : C::ACC_BUFS;
    int t = split ? 0 : g;
    float* vec = epi_vec + g * 3 * BN;
    for (int tile = blockIdx.x + t * gridDim.x; tile < p.num_tiles; tile += step * gridDim.x, t += step) {
      const int buf = t % C::ACC_BUFS;
      const uint32_t acc_phase = (t / C::ACC_BUFS) & 1;
      int mb, nb;
      tile_coords(p, tile, mb, nb);
      // The tile's constants, loaded while its MMAs run (a piece of the epilogue would otherwise
      // wait for them): this row's activation scale, and into shared memory, once per warpgroup
      // (after all four warps are done with the previous tile's), the columns' weight scale, bias
      // and gate.
      EpiVec ev;
      ev.as = (mb * BM + row < p.M) ? __ldg(p.a_scale + mb * BM + row) : 0.0f;
      if constexpr (LORA) {
        ev.ws = p.w_scale + nb * BN;
        ev.bias = p.bias ? p.bias + nb * BN : nullptr;
        ev.gate = p.gate ? p.gate + p.gate_off + nb * BN : nullptr;
      } else {
        wg_sync_and(g, true);
        const int tid = threadIdx.x - g * 128;
#pragma unroll
        for (int i = tid; i < BN; i += 128) {
          const int n = nb * BN + i;
          vec[i] = __ldg(p.w_scale + n);
          if (p.bias) vec[BN + i] = __ldg(p.bias + n);
          if (p.out_mode == ANIMA_OUT_RESID) {
            if (p.gate) vec[2 * BN + i] = __ldg(p.gate + p.gate_off + n);
          } else if (p.out_mode != ANIMA_OUT_STORE) {
            // the per-head norms: the third vector holds the norm weight of each column's head
            const int nh = n & ~127;
            const bool qkv = p.out_mode == ANIMA_OUT_QKV_NORM_ROPE;
            const bool is_q = !qkv || nh < p.n_q;
            const bool is_k = qkv && !is_q && nh < 2 * p.n_q;
            vec[2 * BN + i] = (is_q || is_k) ? __ldg((is_k ? p.norm_k : p.norm_q) + (n & 127)) : 0.0f;
          }
        }
        ev.ws = vec;
        ev.bias = vec + BN;
        ev.gate = vec + 2 * BN;
      }
      bool ok = warp_wait(&acc_full[buf], acc_phase, abort_flag, kErrTimeoutAcc);
      // the same branch for the four warps after a failed wait; also publishes the vectors (and,
      // in the LoRA build, orders the previous tile's reads of its LoRA slice before the next)
      ok = wg_sync_and(g, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * C::ACC_COLS;
      LoraTile lt;
      lt.bt_s = nullptr;
      lt.r = 0;
      if constexpr (LORA) {
        // the entry covering this tile (entries are BN-aligned): stage its slice of scale * B^T
        const int n0 = nb * BN;
        int e = -1;
        for (int i = 0; i < p.lora_count; ++i)
          if (n0 >= p.lora_off[i] && n0 < p.lora_off[i] + p.lora_n[i]) e = i;
        if (e >= 0) {
          __half* bt_s = lora_smem + g * LORA_R * BN;
          const int r = p.lora_r[e];
          const int tid = threadIdx.x - g * 128;
          for (int k = tid; k < r * BN / 8; k += 128) {  // 8 columns per step: two loads, one store
            const int i = k / (BN / 8), c8 = k % (BN / 8);
            const float4* src =
                reinterpret_cast<const float4*>(p.lora_bt + static_cast<size_t>(p.lora_r0[e] + i) * p.ld_bt + n0) + 2 * c8;
            const float4 a = __ldg(src), b = __ldg(src + 1);
            const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
            reinterpret_cast<uint4*>(bt_s)[k] =
                make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                           *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
          }
          // this row's x_r A^T for the entry's ranks, both partial products summed, into registers
          const int m = mb * BM + row;
          const float* tr = p.lora_t + static_cast<size_t>(m < p.M ? m : 0) * p.ld_t + p.lora_r0[e];
#pragma unroll
          for (int i4 = 0; i4 < LORA_R; i4 += 4) {
            float4 t4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i4 < r) {
              t4 = __ldg(reinterpret_cast<const float4*>(tr + i4));
              if (p.lora_t_lo) {
                const float4 l4 = __ldg(reinterpret_cast<const float4*>(tr + p.lora_t_lo + i4));
                t4.x += l4.x;
                t4.y += l4.y;
                t4.z += l4.z;
                t4.w += l4.w;
              }
            }
            lt.t[i4 / 2] = __floats2half2_rn(t4.x, t4.y);
            lt.t[i4 / 2 + 1] = __floats2half2_rn(t4.z, t4.w);
          }
          wg_sync_and(g, true);
          lt.bt_s = bt_s;
          lt.r = r;
        }
      }
      if (split)
        store_cols<BN, NPLANES, LORA, BN / 2>(p, ev, &tm_out, staging + warp * 2 * STAGE_BUF, taddr, mb * BM + row,
                                              mb * BM + quad * 32, nb * BN, lt, g * (BN / 2), t);
      else
        epilogue_tile<BN, NPLANES, LORA>(p, ev, &tm_out, &pm, staging + warp * 2 * STAGE_BUF, taddr, mb * BM + row,
                                         mb * BM + quad * 32, nb * BN, lt);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    // every staged store has finished (shared memory is read and the global writes are done)
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int BN, int NPLANES, bool LORA>
int launch(anima_ctx* ctx, const anima_qact* x, const anima_weight* W, const anima_linear_opts* o) {
  using C = Cfg<BN, NPLANES, LORA>;
  const int M = x->rows, N = W->N, K = W->K;
  CUtensorMap tm_hi, tm_lo, tm_w;
  uint64_t adims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
  uint64_t astr[1] = {static_cast<uint64_t>(x->ld)};
  uint32_t abox[2] = {BK, BM};
  int st = make_tmap(&tm_hi, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, x->hi, adims, astr, abox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  if (NPLANES == 2) {
    st = make_tmap(&tm_lo, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, x->lo, adims, astr, abox, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  } else {
    tm_lo = tm_hi;
  }
  uint64_t wdims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
  uint64_t wstr[1] = {static_cast<uint64_t>(K)};
  uint32_t wbox[2] = {BK, BN};
  st = make_tmap(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, W->data, wdims, wstr, wbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  // output: boxes of 128 bytes (32 fp32 or 64 16-bit columns) x 32 rows, one per epilogue warp chunk
  CUtensorMap tm_out;
  {
    const int esz = o->out_dtype == ANIMA_F32 ? 4 : 2;
    const CUtensorMapDataType odt = o->out_dtype == ANIMA_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                    : o->out_dtype == ANIMA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    uint64_t odims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
    uint64_t ostr[1] = {static_cast<uint64_t>(o->ldo) * esz};
    uint32_t obox[2] = {static_cast<uint32_t>(128 / esz), 32};
    st = make_tmap(&tm_out, odt, 2, o->out, odims, ostr, obox, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }

  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_scale = x->scale;
  p.w_scale = W->scale;
  p.bias = W->bias;
  p.add = o->add;
  p.ld_add = o->ld_add;
  p.act = o->act;
  p.out_mode = o->out_mode;
  p.out_dtype = o->out_dtype;
  p.out = o->out;
  p.ldo = o->ldo;
  p.gate = o->gate;
  p.gate_off = o->gate_off;
  p.norm_q = o->norm_q;
  p.norm_k = o->norm_k;
  p.rope = o->rope;
  p.rope_rows = o->rope_rows;
  p.n_q = o->n_q;
  p.eps = o->eps > 0 ? o->eps : 1e-6f;
  p.lora_t = o->lora_t;
  p.ld_t = o->ld_t;
  p.lora_t_lo = o->lora_t_lo;
  p.lora_bt = o->lora_bt;
  p.ld_bt = o->ld_bt;
  p.lora_count = o->lora_t ? o->lora_count : 0;
  for (int e = 0; e < 4; ++e) {
    p.lora_off[e] = o->lora_off[e];
    p.lora_n[e] = o->lora_n[e];
    p.lora_r0[e] = o->lora_r0[e];
    p.lora_r[e] = o->lora_r[e];
  }
  PeerMaps pm;
  memset(&pm, 0, sizeof(pm));
  p.peer_count = o->peer_count;
  p.peer_row0 = o->peer_row0;
  p.peer_rows = o->peer_rows > 0 ? o->peer_rows : 1;
  if (o->peer_count > 0) {
    const int esz = o->out_dtype == ANIMA_F32 ? 4 : 2;
    const CUtensorMapDataType odt = o->out_dtype == ANIMA_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                    : o->out_dtype == ANIMA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t cols = static_cast<uint64_t>(N - o->n_q);
    uint64_t dims[3] = {cols, static_cast<uint64_t>(o->peer_item_rows), static_cast<uint64_t>(M / o->peer_rows)};
    uint64_t str[2] = {cols * esz, cols * esz * static_cast<uint64_t>(o->peer_item_rows)};
    uint32_t box[3] = {static_cast<uint32_t>(128 / esz), 32, 1};
    for (int r = 0; r < o->peer_count; ++r) {
      st = make_tmap(&pm.m[r], odt, 3, o->peer_kv[r], dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
      if (st) return st;
    }
  }
  p.num_m_blocks = (M + BM - 1) / BM;
  p.num_n_blocks = N / BN;
  p.num_k_blocks = K / BK;
  p.num_tiles = p.num_m_blocks * p.num_n_blocks;
  static const int group_m_env = [] {
    const char* e = getenv("ANIMA_GEMM_GROUP_M");  // tile-order experiments; default 8
    return e ? atoi(e) : 8;
  }();
  p.group_m = group_m_env > 0 ? group_m_env : 8;

  st = set_max_dynamic_smem(reinterpret_cast<const void*>(gemm_i8_kernel<BN, NPLANES, LORA>), C::SMEM_BYTES);
  if (st) return st;
  const int grid = p.num_tiles < ctx->num_sms ? p.num_tiles : ctx->num_sms;
  ProfScope prof(ctx, NPLANES == 2 ? "linear.i8x2" : "linear.i8", 2.0 * M * N * K,
                 static_cast<double>(M) * K * NPLANES + static_cast<double>(N) * K);
  gemm_i8_kernel<BN, NPLANES, LORA><<<grid, THREADS, C::SMEM_BYTES, ctx->stream>>>(tm_hi, tm_lo, tm_w, tm_out, p, pm);
  return check_launch("gemm_i8_kernel");
}

}  // namespace gemm
}  // namespace anima

using namespace anima;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// W4 weights run as their int8 grid: anima_linear decodes the layer into this context-owned buffer
// right before the GEMM (the same stream, so the GEMM sees the whole grid and the next W4 call
// cannot overwrite it early). The buffer holds at least the DiT's largest linear (8192 x 2048) and
// grows, outside stream capture only, when a larger weight comes.
static int w4_scratch(anima_ctx* ctx, size_t bytes) {
  if (ctx->w4_ws_bytes >= bytes) return ANIMA_OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  ANIMA_CUDA(cudaStreamIsCapturing(ctx->stream, &cap));
  ANIMA_REQUIRE(cap == cudaStreamCaptureStatusNone,
                "anima_linear: the W4 decode buffer would grow to %zu bytes inside stream capture (run the largest "
                "W4 linear once before capturing)",
                bytes);
  if (ctx->w4_ws) {  // kernels of earlier calls may still read the old buffer
    ANIMA_CUDA(cudaDeviceSynchronize());
    ANIMA_CUDA(cudaFree(ctx->w4_ws));
    ctx->w4_ws = nullptr;
    ctx->w4_ws_bytes = 0;
  }
  const size_t want = bytes > size_t(8192) * 2048 ? bytes : size_t(8192) * 2048;
  ANIMA_CUDA(cudaMalloc(reinterpret_cast<void**>(&ctx->w4_ws), want));
  ctx->w4_ws_bytes = want;
  return ANIMA_OK;
}

extern "C" int anima_linear(anima_ctx* ctx, const anima_qact* x, const anima_weight* W, const anima_linear_opts* o) {
  ANIMA_REQUIRE(ctx && x && W && o, "anima_linear: NULL argument");
  ANIMA_ON_DEVICE(ctx);
  ANIMA_REQUIRE(W->kind == ANIMA_W_I8 || W->kind == ANIMA_W_W4,
                "anima_linear: weight kind %d is not a ConvRot int8 or W4A8 weight", W->kind);
  if (W->kind == ANIMA_W_W4)
    ANIMA_REQUIRE(W->s_rel && W->codebook, "anima_linear: a W4 weight needs s_rel and the codebook");
  ANIMA_REQUIRE(x->cols == W->K, "anima_linear: activation has %d columns, weight K is %d", x->cols, W->K);
  ANIMA_REQUIRE(x->rows > 0 && W->N > 0, "anima_linear: empty problem (M=%d, N=%d)", x->rows, W->N);
  ANIMA_REQUIRE(W->K % gemm::BK == 0, "anima_linear: K=%d must be a multiple of %d", W->K, gemm::BK);
  ANIMA_REQUIRE(W->N % 128 == 0, "anima_linear: N=%d must be a multiple of 128", W->N);
  ANIMA_REQUIRE(x->ld % 16 == 0 && x->ld >= x->cols, "anima_linear: activation ld %d must be >= K and a multiple of 16",
                x->ld);
  ANIMA_REQUIRE(x->hi && x->scale && W->data && W->scale && o->out, "anima_linear: missing data pointer");
  ANIMA_REQUIRE(aligned16(x->hi) && (!x->lo || aligned16(x->lo)) && aligned16(W->data) && aligned16(o->out),
                "anima_linear: data pointers must be 16-byte aligned");
  const int esz = o->out_dtype == ANIMA_F32 ? 4 : 2;
  ANIMA_REQUIRE(o->out_dtype == ANIMA_F32 || o->out_dtype == ANIMA_BF16 || o->out_dtype == ANIMA_F16,
                "anima_linear: out_dtype %d unsupported", o->out_dtype);
  ANIMA_REQUIRE((static_cast<long long>(o->ldo) * esz) % 16 == 0 && o->ldo >= W->N,
                "anima_linear: ldo %d must be >= N and 16-byte aligned", o->ldo);
  ANIMA_REQUIRE(o->out_mode >= ANIMA_OUT_STORE && o->out_mode <= ANIMA_OUT_HEAD_NORM, "anima_linear: bad out_mode %d",
                o->out_mode);
  ANIMA_REQUIRE(o->out_mode != ANIMA_OUT_RESID || o->out_dtype == ANIMA_F32,
                "anima_linear: the residual output is fp32 (the reference's residual stream)");
  ANIMA_REQUIRE(!o->add || (aligned16(o->add) && o->ld_add % 4 == 0 && o->ld_add >= W->N),
                "anima_linear: add must be 16-byte aligned with ld_add >= N, multiple of 4");
  if (o->out_mode == ANIMA_OUT_QKV_NORM_ROPE) {
    ANIMA_REQUIRE(o->norm_q && o->norm_k && o->rope && o->rope_rows > 0, "anima_linear: qkv epilogue needs norms and rope");
    ANIMA_REQUIRE(o->n_q % 128 == 0 && 2 * o->n_q <= W->N, "anima_linear: bad n_q %d", o->n_q);
  }
  if (o->out_mode == ANIMA_OUT_HEAD_NORM) ANIMA_REQUIRE(o->norm_q, "anima_linear: head-norm epilogue needs norm_q");
  if (o->peer_count != 0) {
    ANIMA_REQUIRE(o->out_mode == ANIMA_OUT_QKV_NORM_ROPE && o->peer_count > 0 && o->peer_count <= 8,
                  "anima_linear: the k|v exchange takes 1-8 buffers and the qkv epilogue");
    ANIMA_REQUIRE(o->peer_rows > 0 && o->peer_rows % 32 == 0 && x->rows % o->peer_rows == 0 && o->peer_row0 >= 0 &&
                      o->peer_row0 + o->peer_rows <= o->peer_item_rows,
                  "anima_linear: k|v exchange rows (row0 %d, rows %d of %d per image, M %d) invalid", o->peer_row0,
                  o->peer_rows, o->peer_item_rows, x->rows);
    for (int r = 0; r < o->peer_count; ++r)
      ANIMA_REQUIRE(o->peer_kv[r] && aligned16(o->peer_kv[r]), "anima_linear: k|v buffer %d missing or unaligned", r);
  }
  if (o->lora_t) {
    ANIMA_REQUIRE(o->lora_bt && o->lora_count >= 1 && o->lora_count <= 4, "anima_linear: LoRA needs t, bt and 1-4 entries");
    ANIMA_REQUIRE(aligned16(o->lora_t) && aligned16(o->lora_bt) && o->ld_t % 4 == 0 && o->ld_bt % 4 == 0 &&
                      o->lora_t_lo >= 0 && o->lora_t_lo % 4 == 0 &&
                      o->ld_bt >= W->N,
                  "anima_linear: LoRA t/bt must be 16-byte aligned with ld_t, ld_bt multiples of 4 (ld_bt >= N)");
    for (int e = 0; e < o->lora_count; ++e) {
      ANIMA_REQUIRE(o->lora_off[e] >= 0 && o->lora_n[e] > 0 && o->lora_off[e] % 128 == 0 && o->lora_n[e] % 128 == 0 &&
                        o->lora_off[e] + o->lora_n[e] <= W->N && o->lora_r[e] > 0 && o->lora_r[e] % 4 == 0 &&
                        o->lora_r[e] <= gemm::LORA_R &&
                        o->lora_r0[e] >= 0 && o->lora_r0[e] % 4 == 0 &&
                        o->lora_t_lo + o->lora_r0[e] + o->lora_r[e] <= o->ld_t,
                    "anima_linear: LoRA entry %d (off %d, n %d, r0 %d, r %d) invalid", e, o->lora_off[e],
                    o->lora_n[e], o->lora_r0[e], o->lora_r[e]);
    }
  }
  // the epilogue reads per-column vectors 16 bytes at a time
  ANIMA_REQUIRE(aligned16(W->scale) && (!W->bias || aligned16(W->bias)) && (!o->norm_q || aligned16(o->norm_q)) &&
                    (!o->norm_k || aligned16(o->norm_k)) && (!o->rope || aligned16(o->rope)) &&
                    (!o->gate || (aligned16(o->gate) && o->gate_off % 4 == 0)),
                "anima_linear: scale/bias/gate/norm/rope vectors must be 16-byte aligned (gate_off a multiple of 4)");
  anima_weight grid;
  if (W->kind == ANIMA_W_W4) {
    int st = w4_scratch(ctx, static_cast<size_t>(W->N) * W->K);
    if (st) return st;
    st = launch_w4_decode(ctx, static_cast<const uint8_t*>(W->data), W->s_rel, W->codebook, W->N, W->K, ctx->w4_ws);
    if (st) return st;
    grid = *W;
    grid.kind = ANIMA_W_I8;
    grid.data = ctx->w4_ws;
    W = &grid;
  }
  // Two planes: 128-column tiles double-buffer both accumulators (2 x 2 x 128 TMEM columns) so the
  // epilogue overlaps the next tile's MMAs. One plane: 256-column tiles, double-buffered.
  // LoRA side paths: 128-column tiles (each inside one entry), with the entry's B slice staged
  // in shared memory in place of one pipeline stage.
  const bool two = x->lo != nullptr;
  if (o->lora_t) return two ? gemm::launch<128, 2, true>(ctx, x, W, o) : gemm::launch<128, 1, true>(ctx, x, W, o);
  if (two) {
    // 128-column tiles: double-buffered accumulators and three pipeline stages measured faster than
    // 256-column tiles at every block shape, K = 8192 included (135 vs 169 us for the 8192 -> 2048
    // linear at 4096 tokens). ANIMA_GEMM_BN2=256 selects the wide tile for experiments.
    static const int bn2 = [] {
      const char* e = getenv("ANIMA_GEMM_BN2");
      return e ? atoi(e) : 0;
    }();
    const bool wide = bn2 == 256;
    if (W->N % 256 == 0 && wide) return gemm::launch<256, 2, false>(ctx, x, W, o);
    return gemm::launch<128, 2, false>(ctx, x, W, o);
  }
  if (W->N % 256 == 0) return gemm::launch<256, 1, false>(ctx, x, W, o);
  return gemm::launch<128, 1, false>(ctx, x, W, o);
}
