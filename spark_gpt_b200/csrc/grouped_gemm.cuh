// Ragged per-expert grouped GEMM on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM, operands staged by TMA).
//
// One persistent, warp-specialised kernel template covers every contraction
// of the MoE layer (spark-gpt train.py:1625-2063 does the same work with six
// Triton kernels):
//
//   gate_up fwd   xs (R,H) . W_gu[e]^T  -> gu (R,2I), h = silu(g)*u  [kEpiSwigluFwd]
//   down fwd      h  (R,I) . W_d[e]^T   -> y (R,H)                   [kEpiStoreBf16]
//   down dgrad    dy (R,H) . W_d[e]     -> dh, then the SwiGLU backward
//                 in the epilogue       -> d_gu (R,2I)               [kEpiSwigluBwd]
//   gate_up dgrad d_gu (R,2I) . W_gu[e] -> dxs (R,H)                 [kEpiStoreBf16]
//   wgrads        A_e^T . B_e over the rows of expert e -> fp32 (E,M,N) [kEpiStoreF32]
//   router        logits / d_x / d_W_r^T (single group)             [kEpiStoreBf16 / F32T]
//
// Row layout: routed rows are grouped by expert and every expert's block is
// padded to a multiple of 128 rows (zero rows), so a 128-row M tile never
// straddles two experts and a 64-row K block of a weight gradient never mixes
// experts.  `tile_expert[m]` maps an M tile to its expert; `pad_offsets[e]`
// is the first padded row of expert e and pad_offsets[E] the padded total.
//
// Roles (320 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer (one lane): A and B tiles into a STAGES-deep ring
//   warp 1      MMA issuer (one lane): 4 x tcgen05.mma (K=16) per 64-wide K block,
//               into one of two TMEM accumulators (2 x BN fp32 columns)
//   warps 2..9  epilogue: tcgen05.ld TMEM -> registers -> fused math -> global.
//               Warp w reads TMEM lanes 32*(w%4).. (its hardware lane quarter); the two
//               warps of a quarter split the tile's 32-column chunks between them.
//
// Shared-memory tiles use the 128-byte swizzle.  K-major tiles are
// [rows][64] (128 B per row); MN-major tiles (the transposed operands of
// dgrad/wgrad) are [MN/64 chunks][64 k rows][64] with an 8 KB chunk stride.
#pragma once

#include "common.cuh"

namespace b200moe {

enum Epilogue : int {
  kEpiStoreBf16 = 0,
  kEpiSwigluFwd = 1,
  kEpiSwigluBwd = 2,
  kEpiStoreF32 = 3,
  kEpiStoreF32T = 4,
  kEpiSwigluBwdCombine = 5,  // down dgrad from gathered d_out: combine backward fused in
  kEpiAxpby = 6,             // bf16 out = alpha*acc + beta*aux, or fp32 update += neg_lr*bf16(..)
  kEpiStoreF32Tma = 7,       // kEpiStoreF32 through shared memory and TMA stores / reduce-adds
  kEpiSwigluFwdF8 = 8,       // fp8 gate_up: gu, h stored e4m3 with the delayed scales
  kEpiSwigluBwdF8 = 9,       // down dgrad, SwiGLU backward against e4m3 gu, d_gu stored e5m2
};

// Operand kinds of the expert GEMMs: bf16 (tcgen05.mma kind::f16), or fp8
// (kind::f8f6f4) with A and B formats e4m3 x e4m3 or e5m2 x e4m3.  An fp8
// K block holds 128 elements, so a stage's shared-memory tiles have the same
// bytes and the same 128-byte swizzle as a 64-element bf16 K block.
enum OperandKind : int {
  kOpBf16 = 0,
  kOpE4m3 = 1,     // A e4m3, B e4m3
  kOpE5m2E4m3 = 2  // A e5m2, B e4m3
};

template <int OP>
struct OpTraits {
  static constexpr int kBK = OP == kOpBf16 ? 64 : 128;   // elements per K block
  static constexpr int kMmaK = OP == kOpBf16 ? 16 : 32;  // elements per MMA
  static constexpr uint32_t kAFmt = OP == kOpE5m2E4m3 ? 1u : 0u;
};

// Which operand is gathered row by row from a token-major tensor (x or d_out)
// with TMA tile::gather4 instead of being read from a materialised
// routed-row buffer.
enum Gather : int {
  kGatherNone = 0,
  kGatherA = 1,
  kGatherB = 2,
};

enum Schedule : int {
  kRowsRagged = 0,  // M = routed rows (one expert per 128-row tile), K static
  kKRagged = 1,     // K = the routed rows of one expert (weight gradients)
};

struct GemmParams {
  const int* tile_expert;  // kRowsRagged: expert of each M tile (nullptr: one group)
  const int* pad_offsets;  // E+1 padded row starts (nullptr: one group of k_blocks)
  int num_groups;
  int m_tiles;        // kRowsRagged single group / kKRagged: M / 128
  int n_tiles;        // N / BN
  int k_blocks;       // kRowsRagged: K / 64; kKRagged single group: ceil(rows / 64)
  int b_group_rows;   // rows of one group in B's tensor map (outer dimension)
  int b_half_offset;  // kEpiSwigluFwd: rows from the gate half to the up half (I)
  long long m_valid;  // rows that may be written (kRowsRagged)
  int n_valid;        // columns that may be written
  void* out;
  long long ld_out;
  void* out2;
  long long ld_out2;
  const void* aux;
  long long ld_aux;
  int inter;          // I: column offset of the up half inside gu / d_gu
  int accumulate;     // fp32 outputs: add into the existing values
  long long out_group_stride;
  int k_split_blocks; // kKRagged single group split over K: 64-row blocks per split (0: none)
  // gathered operand: padded row p reads token row_flat[p] / gather_k of the
  // token-major tensor; padding rows (row_flat < 0) read token gather_oob
  // (one past the end: zero fill)
  const int* gather_rows;
  int gather_k;
  int gather_oob;
  // kEpiSwigluBwdCombine
  const void* aux2;            // h (Rcap, I)
  long long ld_aux2;
  const __nv_bfloat16* route_w;  // routing weights, flat slot order (T*k)
  float* dw_part;              // per-(N tile, half) partial d_weights, [parts][Rcap]
  long long part_stride;
  // kEpiStoreBf16: when set, padded row p is written to output row
  // scatter_rows[p] (token-major layout t*k+s) and padding rows are skipped
  const int* scatter_rows;
  // kEpiAxpby (the batched Newton-Schulz products of Muon): v = alpha*acc +
  // beta*aux[row, col] (aux bf16, or alpha*acc when aux is null); with `update`
  // set, update[row, col] += neg_lr * bf16(v) (fp32) instead of storing v.
  // Row offsets of a group's output: T.g * out_group_stride (K-ragged Gram
  // products); rows-ragged products index the stacked rows directly.
  float alpha, beta, neg_lr;
  float* update;
  long long ld_update;
  // fp8 path (spark-gpt train.py:1301-1530): the delayed per-site scales
  // (x, gu, h, d_gu, dy) and the amax slots the epilogues raise.  An output is
  // multiplied by 1 / (deq_a[0] * deq_b[0] * deq_g[group]) over the pointers
  // that are set: products of powers of two, so the scaling is exact.
  const float* fp8_scale;
  float* fp8_amax;
  const float* deq_a;
  const float* deq_b;
  const float* deq_g;
  // kKRagged pair tiles over several row segments (the weight gradient of an
  // expert whose rows sit in several buffers of one allocation): with
  // k_segments > 1, pad_offsets holds k_segments rows of num_groups + 1
  // absolute row offsets, and group g's K rows are the union over segments s
  // of [pad_offsets[s][g], pad_offsets[s][g + 1]), in segment order.
  int k_segments;
};

__device__ __forceinline__ float deq_factor(const GemmParams& p, int g) {
  float d = 1.f;
  if (p.deq_a) d *= __ldg(p.deq_a);
  if (p.deq_b) d *= __ldg(p.deq_b);
  if (p.deq_g) d *= __ldg(p.deq_g + g);
  return 1.0f / d;
}

__device__ __forceinline__ int gather_token(const GemmParams& p, int row) {
  const int f = __ldg(p.gather_rows + row);
  return f >= 0 ? f / p.gather_k : p.gather_oob;
}

// sigmoid with the hardware exp2 approximation and approximate divide: about
// 1e-6 relative error, far below the bf16 rounding that follows every use.
__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr uint32_t kABytes = 128 * 64 * 2;
  static constexpr uint32_t kBBytes = BN * 64 * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kBarrierBytes = 256;
  static constexpr uint32_t kTotal = STAGES * kStageBytes + kBarrierBytes + 1024;
};

template <int BN>
struct TmemCols {
  static constexpr uint32_t value = (2 * BN < 32) ? 32 : 2 * BN;
};

struct TileInfo {
  int m, n, g, krow0, kblocks;
};

template <int SCHED>
__device__ __forceinline__ TileInfo decode_tile(const GemmParams& p, int t) {
  TileInfo T;
  if (SCHED == kRowsRagged) {
    T.m = t / p.n_tiles;
    T.n = t - T.m * p.n_tiles;
    T.g = p.tile_expert ? __ldg(p.tile_expert + T.m) : 0;
    T.krow0 = 0;
    T.kblocks = p.k_blocks;
  } else {
    const int per = p.m_tiles * p.n_tiles;
    T.g = t / per;
    const int r = t - T.g * per;
    T.m = r / p.n_tiles;
    T.n = r - T.m * p.n_tiles;
    if (p.pad_offsets) {
      const int s = __ldg(p.pad_offsets + T.g);
      const int e = __ldg(p.pad_offsets + T.g + 1);
      T.krow0 = s;
      T.kblocks = (e - s) / 64;
    } else if (p.k_split_blocks > 0) {
      // group index = K split: blocks [g*ks, min((g+1)*ks, k_blocks))
      const int b0 = T.g * p.k_split_blocks;
      const int b1 = min(b0 + p.k_split_blocks, p.k_blocks);
      T.krow0 = b0 * 64;
      T.kblocks = max(b1 - b0, 0);
    } else {
      T.krow0 = 0;
      T.kblocks = p.k_blocks;
    }
  }
  return T;
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
    w.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
    w.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
    w.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
    d[q] = w;
  }
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float* v) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w = s[q];
    v[8 * q + 0] = bf16_lo(w.x);
    v[8 * q + 1] = bf16_hi(w.x);
    v[8 * q + 2] = bf16_lo(w.y);
    v[8 * q + 3] = bf16_hi(w.y);
    v[8 * q + 4] = bf16_lo(w.z);
    v[8 * q + 5] = bf16_hi(w.z);
    v[8 * q + 6] = bf16_lo(w.w);
    v[8 * q + 7] = bf16_hi(w.w);
  }
}

// SwiGLU-backward epilogue: pull this lane's row of g and u for the tile's
// column half into L2 before the accumulator is ready, so the epilogue's loads
// of them (one chunk ahead) hit L2 instead of waiting on DRAM.
template <int BN>
__device__ __forceinline__ void prefetch_gu_row(const GemmParams& p, const TileInfo& T,
                                                int row_in, int half) {
  const long long row = static_cast<long long>(T.m) * 128 + row_in;
  if (row >= p.m_valid) return;
  const char* gu = reinterpret_cast<const char*>(static_cast<const __nv_bfloat16*>(p.aux) +
                                                 row * p.ld_aux + T.n * BN + half * (BN / 2));
  const long long up = static_cast<long long>(p.inter) * 2;
#pragma unroll
  for (int off = 0; off < BN; off += 128) {  // BN/2 columns = BN bytes, 128-byte lines
    asm volatile("prefetch.global.L2 [%0];" ::"l"(gu + off));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(gu + up + off));
  }
}

// Epilogue of a weight-gradient tile whose expert received no rows: zeros
// (or nothing when accumulating).  Warps split the columns by `half`.
template <int EPI, int BN>
__device__ __forceinline__ void epilogue_empty_tile(const GemmParams& p, const TileInfo& T,
                                                    int row_in, int half) {
  constexpr int BM = 128;
  // a weight-gradient tile of an expert that received no rows
  if ((EPI == kEpiStoreF32 || EPI == kEpiStoreF32Tma || EPI == kEpiStoreF32T) && !p.accumulate) {
    if (EPI == kEpiStoreF32 || EPI == kEpiStoreF32Tma) {
      float* o = static_cast<float*>(p.out) + T.g * p.out_group_stride +
                 static_cast<long long>(T.m * BM + row_in) * p.ld_out + T.n * BN;
      float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c = half * (BN / 2); c < (half + 1) * (BN / 2) && T.n * BN + c < p.n_valid; c += 4)
        *reinterpret_cast<float4*>(o + c) = z;
    } else {
      for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); ++c) {
        const int col = T.n * BN + c;
        if (col < p.n_valid)
          static_cast<float*>(p.out)[T.g * p.out_group_stride +
                                     static_cast<long long>(col) * p.ld_out + T.m * BM +
                                     row_in] = 0.f;
      }
    }
  }
}

// Drain one accumulator tile (this warp's 32 TMEM lanes, its half of the
// 32-column chunks) through the fused epilogue.  `taddr` is the TMEM address
// of the warp's lane quarter at the tile's first column.
template <int EPI, int BN>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, const TileInfo& T,
                                              int row_in, int half, uint32_t taddr) {
  constexpr int BM = 128;
  if (EPI == kEpiStoreBf16) {
    long long row = static_cast<long long>(T.m) * BM + row_in;
    bool row_ok = row < p.m_valid;
    if (p.scatter_rows != nullptr && row_ok) {
      row = __ldg(p.scatter_rows + row);
      row_ok = row >= 0;
    }
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + (row_ok ? row : 0) * p.ld_out;
#pragma unroll 1
    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      const int col0 = T.n * BN + c * 32;
      if (row_ok) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (col0 + 32 <= p.n_valid) {
          store_bf16x32(o + col0, v);
        } else {
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.n_valid) o[col0 + j] = __float2bfloat16_rn(v[j]);
        }
      }
    }
  } else if (EPI == kEpiSwigluFwd) {
    constexpr int HALF = BN / 2;
    const long long row = static_cast<long long>(T.m) * BM + row_in;
    const bool row_ok = row < p.m_valid;
    __nv_bfloat16* gu = static_cast<__nv_bfloat16*>(p.out) + row * p.ld_out;
    __nv_bfloat16* hh = static_cast<__nv_bfloat16*>(p.out2) + row * p.ld_out2;
#pragma unroll 1
    for (int c = half * (HALF / 64); c < (half + 1) * (HALF / 64); ++c) {
      uint32_t rg[32], ru[32];
      tmem_ld32(taddr + c * 32, rg);
      tmem_ld32(taddr + HALF + c * 32, ru);
      tmem_wait_ld();
      if (row_ok) {
        const int col = T.n * HALF + c * 32;
        float g[32], u[32], h[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          g[j] = bf16_round(__uint_as_float(rg[j]));
          u[j] = bf16_round(__uint_as_float(ru[j]));
          h[j] = g[j] * sigmoidf_(g[j]) * u[j];
        }
        store_bf16x32(gu + col, g);
        store_bf16x32(gu + p.inter + col, u);
        store_bf16x32(hh + col, h);
      }
    }
  } else if (EPI == kEpiSwigluBwd) {
    const long long row = static_cast<long long>(T.m) * BM + row_in;
    const bool row_ok = row < p.m_valid;
    const __nv_bfloat16* gu = static_cast<const __nv_bfloat16*>(p.aux) + row * p.ld_aux;
    __nv_bfloat16* dgu = static_cast<__nv_bfloat16*>(p.out) + row * p.ld_out;
#pragma unroll 1
    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      if (row_ok) {
        const int col = T.n * BN + c * 32;
        float g[32], u[32], dg[32], du[32];
        load_bf16x32(gu + col, g);
        load_bf16x32(gu + p.inter + col, u);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float dh = bf16_round(__uint_as_float(r[j]));
          const float sig = sigmoidf_(g[j]);
          dg[j] = dh * u[j] * (sig * (1.0f + g[j] * (1.0f - sig)));
          du[j] = dh * g[j] * sig;
        }
        store_bf16x32(dgu + col, dg);
        store_bf16x32(dgu + p.inter + col, du);
      }
    }
  } else if (EPI == kEpiSwigluFwdF8 || EPI == kEpiSwigluBwdF8) {
    // the fp8 epilogues run only through the TMA-store ring (epilogue_tile_tma)
    if (row_in == 0) raise_fault(kFaultBadShape);
  } else if (EPI == kEpiSwigluBwdCombine) {
    // acc = d_out[token] . W_d[e] (unscaled).  dh = bf16(w * acc); the routing
    // weight's gradient <d_out[token], y[row]> = <acc, h[row]> is summed here;
    // w * h is written for the down-projection weight gradient.
    const long long row = static_cast<long long>(T.m) * BM + row_in;
    const int f = __ldg(p.gather_rows + row);
    const float w = f >= 0 ? __bfloat162float(p.route_w[f]) : 0.f;
    const __nv_bfloat16* gu = static_cast<const __nv_bfloat16*>(p.aux) + row * p.ld_aux;
    const __nv_bfloat16* hh = static_cast<const __nv_bfloat16*>(p.aux2) + row * p.ld_aux2;
    __nv_bfloat16* dgu = static_cast<__nv_bfloat16*>(p.out) + row * p.ld_out;
    __nv_bfloat16* hw = static_cast<__nv_bfloat16*>(p.out2) + row * p.ld_out2;
    float dwp = 0.f;
#pragma unroll 1
    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      const int col = T.n * BN + c * 32;
      float g[32], u[32], hv[32], dg[32], du[32];
      load_bf16x32(gu + col, g);
      load_bf16x32(gu + p.inter + col, u);
      load_bf16x32(hh + col, hv);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float a = __uint_as_float(r[j]);
        dwp += a * hv[j];
        const float dh = bf16_round(w * a);
        const float sig = sigmoidf_(g[j]);
        dg[j] = dh * u[j] * (sig * (1.0f + g[j] * (1.0f - sig)));
        du[j] = dh * g[j] * sig;
        hv[j] *= w;
      }
      store_bf16x32(dgu + col, dg);
      store_bf16x32(dgu + p.inter + col, du);
      store_bf16x32(hw + col, hv);
    }
    p.dw_part[(T.n * 2 + half) * p.part_stride + row] = dwp;
  } else if (EPI == kEpiAxpby) {
    const long long row = static_cast<long long>(T.m) * BM + row_in;
    const long long base = T.g * p.out_group_stride;
    const bool row_ok = row < p.m_valid;
#pragma unroll 1
    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      const int col0 = T.n * BN + c * 32;
      if (!row_ok) continue;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = p.alpha * __uint_as_float(r[j]);
      if (p.aux != nullptr) {
        float cv[32];
        load_bf16x32(static_cast<const __nv_bfloat16*>(p.aux) + base + row * p.ld_aux + col0, cv);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += p.beta * cv[j];
      }
      if (p.update != nullptr) {
        float4* u = reinterpret_cast<float4*>(p.update + base + row * p.ld_update + col0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 w = u[j];
          w.x += p.neg_lr * bf16_round(v[4 * j + 0]);
          w.y += p.neg_lr * bf16_round(v[4 * j + 1]);
          w.z += p.neg_lr * bf16_round(v[4 * j + 2]);
          w.w += p.neg_lr * bf16_round(v[4 * j + 3]);
          u[j] = w;
        }
      } else {
        store_bf16x32(static_cast<__nv_bfloat16*>(p.out) + base + row * p.ld_out + col0, v);
      }
    }
  } else if (EPI == kEpiStoreF32) {
    float* o = static_cast<float*>(p.out) + T.g * p.out_group_stride +
               static_cast<long long>(T.m * BM + row_in) * p.ld_out + T.n * BN;
#pragma unroll 1
    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      float4* d = reinterpret_cast<float4*>(o + c * 32);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 v = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
        if (p.accumulate) {
          const float4 old = d[j];
          v.x += old.x;
          v.y += old.y;
          v.z += old.z;
          v.w += old.w;
        }
        d[j] = v;
      }
    }
  } else {  // kEpiStoreF32T
    float* o = static_cast<float*>(p.out) + T.g * p.out_group_stride + T.m * BM + row_in;
#pragma unroll 1
    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int col = T.n * BN + c * 32 + j;
        if (col < p.n_valid) {
          float* dst = o + static_cast<long long>(col) * p.ld_out;
          const float v = __uint_as_float(r[j]);
          *dst = p.accumulate ? (*dst + v) : v;
        }
      }
    }
  }
}
// ---------------------------------------------------------------------------
// Epilogue through shared memory + TMA stores: each warp owns a ring of kOutRing
// 2 KB buffers; a 32-row x 32-column bf16 chunk of its rows is written there
// (64-byte swizzle, conflict-free) and stored with one TMA tensor store, so
// global writes are full, coalesced rows and asynchronous.  The output tensor
// maps have a {32, 32} box and the 64-byte swizzle.
// ---------------------------------------------------------------------------
#ifndef B200MOE_OUT_RING
#define B200MOE_OUT_RING 2  // 2 KB staging buffers per epilogue warp (2: six operand stages fit)
#endif
constexpr int kOutRing = B200MOE_OUT_RING;

struct OutRing {
  uint8_t* base;  // kOutRing x 2048 bytes, 512-byte aligned
  int next;
  // SwiGLU-backward epilogue of the pair kernel: two 2 KB buffers that a TMA
  // load fills with the warp's 32 x 32 chunk of g and of u, completing on
  // in_bar (one phase per chunk)
  uint8_t* in = nullptr;
  uint64_t* in_bar = nullptr;
  uint32_t in_phase = 0;
  volatile int* abort = nullptr;
};

// Issue the TMA loads of one 32-row x 32-column chunk of g (column col) and of
// u (column inter + col) into the warp's input buffers (64-byte swizzle, the
// layout ring_put writes).  Every lane's earlier reads of the buffers are
// ordered before the asynchronous refill (proxy fence, then the warp
// converges); lane 0 issues; completion on ring.in_bar.
// BYTES: one chunk's size (2048 for bf16, 1024 for the unswizzled fp8 boxes).
template <int BYTES = 2048>
__device__ __forceinline__ void gu_chunk_load(const OutRing& ring, const CUtensorMap* tm,
                                              int col, int inter, int row0, int lane) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    mbar_expect_tx(ring.in_bar, 2 * BYTES);
    tma_load_2d(ring.in, tm, ring.in_bar, col, row0);
    tma_load_2d(ring.in + 2048, tm, ring.in_bar, inter + col, row0);
  }
}

// Chunks of one warp are stored in groups of G: G chunks are written to
// consecutive ring buffers, then one proxy fence and one bulk group of G TMA
// stores cover them.  Within one kernel every group has the same G, so
// "at most kOutRing/G - 1 groups still reading" frees the next G buffers.
template <int G>
__device__ __forceinline__ void ring_acquire(int lane) {
  static_assert(kOutRing % G == 0, "ring size must be a multiple of the store group");
  if (lane == 0) bulk_wait_group_read<kOutRing / G - 1>();
  __syncwarp();
}

// Chunk `slot` of the group: this lane's row of 32 fp32 values as bf16 in the
// 64-byte-swizzled 32 x 32 box.
__device__ __forceinline__ void ring_put(const OutRing& ring, int slot, const float* v, int lane) {
  uint8_t* buf = ring.base + ((ring.next + slot) % kOutRing) * 2048;
  uint4* rowp = reinterpret_cast<uint4*>(buf + lane * 64);
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
    w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
    w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
    w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
    rowp[j ^ sw] = w;
  }
}

// Chunk `slot` of the group: this lane's row of 16 fp32 values (64 bytes) in
// the 64-byte-swizzled 32 x 16 fp32 box.
__device__ __forceinline__ void ring_put_f32(const OutRing& ring, int slot, const float* v,
                                             int lane) {
  uint8_t* buf = ring.base + ((ring.next + slot) % kOutRing) * 2048;
  uint4* rowp = reinterpret_cast<uint4*>(buf + lane * 64);
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    rowp[j ^ sw] = make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                              __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
}

template <int G>
__device__ __forceinline__ void ring_flush(OutRing& ring, const CUtensorMap* const* tm,
                                           const int* col, int row0, int lane) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g)
      tma_store_2d(tm[g], ring.base + ((ring.next + g) % kOutRing) * 2048, col[g], row0);
    bulk_commit_group();
  }
  ring.next = (ring.next + G) % kOutRing;
}

// Chunk `slot` of the group: this lane's row of 32 fp8 bytes in the unswizzled
// 32 x 32-byte box.
__device__ __forceinline__ void ring_put_u8(const OutRing& ring, int slot, const uint32_t* w,
                                            int lane) {
  uint8_t* buf = ring.base + ((ring.next + slot) % kOutRing) * 2048;
  uint4* rowp = reinterpret_cast<uint4*>(buf + lane * 32);
  rowp[0] = make_uint4(w[0], w[1], w[2], w[3]);
  rowp[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

__device__ __forceinline__ void store_chunk_tma_u8(OutRing& ring, const CUtensorMap* tm,
                                                   const uint32_t* w, int lane, int col,
                                                   int row0) {
  ring_acquire<1>(lane);
  ring_put_u8(ring, 0, w, lane);
  ring_flush<1>(ring, &tm, &col, row0, lane);
}

// One 32 x 32 bf16 chunk of a single input tile (the C operand of kEpiAxpby)
// into the warp's first input buffer; lane 0 issues; completion on ring.in_bar.
__device__ __forceinline__ void aux_chunk_load(const OutRing& ring, const CUtensorMap* tm,
                                               int col, int row0, int lane) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    mbar_expect_tx(ring.in_bar, 2048);
    tma_load_2d(ring.in, tm, ring.in_bar, col, row0);
  }
}

__device__ __forceinline__ void store_chunk_tma(OutRing& ring, const CUtensorMap* tm,
                                                const float* v, int lane, int col, int row0) {
  ring_acquire<1>(lane);
  ring_put(ring, 0, v, lane);
  ring_flush<1>(ring, &tm, &col, row0, lane);
}

#ifndef B200MOE_EPI_GROUP
#define B200MOE_EPI_GROUP 1  // chunks per proxy fence in the plain bf16 epilogue
#endif
#ifndef B200MOE_WIDE_BF16
#define B200MOE_WIDE_BF16 1  // plain bf16 stores as 32 x 64 boxes (128-byte swizzle)
#endif
constexpr bool kWideBf16Store = B200MOE_WIDE_BF16 != 0;
#ifndef B200MOE_WIDE_F32
#define B200MOE_WIDE_F32 1  // fp32 weight-gradient stores as 32 x 32 boxes (128-byte swizzle)
#endif
constexpr bool kWideF32Store = B200MOE_WIDE_F32 != 0;

// The bf16-output epilogues (plain store, SwiGLU forward, SwiGLU backward) with
// TMA stores.  Outputs: O0 = out (or gu / d_gu), O1 = h (SwiGLU forward).
// SCALED: multiply the accumulator by deq_factor (the fp8 GEMMs' dequantization).
template <int EPI, int BN, bool SCALED = false>
__device__ __forceinline__ void epilogue_tile_tma(const GemmParams& p, const TileInfo& T,
                                                  int quarter, int lane, int half,
                                                  uint32_t taddr, const CUtensorMap* tmO0,
                                                  const CUtensorMap* tmO1, OutRing& ring,
                                                  unsigned long long* prof = nullptr) {
  constexpr int BM = 128;
  const int row0 = T.m * BM + quarter * 32;
  if (EPI == kEpiStoreF32Tma && kWideF32Store) {
    // fp32 weight-gradient tile: each 32-column TMEM chunk leaves as one 32 x 32
    // box (4 KB, 128-byte swizzle) in the ring's two buffers, stored (or
    // reduce-added into the gradient when accumulating)
    static_assert(kOutRing % 2 == 0, "wide stores take buffer pairs");
    const int rowg = T.g * p.m_tiles * BM + row0;  // (E*M, N) view of the output
    const float sc = SCALED ? deq_factor(p, T.g) : 1.f;
#pragma unroll 1
    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
      if (T.n * BN + c * 32 >= p.n_valid) break;
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      ring_acquire<2>(lane);
      uint4* rowp = reinterpret_cast<uint4*>(ring.base + ring.next * 2048 + lane * 128);
      const int sw = lane & 7;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          v[q] = SCALED ? __uint_as_float(r[4 * j + q]) * sc : __uint_as_float(r[4 * j + q]);
        rowp[j ^ sw] = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]),
                                  __float_as_uint(v[2]), __float_as_uint(v[3]));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const uint8_t* buf = ring.base + ring.next * 2048;
        const int col = T.n * BN + c * 32;
        if (p.accumulate)
          tma_reduce_add_2d(tmO0, buf, col, rowg);
        else
          tma_store_2d(tmO0, buf, col, rowg);
        bulk_commit_group();
      }
      ring.next = (ring.next + 2) % kOutRing;
    }
  } else if (EPI == kEpiStoreF32Tma) {
    // fp32 weight-gradient tile: each 32-column TMEM chunk leaves as two 32 x 16
    // boxes, stored (or reduce-added into the gradient when accumulating)
    const int rowg = T.g * p.m_tiles * BM + row0;  // (E*M, N) view of the output
    const float sc = SCALED ? deq_factor(p, T.g) : 1.f;
#pragma unroll 1
    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
      // columns past N (a last tile wider than what is left of N) are not stored
      if (T.n * BN + c * 32 >= p.n_valid) break;
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        ring_acquire<1>(lane);
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = SCALED ? __uint_as_float(r[16 * part + j]) * sc
                                                   : __uint_as_float(r[16 * part + j]);
        ring_put_f32(ring, 0, v, lane);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const uint8_t* buf = ring.base + ring.next * 2048;
          const int col = T.n * BN + c * 32 + 16 * part;
          if (p.accumulate)
            tma_reduce_add_2d(tmO0, buf, col, rowg);
          else
            tma_store_2d(tmO0, buf, col, rowg);
          bulk_commit_group();
        }
        ring.next = (ring.next + 1) % kOutRing;
      }
    }
  } else if (EPI == kEpiAxpby) {
    // Newton-Schulz products (Muon): v = alpha*acc + beta*C, C's chunks arriving
    // by TMA in the warp's input buffer (the first one loaded before the
    // accumulator wait); v leaves as bf16 through the ring, or, with `update`,
    // update += neg_lr * bf16(v) as fp32 TMA reduce-adds.  Rows: the (groups x
    // M, N) view for weight-gradient-shaped (K-ragged) products, the stacked
    // rows otherwise (m_tiles is 0 there).
    const int rowg = T.g * p.m_tiles * BM + row0;
    const bool has_c = p.aux != nullptr;
    const int c0 = half * (BN / 64), c1 = (half + 1) * (BN / 64);
    const int sw = (lane >> 1) & 3;
#pragma unroll 1
    for (int c = c0; c < c1; ++c) {
      const int col = T.n * BN + c * 32;
      float v[32];
      uint4 cc[4];
      if (has_c) {
        const bool got =
            __all_sync(0xffffffffu, mbar_wait(ring.in_bar, ring.in_phase, ring.abort));
        if (!got) return;
        ring.in_phase ^= 1u;
        const uint4* cs = reinterpret_cast<const uint4*>(ring.in + lane * 64);
#pragma unroll
        for (int j = 0; j < 4; ++j) cc[j] = cs[j ^ sw];
        if (c + 1 < c1) aux_chunk_load(ring, tmO1, col + 32, rowg, lane);
      }
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = p.alpha * __uint_as_float(r[j]);
      if (has_c) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[8 * j + 0] += p.beta * bf16_lo(cc[j].x); v[8 * j + 1] += p.beta * bf16_hi(cc[j].x);
          v[8 * j + 2] += p.beta * bf16_lo(cc[j].y); v[8 * j + 3] += p.beta * bf16_hi(cc[j].y);
          v[8 * j + 4] += p.beta * bf16_lo(cc[j].z); v[8 * j + 5] += p.beta * bf16_hi(cc[j].z);
          v[8 * j + 6] += p.beta * bf16_lo(cc[j].w); v[8 * j + 7] += p.beta * bf16_hi(cc[j].w);
        }
      }
      if (p.update != nullptr) {
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          ring_acquire<1>(lane);
          float w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = p.neg_lr * bf16_round(v[16 * part + j]);
          ring_put_f32(ring, 0, w, lane);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_2d(tmO0, ring.base + ring.next * 2048, col + 16 * part, rowg);
            bulk_commit_group();
          }
          ring.next = (ring.next + 1) % kOutRing;
        }
      } else {
        store_chunk_tma(ring, tmO0, v, lane, col, rowg);
      }
    }
  } else if (EPI == kEpiStoreBf16 && kWideBf16Store) {
    // two 32-column TMEM chunks leave as one 32 x 64 bf16 box (4 KB, 128-byte
    // swizzle) in two consecutive ring buffers: half the TMA stores
    static_assert(kOutRing % 2 == 0 && (BN / 64) % 2 == 0, "wide stores take buffer pairs");
    const float sc = SCALED ? deq_factor(p, T.g) : 1.f;
#pragma unroll 1
    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); c += 2) {
      uint32_t r0[32], r1[32];
      tmem_ld32(taddr + c * 32, r0);
      tmem_ld32(taddr + (c + 1) * 32, r1);
      tmem_wait_ld();
      ring_acquire<2>(lane);
      uint4* rowp = reinterpret_cast<uint4*>(ring.base + ring.next * 2048 + lane * 128);
      const int sw = lane & 7;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t* r = j < 4 ? r0 + 8 * j : r1 + 8 * (j - 4);
        float v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = SCALED ? __uint_as_float(r[q]) * sc : __uint_as_float(r[q]);
        rowp[j ^ sw] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                  pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmO0, ring.base + ring.next * 2048, T.n * BN + c * 32, row0);
        bulk_commit_group();
      }
      ring.next = (ring.next + 2) % kOutRing;
    }
  } else if (EPI == kEpiStoreBf16) {
    constexpr int G = B200MOE_EPI_GROUP < BN / 64 ? B200MOE_EPI_GROUP : BN / 64;
    const float sc = SCALED ? deq_factor(p, T.g) : 1.f;
#pragma unroll 1
    for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); c += G) {
      uint32_t r[G][32];
      B200_PROF(long long q0 = clock64();)
#pragma unroll
      for (int g = 0; g < G; ++g) tmem_ld32(taddr + (c + g) * 32, r[g]);
      tmem_wait_ld();
      B200_PROF(long long q1 = clock64(); prof[0] += q1 - q0;)
      ring_acquire<G>(lane);
      B200_PROF(long long q2 = clock64(); prof[1] += q2 - q1;)
      const CUtensorMap* tms[G];
      int cols[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = SCALED ? __uint_as_float(r[g][j]) * sc
                                                   : __uint_as_float(r[g][j]);
        ring_put(ring, g, v, lane);
        tms[g] = tmO0;
        cols[g] = T.n * BN + (c + g) * 32;
      }
      ring_flush<G>(ring, tms, cols, row0, lane);
      B200_PROF(prof[2] += clock64() - q2;)
    }
  } else if (EPI == kEpiSwigluFwdF8) {
    // fp8 gate_up (train.py:1317-1354): g, u = bf16(acc / (s_x q_e)), h = silu(g) u;
    // gu and h leave as e4m3 boxes with the gu / h scales; amax of g, u and h
    constexpr int HALF = BN / 2;
    const float deq = deq_factor(p, T.g);
    const float s_gu = __ldg(p.fp8_scale + 1), s_h = __ldg(p.fp8_scale + 2);
    float m_gu = 0.f, m_h = 0.f;
#pragma unroll 1
    for (int c = half * (HALF / 64); c < (half + 1) * (HALF / 64); ++c) {
      uint32_t rg[32], ru[32];
      tmem_ld32(taddr + c * 32, rg);
      tmem_ld32(taddr + HALF + c * 32, ru);
      tmem_wait_ld();
      const int col = T.n * HALF + c * 32;
      uint32_t wg[8], wu[8], wh[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float g[4], u[4], h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          g[j] = bf16_round(__uint_as_float(rg[4 * q + j]) * deq);
          u[j] = bf16_round(__uint_as_float(ru[4 * q + j]) * deq);
          h[j] = g[j] * sigmoidf_(g[j]) * u[j];
          m_gu = fmaxf(m_gu, fmaxf(fabsf(g[j]), fabsf(u[j])));
          m_h = fmaxf(m_h, fabsf(h[j]));
        }
        wg[q] = pack_fp8x4<kE4M3>(g[0] * s_gu, g[1] * s_gu, g[2] * s_gu, g[3] * s_gu);
        wu[q] = pack_fp8x4<kE4M3>(u[0] * s_gu, u[1] * s_gu, u[2] * s_gu, u[3] * s_gu);
        wh[q] = pack_fp8x4<kE4M3>(h[0] * s_h, h[1] * s_h, h[2] * s_h, h[3] * s_h);
      }
      store_chunk_tma_u8(ring, tmO0, wg, lane, col, row0);
      store_chunk_tma_u8(ring, tmO0, wu, lane, p.inter + col, row0);
      store_chunk_tma_u8(ring, tmO1, wh, lane, col, row0);
    }
    m_gu = warp_max(m_gu);
    m_h = warp_max(m_h);
    if (lane == 0) {
      atomic_max_nonneg(p.fp8_amax + 1, m_gu);
      atomic_max_nonneg(p.fp8_amax + 2, m_h);
    }
  } else if (EPI == kEpiSwigluBwdF8) {
    // down dgrad with the SwiGLU backward against the e4m3 gu (train.py:1382-1423):
    // dh = bf16(acc); g, u = gu8 / s_gu; d_gu leaves as e5m2 boxes with the d_gu
    // scale; amax of d_gate, d_up.  The gu8 chunks arrive by TMA in the warp's
    // input buffers (32 rows x 32 bytes, unswizzled), as in the bf16 version.
    const float inv_s_gu = 1.0f / __ldg(p.fp8_scale + 1);
    const float s_dgu = __ldg(p.fp8_scale + 3);
    float m_d = 0.f;
    const int c0 = half * (BN / 64), c1 = (half + 1) * (BN / 64);
#pragma unroll 1
    for (int c = c0; c < c1; ++c) {
      const int col = T.n * BN + c * 32;
      const bool got = __all_sync(0xffffffffu, mbar_wait(ring.in_bar, ring.in_phase, ring.abort));
      if (!got) return;
      ring.in_phase ^= 1u;
      const uint4* gs = reinterpret_cast<const uint4*>(ring.in + lane * 32);
      const uint4* us = reinterpret_cast<const uint4*>(ring.in + 2048 + lane * 32);
      const uint4 g0 = gs[0], g1 = gs[1], u0 = us[0], u1 = us[1];
      if (c + 1 < c1) gu_chunk_load<1024>(ring, tmO1, col + 32, p.inter, row0, lane);
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      const uint32_t gw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const uint32_t uw[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      uint32_t wg[8], wu[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float g[4], u[4], dg[4], du[4];
        unpack_fp8x4<kE4M3>(gw[q], g);
        unpack_fp8x4<kE4M3>(uw[q], u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          g[j] *= inv_s_gu;
          u[j] *= inv_s_gu;
          const float dh = bf16_round(__uint_as_float(r[4 * q + j]));
          const float sig = sigmoidf_(g[j]);
          dg[j] = dh * u[j] * (sig * (1.0f + g[j] * (1.0f - sig)));
          du[j] = dh * g[j] * sig;
          m_d = fmaxf(m_d, fmaxf(fabsf(dg[j]), fabsf(du[j])));
        }
        wg[q] = pack_fp8x4<kE5M2>(dg[0] * s_dgu, dg[1] * s_dgu, dg[2] * s_dgu, dg[3] * s_dgu);
        wu[q] = pack_fp8x4<kE5M2>(du[0] * s_dgu, du[1] * s_dgu, du[2] * s_dgu, du[3] * s_dgu);
      }
      store_chunk_tma_u8(ring, tmO0, wg, lane, col, row0);
      store_chunk_tma_u8(ring, tmO0, wu, lane, p.inter + col, row0);
    }
    m_d = warp_max(m_d);
    if (lane == 0) atomic_max_nonneg(p.fp8_amax + 3, m_d);
  } else if (EPI == kEpiSwigluFwd) {
    constexpr int HALF = BN / 2;
#pragma unroll 1
    for (int c = half * (HALF / 64); c < (half + 1) * (HALF / 64); ++c) {
      uint32_t rg[32], ru[32];
      tmem_ld32(taddr + c * 32, rg);
      tmem_ld32(taddr + HALF + c * 32, ru);
      tmem_wait_ld();
      const int col = T.n * HALF + c * 32;
      float g[32], u[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        g[j] = bf16_round(__uint_as_float(rg[j]));
        u[j] = bf16_round(__uint_as_float(ru[j]));
      }
      store_chunk_tma(ring, tmO0, g, lane, col, row0);
      store_chunk_tma(ring, tmO0, u, lane, p.inter + col, row0);
#pragma unroll
      for (int j = 0; j < 32; ++j) g[j] = g[j] * sigmoidf_(g[j]) * u[j];
      store_chunk_tma(ring, tmO1, g, lane, col, row0);
    }
  } else {  // kEpiSwigluBwd
    // g, u of each 32-column chunk arrive by TMA in the warp's input buffers
    // (the first chunk's load was issued before the accumulator wait); the
    // next chunk's load is issued as soon as this one's values are in registers
    const int c0 = half * (BN / 64), c1 = (half + 1) * (BN / 64);
    const int sw = (lane >> 1) & 3;
#pragma unroll 1
    for (int c = c0; c < c1; ++c) {
      const bool got = __all_sync(0xffffffffu, mbar_wait(ring.in_bar, ring.in_phase, ring.abort));
      if (!got) return;
      ring.in_phase ^= 1u;
      uint4 gc[4], uc[4];
      {
        const uint4* gs = reinterpret_cast<const uint4*>(ring.in + lane * 64);
        const uint4* us = reinterpret_cast<const uint4*>(ring.in + 2048 + lane * 64);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          gc[j] = gs[j ^ sw];
          uc[j] = us[j ^ sw];
        }
      }
      if (c + 1 < c1) gu_chunk_load(ring, tmO1, T.n * BN + (c + 1) * 32, p.inter, row0, lane);
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      const int col = T.n * BN + c * 32;
      float g[32], u[32], dg[32];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        g[8 * j + 0] = bf16_lo(gc[j].x); g[8 * j + 1] = bf16_hi(gc[j].x);
        g[8 * j + 2] = bf16_lo(gc[j].y); g[8 * j + 3] = bf16_hi(gc[j].y);
        g[8 * j + 4] = bf16_lo(gc[j].z); g[8 * j + 5] = bf16_hi(gc[j].z);
        g[8 * j + 6] = bf16_lo(gc[j].w); g[8 * j + 7] = bf16_hi(gc[j].w);
        u[8 * j + 0] = bf16_lo(uc[j].x); u[8 * j + 1] = bf16_hi(uc[j].x);
        u[8 * j + 2] = bf16_lo(uc[j].y); u[8 * j + 3] = bf16_hi(uc[j].y);
        u[8 * j + 4] = bf16_lo(uc[j].z); u[8 * j + 5] = bf16_hi(uc[j].z);
        u[8 * j + 6] = bf16_lo(uc[j].w); u[8 * j + 7] = bf16_hi(uc[j].w);
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float dh = bf16_round(__uint_as_float(r[j]));
        const float sig = sigmoidf_(g[j]);
        dg[j] = dh * u[j] * (sig * (1.0f + g[j] * (1.0f - sig)));
        u[j] = dh * g[j] * sig;  // d_up, reusing u's registers
      }
      store_chunk_tma(ring, tmO0, dg, lane, col, row0);
      store_chunk_tma(ring, tmO0, u, lane, p.inter + col, row0);
    }
  }
}

constexpr int kEpilogueWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpilogueWarps;

template <int BN, bool A_MN, bool B_MN, int EPI, int SCHED, int STAGES, int GATHER = kGatherNone>
__global__ void __launch_bounds__(kGemmThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN");
  static_assert(SCHED == kRowsRagged ? !A_MN : (A_MN && B_MN), "operand majors vs schedule");
  static_assert(GATHER != kGatherB || (SCHED == kKRagged && B_MN), "B gathers only in wgrads");
  constexpr int BM = 128;
  constexpr int BK = 64;
  using S = GemmSmem<BN, STAGES>;
  constexpr uint32_t kTmemCols = TmemCols<BN>::value;
  constexpr uint32_t kIdesc = make_idesc_bf16(BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * S::kBBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpilogueWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  int num_tiles;
  if (SCHED == kRowsRagged) {
    const int mt = p.tile_expert ? (__ldg(p.pad_offsets + p.num_groups) / BM) : p.m_tiles;
    num_tiles = mt * p.n_tiles;
  } else {
    num_tiles = p.num_groups * p.m_tiles * p.n_tiles;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Lane 0 waits for a free stage, arms the barrier and issues the plain
    // tile loads; with a gathered operand every lane then issues gather4 loads
    // of 4 rows each.
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    // Gathered rows are looked up ahead of use so the index loads never sit on
    // the producer's critical path: the next tile's 4 rows per lane (row-ragged
    // A), or the rows of K blocks kb+1..kb+4 (K-ragged gathers), in registers.
    int4 tok_next = make_int4(0, 0, 0, 0);
    if (GATHER == kGatherA && SCHED == kRowsRagged && blockIdx.x < num_tiles) {
      const int r = (blockIdx.x / p.n_tiles) * BM + 4 * lane;
      tok_next = make_int4(gather_token(p, r), gather_token(p, r + 1), gather_token(p, r + 2),
                           gather_token(p, r + 3));
    }
    for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
      const TileInfo T = decode_tile<SCHED>(p, t);
      const int4 tok = tok_next;
      if (GATHER == kGatherA && SCHED == kRowsRagged && t + gridDim.x < num_tiles) {
        const int r = ((t + gridDim.x) / p.n_tiles) * BM + 4 * lane;
        tok_next = make_int4(gather_token(p, r), gather_token(p, r + 1), gather_token(p, r + 2),
                             gather_token(p, r + 3));
      }
      // K-ragged gathers: rows 4*(lane%16).. of K block kb live in q0 (kb), q1 (kb+1), ...
      int4 q0 = make_int4(0, 0, 0, 0), q1 = q0, q2 = q0, q3 = q0;
      auto k_rows = [&](int kb) -> int4 {
        if (kb >= T.kblocks) return make_int4(0, 0, 0, 0);
        const int r = T.krow0 + kb * BK + 4 * (lane & 15);
        return make_int4(gather_token(p, r), gather_token(p, r + 1), gather_token(p, r + 2),
                         gather_token(p, r + 3));
      };
      if (GATHER != kGatherNone && SCHED == kKRagged) {
        q0 = k_rows(0);
        q1 = k_rows(1);
        q2 = k_rows(2);
        q3 = k_rows(3);
      }
      for (int kb = 0; kb < T.kblocks; ++kb) {
        int good = 1;
        uint8_t* a = sA + stage * S::kABytes;
        uint8_t* b = sB + stage * S::kBBytes;
        int4 cur = q0;
        if (GATHER != kGatherNone && SCHED == kKRagged) {
          q0 = q1;
          q1 = q2;
          q2 = q3;
          q3 = k_rows(kb + 4);
        }
        if (lane == 0) {
          good = mbar_wait(&empty[stage], phase ^ 1u, abort_flag) ? 1 : 0;
          if (good) {
            mbar_expect_tx(&full[stage], S::kStageBytes);
            if (GATHER != kGatherA) {
              if (!A_MN) {
                tma_load_2d(a, &tmA, &full[stage], kb * BK, T.m * BM);
              } else {
                const int krow = T.krow0 + kb * BK;
                tma_load_2d(a, &tmA, &full[stage], T.m * BM, krow);
                tma_load_2d(a + 8192, &tmA, &full[stage], T.m * BM + 64, krow);
              }
            }
            if (GATHER != kGatherB) {
              if (!B_MN) {
                if (EPI == kEpiSwigluFwd) {
                  const int row = T.g * p.b_group_rows + T.n * (BN / 2);
                  tma_load_2d(b, &tmB, &full[stage], kb * BK, row);
                  tma_load_2d(b + S::kBBytes / 2, &tmB, &full[stage], kb * BK,
                              row + p.b_half_offset);
                } else {
                  tma_load_2d(b, &tmB, &full[stage], kb * BK, T.g * p.b_group_rows + T.n * BN);
                }
              } else {
                const int krow =
                    (SCHED == kKRagged) ? (T.krow0 + kb * BK) : (T.g * p.b_group_rows + kb * BK);
#pragma unroll
                for (int j = 0; j < BN / 64; ++j)
                  tma_load_2d(b + j * 8192, &tmB, &full[stage], T.n * BN + 64 * j, krow);
              }
            }
          }
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) {
          ok = false;
          break;
        }
        if (GATHER == kGatherA) {
          if (SCHED == kRowsRagged) {
            tma_gather4(a + lane * 512, &tmA, &full[stage], kb * BK, tok.x, tok.y, tok.z, tok.w);
          } else {
            // MN-major A: 2 chunks of [64 k rows][64 m]; lane l: rows 4(l%16).., chunk l/16
            const int c = lane >> 4;
            tma_gather4(a + c * 8192 + (lane & 15) * 512, &tmA, &full[stage], T.m * BM + 64 * c,
                        cur.x, cur.y, cur.z, cur.w);
          }
        }
        if (GATHER == kGatherB) {
          // MN-major B: BN/64 chunks of [64 k rows][64 n]
          for (int j = lane >> 4; j < BN / 64; j += 2)
            tma_gather4(b + j * 8192 + (lane & 15) * 512, &tmB, &full[stage], T.n * BN + 64 * j,
                        cur.x, cur.y, cur.z, cur.w);
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
        const TileInfo T = decode_tile<SCHED>(p, t);
        if (T.kblocks == 0) continue;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        ++local;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < T.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * S::kABytes);
          const uint32_t b0 = smem_u32(sB + stage * S::kBBytes);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad =
                A_MN ? make_sdesc(a0 + kk * 2048, 8192, 1024) : make_sdesc(a0 + kk * 32, 16, 1024);
            const uint64_t bd =
                B_MN ? make_sdesc(b0 + kk * 2048, 8192, 1024) : make_sdesc(b0 + kk * 32, 16, 1024);
            umma_bf16(d_tmem, ad, bd, kIdesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;  // which half of the tile's column chunks
    const int row_in = q * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const TileInfo T = decode_tile<SCHED>(p, t);
      if (T.kblocks == 0) {
        epilogue_empty_tile<EPI, BN>(p, T, row_in, half);
        continue;
      }
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      ++local;
      if (EPI == kEpiSwigluBwd) prefetch_gu_row<BN>(p, T, row_in, half);
      // every lane waits; the warp leaves together if any lane gave up (the TMEM
      // loads below are warp-collective)
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort_flag))) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;

      epilogue_tile<EPI, BN>(p, T, row_in, half, taddr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace b200moe
