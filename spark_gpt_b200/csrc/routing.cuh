// HBM-bound kernels of the MoE layer: weight cast, dispatch (histogram, scan,
// stable permutation into 128-row-padded expert blocks), row gather and its
// top-k sum backward, weighted combine and its backward.  (Router and
// load-balancing kernels: router.cuh.)
//
// Row kernels are one warp per row or per token with 16-byte vector accesses;
// nothing allocates and nothing uses atomics on global memory, so every
// result is deterministic.
#pragma once

#include "common.cuh"
#include "router.cuh"

namespace b200moe {

constexpr int kRowTile = 128;       // padding granule of an expert's row block
constexpr int kDispatchChunk = 4096;  // flat routed slots per dispatch block
constexpr int kDispatchThreads = 1024;  // count kernel: 4 slots per thread

// ---------------------------------------------------------------------------
// fp32 master -> bf16 compute copy, rows >= rows_in zero-filled
// ---------------------------------------------------------------------------
__global__ void cast_f32_bf16_kernel(const float* __restrict__ src, long long rows_in,
                                     long long cols, long long rows_out,
                                     __nv_bfloat16* __restrict__ dst) {
  const long long n_in = rows_in * cols;
  const long long n_out = rows_out * cols;
  const long long n4 = n_out / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = i * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e + 3 < n_in) {
      v = *reinterpret_cast<const float4*>(src + e);
    } else {
      if (e + 0 < n_in) v.x = src[e + 0];
      if (e + 1 < n_in) v.y = src[e + 1];
      if (e + 2 < n_in) v.z = src[e + 2];
    }
    uint2 o;
    o.x = pack_bf16x2(v.x, v.y);
    o.y = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2*>(dst + e) = o;
  }
}

// out[i] (+)= sum_s partial[s*n + i], fixed order over s (n % 4 == 0)
__global__ void reduce_splits_kernel(const float* __restrict__ partial, int splits, long long n,
                                     float* __restrict__ out, int accumulate) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 acc = accumulate ? reinterpret_cast<const float4*>(out)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < splits; ++s) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(partial + s * n) + i);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = acc;
  }
}

// ---------------------------------------------------------------------------
// dispatch (spark-gpt train.py:2271-2290): stable counting sort of the flat
// expert ids into expert blocks padded to kRowTile rows.  A negative id marks
// a slot that goes to no expert (the expert-parallel layer's rows carry only
// the slots of one rank's experts): it gets no row and inv_pad = -1.
//   block_base[e * nblk + b]: rows of expert e in chunk b (pass 1), then the
//   padded start of those rows (pass 2).
// ---------------------------------------------------------------------------
__global__ void dispatch_count_kernel(const long long* __restrict__ sel, long long R, int E,
                                      int nblk, int* __restrict__ block_base) {
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const long long base = static_cast<long long>(blockIdx.x) * kDispatchChunk;
  for (int i = threadIdx.x; i < kDispatchChunk; i += blockDim.x) {
    const long long f = base + i;
    if (f < R) {
      const long long e = sel[f];
      if (e >= 0 && e < E)
        atomicAdd(&hist[e], 1);
      else if (e >= E)
        raise_fault(kFaultBadExpert);  // negative: the slot goes to no expert
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) block_base[e * nblk + blockIdx.x] = hist[e];
}

// Lanes per expert in the dispatch scan: a power of two <= 32 with
// lanes * E <= threads (1 when E >= threads).
__device__ __forceinline__ int scan_parts(int E, int threads) {
  int p = 1;
  while (p < 32 && 2 * p * E <= threads) p *= 2;
  return p;
}

// One block.  Each expert's nblk per-block counts are handled by P lanes of
// one warp (a contiguous chunk of blocks per lane): totals, then the expert
// scans (warp 0), then each block's starting padded row, the padding rows
// (row_flat = -1) and the tile -> expert table, all spread over the lanes.
__global__ void dispatch_scan_kernel(int* __restrict__ block_base, int nblk, int E,
                                     int* __restrict__ counts, int* __restrict__ offsets,
                                     int* __restrict__ pad_offsets, int* __restrict__ row_flat,
                                     int* __restrict__ tile_expert) {
  extern __shared__ int sh[];  // counts[E], pad_start[E+1]
  int* cnt = sh;
  int* pst = sh + E;
  const int P = scan_parts(E, blockDim.x);
  const int groups = blockDim.x / P;
  const int part = threadIdx.x % P;
  const int slot = threadIdx.x / P;
  const int lane = threadIdx.x & 31;
  const int per = (nblk + P - 1) / P;
  const int b0 = part * per;
  const int b1 = min(nblk, b0 + per);
  for (int e0 = 0; e0 < E; e0 += groups) {  // same trip count for every thread
    const int e = e0 + slot;
    int c = 0;
    if (e < E)
      for (int b = b0; b < b1; ++b) c += block_base[static_cast<long long>(e) * nblk + b];
    for (int o = 1; o < P; o <<= 1) c += __shfl_xor_sync(0xffffffffu, c, o, P);
    if (e < E && part == 0) cnt[e] = c;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int per_l = (E + 31) / 32;
    const int a = min(E, lane * per_l), z = min(E, a + per_l);
    int s = 0, ps = 0;
    for (int e = a; e < z; ++e) {
      s += cnt[e];
      ps += (cnt[e] + kRowTile - 1) / kRowTile * kRowTile;
    }
    int is = s, ips = ps;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, is, o);
      const int w = __shfl_up_sync(0xffffffffu, ips, o);
      if (lane >= o) {
        is += v;
        ips += w;
      }
    }
    int run = is - s, prun = ips - ps;
    for (int e = a; e < z; ++e) {
      run += cnt[e];
      offsets[e] = run;
      counts[e] = cnt[e];
      pst[e] = prun;
      pad_offsets[e] = prun;
      prun += (cnt[e] + kRowTile - 1) / kRowTile * kRowTile;
    }
    if (lane == 31) {
      pst[E] = ips;
      pad_offsets[E] = ips;
    }
  }
  __syncthreads();
  for (int e0 = 0; e0 < E; e0 += groups) {
    const int e = e0 + slot;
    int c = 0;
    if (e < E)
      for (int b = b0; b < b1; ++b) c += block_base[static_cast<long long>(e) * nblk + b];
    int inc = c;
    for (int o = 1; o < P; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, inc, o, P);
      if (part >= o) inc += v;
    }
    if (e < E) {
      int run = pst[e] + inc - c;
      for (int b = b0; b < b1; ++b) {
        const long long i = static_cast<long long>(e) * nblk + b;
        const int v = block_base[i];
        block_base[i] = run;
        run += v;
      }
      for (int r = pst[e] + cnt[e] + part; r < pst[e + 1]; r += P) row_flat[r] = -1;
      for (int j = pst[e] / kRowTile + part; j < pst[e + 1] / kRowTile; j += P) tile_expert[j] = e;
    }
  }
}

// WARPS warps per chunk, each placing a contiguous run of 4096 / WARPS slots
// (32 warps while their per-warp expert tables fit in shared memory).
template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
    dispatch_scatter_kernel(const long long* __restrict__ sel, long long R, int E, int nblk,
                            const int* __restrict__ block_base, int* __restrict__ row_flat,
                            int* __restrict__ inv_pad) {
  extern __shared__ int wbase[];  // [warps][E]
  constexpr int kWarps = WARPS;
  constexpr int kPerWarp = kDispatchChunk / kWarps;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* mine = wbase + warp * E;
  for (int e = lane; e < E; e += 32) mine[e] = 0;
  __syncwarp();
  const long long base = static_cast<long long>(blockIdx.x) * kDispatchChunk + warp * kPerWarp;
  for (int i = lane; i < kPerWarp; i += 32) {
    const long long f = base + i;
    if (f < R) {
      const long long e = sel[f];
      if (e >= 0 && e < E) atomicAdd(&mine[e], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = block_base[e * nblk + blockIdx.x];
    for (int w = 0; w < kWarps; ++w) {
      const int c = wbase[w * E + e];
      wbase[w * E + e] = run;
      run += c;
    }
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int i0 = 0; i0 < kPerWarp; i0 += 32) {
    const long long f = base + i0 + lane;
    int e = -1;
    if (f < R) {
      const long long v = sel[f];
      if (v >= 0 && v < E) e = static_cast<int>(v);
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    int pos = 0;
    if (e >= 0) pos = mine[e] + __popc(peers & lt_mask);
    __syncwarp();
    if (e >= 0 && lane == 31 - __clz(peers)) mine[e] += __popc(peers);
    __syncwarp();
    if (e >= 0) {
      row_flat[pos] = static_cast<int>(f);
      inv_pad[f] = pos;
    } else if (f < R) {
      inv_pad[f] = -1;  // a slot without an expert has no row
    }
  }
}

// ---------------------------------------------------------------------------
// gather (train.py:2195-2217): xs[p] = x[row_flat[p] / k], zero for padding
// ---------------------------------------------------------------------------
// VPL = 16-byte vectors per lane per row (H = 256 * VPL); every load of a row
// is issued before the first store, so a warp keeps VPL loads in flight.
// VPL == 0: any H (multiple of 8), one vector at a time.
template <int VPL>
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                   const int* __restrict__ row_flat,
                                   const int* __restrict__ total_rows, int k, int H,
                                   __nv_bfloat16* __restrict__ xs) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const long long total = *total_rows;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       r < total; r += warps) {
    const int f = row_flat[r];
    uint4* dst = reinterpret_cast<uint4*>(xs + r * H);
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(f < 0 ? 0 : f / k) * H);
    if (VPL > 0) {
      uint4 v[VPL > 0 ? VPL : 1];
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        v[j] = f >= 0 ? __ldg(src + lane + 32 * j) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int j = 0; j < VPL; ++j) dst[lane + 32 * j] = v[j];
    } else if (f >= 0) {
      for (int v = lane; v < nvec; v += 32) dst[v] = __ldg(src + v);
    } else {
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      for (int v = lane; v < nvec; v += 32) dst[v] = z;
    }
  }
}

// Zero the padding rows (row_flat < 0) of a padded-row buffer: each warp
// checks 32 rows at a time and clears the padding rows among them together.
template <int VPL>
__device__ __forceinline__ void zero_padding_rows(const int* __restrict__ row_flat,
                                                  long long total, int H, long long warp_id,
                                                  long long warps, int lane,
                                                  __nv_bfloat16* __restrict__ buf) {
  const int nvec = H / 8;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (long long base = warp_id * 32; base < total; base += warps * 32) {
    const long long r = base + lane;
    unsigned m = __ballot_sync(0xffffffffu, r < total && row_flat[r] < 0);
    while (m) {
      const int i = __ffs(m) - 1;
      m &= m - 1;
      uint4* dst = reinterpret_cast<uint4*>(buf + (base + i) * H);
      if (VPL > 0) {
#pragma unroll
        for (int j = 0; j < VPL; ++j) dst[lane + 32 * j] = z;
      } else {
        for (int v = lane; v < nvec; v += 32) dst[v] = z;
      }
    }
  }
}

// Token-order gather: warp per token; x[t] is read once and written to the
// padded rows of its k slots (inv_pad), then the padding rows are zeroed.
// Reads each token row once instead of once per slot.
template <int VPL>
__global__ void scatter_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                    const int* __restrict__ inv_pad,
                                    const int* __restrict__ row_flat,
                                    const int* __restrict__ total_rows, long long T, int k, int H,
                                    __nv_bfloat16* __restrict__ xs) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long warp_id = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
  for (long long t = warp_id; t < T; t += warps) {
    const int rl = lane < k ? inv_pad[t * k + lane] : 0;
    const uint4* src = reinterpret_cast<const uint4*>(x + t * H);
    if (VPL > 0) {
      uint4 v[VPL > 0 ? VPL : 1];
#pragma unroll
      for (int j = 0; j < VPL; ++j) v[j] = __ldg(src + lane + 32 * j);
      for (int s = 0; s < k; ++s) {
        const long long r = __shfl_sync(0xffffffffu, rl, s);
        if (r < 0) continue;  // slot without an expert
        uint4* dst = reinterpret_cast<uint4*>(xs + r * H);
#pragma unroll
        for (int j = 0; j < VPL; ++j) dst[lane + 32 * j] = v[j];
      }
    } else {
      for (int s = 0; s < k; ++s) {
        const long long r = __shfl_sync(0xffffffffu, rl, s);
        if (r < 0) continue;
        uint4* dst = reinterpret_cast<uint4*>(xs + r * H);
        for (int v = lane; v < nvec; v += 32) dst[v] = __ldg(src + v);
      }
    }
  }
  zero_padding_rows<VPL>(row_flat, *total_rows, H, warp_id, warps, lane, xs);
}

// Token-order combine backward over the padded layout: warp per token; d_out[t]
// is read once and the rows of its k slots are visited through inv_pad (the
// next slot's y row is loaded while the current one is processed):
//   dy[r] = bf16(d_out[t] * w[t,s]),  d_weights[t*k+s] = <d_out[t], y[r]>,
// then the padding rows of dy are zeroed.  F8: the same rows also leave as
// dy8 = e5m2(dy * q_scale[0]) (the fp8 down weight gradient's operand), with
// the amax of |dy| raised in q_amax[0].
template <int VPL, bool F8 = false>
__global__ void combine_bwd_tokens_kernel(const __nv_bfloat16* __restrict__ d_out,
                                          const __nv_bfloat16* __restrict__ y,
                                          const int* __restrict__ inv_pad,
                                          const int* __restrict__ row_flat,
                                          const int* __restrict__ total_rows,
                                          const __nv_bfloat16* __restrict__ weights, long long T,
                                          int k, int H, __nv_bfloat16* __restrict__ dy,
                                          float* __restrict__ d_weights,
                                          const float* __restrict__ q_scale = nullptr,
                                          float* __restrict__ q_amax = nullptr,
                                          uint8_t* __restrict__ dy8 = nullptr) {
  static_assert(VPL > 0, "token-order combine backward needs H in {256, 512, 1024, 2048}");
  const int lane = threadIdx.x & 31;
  const float qs = F8 ? __ldg(q_scale) : 0.f;
  float qm = 0.f;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long warp_id = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
  for (long long t = warp_id; t < T; t += warps) {
    int rl = 0;
    float wl = 0.f;
    if (lane < k) {
      rl = inv_pad[t * k + lane];
      wl = __bfloat162float(weights[t * k + lane]);
    }
    const uint4* g = reinterpret_cast<const uint4*>(d_out + t * H);
    float ga[VPL][8];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint4 a = __ldg(g + lane + 32 * j);
      ga[j][0] = bf16_lo(a.x); ga[j][1] = bf16_hi(a.x);
      ga[j][2] = bf16_lo(a.y); ga[j][3] = bf16_hi(a.y);
      ga[j][4] = bf16_lo(a.z); ga[j][5] = bf16_hi(a.z);
      ga[j][6] = bf16_lo(a.w); ga[j][7] = bf16_hi(a.w);
    }
    float my_dot = 0.f;
    uint4 bn[VPL];
    {
      const long long r0 = __shfl_sync(0xffffffffu, rl, 0);
      const uint4* yy = reinterpret_cast<const uint4*>(y + (r0 < 0 ? 0 : r0) * H);
#pragma unroll
      for (int j = 0; j < VPL; ++j) bn[j] = r0 >= 0 ? __ldg(yy + lane + 32 * j) : make_uint4(0u, 0u, 0u, 0u);
    }
    for (int s = 0; s < k; ++s) {
      const long long r = __shfl_sync(0xffffffffu, rl, s);
      const float w = __shfl_sync(0xffffffffu, wl, s);
      uint4 b[VPL];
#pragma unroll
      for (int j = 0; j < VPL; ++j) b[j] = bn[j];
      const long long rn = __shfl_sync(0xffffffffu, rl, s + 1 < k ? s + 1 : s);
      if (s + 1 < k && rn >= 0) {
        const uint4* yy = reinterpret_cast<const uint4*>(y + rn * H);
#pragma unroll
        for (int j = 0; j < VPL; ++j) bn[j] = __ldg(yy + lane + 32 * j);
      }
      if (r < 0) continue;  // slot without an expert: d_weights stays 0
      uint4* dst = reinterpret_cast<uint4*>(dy + r * H);
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const float yb[8] = {bf16_lo(b[j].x), bf16_hi(b[j].x), bf16_lo(b[j].y), bf16_hi(b[j].y),
                             bf16_lo(b[j].z), bf16_hi(b[j].z), bf16_lo(b[j].w), bf16_hi(b[j].w)};
#pragma unroll
        for (int e = 0; e < 8; ++e) dot += ga[j][e] * yb[e];
        uint4 o;
        o.x = pack_bf16x2(ga[j][0] * w, ga[j][1] * w);
        o.y = pack_bf16x2(ga[j][2] * w, ga[j][3] * w);
        o.z = pack_bf16x2(ga[j][4] * w, ga[j][5] * w);
        o.w = pack_bf16x2(ga[j][6] * w, ga[j][7] * w);
        dst[lane + 32 * j] = o;
        if constexpr (F8) {
          const float v[8] = {bf16_lo(o.x), bf16_hi(o.x), bf16_lo(o.y), bf16_hi(o.y),
                              bf16_lo(o.z), bf16_hi(o.z), bf16_lo(o.w), bf16_hi(o.w)};
#pragma unroll
          for (int e = 0; e < 8; ++e) qm = fmaxf(qm, fabsf(v[e]));
          reinterpret_cast<uint2*>(dy8 + r * H)[lane + 32 * j] =
              make_uint2(pack_fp8x4<kE5M2>(v[0] * qs, v[1] * qs, v[2] * qs, v[3] * qs),
                         pack_fp8x4<kE5M2>(v[4] * qs, v[5] * qs, v[6] * qs, v[7] * qs));
        }
      }
      dot = warp_sum(dot);
      if (lane == s) my_dot = dot;
    }
    if (lane < k) d_weights[t * k + lane] = my_dot;
  }
  zero_padding_rows<VPL>(row_flat, *total_rows, H, warp_id, warps, lane, dy);
  if constexpr (F8) {
    // the padding rows of dy8 (H bytes each)
    const long long total = *total_rows;
    for (long long base = warp_id * 32; base < total; base += warps * 32) {
      const long long r = base + lane;
      unsigned pad = __ballot_sync(0xffffffffu, r < total && row_flat[r] < 0);
      while (pad) {
        const int i = __ffs(pad) - 1;
        pad &= pad - 1;
        uint4* d8 = reinterpret_cast<uint4*>(dy8 + (base + i) * H);
        for (int v = lane; v < H / 16; v += 32) d8[v] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    qm = warp_max(qm);
    if (lane == 0 && qm > 0.f) atomic_max_nonneg(q_amax, qm);
  }
}

// dx[t] = sum_s dxs[inv_pad[t*k+s]] (+ addend[t]); fp32 accumulation.  With
// inv_pad == nullptr the rows are token-major (slot t*k+s in row t*k+s).  Used
// when one token's k rows do not fit the shared-memory ring of row_reduce_kernel.
__global__ void gather_rows_bwd_kernel(const __nv_bfloat16* __restrict__ dxs,
                                       const int* __restrict__ inv_pad,
                                       const __nv_bfloat16* __restrict__ addend, long long T,
                                       int k, int H, __nv_bfloat16* __restrict__ dx) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       t < T; t += warps) {
    int rows[kMaxTopK];
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s)
      rows[s] = s < k ? (inv_pad ? inv_pad[t * k + s] : static_cast<int>(t * k + s)) : 0;
    for (int v = lane; v < nvec; v += 32) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int s = 0; s < kMaxTopK; ++s) {
        if (s < k && rows[s] >= 0) {
          const uint4 w = __ldg(reinterpret_cast<const uint4*>(dxs + static_cast<long long>(rows[s]) * H) + v);
          acc[0] += bf16_lo(w.x); acc[1] += bf16_hi(w.x);
          acc[2] += bf16_lo(w.y); acc[3] += bf16_hi(w.y);
          acc[4] += bf16_lo(w.z); acc[5] += bf16_hi(w.z);
          acc[6] += bf16_lo(w.w); acc[7] += bf16_hi(w.w);
        }
      }
      if (addend) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(addend + t * H) + v);
        acc[0] += bf16_lo(w.x); acc[1] += bf16_hi(w.x);
        acc[2] += bf16_lo(w.y); acc[3] += bf16_hi(w.y);
        acc[4] += bf16_lo(w.z); acc[5] += bf16_hi(w.z);
        acc[6] += bf16_lo(w.w); acc[7] += bf16_hi(w.w);
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(dx + t * H)[v] = o;
    }
  }
}

// ---------------------------------------------------------------------------
// combine (train.py:2220-2241)
//   fwd: out[t] = sum_s bf16(y[j] * w[t,s]), j = inv_pad[t*k+s]  (fp32 sum)
//   bwd: dy[p] = bf16(d_out[t] * w), d_w[t*k+s] = <d_out[t], y[p]>
// ---------------------------------------------------------------------------
__global__ void combine_fwd_kernel(const __nv_bfloat16* __restrict__ y,
                                   const int* __restrict__ inv_pad,
                                   const __nv_bfloat16* __restrict__ weights, long long T, int k,
                                   int H, __nv_bfloat16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       t < T; t += warps) {
    int rows[kMaxTopK];
    float w[kMaxTopK];
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s) {
      rows[s] = s < k ? (inv_pad ? inv_pad[t * k + s] : static_cast<int>(t * k + s)) : 0;
      w[s] = s < k ? __bfloat162float(weights[t * k + s]) : 0.f;
    }
    for (int v = lane; v < nvec; v += 32) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int s = 0; s < kMaxTopK; ++s) {
        if (s < k && rows[s] >= 0) {
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(y + static_cast<long long>(rows[s]) * H) + v);
          acc[0] += bf16_round(bf16_lo(q.x) * w[s]); acc[1] += bf16_round(bf16_hi(q.x) * w[s]);
          acc[2] += bf16_round(bf16_lo(q.y) * w[s]); acc[3] += bf16_round(bf16_hi(q.y) * w[s]);
          acc[4] += bf16_round(bf16_lo(q.z) * w[s]); acc[5] += bf16_round(bf16_hi(q.z) * w[s]);
          acc[6] += bf16_round(bf16_lo(q.w) * w[s]); acc[7] += bf16_round(bf16_hi(q.w) * w[s]);
        }
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(out + t * H)[v] = o;
    }
  }
}

template <int VPL>
__global__ void combine_bwd_kernel(const __nv_bfloat16* __restrict__ d_out,
                                   const __nv_bfloat16* __restrict__ y,
                                   const int* __restrict__ row_flat,
                                   const int* __restrict__ total_rows,
                                   const __nv_bfloat16* __restrict__ weights, int k, int H,
                                   __nv_bfloat16* __restrict__ dy, float* __restrict__ d_weights) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const long long total = *total_rows;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       r < total; r += warps) {
    const int f = row_flat[r];
    uint4* dst = reinterpret_cast<uint4*>(dy + r * H);
    if (f < 0) {
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      for (int v = lane; v < nvec; v += 32) dst[v] = z;
      continue;
    }
    const float w = __bfloat162float(weights[f]);
    const uint4* g = reinterpret_cast<const uint4*>(d_out + static_cast<long long>(f / k) * H);
    const uint4* yy = reinterpret_cast<const uint4*>(y + r * H);
    float dot = 0.f;
    auto one = [&](const uint4 a, const uint4 b, int v) {
      float ga[8] = {bf16_lo(a.x), bf16_hi(a.x), bf16_lo(a.y), bf16_hi(a.y),
                     bf16_lo(a.z), bf16_hi(a.z), bf16_lo(a.w), bf16_hi(a.w)};
      float yb[8] = {bf16_lo(b.x), bf16_hi(b.x), bf16_lo(b.y), bf16_hi(b.y),
                     bf16_lo(b.z), bf16_hi(b.z), bf16_lo(b.w), bf16_hi(b.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) dot += ga[j] * yb[j];
      uint4 o;
      o.x = pack_bf16x2(ga[0] * w, ga[1] * w);
      o.y = pack_bf16x2(ga[2] * w, ga[3] * w);
      o.z = pack_bf16x2(ga[4] * w, ga[5] * w);
      o.w = pack_bf16x2(ga[6] * w, ga[7] * w);
      dst[v] = o;
    };
    if (VPL > 0) {
      uint4 a[VPL > 0 ? VPL : 1], b[VPL > 0 ? VPL : 1];
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        a[j] = __ldg(g + lane + 32 * j);
        b[j] = __ldg(yy + lane + 32 * j);
      }
#pragma unroll
      for (int j = 0; j < VPL; ++j) one(a[j], b[j], lane + 32 * j);
    } else {
      for (int v = lane; v < nvec; v += 32) one(__ldg(g + v), __ldg(yy + v), v);
    }
    dot = warp_sum(dot);
    if (lane == 0) d_weights[f] = dot;
  }
}

// Token-major combine backward: y_tok (T*k, H) holds the down projection of
// slot f = t*k+s in row f.  Warp per slot, in slot order (sequential reads of
// y_tok and d_out): dy[inv_pad[f]] = bf16(d_out[t] * w[f]) (scattered 2*H-byte
// row writes), d_weights[f] = <d_out[t], y_tok[f]>.
__global__ void combine_bwd_token_major_kernel(const __nv_bfloat16* __restrict__ d_out,
                                               const __nv_bfloat16* __restrict__ y_tok,
                                               const int* __restrict__ inv_pad,
                                               const __nv_bfloat16* __restrict__ weights,
                                               long long R, int k, int H,
                                               __nv_bfloat16* __restrict__ dy,
                                               float* __restrict__ d_weights) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long f = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       f < R; f += warps) {
    const int row = inv_pad[f];
    if (row < 0) {  // slot without an expert
      if (lane == 0) d_weights[f] = 0.f;
      continue;
    }
    const float w = __bfloat162float(weights[f]);
    const uint4* g = reinterpret_cast<const uint4*>(d_out + (f / k) * H);
    const uint4* yy = reinterpret_cast<const uint4*>(y_tok + f * H);
    uint4* dst = reinterpret_cast<uint4*>(dy + static_cast<long long>(row) * H);
    float dot = 0.f;
    for (int v = lane; v < nvec; v += 32) {
      const uint4 a = __ldg(g + v);
      const uint4 b = __ldg(yy + v);
      float ga[8] = {bf16_lo(a.x), bf16_hi(a.x), bf16_lo(a.y), bf16_hi(a.y),
                     bf16_lo(a.z), bf16_hi(a.z), bf16_lo(a.w), bf16_hi(a.w)};
      float yb[8] = {bf16_lo(b.x), bf16_hi(b.x), bf16_lo(b.y), bf16_hi(b.y),
                     bf16_lo(b.z), bf16_hi(b.z), bf16_lo(b.w), bf16_hi(b.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) dot += ga[j] * yb[j];
      uint4 o;
      o.x = pack_bf16x2(ga[0] * w, ga[1] * w);
      o.y = pack_bf16x2(ga[2] * w, ga[3] * w);
      o.z = pack_bf16x2(ga[4] * w, ga[5] * w);
      o.w = pack_bf16x2(ga[6] * w, ga[7] * w);
      dst[v] = o;
    }
    dot = warp_sum(dot);
    if (lane == 0) d_weights[f] = dot;
  }
}

// Zero the padding rows (row_flat < 0) of a (Rcap, H) bf16 buffer.
__global__ void zero_pad_rows_kernel(const int* __restrict__ row_flat,
                                     const int* __restrict__ total_rows, int H,
                                     __nv_bfloat16* __restrict__ buf) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const long long total = *total_rows;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       r < total; r += warps) {
    if (row_flat[r] >= 0) continue;
    uint4* dst = reinterpret_cast<uint4*>(buf + r * H);
    for (int v = lane; v < nvec; v += 32) dst[v] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// ---------------------------------------------------------------------------
// k-row reductions per token, streamed through shared memory with bulk copies
// (the combine forward and the gather backward):
//   out[t] = sum_s c(s) + addend[t],   c(s) = bf16(rows[j] * w[t,s])  (weights)
//                                       c(s) = rows[j]                 (no weights)
//   j = inv_pad[t*k+s] (or t*k+s when rows are token-major); fp32 accumulation
//   in slot order, one rounding to bf16.  Slots with j = -1 (no expert)
//   contribute nothing and are not copied.
// Warp 0 produces: lane s < k issues the 2*H-byte bulk copy of row s of a
// token into a ring slot.  Consumers are kReduceGroups groups of
// kReduceWarpsPerToken warps; the warps of a group split the H columns of one
// token.  The slot count is a multiple of the group count, so each slot always
// has the same consumer group and its phases are waited in order.  Each block
// owns a contiguous range of tokens, so the k indices of several tokens are
// one coalesced read, issued a group of tokens ahead of use.
// ---------------------------------------------------------------------------
constexpr int kReduceWarpsPerToken = 4;
constexpr int kReduceGroups = 2;
constexpr int kMaxReduceSlots = 4 * kReduceGroups;
constexpr int kReduceThreads = 32 * (1 + kReduceGroups * kReduceWarpsPerToken);

// The post-attention RMSNorm's backward fused into the gather backward
// (NORM = true).  The reference normalises before the layer (train.py:162-170,
// :2370): x_n = bf16(bf16(x * r) * bf16(w)), r = rsqrt(mean(x^2) + eps).  With
// g = bf16(sum of the token's rows + addend) = dL/dx_n (the plain gather
// backward's output, never written here):
//   dy_j   = bf16(g_j * bf16(w_j))                 (d of the bf16 product)
//   dx_j   = bf16(r * dy_j - (r^3 / H) * x_j * sum_i dy_i x_i)
//   dw_j  += g_j * bf16(x_j * r)                   (summed over tokens)
// The row-wide sum needs the whole row: the kReduceWarpsPerToken warps of a
// group each add their columns, exchange the partial sums through shared
// memory and a per-group mbarrier (bounded wait), and make a second pass over
// the slot's rows (still in shared memory) to write dx.  Each group keeps its
// columns' dw sums in registers and writes one partial row at the end.
struct NormBwd {
  const __nv_bfloat16* x;  // (T, H) the norm's input
  const float* w;          // (H,) norm weight (fp32 master, used as bf16)
  const float* rstd;       // (T,) r of the forward
  float* dw_part;          // (gridDim.x * kReduceGroups, H) partial weight gradients
  float inv_h;             // 1 / H
};
constexpr int kNormVecsMax = 4;  // 16-byte column vectors per lane: H <= 4096

__device__ __forceinline__ void unpack8(const uint4 a, float (&f)[8]) {
  f[0] = bf16_lo(a.x); f[1] = bf16_hi(a.x); f[2] = bf16_lo(a.y); f[3] = bf16_hi(a.y);
  f[4] = bf16_lo(a.z); f[5] = bf16_hi(a.z); f[6] = bf16_lo(a.w); f[7] = bf16_hi(a.w);
}

// g = bf16(sum over the token's rows in the ring slot + addend row) for the 8
// columns of 16-byte vector v (fp32 in slot order, one rounding)
template <bool SKIP>
__device__ __forceinline__ void norm_row_sum(const uint8_t* slot, uint32_t row_bytes, int k,
                                             unsigned have, const uint4* arow, int v,
                                             float (&g)[8]) {
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
  for (int r = 0; r < kMaxTopK; ++r) {
    if (r < k && (!SKIP || ((have >> r) & 1u))) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(slot + r * row_bytes + v * 16), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
  }
  if (arow) {
    float f[8];
    unpack8(__ldg(arow + v), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] += f[j];
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) g[j] = bf16_round(acc[j]);
}

// SKIP: some slots may have no row (inv_pad -1, the expert-parallel layouts);
// without it every one of a token's k slots is copied and summed.
// NV > 0: the RMSNorm backward is fused in, with NV 16-byte column vectors per
// lane (H <= NV * 1024); the plain reduction keeps three blocks per SM.
template <bool SKIP, int NV = 0>
__global__ void __launch_bounds__(kReduceThreads, NV == 0 ? 3 : (NV == 1 ? 3 : (NV == 2 ? 2 : 1)))
    row_reduce_kernel(const __nv_bfloat16* __restrict__ rows, const int* __restrict__ inv_pad,
                      const __nv_bfloat16* __restrict__ weights,
                      const __nv_bfloat16* __restrict__ addend, long long T, int k, int H,
                      int slots, __nv_bfloat16* __restrict__ out, NormBwd nb = NormBwd{}) {
  extern __shared__ __align__(128) uint8_t rsm[];
  constexpr bool kNorm = NV > 0;
  // NORM: per group, the row-dot partials of its warps (two token buffers) and
  // the mbarrier their exchange completes on
  __shared__ float red_sh[kReduceGroups][2][kReduceWarpsPerToken];
  __shared__ __align__(8) uint64_t red_bar[kReduceGroups];
  const uint32_t row_bytes = static_cast<uint32_t>(H) * 2;
  const uint32_t slot_bytes = row_bytes * k;
  uint64_t* full = reinterpret_cast<uint64_t*>(rsm + static_cast<size_t>(slots) * slot_bytes);
  uint64_t* empty = full + slots;
  __shared__ int abort_flag_s;
  // per ring slot: which of the token's k rows were copied (bit s = slot s),
  // written by the producer before it arms the slot's full barrier
  __shared__ unsigned slot_mask[kMaxReduceSlots];
  volatile int* abort_flag = &abort_flag_s;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kReduceWarpsPerToken);
    }
    if (kNorm)
      for (int g = 0; g < kReduceGroups; ++g) mbar_init(&red_bar[g], kReduceWarpsPerToken);
    abort_flag_s = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const long long per_block = (T + gridDim.x - 1) / gridDim.x;
  const long long t0 = blockIdx.x * per_block;
  const long long n = max(0LL, min(T, t0 + per_block) - t0);
  if (warp == 0) {
    const int tpg = 32 / k;  // tokens whose k indices one warp load covers
    const bool active_lane = lane < tpg * k;
    // row of slot s of token t: inv_pad[t*k+s], or t*k+s itself when the rows
    // are stored token-major (inv_pad == nullptr)
    auto slot_row = [&](long long f) -> long long { return inv_pad ? inv_pad[f] : f; };
    long long idx_next = 0;
    if (active_lane && lane / k < n) idx_next = slot_row((t0 + lane / k) * k + lane % k);
    for (long long g = 0; g < n; g += tpg) {
      const long long idx = idx_next;
      if (active_lane && g + tpg + lane / k < n)
        idx_next = slot_row((t0 + g + tpg + lane / k) * k + lane % k);
      for (int tt = 0; tt < tpg && g + tt < n; ++tt) {
        const long long i = g + tt;
        const int s = static_cast<int>(i % slots);
        const uint32_t ph = static_cast<uint32_t>((i / slots) & 1);
        // slots without an expert (row -1) are not copied; the barrier expects
        // the bytes of the token's real rows only (zero bytes complete it at once)
        const bool mine = active_lane && lane / k == tt && (!SKIP || idx >= 0);
        const unsigned have = SKIP ? __ballot_sync(0xffffffffu, mine) : 0u;
        int good = 1;
        if (lane == 0) {
          good = mbar_wait(&empty[s], ph ^ 1u, abort_flag) ? 1 : 0;
          if (good) {
            if (SKIP) {
              slot_mask[s] = (have >> (tt * k)) & ((1u << k) - 1u);
              mbar_expect_tx(&full[s], __popc(have) * row_bytes);  // release: orders the mask
            } else {
              mbar_expect_tx(&full[s], slot_bytes);
            }
          }
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) break;
        if (mine)
          bulk_load(rsm + static_cast<size_t>(s) * slot_bytes + (lane % k) * row_bytes,
                    rows + idx * H, row_bytes, &full[s]);
      }
      if (*abort_flag) break;
    }
  } else {
    const int cw = warp - 1;
    const int group = cw / kReduceWarpsPerToken;
    const int part = cw % kReduceWarpsPerToken;
    const int nvec = H / 8;
    const int v0 = part * (nvec / kReduceWarpsPerToken);
    const int v1 = (part + 1 == kReduceWarpsPerToken) ? nvec : v0 + nvec / kReduceWarpsPerToken;
    // NORM: this lane's columns' weight (as bf16) and weight-gradient sums
    constexpr bool NORM = NV > 0;
    constexpr int kNormVecs = NV > 0 ? NV : 1;
    float wb[kNormVecs][8], dw[kNormVecs][8];
    if constexpr (NORM) {
#pragma unroll
      for (int q = 0; q < kNormVecs; ++q) {
        const int v = v0 + lane + 32 * q;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          wb[q][j] = v < v1 ? bf16_round(nb.w[v * 8 + j]) : 0.f;
          dw[q][j] = 0.f;
        }
      }
    }
    uint32_t red_phase = 0;
    for (long long i = group; i < n; i += kReduceGroups) {
      const int s = static_cast<int>(i % slots);
      const uint32_t ph = static_cast<uint32_t>((i / slots) & 1);
      // every lane waits (acquire); the warp leaves together if any lane gave up
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, abort_flag))) break;
      const long long t = t0 + i;
      // routing weights of the token's k slots, broadcast to every lane before
      // the column loop (lanes past the last column skip it: no shuffle inside)
      float wv = 1.f;
      if (weights && lane < k) wv = __bfloat162float(weights[t * k + lane]);
      // slots with a row (inv_pad >= 0); the others were not copied
      const unsigned have = SKIP ? slot_mask[s] : 0xffffffffu;
      __nv_bfloat162 wr[kMaxTopK];
#pragma unroll
      for (int r = 0; r < kMaxTopK; ++r)
        wr[r] = __float2bfloat162_rn(__shfl_sync(0xffffffffu, wv, r));
      const uint8_t* slot = rsm + static_cast<size_t>(s) * slot_bytes;
      if constexpr (NORM) {
        const float r = nb.rstd[t];
        const uint4* xrow = reinterpret_cast<const uint4*>(nb.x + t * H);
        const uint4* arow = addend ? reinterpret_cast<const uint4*>(addend + t * H) : nullptr;
        float dot = 0.f;
#pragma unroll
        for (int q = 0; q < kNormVecs; ++q) {
          const int v = v0 + lane + 32 * q;
          if (v < v1) {
            float g[8], xf[8];
            norm_row_sum<SKIP>(slot, row_bytes, k, have, arow, v, g);
            unpack8(__ldg(xrow + v), xf);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              dot += bf16_round(g[j] * wb[q][j]) * xf[j];
              dw[q][j] += g[j] * bf16_round(xf[j] * r);
            }
          }
        }
        // the group's row-wide sum: each warp's partial through shared memory
        dot = warp_sum(dot);
        const int buf = static_cast<int>(red_phase & 1u);
        if (lane == 0) {
          red_sh[group][buf][part] = dot;
          mbar_arrive(&red_bar[group]);
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&red_bar[group], red_phase, abort_flag))) break;
        red_phase ^= 1u;
        float row_dot = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < kReduceWarpsPerToken; ++w2) row_dot += red_sh[group][buf][w2];
        const float c = r * r * r * nb.inv_h * row_dot;
#pragma unroll
        for (int q = 0; q < kNormVecs; ++q) {
          const int v = v0 + lane + 32 * q;
          if (v < v1) {
            float g[8], xf[8];
            norm_row_sum<SKIP>(slot, row_bytes, k, have, arow, v, g);
            unpack8(__ldg(xrow + v), xf);
#pragma unroll
            for (int j = 0; j < 8; ++j) g[j] = r * bf16_round(g[j] * wb[q][j]) - c * xf[j];
            uint4 o;
            o.x = pack_bf16x2(g[0], g[1]);
            o.y = pack_bf16x2(g[2], g[3]);
            o.z = pack_bf16x2(g[4], g[5]);
            o.w = pack_bf16x2(g[6], g[7]);
            reinterpret_cast<uint4*>(out + t * H)[v] = o;
          }
        }
      } else {
      for (int v = v0 + lane; v < v1; v += 32) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxTopK; ++r) {
          if (r < k && (!SKIP || ((have >> r) & 1u))) {
            uint4 q = *reinterpret_cast<const uint4*>(slot + r * row_bytes + v * 16);
            if (weights) {
              // bf16 x bf16 product rounded once to bf16 (= bf16(float(a)*float(b)))
              __nv_bfloat162* q2 = reinterpret_cast<__nv_bfloat162*>(&q);
#pragma unroll
              for (int j = 0; j < 4; ++j) q2[j] = __hmul2(q2[j], wr[r]);
            }
            acc[0] += bf16_lo(q.x); acc[1] += bf16_hi(q.x);
            acc[2] += bf16_lo(q.y); acc[3] += bf16_hi(q.y);
            acc[4] += bf16_lo(q.z); acc[5] += bf16_hi(q.z);
            acc[6] += bf16_lo(q.w); acc[7] += bf16_hi(q.w);
          }
        }
        if (addend) {
          const uint4 a = __ldg(reinterpret_cast<const uint4*>(addend + t * H) + v);
          acc[0] += bf16_lo(a.x); acc[1] += bf16_hi(a.x);
          acc[2] += bf16_lo(a.y); acc[3] += bf16_hi(a.y);
          acc[4] += bf16_lo(a.z); acc[5] += bf16_hi(a.z);
          acc[6] += bf16_lo(a.w); acc[7] += bf16_hi(a.w);
        }
        uint4 o;
        o.x = pack_bf16x2(acc[0], acc[1]);
        o.y = pack_bf16x2(acc[2], acc[3]);
        o.z = pack_bf16x2(acc[4], acc[5]);
        o.w = pack_bf16x2(acc[6], acc[7]);
        reinterpret_cast<uint4*>(out + t * H)[v] = o;
      }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if constexpr (NORM) {
      float* dst = nb.dw_part + (static_cast<long long>(blockIdx.x) * kReduceGroups + group) * H;
#pragma unroll
      for (int q = 0; q < kNormVecs; ++q) {
        const int v = v0 + lane + 32 * q;
        if (v < v1) {
#pragma unroll
          for (int j = 0; j < 8; ++j) dst[v * 8 + j] = dw[q][j];
        }
      }
    }
  }
}

// out[c] = sum over rows r of part[r][c], r in order (deterministic column sums
// of per-block partials: the RMSNorm weight gradient).
__global__ void sum_columns_kernel(const float* __restrict__ part, int rows, int cols,
                                   float* __restrict__ out) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += gridDim.x * blockDim.x) {
    float a = 0.f;
#pragma unroll 8
    for (int r = 0; r < rows; ++r) a += part[static_cast<long long>(r) * cols + c];
    out[c] = a;
  }
}

// x_n = bf16(bf16(x * r) * bf16(w)), r = rsqrt(mean(x^2) + eps) per token
// (the reference's RMSNorm, train.py:162-170: the mean as the sum times 1/H).
// Warp per token, 16-byte vectors; r is kept for the backward.
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                   const float* __restrict__ w, long long T, int H, float eps,
                                   __nv_bfloat16* __restrict__ x_n, float* __restrict__ rstd) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const float inv_h = 1.0f / static_cast<float>(H);
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       t < T; t += warps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + t * H);
    float ss = 0.f;
    for (int v = lane; v < nvec; v += 32) {
      const uint4 a = __ldg(xr + v);
      const float f[8] = {bf16_lo(a.x), bf16_hi(a.x), bf16_lo(a.y), bf16_hi(a.y),
                          bf16_lo(a.z), bf16_hi(a.z), bf16_lo(a.w), bf16_hi(a.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss * inv_h + eps);
    if (lane == 0) rstd[t] = r;
    uint4* o = reinterpret_cast<uint4*>(x_n + t * H);
    for (int v = lane; v < nvec; v += 32) {
      const uint4 a = __ldg(xr + v);
      const float f[8] = {bf16_lo(a.x), bf16_hi(a.x), bf16_lo(a.y), bf16_hi(a.y),
                          bf16_lo(a.z), bf16_hi(a.z), bf16_lo(a.w), bf16_hi(a.w)};
      float y[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = bf16_round(f[j] * r) * bf16_round(w[v * 8 + j]);
      uint4 q;
      q.x = pack_bf16x2(y[0], y[1]);
      q.y = pack_bf16x2(y[2], y[3]);
      q.z = pack_bf16x2(y[4], y[5]);
      q.w = pack_bf16x2(y[6], y[7]);
      o[v] = q;
    }
  }
}

// d_weights[row_flat[p]] = sum over parts of dw_part[part][p] (fixed order);
// the parts are the per-(N tile, column half) partial sums of the fused
// down-dgrad epilogue.
__global__ void combine_weight_grad_kernel(const float* __restrict__ dw_part, int parts,
                                           long long stride, const int* __restrict__ row_flat,
                                           const int* __restrict__ total_rows,
                                           float* __restrict__ d_weights) {
  const long long total = *total_rows;
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; r < total;
       r += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int f = row_flat[r];
    if (f < 0) continue;
    float acc = 0.f;
    for (int q = 0; q < parts; ++q) acc += dw_part[q * stride + r];
    d_weights[f] = acc;
  }
}

}  // namespace b200moe
