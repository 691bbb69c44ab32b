// HBM-bound kernels of the MoE layer: router softmax/top-k (+ backward),
// dispatch (histogram, scan, stable permutation into 128-row-padded expert
// blocks), row gather / its top-k sum backward, weighted combine (+ backward)
// and the load-balancing statistics.
//
// All of them are one-warp-per-row or one-warp-per-token kernels with 16-byte
// vector accesses; they never allocate and never use atomics on global
// memory, so every result is deterministic.
#pragma once

#include "common.cuh"

namespace b200moe {

constexpr int kRowTile = 128;       // padding granule of an expert's row block
constexpr int kDispatchChunk = 4096;  // flat routed slots per dispatch block
constexpr int kDispatchThreads = 256;
constexpr int kMaxTopK = 16;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

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

// ---------------------------------------------------------------------------
// router: fp32 softmax over E logits, top-k, renormalisation
// (spark-gpt train.py:2144-2158).  One warp per token, expert e in lane e%32,
// register slot e/32.  Selection order: probability desc, lower index first
// on ties (torch CUDA's top-k takes the lowest indices among values equal to
// the k-th).
// ---------------------------------------------------------------------------
template <int VPT, typename LT>
__device__ __forceinline__ void softmax_row(const LT* __restrict__ row, int E, int lane,
                                            float (&p)[VPT]) {
  float z[VPT];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = lane + 32 * j;
    z[j] = e < E ? to_f32(row[e]) : -INFINITY;
    m = fmaxf(m, z[j]);
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = lane + 32 * j;
    p[j] = e < E ? expf(z[j] - m) : 0.f;
    s += p[j];
  }
  s = warp_sum(s);
#pragma unroll
  for (int j = 0; j < VPT; ++j) p[j] = p[j] / s;
}

template <int VPT, typename LT>
__global__ void router_topk_fwd_kernel(const LT* __restrict__ logits, long long ld, long long T,
                                       int E, int k, int norm, long long* __restrict__ selected,
                                       __nv_bfloat16* __restrict__ weights) {
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       t < T; t += warps) {
    float p[VPT];
    softmax_row<VPT>(logits + t * ld, E, lane, p);
#pragma unroll
    for (int j = 0; j < VPT; ++j)
      if (lane + 32 * j >= E) p[j] = -1.f;
    float sv[kMaxTopK];
    int si[kMaxTopK];
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
      sv[r] = 0.f;
      si[r] = 0;
      if (r < k) {
        float bv = -2.f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const int e = lane + 32 * j;
          if (p[j] > bv || (p[j] == bv && e < bi)) {
            bv = p[j];
            bi = e;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
#pragma unroll
        for (int j = 0; j < VPT; ++j)
          if (lane + 32 * j == bi) p[j] = -3.f;
        sv[r] = bv;
        si[r] = bi;
      }
    }
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r)
      if (r < k) sum += sv[r];
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
      if (r < k && lane == r) {
        selected[t * k + r] = si[r];
        weights[t * k + r] = __float2bfloat16_rn(norm ? sv[r] / sum : sv[r]);
      }
    }
  }
}

// d logits of the router given d(routing weights) (T,k) fp32 in slot order,
// plus an optional extra bf16 logit gradient (the load-balancing loss).
template <int VPT>
__global__ void router_topk_bwd_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                       const long long* __restrict__ selected,
                                       const float* __restrict__ d_weights,
                                       const __nv_bfloat16* __restrict__ d_extra, long long T,
                                       int E, int k, int norm,
                                       __nv_bfloat16* __restrict__ d_logits) {
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       t < T; t += warps) {
    float p[VPT];
    softmax_row<VPT>(logits + t * ld, E, lane, p);
    int si[kMaxTopK];
    float ps[kMaxTopK];
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
      si[r] = -1;
      ps[r] = 0.f;
      if (r < k) {
        const int e = static_cast<int>(selected[t * k + r]);
        float v = 0.f;
#pragma unroll
        for (int j = 0; j < VPT; ++j)
          if (lane + 32 * j == e) v = p[j];
        si[r] = e;
        ps[r] = warp_sum(v);
        s += ps[r];
      }
    }
    float dot = 0.f;
    float dw[kMaxTopK];
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
      dw[r] = r < k ? d_weights[t * k + r] : 0.f;
      if (r < k) dot += dw[r] * (ps[r] / s);
    }
    float g[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) g[j] = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
      if (r < k) {
        const float dp = norm ? (dw[r] - dot) / s : dw[r];
#pragma unroll
        for (int j = 0; j < VPT; ++j)
          if (lane + 32 * j == si[r]) g[j] = dp;
      }
    }
    float pg = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) pg += p[j] * g[j];
    pg = warp_sum(pg);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int e = lane + 32 * j;
      if (e < ld) {
        float v = 0.f;
        if (e < E) {
          v = p[j] * (g[j] - pg);
          if (d_extra) v += __bfloat162float(d_extra[t * ld + e]);
        }
        d_logits[t * ld + e] = __float2bfloat16_rn(v);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// dispatch (spark-gpt train.py:2271-2290): stable counting sort of the flat
// expert ids into expert blocks padded to kRowTile rows.
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
      else
        raise_fault(kFaultBadExpert);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) block_base[e * nblk + blockIdx.x] = hist[e];
}

__global__ void dispatch_scan_kernel(int* __restrict__ block_base, int nblk, int E,
                                     int* __restrict__ counts, int* __restrict__ offsets,
                                     int* __restrict__ pad_offsets, int* __restrict__ row_flat,
                                     int* __restrict__ tile_expert) {
  extern __shared__ int sh[];  // counts[E], pad_start[E+1]
  int* cnt = sh;
  int* pst = sh + E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
    for (int b = 0; b < nblk; ++b) c += block_base[e * nblk + b];
    cnt[e] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0, prun = 0;
    for (int e = 0; e < E; ++e) {
      run += cnt[e];
      offsets[e] = run;
      counts[e] = cnt[e];
      pst[e] = prun;
      pad_offsets[e] = prun;
      prun += (cnt[e] + kRowTile - 1) / kRowTile * kRowTile;
    }
    pst[E] = prun;
    pad_offsets[E] = prun;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = pst[e];
    for (int b = 0; b < nblk; ++b) {
      const int c = block_base[e * nblk + b];
      block_base[e * nblk + b] = run;
      run += c;
    }
    for (int r = pst[e] + cnt[e]; r < pst[e + 1]; ++r) row_flat[r] = -1;
    for (int j = pst[e] / kRowTile; j < pst[e + 1] / kRowTile; ++j) tile_expert[j] = e;
  }
}

__global__ void dispatch_scatter_kernel(const long long* __restrict__ sel, long long R, int E,
                                        int nblk, const int* __restrict__ block_base,
                                        int* __restrict__ row_flat, int* __restrict__ inv_pad) {
  extern __shared__ int wbase[];  // [warps][E]
  constexpr int kWarps = kDispatchThreads / 32;
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
    }
  }
}

// ---------------------------------------------------------------------------
// gather (train.py:2195-2217): xs[p] = x[row_flat[p] / k], zero for padding
// ---------------------------------------------------------------------------
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
    if (f >= 0) {
      const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(f / k) * H);
      for (int v = lane; v < nvec; v += 32) dst[v] = __ldg(src + v);
    } else {
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      for (int v = lane; v < nvec; v += 32) dst[v] = z;
    }
  }
}

// dx[t] = sum_s dxs[inv_pad[t*k+s]] (+ addend[t]); fp32 accumulation.
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
    for (int s = 0; s < kMaxTopK; ++s) rows[s] = s < k ? inv_pad[t * k + s] : 0;
    for (int v = lane; v < nvec; v += 32) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int s = 0; s < kMaxTopK; ++s) {
        if (s < k) {
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
      rows[s] = s < k ? inv_pad[t * k + s] : 0;
      w[s] = s < k ? __bfloat162float(weights[t * k + s]) : 0.f;
    }
    for (int v = lane; v < nvec; v += 32) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int s = 0; s < kMaxTopK; ++s) {
        if (s < k) {
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

// ---------------------------------------------------------------------------
// load-balancing statistics (train.py:3141-3153), deterministic two-pass:
//   partials[b][0:E]   hard counts (masked top-k bincount)
//   partials[b][E:2E]  soft sums   (masked softmax sums)
//   partials[b][2E]    entropy sum, partials[b][2E+1] valid rows
// ---------------------------------------------------------------------------
constexpr int kLbThreads = 256;
constexpr int kLbTokensPerBlock = 256;

template <int VPT>
__global__ void lb_partials_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                   const long long* __restrict__ selected,
                                   const unsigned char* __restrict__ valid, long long T, int E,
                                   int k, float* __restrict__ partials) {
  extern __shared__ float lsh[];  // [warps][2E+2]
  constexpr int kWarps = kLbThreads / 32;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int W = 2 * E + 2;
  float* mine = lsh + warp * W;
  for (int i = lane; i < W; i += 32) mine[i] = 0.f;
  __syncwarp();
  float soft[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) soft[j] = 0.f;
  float ent = 0.f;
  float rows = 0.f;
  const long long t0 = static_cast<long long>(blockIdx.x) * kLbTokensPerBlock;
  const float tiny = 1.17549435e-38f;
  for (int i = warp; i < kLbTokensPerBlock; i += kWarps) {
    const long long t = t0 + i;
    if (t >= T) break;
    if (valid && !valid[t]) continue;
    float p[VPT];
    softmax_row<VPT>(logits + t * ld, E, lane, p);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      if (lane + 32 * j < E) {
        soft[j] += p[j];
        ent -= p[j] * logf(fmaxf(p[j], tiny));
      }
    }
    rows += 1.f;
    if (lane < k) {
      const long long e = selected[t * k + lane];
      if (e >= 0 && e < E) atomicAdd(&mine[e], 1.f);
    }
    __syncwarp();
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j)
    if (lane + 32 * j < E) mine[E + lane + 32 * j] = soft[j];
  ent = warp_sum(ent);
  if (lane == 0) {
    mine[2 * E] = ent;
    mine[2 * E + 1] = rows;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < W; i += blockDim.x) {
    float acc = 0.f;
    for (int w = 0; w < kWarps; ++w) acc += lsh[w * W + i];
    partials[static_cast<long long>(blockIdx.x) * W + i] = acc;
  }
}

__global__ void lb_accumulate_kernel(const float* __restrict__ partials, int nblk, int W,
                                     float* __restrict__ packed) {
  for (int i = threadIdx.x; i < W; i += blockDim.x) {
    float acc = 0.f;
    for (int b = 0; b < nblk; ++b) acc += partials[static_cast<long long>(b) * W + i];
    packed[i] += acc;
  }
}

// aux value, stats and the per-expert gradient coefficient from the
// all-reduced packed sums (train.py:3163-3196).
// stats: [min_frac, max_frac, cv, entropy, unused]
__global__ void lb_finalize_kernel(const float* __restrict__ packed, int E, int k, int world,
                                   float* __restrict__ aux, float* __restrict__ stats,
                                   float* __restrict__ coef) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const float rows = packed[2 * E + 1];
  const float safe = fmaxf(rows, 1.f);
  const float has = rows > 0.f ? 1.f : 0.f;
  float dot = 0.f, mn = INFINITY, mx = -INFINITY, sum = 0.f, unused = 0.f;
  for (int e = 0; e < E; ++e) {
    const float a = packed[e] / safe;
    dot += a * (packed[E + e] / safe);
    const float fr = packed[e] / (safe * k);
    mn = fminf(mn, fr);
    mx = fmaxf(mx, fr);
    sum += fr;
    unused += packed[e] == 0.f ? 1.f : 0.f;
    coef[e] = has * static_cast<float>(world) * static_cast<float>(E) / safe * a;
  }
  const float mean = sum / E;
  float var = 0.f;
  for (int e = 0; e < E; ++e) {
    const float d = packed[e] / (safe * k) - mean;
    var += d * d;
  }
  var /= E;
  *aux = has * static_cast<float>(E) * dot;
  stats[0] = mn;
  stats[1] = mx;
  stats[2] = sqrtf(var) / fmaxf(mean, 1e-12f);
  stats[3] = packed[2 * E] / safe;
  stats[4] = unused;
}

// d aux / d logits[t,e] = g * mask_t * p_e (coef_e - <p, coef>), g = *grad
template <int VPT>
__global__ void lb_grad_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                               const unsigned char* __restrict__ valid, long long T, int E,
                               const float* __restrict__ coef, const float* __restrict__ grad,
                               __nv_bfloat16* __restrict__ d_logits) {
  const int lane = threadIdx.x & 31;
  const float g = *grad;
  float c[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) c[j] = (lane + 32 * j < E) ? coef[lane + 32 * j] : 0.f;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       t < T; t += warps) {
    const bool on = valid ? valid[t] != 0 : true;
    float p[VPT];
    softmax_row<VPT>(logits + t * ld, E, lane, p);
    float pc = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) pc += p[j] * c[j];
    pc = warp_sum(pc);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int e = lane + 32 * j;
      if (e < ld) {
        const float v = (on && e < E) ? g * p[j] * (c[j] - pc) : 0.f;
        d_logits[t * ld + e] = __float2bfloat16_rn(v);
      }
    }
  }
}

}  // namespace b200moe
