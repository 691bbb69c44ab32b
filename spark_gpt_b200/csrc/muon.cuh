// Muon on the packed 3-D expert weights (spark-gpt train.py:2877-3024): the
// momentum stage and the per-matrix normalisation of the batched
// Newton-Schulz iteration.  The iteration's three products per step run on
// the grouped tcgen05 GEMM (grouped_gemm.cuh, kEpiAxpby epilogue); every
// matrix of the stack is one group of rows.
#pragma once

#include "common.cuh"

namespace b200moe {

constexpr int kNsChunk = 16384;  // elements per partial sum of squares

// v <- lerp(v, g, 1 - m) in place (fp32); u <- lerp(g, v, m) as bf16 (nesterov),
// or u <- v.  torch.lerp's two branches, coeff * (end - start) + base with
// coeff = w below 0.5 (base = start) and w - 1 from 0.5 up (base = end).
__global__ void muon_momentum_kernel(const float* __restrict__ g, float* __restrict__ v,
                                     __nv_bfloat16* __restrict__ u, long long n, float w_v,
                                     float w_u, int nesterov) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    const float gs[4] = {gg.x, gg.y, gg.z, gg.w};
    float vs[4] = {vv.x, vv.y, vv.z, vv.w};
    float us[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      vs[j] = w_v < 0.5f ? fmaf(w_v, gs[j] - vs[j], vs[j]) : fmaf(w_v - 1.0f, gs[j] - vs[j], gs[j]);
      us[j] = nesterov ? (w_u < 0.5f ? fmaf(w_u, vs[j] - gs[j], gs[j])
                                     : fmaf(w_u - 1.0f, vs[j] - gs[j], vs[j]))
                       : vs[j];
    }
    reinterpret_cast<float4*>(v)[i] = make_float4(vs[0], vs[1], vs[2], vs[3]);
    uint2 o;
    o.x = pack_bf16x2(us[0], us[1]);
    o.y = pack_bf16x2(us[2], us[3]);
    reinterpret_cast<uint2*>(u)[i] = o;
  }
}

// partial[b * chunks + c] = sum of squares of chunk c of matrix b (fp32)
__global__ void ns_sumsq_kernel(const __nv_bfloat16* __restrict__ x, long long per_matrix,
                                int chunks, float* __restrict__ partial) {
  const int b = blockIdx.x / chunks;
  const int c = blockIdx.x - b * chunks;
  const long long lo = static_cast<long long>(c) * kNsChunk;
  const long long hi = min(per_matrix, lo + kNsChunk);
  const __nv_bfloat16* xm = x + static_cast<long long>(b) * per_matrix;
  float s = 0.f;
  for (long long i = lo + 8 * threadIdx.x; i < hi; i += 8 * blockDim.x) {
    const uint4 w = *reinterpret_cast<const uint4*>(xm + i);
    const float f[8] = {bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y),
                        bf16_lo(w.z), bf16_hi(w.z), bf16_lo(w.w), bf16_hi(w.w)};
#pragma unroll
    for (int j = 0; j < 8; ++j) s = fmaf(f[j], f[j], s);
  }
  s = warp_sum(s);
  __shared__ float ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? ws[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) partial[blockIdx.x] = t;
  }
}

// x[b] <- bf16(x[b] / d[b]), d[b] = bf16(bf16(||x[b]||_F) + 1e-7): the bf16
// X.div_(X.norm(dim=(-2,-1), keepdim=True) + 1e-7) of train.py:2902.  The
// chunk partials are summed in a fixed order, so the result is deterministic.
__global__ void ns_normalize_kernel(__nv_bfloat16* __restrict__ x, long long per_matrix,
                                    int chunks, const float* __restrict__ partial) {
  const int b = blockIdx.y;
  __shared__ float d_s;
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int c = 0; c < chunks; ++c) s += partial[b * chunks + c];
    const float nrm = bf16_round(sqrtf(s));
    d_s = bf16_round(nrm + 1e-7f);
  }
  __syncthreads();
  const float d = d_s;
  __nv_bfloat16* xm = x + static_cast<long long>(b) * per_matrix;
  for (long long i = 8 * (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x);
       i < per_matrix; i += 8LL * gridDim.x * blockDim.x) {
    uint4 w = *reinterpret_cast<const uint4*>(xm + i);
    w.x = pack_bf16x2(__fdiv_rn(bf16_lo(w.x), d), __fdiv_rn(bf16_hi(w.x), d));
    w.y = pack_bf16x2(__fdiv_rn(bf16_lo(w.y), d), __fdiv_rn(bf16_hi(w.y), d));
    w.z = pack_bf16x2(__fdiv_rn(bf16_lo(w.z), d), __fdiv_rn(bf16_hi(w.z), d));
    w.w = pack_bf16x2(__fdiv_rn(bf16_lo(w.w), d), __fdiv_rn(bf16_hi(w.w), d));
    *reinterpret_cast<uint4*>(xm + i) = w;
  }
}

// Group tables of a stack of `batch` matrices of `rows` rows each, as the
// grouped GEMM reads them: pad[b] = b*rows (b <= batch), tile[m] = m / (rows/128).
__global__ void ns_tables_kernel(int batch, int rows, int* __restrict__ pad,
                                 int* __restrict__ tile) {
  const int tiles_per = rows / 128;
  const int n_tiles = batch * tiles_per;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i <= batch || i < n_tiles;
       i += gridDim.x * blockDim.x) {
    if (i <= batch) pad[i] = i * rows;
    if (i < n_tiles) tile[i] = i / tiles_per;
  }
}

}  // namespace b200moe
