// The fp8 expert path's element-wise kernels (spark-gpt's --fp8-mlp on MoE
// layers, train.py:1301-1604): the gather of x fused with its e4m3
// quantization, the per-expert e4m3 weight copies with their power-of-two
// scales, and the e5m2 quantization of the expert rows' gradient.  The
// delayed per-site scales (x, gu, h, d_gu, dy) are read from device memory and
// every kernel raises the amax slot of the tensor it quantizes (the absolute
// maximum of the unquantized values), so nothing here waits for the host.
#pragma once

#include "common.cuh"

namespace b200moe {

constexpr float kE4m3Max = 448.0f;

// ---------------------------------------------------------------------------
// x8[r] = e4m3(x[token(r)] * scale_x) over the padded expert-order rows
// (train.py:1301-1313), padding rows zero; amax of |x| over the routed tokens.
// Warp per token: the bf16 row is read once, quantized once and written to
// the padded rows of its k slots (inv_pad).
// ---------------------------------------------------------------------------
__global__ void fp8_gather_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                        const int* __restrict__ inv_pad,
                                        const int* __restrict__ row_flat,
                                        const int* __restrict__ total_rows, long long T, int k,
                                        int H, const float* __restrict__ scale,
                                        float* __restrict__ amax, uint8_t* __restrict__ x8) {
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;  // 8 bf16 in, 8 e4m3 bytes out per vector
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long warp_id = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
  const float s = __ldg(scale);
  float m = 0.f;
  for (long long t = warp_id; t < T; t += warps) {
    const int rl = lane < k ? inv_pad[t * k + lane] : -1;
    if (__ballot_sync(0xffffffffu, rl >= 0) == 0u) continue;  // no slot has an expert
    const uint4* src = reinterpret_cast<const uint4*>(x + t * H);
    for (int v = lane; v < nvec; v += 32) {
      const uint4 w = __ldg(src + v);
      const float f[8] = {bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y),
                          bf16_lo(w.z), bf16_hi(w.z), bf16_lo(w.w), bf16_hi(w.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(f[j]));
      const uint2 q = make_uint2(pack_fp8x4<kE4M3>(f[0] * s, f[1] * s, f[2] * s, f[3] * s),
                                 pack_fp8x4<kE4M3>(f[4] * s, f[5] * s, f[6] * s, f[7] * s));
      for (int j = 0; j < k; ++j) {
        const long long r = __shfl_sync(0xffffffffu, rl, j);
        if (r >= 0) reinterpret_cast<uint2*>(x8 + r * H)[v] = q;
      }
    }
  }
  // padding rows
  const long long total = *total_rows;
  const int nv16 = H / 16;
  for (long long base = warp_id * 32; base < total; base += warps * 32) {
    const long long r = base + lane;
    unsigned pad = __ballot_sync(0xffffffffu, r < total && row_flat[r] < 0);
    while (pad) {
      const int i = __ffs(pad) - 1;
      pad &= pad - 1;
      uint4* dst = reinterpret_cast<uint4*>(x8 + (base + i) * H);
      for (int v = lane; v < nv16; v += 32) dst[v] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  m = warp_max(m);
  if (lane == 0 && m > 0.f) atomic_max_nonneg(amax, m);
}

// ---------------------------------------------------------------------------
// Per-expert e4m3 copies of fp32 (E, rows, cols) master weights
// (train.py:1536-1540): q_e = 2^floor(log2(448 / max|w_e|)), w8 = e4m3(w * q_e).
// Pass 1: per-(expert, split) maxima; pass 2: q_e; pass 3: the copies.
// ---------------------------------------------------------------------------
constexpr int kWeightAmaxThreads = 256;

__global__ void fp8_weight_amax_kernel(const float* __restrict__ w, long long per_expert,
                                       int splits, float* __restrict__ partial) {
  __shared__ float red[kWeightAmaxThreads / 32];
  const int e = blockIdx.y;
  const long long n4 = per_expert / 4;
  const long long chunk = (n4 + splits - 1) / splits;
  const long long a = blockIdx.x * chunk;
  const long long b = min(n4, a + chunk);
  const float4* src = reinterpret_cast<const float4*>(w + e * per_expert);
  float m = 0.f;
  for (long long i = a + threadIdx.x; i < b; i += blockDim.x) {
    const float4 v = __ldg(src + i);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < kWeightAmaxThreads / 32 ? red[threadIdx.x] : 0.f;
    m = warp_max(m);
    if (threadIdx.x == 0) partial[static_cast<long long>(e) * splits + blockIdx.x] = m;
  }
}

__global__ void fp8_weight_scale_kernel(const float* __restrict__ partial, int E, int splits,
                                        float* __restrict__ q) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  float m = 0.f;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, partial[static_cast<long long>(e) * splits + s]);
  m = fmaxf(m, 1e-30f);
  q[e] = exp2f(floorf(log2f(kE4m3Max / m)));
}

__global__ void fp8_weight_quant_kernel(const float* __restrict__ w, long long per_expert,
                                        long long total, const float* __restrict__ q,
                                        uint8_t* __restrict__ w8) {
  const long long n4 = total / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += stride) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(w) + i);
    const float s = __ldg(q + (4 * i) / per_expert);
    reinterpret_cast<uint32_t*>(w8)[i] = pack_fp8x4<kE4M3>(v.x * s, v.y * s, v.z * s, v.w * s);
  }
}

// ---------------------------------------------------------------------------
// dst = fp8(src * scale) element-wise over the first rows of a bf16 (rows,
// cols) matrix (all rows, or *total_rows of them), amax of |src| raised (the
// e5m2 copy of the expert rows' gradient that the down projection's weight
// gradient reads, train.py:1504-1530).
// ---------------------------------------------------------------------------
template <int FMT>
__global__ void fp8_quantize_rows_kernel(const __nv_bfloat16* __restrict__ src, long long n8,
                                         int cols, const int* __restrict__ total_rows,
                                         const float* __restrict__ scale, float* __restrict__ amax,
                                         uint8_t* __restrict__ dst) {
  const float s = __ldg(scale);
  // rows past the padded total (the buffer's spare capacity) hold no data
  if (total_rows) n8 = min(n8, static_cast<long long>(*total_rows) * cols / 8);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  float m = 0.f;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8;
       i += stride) {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(src) + i);
    const float f[8] = {bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y),
                        bf16_lo(w.z), bf16_hi(w.z), bf16_lo(w.w), bf16_hi(w.w)};
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(f[j]));
    reinterpret_cast<uint2*>(dst)[i] =
        make_uint2(pack_fp8x4<FMT>(f[0] * s, f[1] * s, f[2] * s, f[3] * s),
                   pack_fp8x4<FMT>(f[4] * s, f[5] * s, f[6] * s, f[7] * s));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0 && m > 0.f) atomic_max_nonneg(amax, m);
}

}  // namespace b200moe
