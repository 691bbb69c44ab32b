// Router softmax / top-k / renormalisation and the load-balancing statistics
// (spark-gpt train.py:2144-2158, 3098-3197).
//
// A token is handled by a group of L lanes (L = 2..32, a power of two) that
// hold 8 logits each: expert e lives in lane e / 8 of the group, register
// slot e % 8, so a lane's logits are one 16-byte load.  E = 64 uses 8 lanes,
// so one warp works on 4 tokens at once and every reduction is log2(L)
// shuffles.  Loops run in whole-warp rounds so every lane of a warp executes
// every shuffle.
#pragma once

#include "common.cuh"

namespace b200moe {

constexpr int kMaxTopK = 16;
constexpr int kVpt = 8;  // logits per lane

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <int L>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <int L>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Logits [e0, e0+8) of a row as fp32, -inf at e >= E or for an invalid row.
// vec: the row start is 16-byte aligned and ld is a multiple of 16 bytes, so a
// chunk that lies inside E is one vector load.
template <typename LT>
__device__ __forceinline__ void load_chunk(const LT* __restrict__ row, int e0, int E, bool valid,
                                           bool vec, float (&z)[kVpt]) {
  if (valid && vec && e0 + kVpt <= E) {
    if constexpr (sizeof(LT) == 2) {
      const uint4 v = *reinterpret_cast<const uint4*>(row + e0);
      z[0] = bf16_lo(v.x); z[1] = bf16_hi(v.x); z[2] = bf16_lo(v.y); z[3] = bf16_hi(v.y);
      z[4] = bf16_lo(v.z); z[5] = bf16_hi(v.z); z[6] = bf16_lo(v.w); z[7] = bf16_hi(v.w);
    } else {
      const float4 a = *reinterpret_cast<const float4*>(row + e0);
      const float4 b = *reinterpret_cast<const float4*>(row + e0 + 4);
      z[0] = a.x; z[1] = a.y; z[2] = a.z; z[3] = a.w;
      z[4] = b.x; z[5] = b.y; z[6] = b.z; z[7] = b.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kVpt; ++j) {
      const int e = e0 + j;
      z[j] = (valid && e < E) ? to_f32(row[e]) : -INFINITY;
    }
  }
}

// p = softmax(row[0:E]) in fp32 (max-subtract, exp, sum, divide) for this
// lane's experts e = 8*sub + j; entries beyond E are 0.  FAST (gradient and
// statistics kernels): __expf and one reciprocal; otherwise expf and a
// division per entry (the forward selection).  `valid` false: row is not
// read, p is garbage but every shuffle still runs.
template <int L, bool FAST, typename LT>
__device__ __forceinline__ void softmax_group(const LT* __restrict__ row, int E, int sub,
                                              bool valid, bool vec, float (&p)[kVpt]) {
  float z[kVpt];
  load_chunk(row, sub * kVpt, E, valid, vec, z);
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kVpt; ++j) m = fmaxf(m, z[j]);
  m = group_max<L>(m);
  if (!valid) m = 0.f;
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kVpt; ++j) {
    const bool in = valid && sub * kVpt + j < E;
    p[j] = in ? (FAST ? __expf(z[j] - m) : expf(z[j] - m)) : 0.f;
    s += p[j];
  }
  s = group_sum<L>(s);
  if (!valid) s = 1.f;
  if (FAST) {
    const float inv = 1.0f / s;
#pragma unroll
    for (int j = 0; j < kVpt; ++j) p[j] *= inv;
  } else {
#pragma unroll
    for (int j = 0; j < kVpt; ++j) p[j] = p[j] / s;
  }
}

// Value of register slot e % 8 from lane e / 8 of the group (all lanes call).
template <int L>
__device__ __forceinline__ float group_fetch(const float (&v)[kVpt], int e) {
  float x = 0.f;
#pragma unroll
  for (int j = 0; j < kVpt; ++j)
    if ((e & (kVpt - 1)) == j) x = v[j];
  return __shfl_sync(0xffffffffu, x, (e >> 3) & (L - 1), L);
}

// Grid-stride over tokens in whole-grid rounds: every thread runs the same
// number of rounds (t may be past T: `valid` false), so no lane of a warp
// leaves a shuffle early.
struct GroupTokens {
  long long first, stride, rounds;
  template <int L>
  __device__ __forceinline__ static GroupTokens make(long long T) {
    GroupTokens g;
    const long long per_block = blockDim.x / L;
    g.stride = per_block * gridDim.x;
    g.first = blockIdx.x * per_block + threadIdx.x / L;
    g.rounds = (T + g.stride - 1) / g.stride;
    return g;
  }
};

// The order torch.topk on CUDA lists its k winners in (the reference's router,
// train.py:2147; torch 2.11: TensorTopK.cu gatherTopK, Sort.cu SmallBitonicSort,
// SortUtils.cuh bitonicSort / bitonicSwap).  The winners are gathered as
// [values above the k-th, by ascending index] + [values equal to the k-th, by
// ascending index] into 32 slots (slots >= k invalid) and sorted by a bitonic
// key/value network, descending and unstable, so equal values come out in a
// fixed, shape-dependent order.  In: (sv, si) in (value desc, index asc) order,
// as the selection produces them.  Out: the same winners in torch's order.
// Only called for rows with a tie among their winners (without one the order
// is the unique descending order); every index below is static.
__device__ __forceinline__ void torch_topk_order(float (&sv)[kMaxTopK], int (&si)[kMaxTopK],
                                                 int k) {
  const float kth = sv[k - 1];
  // rank of each winner in the gathered order
  int rank[kMaxTopK];
#pragma unroll
  for (int i = 0; i < kMaxTopK; ++i) {
    int r = 0;
    const bool ai = sv[i] > kth;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      if (j >= k) continue;
      const bool aj = sv[j] > kth;
      // above-kth winners first, each group by ascending expert index
      r += (aj && !ai) || (aj == ai && si[j] < si[i]) ? 1 : 0;
    }
    rank[i] = r;
  }
  float K[32];
  int V[32];  // -1: an invalid slot (sorts to the end)
#pragma unroll
  for (int d = 0; d < 32; ++d) {
    K[d] = 0.f;
    V[d] = -1;
  }
#pragma unroll
  for (int d = 0; d < kMaxTopK; ++d) {
#pragma unroll
    for (int i = 0; i < kMaxTopK; ++i) {
      if (i < k && rank[i] == d) {
        K[d] = sv[i];
        V[d] = si[i];
      }
    }
  }
  // 16 "threads" t, each owning one compare-exchange (pos, pos + stride) per
  // substep; swap when (K[a] > K[b] && a valid) || b invalid equals the
  // substep's direction flag
#pragma unroll
  for (int size = 2; size <= 32; size *= 2) {
#pragma unroll
    for (int stride = size / 2; stride > 0; stride /= 2) {
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const bool flag = size < 32 && (t & (size / 2)) != 0;
        const int a = 2 * t - (t & (stride - 1));
        const int b = a + stride;
        const bool sw = (K[a] > K[b] && V[a] >= 0) || V[b] < 0;
        if (sw == flag) {
          const float tk = K[a];
          K[a] = K[b];
          K[b] = tk;
          const int tv = V[a];
          V[a] = V[b];
          V[b] = tv;
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kMaxTopK; ++r) {
    sv[r] = K[r];
    si[r] = V[r];
  }
}

template <int L, typename LT>
__global__ void router_topk_fwd_kernel(const LT* __restrict__ logits, long long ld, long long T,
                                       int E, int k, int norm, int vec,
                                       long long* __restrict__ selected,
                                       __nv_bfloat16* __restrict__ weights) {
  const int sub = threadIdx.x & (L - 1);
  const GroupTokens gt = GroupTokens::make<L>(T);
  for (long long rnd = 0; rnd < gt.rounds; ++rnd) {
    const long long t = gt.first + rnd * gt.stride;
    const bool valid = t < T;
    float p[kVpt];
    softmax_group<L, false>(logits + (valid ? t : 0) * ld, E, sub, valid, vec != 0, p);
#pragma unroll
    for (int j = 0; j < kVpt; ++j)
      if (sub * kVpt + j >= E) p[j] = -1.f;
    float sv[kMaxTopK];
    int si[kMaxTopK];
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
      sv[r] = 0.f;
      si[r] = 0;
      if (r < k) {
        // lane-local best (ascending e: the first maximum is the lowest index)
        float bv = -2.f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < kVpt; ++j) {
          if (p[j] > bv) {
            bv = p[j];
            bi = sub * kVpt + j;
          }
        }
#pragma unroll
        for (int o = L / 2; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
#pragma unroll
        for (int j = 0; j < kVpt; ++j)
          if (sub * kVpt + j == bi) p[j] = -3.f;
        sv[r] = bv;
        si[r] = bi;
      }
    }
    bool tie = false;
#pragma unroll
    for (int r = 0; r + 1 < kMaxTopK; ++r)
      if (r + 1 < k) tie |= sv[r] == sv[r + 1];
    if (tie) torch_topk_order(sv, si, k);
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r)
      if (r < k) sum += sv[r];
    if (valid) {
#pragma unroll
      for (int r = 0; r < kMaxTopK; ++r) {
        if (r < k && (r & (L - 1)) == sub) {
          selected[t * k + r] = si[r];
          weights[t * k + r] = __float2bfloat16_rn(norm ? sv[r] / sum : sv[r]);
        }
      }
    }
  }
}

// d logits (T, ld) of the router from d(routing weights) (T,k) fp32 in slot
// order, plus an optional extra bf16 logit gradient (the load-balancing loss);
// columns in [E, ld) are written as zero.  8L >= ld.
template <int L>
__global__ void router_topk_bwd_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                       const long long* __restrict__ selected,
                                       const float* __restrict__ d_weights,
                                       const __nv_bfloat16* __restrict__ d_extra, long long T,
                                       int E, int k, int norm, int vec,
                                       __nv_bfloat16* __restrict__ d_logits) {
  constexpr int kSlots = (kMaxTopK + L - 1) / L;  // slots r = sub + L*i held by this lane
  const int sub = threadIdx.x & (L - 1);
  const int e0 = sub * kVpt;
  const GroupTokens gt = GroupTokens::make<L>(T);
  for (long long rnd = 0; rnd < gt.rounds; ++rnd) {
    const long long t = gt.first + rnd * gt.stride;
    const bool valid = t < T;
    const long long tt = valid ? t : 0;
    float p[kVpt];
    softmax_group<L, true>(logits + tt * ld, E, sub, valid, vec != 0, p);
    int sl[kSlots];
    float dl[kSlots];
#pragma unroll
    for (int i = 0; i < kSlots; ++i) {
      const int r = sub + L * i;
      const bool on = valid && r < k;
      sl[i] = on ? static_cast<int>(selected[tt * k + r]) : -1;
      dl[i] = on ? d_weights[tt * k + r] : 0.f;
    }
    int si[kMaxTopK];
    float ps[kMaxTopK], dw[kMaxTopK];
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
      si[r] = -1;
      ps[r] = 0.f;
      dw[r] = 0.f;
      if (r < k) {
        const int e = __shfl_sync(0xffffffffu, sl[r / L], r % L, L);
        dw[r] = __shfl_sync(0xffffffffu, dl[r / L], r % L, L);
        si[r] = e;
        const float pe = group_fetch<L>(p, e < 0 ? 0 : e);  // every lane shuffles
        ps[r] = e >= 0 ? pe : 0.f;
        s += ps[r];
      }
    }
    if (!valid || s == 0.f) s = 1.f;
    const float inv_s = 1.0f / s;
    float dot = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r)
      if (r < k) dot += dw[r] * (ps[r] * inv_s);
    float g[kVpt];
#pragma unroll
    for (int j = 0; j < kVpt; ++j) g[j] = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
      if (r < k) {
        const float dp = norm ? (dw[r] - dot) * inv_s : dw[r];
#pragma unroll
        for (int j = 0; j < kVpt; ++j)
          if (e0 + j == si[r]) g[j] = dp;
      }
    }
    float pg = 0.f;
#pragma unroll
    for (int j = 0; j < kVpt; ++j) pg += p[j] * g[j];
    pg = group_sum<L>(pg);
    if (valid) {
      float ex[kVpt];
#pragma unroll
      for (int j = 0; j < kVpt; ++j) ex[j] = 0.f;
      const bool vio = vec && e0 + kVpt <= ld;
      if (d_extra) {
        if (vio) {
          const uint4 v = *reinterpret_cast<const uint4*>(d_extra + tt * ld + e0);
          ex[0] = bf16_lo(v.x); ex[1] = bf16_hi(v.x); ex[2] = bf16_lo(v.y); ex[3] = bf16_hi(v.y);
          ex[4] = bf16_lo(v.z); ex[5] = bf16_hi(v.z); ex[6] = bf16_lo(v.w); ex[7] = bf16_hi(v.w);
        } else {
#pragma unroll
          for (int j = 0; j < kVpt; ++j)
            if (e0 + j < ld) ex[j] = __bfloat162float(d_extra[tt * ld + e0 + j]);
        }
      }
      float v[kVpt];
#pragma unroll
      for (int j = 0; j < kVpt; ++j) v[j] = (e0 + j < E) ? p[j] * (g[j] - pg) + ex[j] : 0.f;
      if (vio) {
        uint4 o;
        o.x = pack_bf16x2(v[0], v[1]);
        o.y = pack_bf16x2(v[2], v[3]);
        o.z = pack_bf16x2(v[4], v[5]);
        o.w = pack_bf16x2(v[6], v[7]);
        *reinterpret_cast<uint4*>(d_logits + tt * ld + e0) = o;
      } else {
#pragma unroll
        for (int j = 0; j < kVpt; ++j)
          if (e0 + j < ld) d_logits[tt * ld + e0 + j] = __float2bfloat16_rn(v[j]);
      }
    }
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

template <int L>
__global__ void lb_partials_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                   const long long* __restrict__ selected,
                                   const unsigned char* __restrict__ valid_mask, long long T,
                                   int E, int k, int vec, float* __restrict__ partials) {
  constexpr int kGroups = kLbThreads / L;
  // [groups][8L] soft sums, then [E] hard counts, then [groups] entropy, [groups] rows
  extern __shared__ float lsh[];
  float* soft_sh = lsh;
  float* hard_sh = lsh + kGroups * kVpt * L;
  float* ent_sh = hard_sh + E;
  float* rows_sh = ent_sh + kGroups;
  const int sub = threadIdx.x & (L - 1);
  const int grp = threadIdx.x / L;
  for (int i = threadIdx.x; i < E; i += blockDim.x) hard_sh[i] = 0.f;
  __syncthreads();
  float soft[kVpt];
#pragma unroll
  for (int j = 0; j < kVpt; ++j) soft[j] = 0.f;
  float ent = 0.f, rows = 0.f;
  const float tiny = 1.17549435e-38f;
  const long long t0 = static_cast<long long>(blockIdx.x) * kLbTokensPerBlock;
  for (int i = grp; i < kLbTokensPerBlock; i += kGroups) {  // uniform trip count per warp
    const long long t = t0 + i;
    const bool valid = t < T && (valid_mask == nullptr || valid_mask[t] != 0);
    float p[kVpt];
    softmax_group<L, true>(logits + (valid ? t : 0) * ld, E, sub, valid, vec != 0, p);
    if (valid) {
#pragma unroll
      for (int j = 0; j < kVpt; ++j) {
        if (sub * kVpt + j < E) {
          soft[j] += p[j];
          ent -= p[j] * logf(fmaxf(p[j], tiny));
        }
      }
      rows += 1.f;
      for (int r = sub; r < k; r += L) {
        const long long e = selected[t * k + r];
        if (e >= 0 && e < E) atomicAdd(&hard_sh[e], 1.f);  // integer-valued: exact
      }
    }
  }
  ent = group_sum<L>(ent);
#pragma unroll
  for (int j = 0; j < kVpt; ++j) soft_sh[grp * kVpt * L + sub * kVpt + j] = soft[j];
  if (sub == 0) {
    ent_sh[grp] = ent;
    rows_sh[grp] = rows;
  }
  __syncthreads();
  const int W = 2 * E + 2;
  float* out = partials + static_cast<long long>(blockIdx.x) * W;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    float acc = 0.f;
    for (int g = 0; g < kGroups; ++g) acc += soft_sh[g * kVpt * L + e];
    out[E + e] = acc;
    out[e] = hard_sh[e];
  }
  if (threadIdx.x == 0) {
    float a = 0.f, b = 0.f;
    for (int g = 0; g < kGroups; ++g) {
      a += ent_sh[g];
      b += rows_sh[g];
    }
    out[2 * E] = a;
    out[2 * E + 1] = b;
  }
}

template <int L>
constexpr size_t lb_partials_smem(int E) {
  return (static_cast<size_t>(kLbThreads / L) * kVpt * L + E + 2 * (kLbThreads / L)) *
         sizeof(float);
}

// packed[i] += sum over blocks of partials[b][i], fixed block order.
// packed[i] += sum over blocks of partials[b][i]: warp w sums the blocks
// b = w (mod warps) for its lane's columns, then the warps' sums are added in
// warp order (a fixed order: deterministic).  Shared memory: warps * W floats.
__global__ void lb_accumulate_kernel(const float* __restrict__ partials, int nblk, int W,
                                     float* __restrict__ packed) {
  extern __shared__ float acc_sh[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  for (int i = lane; i < W; i += 32) {
    float a = 0.f;
#pragma unroll 4
    for (int b = warp; b < nblk; b += nw) a += partials[static_cast<long long>(b) * W + i];
    acc_sh[warp * W + i] = a;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < W; i += blockDim.x) {
    float a = 0.f;
    for (int w = 0; w < nw; ++w) a += acc_sh[w * W + i];
    packed[i] += a;
  }
}

// aux value, stats and the per-expert gradient coefficient from the
// all-reduced packed sums (train.py:3163-3196).
// stats: [min_frac, max_frac, cv, entropy, unused]
__global__ void lb_finalize_kernel(const float* __restrict__ packed, int E, int k, int world,
                                   float* __restrict__ aux, float* __restrict__ stats,
                                   float* __restrict__ coef) {
  extern __shared__ float fsh[];  // [2E+2]
  for (int i = threadIdx.x; i < 2 * E + 2; i += blockDim.x) fsh[i] = packed[i];
  __syncthreads();
  const float rows = fsh[2 * E + 1];
  const float safe = fmaxf(rows, 1.f);
  const float has = rows > 0.f ? 1.f : 0.f;
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    coef[e] = has * static_cast<float>(world) * static_cast<float>(E) / safe * (fsh[e] / safe);
  if (threadIdx.x != 0) return;
  float dot = 0.f, mn = INFINITY, mx = -INFINITY, sum = 0.f, unused = 0.f;
  for (int e = 0; e < E; ++e) {
    const float a = fsh[e] / safe;
    dot += a * (fsh[E + e] / safe);
    const float fr = fsh[e] / (safe * k);
    mn = fminf(mn, fr);
    mx = fmaxf(mx, fr);
    sum += fr;
    unused += fsh[e] == 0.f ? 1.f : 0.f;
  }
  const float mean = sum / E;
  float var = 0.f;
  for (int e = 0; e < E; ++e) {
    const float d = fsh[e] / (safe * k) - mean;
    var += d * d;
  }
  var /= E;
  *aux = has * static_cast<float>(E) * dot;
  stats[0] = mn;
  stats[1] = mx;
  stats[2] = sqrtf(var) / fmaxf(mean, 1e-12f);
  stats[3] = fsh[2 * E] / safe;
  stats[4] = unused;
}

// d aux / d logits[t,e] = g * mask_t * p_e (coef_e - <p, coef>), g = *grad;
// columns in [E, ld) are zero.  8L >= ld.
template <int L>
__global__ void lb_grad_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                               const unsigned char* __restrict__ valid_mask, long long T, int E,
                               const float* __restrict__ coef, const float* __restrict__ grad,
                               int vec, __nv_bfloat16* __restrict__ d_logits) {
  const float g = *grad;
  const int sub = threadIdx.x & (L - 1);
  const int e0 = sub * kVpt;
  float c[kVpt];
#pragma unroll
  for (int j = 0; j < kVpt; ++j) c[j] = (e0 + j < E) ? coef[e0 + j] : 0.f;
  const bool vio = vec && e0 + kVpt <= ld;
  const GroupTokens gt = GroupTokens::make<L>(T);
  for (long long rnd = 0; rnd < gt.rounds; ++rnd) {
    const long long t = gt.first + rnd * gt.stride;
    const bool valid = t < T;
    const long long tt = valid ? t : 0;
    const bool on = valid && (valid_mask == nullptr || valid_mask[tt] != 0);
    float p[kVpt];
    softmax_group<L, true>(logits + tt * ld, E, sub, valid, vec != 0, p);
    float pc = 0.f;
#pragma unroll
    for (int j = 0; j < kVpt; ++j) pc += p[j] * c[j];
    pc = group_sum<L>(pc);
    if (valid) {
      float v[kVpt];
#pragma unroll
      for (int j = 0; j < kVpt; ++j) v[j] = (on && e0 + j < E) ? g * p[j] * (c[j] - pc) : 0.f;
      if (vio) {
        uint4 o;
        o.x = pack_bf16x2(v[0], v[1]);
        o.y = pack_bf16x2(v[2], v[3]);
        o.z = pack_bf16x2(v[4], v[5]);
        o.w = pack_bf16x2(v[6], v[7]);
        *reinterpret_cast<uint4*>(d_logits + tt * ld + e0) = o;
      } else {
#pragma unroll
        for (int j = 0; j < kVpt; ++j)
          if (e0 + j < ld) d_logits[tt * ld + e0 + j] = __float2bfloat16_rn(v[j]);
      }
    }
  }
}

}  // namespace b200moe
