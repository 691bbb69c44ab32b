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
constexpr int kRouterThreads = 256;  // threads per block of the router kernels
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
// fixed, shape-dependent order.
//
// Here the L lanes of a token's group hold the 32 slots (32/L each: slot s in
// lane s / (32/L)) and run that network together: a compare-exchange whose
// slots lie in one lane is done in registers, one across lanes by a shuffle
// with the partner lane (both lanes evaluate the same comparison).  The
// gathered order is built from the lanes' own experts: lane `sub` holds the
// probabilities of experts 8*sub .. 8*sub+7 (`pe`, as the selection saw them),
// so the winners above the k-th value in ascending index order are each
// lane's such experts placed after those of the lower lanes (a prefix sum of
// per-lane counts), and likewise the first k - above experts equal to it.
// In: `kth` the k-th largest probability.  Out: this lane's slots (K, V) in
// torch's order; V = -1 marks a slot >= k.  `sh_k`, `sh_v`: the group's
// 32-slot shared-memory staging area.  Every lane of the warp must call it.
template <int L>
__device__ __forceinline__ int lane_exclusive_sum(int v, int sub) {
  int incl = v;
#pragma unroll
  for (int o = 1; o < L; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o, L);
    if (sub >= o) incl += u;
  }
  return incl - v;
}

template <int L>
__device__ __forceinline__ void stage_gathered_winners(const float (&pe)[kVpt], float kth, int k,
                                                       int sub, float* sh_k, int* sh_v) {
  int n_above = 0, n_equal = 0;
#pragma unroll
  for (int j = 0; j < kVpt; ++j) {
    n_above += pe[j] > kth ? 1 : 0;
    n_equal += pe[j] == kth ? 1 : 0;
  }
  int above_at = lane_exclusive_sum<L>(n_above, sub);
  int equal_at = lane_exclusive_sum<L>(n_equal, sub);
  const int above_total = __shfl_sync(0xffffffffu, above_at + n_above, L - 1, L);
  equal_at += above_total;
#pragma unroll
  for (int j = 0; j < kVpt; ++j) {
    if (pe[j] > kth) {
      sh_k[above_at] = pe[j];
      sh_v[above_at] = sub * kVpt + j;
      ++above_at;
    } else if (pe[j] == kth) {
      if (equal_at < k) {
        sh_k[equal_at] = pe[j];
        sh_v[equal_at] = sub * kVpt + j;
      }
      ++equal_at;
    }
  }
  __syncwarp();
}

// The general case (any k <= 16, any L): 32 slots over the group's lanes.
template <int L>
__device__ __forceinline__ void torch_topk_order(const float (&pe)[kVpt], float kth, int k, int sub,
                                                 float* sh_k, int* sh_v, float (&K)[32 / L],
                                                 int (&V)[32 / L]) {
  constexpr int SPL = 32 / L;  // slots per lane
  stage_gathered_winners<L>(pe, kth, k, sub, sh_k, sh_v);
#pragma unroll
  for (int j = 0; j < SPL; ++j) {
    const int d = sub * SPL + j;
    K[j] = d < k ? sh_k[d] : 0.f;
    V[j] = d < k ? sh_v[d] : -1;
  }
  __syncwarp();  // the staging area is free for the next token
  // pair (a, a + stride) exchanges when (K[a] > K[b] && a valid) || b invalid
  // equals the direction flag, which is bit `size` of a (false in the last merge)
#pragma unroll
  for (int size = 2; size <= 32; size *= 2) {
#pragma unroll
    for (int stride = size / 2; stride > 0; stride /= 2) {
      if (stride >= SPL) {
        const int lane_mask = stride / SPL;
#pragma unroll
        for (int j = 0; j < SPL; ++j) {
          const float ok = __shfl_xor_sync(0xffffffffu, K[j], lane_mask);
          const int ov = __shfl_xor_sync(0xffffffffu, V[j], lane_mask);
          const int slot = sub * SPL + j;
          const bool lower = (slot & stride) == 0;
          const bool flag = size < 32 && (slot & size) != 0;
          const float ka = lower ? K[j] : ok, kb = lower ? ok : K[j];
          const int va = lower ? V[j] : ov, vb = lower ? ov : V[j];
          const bool sw = (ka > kb && va >= 0) || vb < 0;
          if (sw == flag) {
            K[j] = ok;
            V[j] = ov;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < SPL; ++j) {
          if ((j & stride) == 0) {
            const bool flag = size < 32 && ((sub * SPL + j) & size) != 0;
            const bool sw = (K[j] > K[j + stride] && V[j] >= 0) || V[j + stride] < 0;
            if (sw == flag) {
              const float tk = K[j];
              K[j] = K[j + stride];
              K[j + stride] = tk;
              const int tv = V[j];
              V[j] = V[j + stride];
              V[j + stride] = tv;
            }
          }
        }
      }
    }
  }
}

// k a power of two and k <= L (every MoE shape here: top-2/4/8/16): the valid
// slots never leave [0, k) -- an invalid slot always sorts behind a valid one,
// and a pair (a, a + stride >= k) has direction flag bit `size` of a < k, i.e.
// false, so it never exchanges -- so the network reduces to its substeps with
// stride < k on lanes 0..k-1, one winner per lane.  Out: lane `sub` < k holds
// slot `sub` (K, V).
template <int L>
__device__ __forceinline__ void torch_topk_order_small(const float (&pe)[kVpt], float kth, int k,
                                                       int sub, float* sh_k, int* sh_v, float& K,
                                                       int& V) {
  stage_gathered_winners<L>(pe, kth, k, sub, sh_k, sh_v);
  K = sub < k ? sh_k[sub] : 0.f;
  V = sub < k ? sh_v[sub] : -1;
  __syncwarp();  // the staging area is free for the next token
#pragma unroll
  for (int size = 2; size <= 32; size *= 2) {
#pragma unroll
    for (int stride = size / 2; stride > 0; stride /= 2) {
      if (stride < L) {  // (stride < k is checked at run time: k <= L)
        const float ok = __shfl_xor_sync(0xffffffffu, K, stride);
        const int ov = __shfl_xor_sync(0xffffffffu, V, stride);
        if (stride < k) {
          const bool lower = (sub & stride) == 0;
          const bool flag = size < 32 && (sub & size) != 0;
          const float ka = lower ? K : ok, kb = lower ? ok : K;
          if ((ka > kb) == flag) {
            K = ok;
            V = ov;
          }
        }
      }
    }
  }
}

// KMAX: the largest k this instantiation takes (8 or KMAX): fewer registers
// for the common top-8, so more tokens are in flight per SM.
template <int L, int KMAX, typename LT>
__global__ void router_topk_fwd_kernel(const LT* __restrict__ logits, long long ld, long long T,
                                       int E, int k, int norm, int vec,
                                       long long* __restrict__ selected,
                                       __nv_bfloat16* __restrict__ weights) {
  __shared__ float sh_k[kRouterThreads / L][32];  // tie-order staging, 32 slots per token group
  __shared__ int sh_v[kRouterThreads / L][32];
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
    float pe[kVpt];  // the probabilities as selected (entries >= E: -1)
#pragma unroll
    for (int j = 0; j < kVpt; ++j) pe[j] = p[j];
    float sv[KMAX];
    int si[KMAX];
    float kth = 0.f;  // the k-th largest probability
#pragma unroll
    for (int r = 0; r < KMAX; ++r) {
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
        if (r == k - 1) kth = bv;
      }
    }
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < KMAX; ++r)
      if (r < k) sum += sv[r];
    // winners with equal probabilities leave in torch's order; the network
    // runs (warp-uniformly) only when some token of the warp has such a tie
    bool tie = false;
#pragma unroll
    for (int r = 0; r + 1 < KMAX; ++r)
      if (r + 1 < k) tie |= sv[r] == sv[r + 1];
    if (!__any_sync(0xffffffffu, valid && tie)) {
      if (valid) {
#pragma unroll
        for (int r = 0; r < KMAX; ++r) {
          if (r < k && (r & (L - 1)) == sub) {
            selected[t * k + r] = si[r];
            weights[t * k + r] = __float2bfloat16_rn(norm ? sv[r] / sum : sv[r]);
          }
        }
      }
    } else if ((k & (k - 1)) == 0 && k <= L) {
      float K;
      int V;
      const int grp = threadIdx.x / L;
      torch_topk_order_small<L>(pe, kth, k, sub, sh_k[grp], sh_v[grp], K, V);
      if (valid && sub < k) {
        selected[t * k + sub] = V;
        weights[t * k + sub] = __float2bfloat16_rn(norm ? K / sum : K);
      }
    } else {
      constexpr int SPL = 32 / L;
      float K[SPL];
      int V[SPL];
      const int grp = threadIdx.x / L;
      torch_topk_order<L>(pe, kth, k, sub, sh_k[grp], sh_v[grp], K, V);
      if (valid) {
#pragma unroll
        for (int j = 0; j < SPL; ++j) {
          const int d = sub * SPL + j;
          if (d < k) {
            selected[t * k + d] = V[j];
            weights[t * k + d] = __float2bfloat16_rn(norm ? K[j] / sum : K[j]);
          }
        }
      }
    }
  }
}

// d logits (T, ld) of the router from d(routing weights) (T,k) fp32 in slot
// order, plus an optional extra bf16 logit gradient (the load-balancing loss);
// columns in [E, ld) are written as zero.  8L >= ld.
template <int L, int KMAX>
__global__ void router_topk_bwd_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                       const long long* __restrict__ selected,
                                       const float* __restrict__ d_weights,
                                       const __nv_bfloat16* __restrict__ d_extra, long long T,
                                       int E, int k, int norm, int vec,
                                       __nv_bfloat16* __restrict__ d_logits) {
  constexpr int kSlots = (KMAX + L - 1) / L;  // slots r = sub + L*i held by this lane
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
    int si[KMAX];
    float ps[KMAX], dw[KMAX];
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < KMAX; ++r) {
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
    for (int r = 0; r < KMAX; ++r)
      if (r < k) dot += dw[r] * (ps[r] * inv_s);
    float g[kVpt];
#pragma unroll
    for (int j = 0; j < kVpt; ++j) g[j] = 0.f;
#pragma unroll
    for (int r = 0; r < KMAX; ++r) {
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
// Blocks of the statistics kernel: one token per lane group and round, at
// most 8 blocks per SM of B200's 148 (more tokens loop over the grid in
// rounds), so the partials stay under 1184 rows.
constexpr int kLbMaxBlocks = 148 * 8;

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
  const long long stride = static_cast<long long>(gridDim.x) * kGroups;
  const long long rounds = (T + stride - 1) / stride;  // the same for every warp
  for (long long rnd = 0; rnd < rounds; ++rnd) {
    const long long t = rnd * stride + static_cast<long long>(blockIdx.x) * kGroups + grp;
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

// Deterministic two-level sum of the per-block partial rows (W floats each):
// block b of level one adds rows [kLbRowsPerSum*b, kLbRowsPerSum*(b+1)) in row
// order into out[b]; level two (one block, accumulate = 1) adds those rows in
// order into packed.  Each thread owns columns i = threadIdx.x + blockDim.x*j,
// so a row is read coalesced and every sum has a fixed order.
constexpr int kLbRowsPerSum = 32;

__global__ void lb_sum_rows_kernel(const float* __restrict__ rows_in, int nrows, int W,
                                   float* __restrict__ out, int accumulate) {
  const int r0 = blockIdx.x * kLbRowsPerSum;
  const int r1 = min(nrows, r0 + kLbRowsPerSum);
  for (int i = threadIdx.x; i < W; i += blockDim.x) {
    float a = 0.f;
#pragma unroll 8
    for (int r = r0; r < r1; ++r) a += rows_in[static_cast<long long>(r) * W + i];
    if (accumulate)
      out[i] += a;
    else
      out[static_cast<long long>(blockIdx.x) * W + i] = a;
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
