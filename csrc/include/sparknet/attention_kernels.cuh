// Split-KV flash-decoding kernels for grouped-query attention (sm_100a), shared by
// the torch entry point (decode_ops.cu) and the allocation-free C entry point
// (attention_noalloc.cu).  One query token per sequence; head_dim 128.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace sn {
namespace attn {

constexpr int kHead = 128;   // head_dim
constexpr int kTile = 32;    // keys per tile
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

// Number of KV spans per (sequence, KV head): enough blocks for two waves of the
// SMs, spans of at least 64 keys.
static inline int splits(int B, int Hkv, int max_len, int sms) {
  int want = (2 * sms + B * Hkv - 1) / (B * Hkv);
  if (want < 1) want = 1;
  int max_splits = (max_len + 63) / 64;
  if (max_splits < 1) max_splits = 1;
  return want < max_splits ? want : max_splits;
}

// Floats of scratch the kernels need: partial outputs [B, Hq, nsplit, 128] and
// (max, sum) pairs [B, Hq, nsplit, 2].
static inline size_t scratch_floats(int B, int Hq, int Hkv, int max_len, int sms) {
  return size_t(B) * Hq * splits(B, Hkv, max_len, sms) * (kHead + 2);
}

// ---------------------------------------------------------------------------
// Split-KV decode attention.  grid (B * Hkv, nsplit), block 128 threads.
// q: [B, Hq, 128] with Hq = G * Hkv; caches [B, Lmax, Hkv, 128]; lengths [B].
// part_o: [B, Hq, nsplit, 128] fp32 (unnormalised), part_ml: [B, Hq, nsplit, 2] (max, sum),
// both in log2 units.
// ---------------------------------------------------------------------------
template <int G>
static __global__ void __launch_bounds__(128) k_decode_attn(const __nv_bfloat16* __restrict__ q,
                                                     const __nv_bfloat16* __restrict__ k_cache,
                                                     const __nv_bfloat16* __restrict__ v_cache,
                                                     const int* __restrict__ lengths, float* __restrict__ part_o,
                                                     float* __restrict__ part_ml, int Hkv, int Lmax, int chunk,
                                                     float scale_log2) {
  __shared__ float qs[G][kHead];
  // rows padded by 16 bytes: lane-per-key 16-byte reads hit distinct bank groups
  __shared__ __align__(16) __nv_bfloat16 tile[kTile][kHead + 8];
  __shared__ float ps[G][kTile];
  __shared__ float corr[G];
  const int b = blockIdx.x / Hkv, h = blockIdx.x % Hkv, s = blockIdx.y, nsplit = gridDim.y;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int Hq = G * Hkv;
  const int len = lengths[b];
  const int start = s * chunk, end = min(start + chunk, len);
  for (int i = t; i < G * kHead; i += blockDim.x) {
    int g = i / kHead, d = i % kHead;
    qs[g][d] = bf(q[(size_t(b) * Hq + h * G + g) * kHead + d]) * scale_log2;
  }
  float m[G], l[G], acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
    acc[g] = 0.0f;
  }
  const size_t row_stride = size_t(Hkv) * kHead;
  const __nv_bfloat16* kbase = k_cache + (size_t(b) * Lmax * Hkv + h) * kHead;
  const __nv_bfloat16* vbase = v_cache + (size_t(b) * Lmax * Hkv + h) * kHead;
  __syncthreads();
  for (int k0 = start; k0 < end; k0 += kTile) {
    const int nk = min(kTile, end - k0);
    // K tile -> shared (each thread moves 4 x 16 bytes)
    for (int i = t; i < kTile * (kHead / 8); i += blockDim.x) {
      int key = i / (kHead / 8), c = i % (kHead / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (key < nk) v = *reinterpret_cast<const uint4*>(kbase + size_t(k0 + key) * row_stride + c * 8);
      *reinterpret_cast<uint4*>(&tile[key][c * 8]) = v;
    }
    __syncthreads();
    // scores: thread (warp w, lane = key) computes heads g = w, w + 4, ...
    for (int g = warp; g < G; g += 4) {
      float sc = -INFINITY;
      if (lane < nk) {
        float dot = 0.0f;
#pragma unroll
        for (int c = 0; c < kHead / 8; ++c) {
          uint4 kv = *reinterpret_cast<const uint4*>(&tile[lane][c * 8]);
          const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float2 kf = __bfloat1622float2(k2[e]);
            dot += qs[g][c * 8 + 2 * e] * kf.x + qs[g][c * 8 + 2 * e + 1] * kf.y;
          }
        }
        sc = dot;
      }
      float tmax = sc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      float mnew = fmaxf(m[g], tmax);
      float p = lane < nk ? exp2f(sc - mnew) : 0.0f;
      float psum = p;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      float c = exp2f(m[g] - mnew);  // m = -inf first: exp2(-inf) = 0
      l[g] = l[g] * c + psum;
      m[g] = mnew;
      ps[g][lane] = p;
      if (lane == 0) corr[g] = c;
    }
    __syncthreads();
    // V tile -> shared
    for (int i = t; i < kTile * (kHead / 8); i += blockDim.x) {
      int key = i / (kHead / 8), c = i % (kHead / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (key < nk) v = *reinterpret_cast<const uint4*>(vbase + size_t(k0 + key) * row_stride + c * 8);
      *reinterpret_cast<uint4*>(&tile[key][c * 8]) = v;
    }
    __syncthreads();
    // accumulate: thread t owns dimension d = t for every head of the group
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float a = acc[g] * corr[g];
      for (int key = 0; key < nk; ++key) a += ps[g][key] * bf(tile[key][t]);
      acc[g] = a;
    }
    __syncthreads();
  }
  // m/l live in the warps that own each head; publish them through shared memory
  __shared__ float mls[G][2];
  for (int g = warp; g < G; g += 4)
    if (lane == 0) {
      mls[g][0] = m[g];
      mls[g][1] = l[g];
    }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    size_t row = (size_t(b) * Hq + h * G + g) * nsplit + s;
    part_o[row * kHead + t] = acc[g];
    if (t == 0) {
      part_ml[row * 2] = mls[g][0];
      part_ml[row * 2 + 1] = mls[g][1];
    }
  }
}

// grid B * Hq, block 128: merge the spans of one (sequence, head).
static __global__ void k_decode_combine(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                 __nv_bfloat16* __restrict__ out, int nsplit) {
  const size_t bh = blockIdx.x;
  const int t = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part_ml[(bh * nsplit + s) * 2]);
  float L = 0.0f, o = 0.0f;
  for (int s = 0; s < nsplit; ++s) {
    float ms = part_ml[(bh * nsplit + s) * 2], ls = part_ml[(bh * nsplit + s) * 2 + 1];
    if (ls == 0.0f) continue;
    float w = exp2f(ms - M);
    L += ls * w;
    o += part_o[(bh * nsplit + s) * kHead + t] * w;
  }
  out[bh * kHead + t] = __float2bfloat16_rn(L > 0.0f ? o / L : 0.0f);
}

}  // namespace attn
}  // namespace sn
