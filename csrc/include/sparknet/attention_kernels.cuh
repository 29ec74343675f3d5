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
  if (max_splits > 64) max_splits = 64;  // kMaxSplits
  return want < max_splits ? want : max_splits;
}

// Split counters (one int per (sequence, KV head)) sit at the front of the scratch in
// a region of fixed size, so a later call with other shapes finds them where it left
// them: zero.  The scratch must be zero there before its first use; every call that
// completes leaves them zero.
constexpr int kCounterSlots = 4096;

// The tensor-core kernel (attention_tc.cuh) splits a sequence into spans of T tiles of
// 128 keys, T = 1 or 2, at most kTcMaxSpans spans; 0 tiles = it does not take the problem.
constexpr int kTcKeys = 128;
constexpr int kTcMaxSpans = 64;
static inline int tc_tiles(int max_len) {
  if (max_len <= kTcMaxSpans * kTcKeys) return 1;
  if (max_len <= kTcMaxSpans * 2 * kTcKeys) return 2;
  return 0;
}
static inline int tc_splits(int max_len) {
  const int T = tc_tiles(max_len);
  return T ? (max_len + T * kTcKeys - 1) / (T * kTcKeys) : 0;
}

// Floats of scratch the kernels need: the counters, partial outputs [B, Hq, nsplit,
// 128] and (max, sum) pairs [B, Hq, nsplit, 2], for the larger split count of the two
// kernels (either may run: the tensor-core one where it is eligible).
static inline size_t scratch_floats(int B, int Hq, int Hkv, int max_len, int sms) {
  const int a = splits(B, Hkv, max_len, sms), b = tc_splits(max_len);
  return size_t(kCounterSlots) + size_t(B) * Hq * (a > b ? a : b) * (kHead + 2);
}

// ---------------------------------------------------------------------------
// Split-KV decode attention.  grid (B * Hkv, nsplit), block 256 threads.
// q: [B, Hq, 128] with Hq = G * Hkv; caches [B, Lmax, Hkv, 128]; lengths [B]; out
// [B, Hq, 128].  Each block streams its span of keys in tiles of 32 keys: the K and
// V rows of two tiles are in flight at once (cp.async, 16 bytes per copy, double
// buffered), so a block pays one memory latency up front instead of two per tile.
// With several spans, each block leaves its unnormalised output and (max, sum) in
// the scratch, and the last block of a (sequence, KV head) to finish (a counter)
// merges the spans in span order and writes `out`.  Scores are in log2 units.
// ---------------------------------------------------------------------------
constexpr int kRowPad = kHead + 8;  // +16 bytes: lane-per-key 16-byte reads spread over banks
constexpr int kMaxSplits = 64;      // spans per (sequence, KV head)
constexpr int kMergeBatch = 32;     // partial outputs loaded at once in the merge

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int src_bytes = valid ? 16 : 0;  // 0: fill the 16 bytes with zeros
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

constexpr int kAttnThreads = 256;  // 8 warps

template <int G>
static __global__ void __launch_bounds__(kAttnThreads) k_decode_attn(const __nv_bfloat16* __restrict__ q,
                                                                     const __nv_bfloat16* __restrict__ k_cache,
                                                                     const __nv_bfloat16* __restrict__ v_cache,
                                                                     const int* __restrict__ lengths,
                                                                     __nv_bfloat16* __restrict__ out, int* counters,
                                                                     float* part_o, float* part_ml, int Hkv, int Lmax,
                                                                     int chunk, float scale_log2) {
  // Roles.  Scores: warp w owns heads w, w + 8 (G = 16); lane = key of the tile.  P V:
  // thread t owns dimensions 2*(t % 64), +1 of heads t / 64, t / 64 + 4, ...
  constexpr int kHW = (G + 7) / 8;     // heads per warp in the score phase
  constexpr int kHT = (G + 3) / 4;     // heads per thread in the P V phase
  __shared__ __align__(16) float qs[G][kHead];
  __shared__ __align__(16) __nv_bfloat16 kt[2][kTile][kRowPad];
  __shared__ __align__(16) __nv_bfloat16 vt[2][kTile][kRowPad];
  __shared__ __align__(16) float ps[G][kTile];
  __shared__ float corr[G];
  __shared__ float mls[G][2];
  __shared__ int last;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // a PDL-launched successor may start early
  const int b = blockIdx.x / Hkv, h = blockIdx.x % Hkv, s = blockIdx.y, nsplit = gridDim.y;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int dp = t & 63, hg = t >> 6;
  const int Hq = G * Hkv;
  // The splits cover nsplit * chunk >= max_len keys (the host sizes chunk from max_len):
  // a sequence longer than that is attended over its first nsplit * chunk keys only.
  const int len = min(min(lengths[b], Lmax), nsplit * chunk);
  const int start = s * chunk, end = min(start + chunk, len);
  const int ntiles = end > start ? (end - start + kTile - 1) / kTile : 0;
  const size_t row_stride = size_t(Hkv) * kHead;
  const __nv_bfloat16* kbase = k_cache + (size_t(b) * Lmax * Hkv + h) * kHead;
  const __nv_bfloat16* vbase = v_cache + (size_t(b) * Lmax * Hkv + h) * kHead;

  // one tile = 32 keys x 256 bytes of K and of V = 1024 copies of 16 bytes, 4 per thread
  auto issue = [&](int tile_idx) {
    if (tile_idx < ntiles) {
      const int k0 = start + tile_idx * kTile, buf = tile_idx & 1;
#pragma unroll
      for (int r = 0; r < (kTile * kHead / 8) / kAttnThreads; ++r) {
        const int i = r * kAttnThreads + t, key = i / (kHead / 8), c = i % (kHead / 8);
        const bool valid = k0 + key < end;
        const size_t off = size_t(valid ? k0 + key : start) * row_stride + c * 8;
        cp_async16(&kt[buf][key][c * 8], kbase + off, valid);
        cp_async16(&vt[buf][key][c * 8], vbase + off, valid);
      }
    }
    cp_async_commit();  // possibly empty: keeps the group count uniform
  };
  // Programmatic dependent launch: K/V tiles wholly below the newest key (lengths[b] - 1,
  // the one the preceding RoPE kernel writes) are requested before griddepcontrol.wait;
  // q and everything else after it.  Without PDL the wait returns at once.
  auto safe = [&](int tile_idx) { return tile_idx < ntiles && start + (tile_idx + 1) * kTile <= len - 1; };
  const bool pre0 = safe(0), pre1 = pre0 && safe(1);
  if (pre0) issue(0);
  if (pre1) issue(1);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (!pre0) issue(0);
  if (!pre1) issue(1);
  for (int i = t; i < G * kHead; i += kAttnThreads) {
    const int g = i / kHead, d = i % kHead;
    qs[g][d] = bf(q[(size_t(b) * Hq + h * G + g) * kHead + d]) * scale_log2;
  }
  float m[kHW], l[kHW];
#pragma unroll
  for (int j = 0; j < kHW; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.0f;
  }
  float2 acc[kHT];
#pragma unroll
  for (int i = 0; i < kHT; ++i) acc[i] = make_float2(0.0f, 0.0f);

  for (int it = 0; it < ntiles; ++it) {
    const int buf = it & 1;
    const int nk = min(kTile, end - (start + it * kTile));
    cp_async_wait1();
    __syncthreads();
    // scores + online softmax, one K row per lane, loaded once for the warp's heads
    if (warp < G) {
      float dot[kHW];
#pragma unroll
      for (int j = 0; j < kHW; ++j) dot[j] = 0.0f;
#pragma unroll
      for (int c = 0; c < kHead / 8; ++c) {
        const uint4 kv = *reinterpret_cast<const uint4*>(&kt[buf][lane][c * 8]);
        const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kv);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(k2[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int j = 0; j < kHW; ++j) {
          const int g = warp + 8 * j;
          if (g < G) {
            const float4 qa = *reinterpret_cast<const float4*>(&qs[g][c * 8]);
            const float4 qb = *reinterpret_cast<const float4*>(&qs[g][c * 8 + 4]);
            dot[j] += qa.x * kf[0] + qa.y * kf[1] + qa.z * kf[2] + qa.w * kf[3] + qb.x * kf[4] + qb.y * kf[5] +
                      qb.z * kf[6] + qb.w * kf[7];
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kHW; ++j) {
        const int g = warp + 8 * j;
        if (g < G) {
          const float sc = lane < nk ? dot[j] : -INFINITY;
          float tmax = sc;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
          const float mnew = fmaxf(m[j], tmax);
          const float pr = lane < nk ? exp2f(sc - mnew) : 0.0f;
          float psum = pr;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
          const float cf = exp2f(m[j] - mnew);  // m = -inf first: exp2(-inf) = 0
          l[j] = l[j] * cf + psum;
          m[j] = mnew;
          ps[g][lane] = pr;
          if (lane == 0) corr[g] = cf;
        }
      }
    }
    __syncthreads();
    // P V: a V pair loaded once, used for every head of the thread
#pragma unroll
    for (int i = 0; i < kHT; ++i) {
      const int g = hg + 4 * i;
      if (g < G) {
        const float cf = corr[g];
        acc[i].x *= cf;
        acc[i].y *= cf;
      }
    }
    for (int key = 0; key < nk; ++key) {
      const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vt[buf][key][2 * dp]));
#pragma unroll
      for (int i = 0; i < kHT; ++i) {
        const int g = hg + 4 * i;
        if (g < G) {
          const float pr = ps[g][key];
          acc[i].x = fmaf(pr, v.x, acc[i].x);
          acc[i].y = fmaf(pr, v.y, acc[i].y);
        }
      }
    }
    __syncthreads();  // buffer `buf` and ps are free again
    issue(it + 2);
  }
  if (warp < G && lane == 0) {
#pragma unroll
    for (int j = 0; j < kHW; ++j) {
      const int g = warp + 8 * j;
      if (g < G) {
        mls[g][0] = m[j];
        mls[g][1] = l[j];
      }
    }
  }
  __syncthreads();
  const size_t head0 = size_t(b) * Hq + h * G;
  if (nsplit == 1) {
#pragma unroll
    for (int i = 0; i < kHT; ++i) {
      const int g = hg + 4 * i;
      if (g < G) {
        const float L = mls[g][1], inv = L > 0.0f ? 1.0f / L : 0.0f;
        *reinterpret_cast<__nv_bfloat162*>(out + (head0 + g) * kHead + 2 * dp) =
            __floats2bfloat162_rn(acc[i].x * inv, acc[i].y * inv);
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < kHT; ++i) {
    const int g = hg + 4 * i;
    if (g < G) {
      const size_t row = (head0 + g) * nsplit + s;
      __stcg(reinterpret_cast<float2*>(part_o + row * kHead + 2 * dp), acc[i]);
      if (dp == 0) {
        __stcg(part_ml + row * 2, mls[g][0]);
        __stcg(part_ml + row * 2 + 1, mls[g][1]);
      }
    }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) last = atomicAdd(&counters[blockIdx.x], 1) == nsplit - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // Merge the spans of each head in span order.  Every load is issued before any sum
  // depends on it: (max, sum) pairs first, then the weights in shared memory, then the
  // partial outputs in batches of kMergeBatch spans.
  asm volatile("cp.async.wait_all;" ::: "memory");
  float(*wts)[kMaxSplits] = reinterpret_cast<float(*)[kMaxSplits]>(&kt[0][0][0]);  // K tiles are free now
  float(*sums)[kMaxSplits] = reinterpret_cast<float(*)[kMaxSplits]>(&vt[0][0][0]);  // V tiles too
  static_assert(sizeof(float) * G * kMaxSplits <= sizeof(kt), "merge weights must fit the K tile buffers");
  __shared__ float lsum[G];
  for (int i = t; i < G * nsplit; i += kAttnThreads) {  // every (max, sum) pair in one parallel pass
    const int g = i / nsplit, sp = i % nsplit;
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(part_ml + ((head0 + g) * nsplit + sp) * 2));
    wts[g][sp] = ml.x;  // max (log2 units)
    sums[g][sp] = ml.y;
  }
  __syncthreads();
  if (t < G) {
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, wts[t][sp]);
    float L = 0.0f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float ls = sums[t][sp];
      const float w = ls > 0.0f ? exp2f(wts[t][sp] - M) : 0.0f;
      wts[t][sp] = w;
      L += ls * w;
    }
    lsum[t] = L;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kHT; ++i) {
    const int g = hg + 4 * i;
    if (g >= G) continue;
    const float* po = part_o + (head0 + g) * nsplit * kHead + 2 * dp;
    float2 o = make_float2(0.0f, 0.0f);
    for (int sp0 = 0; sp0 < nsplit; sp0 += kMergeBatch) {
      float2 v[kMergeBatch];
#pragma unroll
      for (int j = 0; j < kMergeBatch; ++j)
        v[j] = sp0 + j < nsplit ? __ldcg(reinterpret_cast<const float2*>(po + (sp0 + j) * kHead)) : make_float2(0, 0);
#pragma unroll
      for (int j = 0; j < kMergeBatch; ++j)
        if (sp0 + j < nsplit) {
          o.x += v[j].x * wts[g][sp0 + j];
          o.y += v[j].y * wts[g][sp0 + j];
        }
    }
    const float L = lsum[g], inv = L > 0.0f ? 1.0f / L : 0.0f;
    *reinterpret_cast<__nv_bfloat162*>(out + (head0 + g) * kHead + 2 * dp) = __floats2bfloat162_rn(o.x * inv, o.y * inv);
  }
  if (t == 0) counters[blockIdx.x] = 0;
}

// Launch over a scratch laid out as [kCounterSlots ints][part_o][part_ml].  Returns the
// launch's error (or cudaErrorInvalidValue for an unsupported group size or too many
// (sequence, KV head) pairs).
static inline cudaError_t launch_decode_attention_simt(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                                                  const __nv_bfloat16* v_cache, const int* lengths,
                                                  __nv_bfloat16* out, float* scratch, int B, int Hq, int Hkv,
                                                  int Lmax, int max_len, float scale, int sms, cudaStream_t st,
                                                  bool pdl = false) {
  if (Hkv <= 0 || Hq % Hkv || B * Hkv > kCounterSlots) return cudaErrorInvalidValue;
  const int G = Hq / Hkv;
  const int nsplit = splits(B, Hkv, max_len, sms);
  const int chunk = ((max_len + nsplit - 1) / nsplit + kTile - 1) / kTile * kTile;
  int* counters = reinterpret_cast<int*>(scratch);
  float* part_o = scratch + kCounterSlots;
  float* part_ml = part_o + size_t(B) * Hq * nsplit * kHead;
  const float scale_log2 = scale * kLog2e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B * Hkv, nsplit, 1);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  switch (G) {
#define SN_ATT(GG)                                                                                       \
  case GG:                                                                                               \
    return cudaLaunchKernelEx(&cfg, k_decode_attn<GG>, q, k_cache, v_cache, lengths, out, counters, part_o, \
                              part_ml, Hkv, Lmax, chunk, scale_log2);
    SN_ATT(1)
    SN_ATT(2)
    SN_ATT(4)
    SN_ATT(8)
    SN_ATT(16)
#undef SN_ATT
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace attn
}  // namespace sn
