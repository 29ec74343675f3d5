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

// Floats of scratch the kernels need: the counters, partial outputs [B, Hq, nsplit,
// 128] and (max, sum) pairs [B, Hq, nsplit, 2].
static inline size_t scratch_floats(int B, int Hq, int Hkv, int max_len, int sms) {
  return size_t(kCounterSlots) + size_t(B) * Hq * splits(B, Hkv, max_len, sms) * (kHead + 2);
}

// ---------------------------------------------------------------------------
// Split-KV decode attention.  grid (B * Hkv, nsplit), block 128 threads.
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
constexpr int kMergeBatch = 8;      // partial outputs loaded at once in the merge

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int src_bytes = valid ? 16 : 0;  // 0: fill the 16 bytes with zeros
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

template <int G>
static __global__ void __launch_bounds__(128) k_decode_attn(const __nv_bfloat16* __restrict__ q,
                                                            const __nv_bfloat16* __restrict__ k_cache,
                                                            const __nv_bfloat16* __restrict__ v_cache,
                                                            const int* __restrict__ lengths,
                                                            __nv_bfloat16* __restrict__ out, int* counters,
                                                            float* part_o, float* part_ml, int Hkv, int Lmax,
                                                            int chunk, float scale_log2) {
  __shared__ float qs[G][kHead];
  __shared__ __align__(16) __nv_bfloat16 kt[2][kTile][kRowPad];
  __shared__ __align__(16) __nv_bfloat16 vt[2][kTile][kRowPad];
  __shared__ float ps[G][kTile];
  __shared__ float corr[G];
  __shared__ float mls[G][2];
  __shared__ int last;
  const int b = blockIdx.x / Hkv, h = blockIdx.x % Hkv, s = blockIdx.y, nsplit = gridDim.y;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int Hq = G * Hkv;
  const int len = min(lengths[b], Lmax);
  const int start = s * chunk, end = min(start + chunk, len);
  const int ntiles = end > start ? (end - start + kTile - 1) / kTile : 0;
  const size_t row_stride = size_t(Hkv) * kHead;
  const __nv_bfloat16* kbase = k_cache + (size_t(b) * Lmax * Hkv + h) * kHead;
  const __nv_bfloat16* vbase = v_cache + (size_t(b) * Lmax * Hkv + h) * kHead;

  // one tile = 32 keys x 256 bytes of K and of V = 1024 copies of 16 bytes, 8 per thread
  auto issue = [&](int tile_idx) {
    if (tile_idx < ntiles) {
      const int k0 = start + tile_idx * kTile, buf = tile_idx & 1;
#pragma unroll
      for (int r = 0; r < (kTile * kHead / 8) / 128; ++r) {
        const int i = r * 128 + t, key = i / (kHead / 8), c = i % (kHead / 8);
        const bool valid = k0 + key < end;
        const size_t off = size_t(valid ? k0 + key : start) * row_stride + c * 8;
        cp_async16(&kt[buf][key][c * 8], kbase + off, valid);
        cp_async16(&vt[buf][key][c * 8], vbase + off, valid);
      }
    }
    cp_async_commit();  // possibly empty: keeps the group count uniform
  };
  issue(0);
  issue(1);
  for (int i = t; i < G * kHead; i += blockDim.x) {
    int g = i / kHead, d = i % kHead;
    qs[g][d] = bf(q[(size_t(b) * Hq + h * G + g) * kHead + d]) * scale_log2;
  }
  // per-head running max / sum live in the warp that owns the head (g = warp + 4j)
  float m[(G + 3) / 4], l[(G + 3) / 4];
#pragma unroll
  for (int j = 0; j < (G + 3) / 4; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.0f;
  }
  float acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = 0.0f;

  for (int it = 0; it < ntiles; ++it) {
    const int buf = it & 1;
    const int nk = min(kTile, end - (start + it * kTile));
    cp_async_wait1();
    __syncthreads();
    // scores and online softmax: warp w owns heads w, w + 4, ...; lane = key
#pragma unroll
    for (int j = 0; j < (G + 3) / 4; ++j) {
      const int g = warp + 4 * j;
      if (g < G) {
        float sc = -INFINITY;
        if (lane < nk) {
          float dot = 0.0f;
#pragma unroll
          for (int c = 0; c < kHead / 8; ++c) {
            uint4 kv = *reinterpret_cast<const uint4*>(&kt[buf][lane][c * 8]);
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
        const float mnew = fmaxf(m[j], tmax);
        const float p = lane < nk ? exp2f(sc - mnew) : 0.0f;
        float psum = p;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
        const float cf = exp2f(m[j] - mnew);  // m = -inf first: exp2(-inf) = 0
        l[j] = l[j] * cf + psum;
        m[j] = mnew;
        ps[g][lane] = p;
        if (lane == 0) corr[g] = cf;
      }
    }
    __syncthreads();
    // P V: thread t owns dimension t of every head of the group
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float a = acc[g] * corr[g];
      for (int key = 0; key < nk; ++key) a += ps[g][key] * bf(vt[buf][key][t]);
      acc[g] = a;
    }
    __syncthreads();  // buffer `buf` is free again
    issue(it + 2);
  }
#pragma unroll
  for (int j = 0; j < (G + 3) / 4; ++j) {
    const int g = warp + 4 * j;
    if (g < G && lane == 0) {
      mls[g][0] = m[j];
      mls[g][1] = l[j];
    }
  }
  __syncthreads();
  const size_t head0 = size_t(b) * Hq + h * G;
  if (nsplit == 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float L = mls[g][1];
      out[(head0 + g) * kHead + t] = __float2bfloat16_rn(L > 0.0f ? acc[g] / L : 0.0f);
    }
    return;
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const size_t row = (head0 + g) * nsplit + s;
    __stcg(part_o + row * kHead + t, acc[g]);
    if (t == 0) {
      __stcg(part_ml + row * 2, mls[g][0]);
      __stcg(part_ml + row * 2 + 1, mls[g][1]);
    }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) last = atomicAdd(&counters[blockIdx.x], 1) == nsplit - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // Merge the spans of each head in span order.  Every load is issued before any sum
  // depends on it: (max, sum) pairs first (one per thread), then the weights in shared
  // memory, then the partial outputs in batches of kMergeBatch spans.
  asm volatile("cp.async.wait_all;" ::: "memory");
  float(*wts)[kMaxSplits] = reinterpret_cast<float(*)[kMaxSplits]>(&kt[0][0][0]);  // K tiles are free now
  static_assert(sizeof(float) * G * kMaxSplits <= sizeof(kt), "merge weights must fit the K tile buffers");
  __shared__ float lsum[G];
  for (int i = t; i < G * nsplit; i += blockDim.x) {
    const int g = i / nsplit, sp = i % nsplit;
    wts[g][sp] = __ldcg(part_ml + ((head0 + g) * nsplit + sp) * 2);      // max (log2 units)
  }
  __syncthreads();
  if (t < G) {
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, wts[t][sp]);
    float L = 0.0f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float ls = __ldcg(part_ml + ((head0 + t) * nsplit + sp) * 2 + 1);
      const float w = ls > 0.0f ? exp2f(wts[t][sp] - M) : 0.0f;
      wts[t][sp] = w;
      L += ls * w;
    }
    lsum[t] = L;
  }
  __syncthreads();
#pragma unroll 1
  for (int g = 0; g < G; ++g) {
    const float* po = part_o + (head0 + g) * nsplit * kHead + t;
    float o = 0.0f;
    for (int sp0 = 0; sp0 < nsplit; sp0 += kMergeBatch) {
      float v[kMergeBatch];
#pragma unroll
      for (int j = 0; j < kMergeBatch; ++j) v[j] = sp0 + j < nsplit ? __ldcg(po + (sp0 + j) * kHead) : 0.0f;
#pragma unroll
      for (int j = 0; j < kMergeBatch; ++j)
        if (sp0 + j < nsplit) o += v[j] * wts[g][sp0 + j];
    }
    const float L = lsum[g];
    out[(head0 + g) * kHead + t] = __float2bfloat16_rn(L > 0.0f ? o / L : 0.0f);
  }
  if (t == 0) counters[blockIdx.x] = 0;
}

// Launch over a scratch laid out as [kCounterSlots ints][part_o][part_ml].  Returns the
// launch's error (or cudaErrorInvalidValue for an unsupported group size or too many
// (sequence, KV head) pairs).
static inline cudaError_t launch_decode_attention(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                                                  const __nv_bfloat16* v_cache, const int* lengths,
                                                  __nv_bfloat16* out, float* scratch, int B, int Hq, int Hkv,
                                                  int Lmax, int max_len, float scale, int sms, cudaStream_t st) {
  if (Hkv <= 0 || Hq % Hkv || B * Hkv > kCounterSlots) return cudaErrorInvalidValue;
  const int G = Hq / Hkv;
  const int nsplit = splits(B, Hkv, max_len, sms);
  const int chunk = ((max_len + nsplit - 1) / nsplit + kTile - 1) / kTile * kTile;
  int* counters = reinterpret_cast<int*>(scratch);
  float* part_o = scratch + kCounterSlots;
  float* part_ml = part_o + size_t(B) * Hq * nsplit * kHead;
  const float scale_log2 = scale * kLog2e;
  const dim3 grid(B * Hkv, nsplit);
  switch (G) {
#define SN_ATT(GG)                                                                                              \
  case GG:                                                                                                      \
    k_decode_attn<GG><<<grid, 128, 0, st>>>(q, k_cache, v_cache, lengths, out, counters, part_o, part_ml, Hkv,   \
                                            Lmax, chunk, scale_log2);                                           \
    break;
    SN_ATT(1)
    SN_ATT(2)
    SN_ATT(4)
    SN_ATT(8)
    SN_ATT(16)
#undef SN_ATT
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace attn
}  // namespace sn
