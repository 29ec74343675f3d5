// Split-KV flash-decoding kernels for grouped-query attention (sm_100a), shared by
// the torch entry point (decode_ops.cu) and the allocation-free C entry point
// (attention_noalloc.cu).  One query token per sequence; head_dim 128.
#pragma once

#include <cooperative_groups.h>
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

// ---------------------------------------------------------------------------
// Cluster split-KV decode attention.  grid (S, B * Hkv), cluster (S, 1, 1), block 256,
// S = 8 or 16.  The S spans of one (sequence, KV head) are the S CTAs of one
// thread-block cluster.  Each CTA keeps NT tiles of K and V in flight (a ring of NT
// buffers in dynamic shared memory, so a span of up to NT * 32 keys costs one memory
// latency), parks its unnormalised output and (max, sum) in its own shared memory, and
// after a cluster barrier the cluster merges the S spans through distributed shared
// memory in span order.  Compared with k_decode_attn there is no workspace, no
// counter, no global round trip between the spans and the merge.  Scores are in log2
// units; the score and P V phases are those of k_decode_attn.
// ---------------------------------------------------------------------------
constexpr int kClusterNT = 4;  // tiles in flight per CTA

template <int G, int NT>
struct ClusterSmem {  // every array 16-byte aligned (vector accesses), whatever G is
  alignas(16) float qs[G][kHead];
  alignas(16) __nv_bfloat16 kt[NT][kTile][kRowPad];
  alignas(16) __nv_bfloat16 vt[NT][kTile][kRowPad];
  alignas(16) float ps[G][kTile];
  alignas(16) float corr[G];
  alignas(16) float po[G][kHead];  // this span's unnormalised output, read by the cluster's merge
  alignas(16) float pml[G][2];     // this span's (max, sum)
};

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int G, int S, int NT>
static __global__ void __launch_bounds__(kAttnThreads) k_decode_attn_cluster(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_cache,
    const __nv_bfloat16* __restrict__ v_cache, const int* __restrict__ lengths, __nv_bfloat16* __restrict__ out,
    int Hkv, int Lmax, int chunk, float scale_log2) {
  namespace cg = cooperative_groups;
  constexpr int kHW = (G + 7) / 8;  // heads per warp in the score phase
  constexpr int kHT = (G + 3) / 4;  // heads per thread in the P V phase
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ClusterSmem<G, NT>& sm = *reinterpret_cast<ClusterSmem<G, NT>*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // a PDL-launched successor may start early
  // The merge reads S CTAs' shared memory: a launch that arrives without its S-CTA
  // cluster (re-issued by a tool without the attribute) must not touch it.  Every CTA
  // returns before any access; the output rows keep their previous contents.
  if (cluster.num_blocks() != unsigned(S)) return;
  const int s = blockIdx.x, b = blockIdx.y / Hkv, h = blockIdx.y % Hkv;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int dp = t & 63, hg = t >> 6;
  const int Hq = G * Hkv;
  const int len = min(lengths[b], Lmax);
  const int start = s * chunk, end = min(start + chunk, len);
  const int ntiles = end > start ? (end - start + kTile - 1) / kTile : 0;
  const size_t row_stride = size_t(Hkv) * kHead;
  const __nv_bfloat16* kbase = k_cache + (size_t(b) * Lmax * Hkv + h) * kHead;
  const __nv_bfloat16* vbase = v_cache + (size_t(b) * Lmax * Hkv + h) * kHead;

  // one tile = 32 keys x 256 bytes of K and of V, 4 copies of 16 bytes per thread each;
  // one commit group per tile (possibly empty), so NT groups are always outstanding
  auto issue = [&](int tile_idx) {
    if (tile_idx < ntiles) {
      const int k0 = start + tile_idx * kTile, buf = tile_idx % NT;
#pragma unroll
      for (int r = 0; r < (kTile * kHead / 8) / kAttnThreads; ++r) {
        const int i = r * kAttnThreads + t, key = i / (kHead / 8), c = i % (kHead / 8);
        const bool valid = k0 + key < end;
        const size_t off = size_t(valid ? k0 + key : start) * row_stride + c * 8;
        cp_async16(&sm.kt[buf][key][c * 8], kbase + off, valid);
        cp_async16(&sm.vt[buf][key][c * 8], vbase + off, valid);
      }
    }
    cp_async_commit();
  };
  // Programmatic dependent launch: the leading tiles wholly below the newest key (the
  // one the preceding kernel writes) are requested before griddepcontrol.wait.
  int pre = 0;
  while (pre < NT && pre < ntiles && start + (pre + 1) * kTile <= len - 1) issue(pre++);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int i = pre; i < NT; ++i) issue(i);
  for (int i = t; i < G * kHead; i += kAttnThreads) {
    const int g = i / kHead, d = i % kHead;
    sm.qs[g][d] = bf(q[(size_t(b) * Hq + h * G + g) * kHead + d]) * scale_log2;
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
    const int buf = it % NT;
    const int nk = min(kTile, end - (start + it * kTile));
    cp_async_wait<NT - 1>();  // tile `it` has landed (groups complete in order)
    __syncthreads();
    if (warp < G) {
      float dot[kHW];
#pragma unroll
      for (int j = 0; j < kHW; ++j) dot[j] = 0.0f;
#pragma unroll
      for (int c = 0; c < kHead / 8; ++c) {
        const uint4 kv = *reinterpret_cast<const uint4*>(&sm.kt[buf][lane][c * 8]);
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
            const float4 qa = *reinterpret_cast<const float4*>(&sm.qs[g][c * 8]);
            const float4 qb = *reinterpret_cast<const float4*>(&sm.qs[g][c * 8 + 4]);
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
          const float cf = exp2f(m[j] - mnew);
          l[j] = l[j] * cf + psum;
          m[j] = mnew;
          sm.ps[g][lane] = pr;
          if (lane == 0) sm.corr[g] = cf;
        }
      }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kHT; ++i) {
      const int g = hg + 4 * i;
      if (g < G) {
        const float cf = sm.corr[g];
        acc[i].x *= cf;
        acc[i].y *= cf;
      }
    }
    for (int key = 0; key < nk; ++key) {
      const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.vt[buf][key][2 * dp]));
#pragma unroll
      for (int i = 0; i < kHT; ++i) {
        const int g = hg + 4 * i;
        if (g < G) {
          const float pr = sm.ps[g][key];
          acc[i].x = fmaf(pr, v.x, acc[i].x);
          acc[i].y = fmaf(pr, v.y, acc[i].y);
        }
      }
    }
    __syncthreads();  // buffer `buf`, ps and corr are free again
    issue(it + NT);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");

  // park this span's partial, then merge the cluster's spans in span order
  if (warp < G && lane == 0) {
#pragma unroll
    for (int j = 0; j < kHW; ++j) {
      const int g = warp + 8 * j;
      if (g < G) {
        sm.pml[g][0] = m[j];
        sm.pml[g][1] = l[j];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kHT; ++i) {
    const int g = hg + 4 * i;
    if (g < G) *reinterpret_cast<float2*>(&sm.po[g][2 * dp]) = acc[i];
  }
  cluster.sync();  // every span's partial is parked and visible to the cluster
  const size_t head0 = size_t(b) * Hq + h * G;
  for (int idx = s * kAttnThreads + t; idx < G * (kHead / 2); idx += S * kAttnThreads) {
    const int g = idx / (kHead / 2), d2 = idx % (kHead / 2);
    float mx[S], ls[S];
    float2 ov[S];
#pragma unroll
    for (int r = 0; r < S; ++r) {  // every remote load issued before any is used
      const ClusterSmem<G, NT>* peer = cluster.map_shared_rank(&sm, r);
      mx[r] = peer->pml[g][0];
      ls[r] = peer->pml[g][1];
      ov[r] = *reinterpret_cast<const float2*>(&peer->po[g][2 * d2]);
    }
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < S; ++r) M = fmaxf(M, mx[r]);
    float L = 0.0f;
    float2 o = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int r = 0; r < S; ++r) {
      const float w = ls[r] > 0.0f ? exp2f(mx[r] - M) : 0.0f;
      L += ls[r] * w;
      o.x += ov[r].x * w;
      o.y += ov[r].y * w;
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    *reinterpret_cast<__nv_bfloat162*>(out + (head0 + g) * kHead + 2 * d2) = __floats2bfloat162_rn(o.x * inv, o.y * inv);
  }
  cluster.sync();  // partials stay readable until every CTA of the cluster is done
}

// Cluster size for B * Hkv clusters: 16 spans while that keeps the grid within two
// waves of the SMs, else 8.
static inline int cluster_spans(int B, int Hkv, int sms) { return B * Hkv * 16 <= 2 * sms ? 16 : 8; }

// Whether clusters of 16 CTAs of this kernel can be scheduled at all on the current
// device (the answer depends on the GPU's partitioning): asked once per device.
template <int G>
static inline bool cluster16_fits() {
  static int answer[64] = {0};  // 0 unknown, 1 fits, 2 does not
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (dev >= 0 && dev < 64 && answer[dev]) return answer[dev] == 1;
  auto kernel = k_decode_attn_cluster<G, 16, kClusterNT>;
  const int smem = int(sizeof(ClusterSmem<G, kClusterNT>));
  bool fits = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess &&
              cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
  if (fits) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(16, 1, 1);
    cfg.blockDim = dim3(kAttnThreads, 1, 1);
    cfg.dynamicSmemBytes = size_t(smem);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 16;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    fits = cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) == cudaSuccess && clusters > 0;
  }
  (void)cudaGetLastError();  // clear the error a refused query may leave behind
  if (dev >= 0 && dev < 64) answer[dev] = fits ? 1 : 2;
  return fits;
}

template <int G, int S>
static inline cudaError_t launch_cluster_g(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                                           const __nv_bfloat16* v_cache, const int* lengths, __nv_bfloat16* out,
                                           int B, int Hkv, int Lmax, int chunk, float scale_log2, cudaStream_t st,
                                           bool pdl) {
  auto kernel = k_decode_attn_cluster<G, S, kClusterNT>;
  const int smem = int(sizeof(ClusterSmem<G, kClusterNT>));
  // function attributes belong to each device's context: set once per device (the
  // first call, which is an eager one before any graph capture)
  static int attr_done[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess && S > 8) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_done[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S, B * Hkv, 1);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = S;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, q, k_cache, v_cache, lengths, out, Hkv, Lmax, chunk, scale_log2);
}

// The cluster variant: no workspace.  Returns the launch's error (cudaErrorInvalidValue
// for an unsupported group size).
static inline cudaError_t launch_decode_attention_cluster(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                                                          const __nv_bfloat16* v_cache, const int* lengths,
                                                          __nv_bfloat16* out, int B, int Hq, int Hkv, int Lmax,
                                                          int max_len, float scale, int sms, cudaStream_t st,
                                                          bool pdl = false) {
  if (Hkv <= 0 || Hq % Hkv || B <= 0 || max_len <= 0 || B * Hkv > 65535) return cudaErrorInvalidValue;
  const int G = Hq / Hkv;
  int S = cluster_spans(B, Hkv, sms);
  if (S == 16) {
    bool fits = false;
    switch (G) {
      case 1: fits = cluster16_fits<1>(); break;
      case 2: fits = cluster16_fits<2>(); break;
      case 4: fits = cluster16_fits<4>(); break;
      case 8: fits = cluster16_fits<8>(); break;
      case 16: fits = cluster16_fits<16>(); break;
      default: return cudaErrorInvalidValue;
    }
    if (!fits) S = 8;  // portable cluster size
  }
  const int chunk = ((max_len + S - 1) / S + kTile - 1) / kTile * kTile;
  const float scale_log2 = scale * kLog2e;
#define SN_ATC(GG)                                                                                              \
  case GG:                                                                                                      \
    return S == 16 ? launch_cluster_g<GG, 16>(q, k_cache, v_cache, lengths, out, B, Hkv, Lmax, chunk, scale_log2, \
                                              st, pdl)                                                          \
                   : launch_cluster_g<GG, 8>(q, k_cache, v_cache, lengths, out, B, Hkv, Lmax, chunk, scale_log2,  \
                                             st, pdl);
  switch (G) {
    SN_ATC(1)
    SN_ATC(2)
    SN_ATC(4)
    SN_ATC(8)
    SN_ATC(16)
    default:
      return cudaErrorInvalidValue;
  }
#undef SN_ATC
}

}  // namespace attn
}  // namespace sn
