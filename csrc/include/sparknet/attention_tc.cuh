// Decode attention on the 5th-generation tensor cores (sm_100a): one query token per
// sequence, grouped-query heads, head_dim 128, bf16 in, fp32 softmax and accumulation.
//
// One CTA per (sequence, KV head, span of up to T x 128 keys), 128 threads (the four
// TMEM lane quadrants).  Per 128-key tile:
//
//   S^T[key, head] = K_tile[key, :] . Q[head, :]          tcgen05.mma, M = 128 keys,
//                                                          N = 16 heads (padded), K = 128
//   softmax over the span's keys, per head, in fp32        thread i owns key i (TMEM lane i)
//   O^T[dim, head] += V_tile^T[dim, key] . P^T[key, head]  tcgen05.mma, M = 128 dims,
//                                                          N = 16 heads, K = 128 keys
//
// K and V tiles arrive by TMA (a 3-D map over the [B, Lmax, Hkv, 128] cache, one KV head,
// 128 keys, 128-byte swizzle); V is read by the second MMA straight from the TMA image as
// an MN-major operand, so nothing is transposed.  Q is tiny and comes in by plain loads.
// Scores and the output accumulator live in TMEM.  All scores of the span are held in
// TMEM before the softmax, so the span's maximum is known before P is formed and the
// accumulator is never rescaled.  A sequence split over several spans leaves its
// unnormalised output and (max, sum) per head in a workspace; the last CTA of the
// (sequence, KV head) merges the spans in span order, as the CUDA-core kernel of
// attention_kernels.cuh does (whose workspace layout this shares).
//
// Waits on mbarriers are bounded: a wait that runs out sets the workspace's error word,
// the CTA waits (bounded) for its own copies in flight, frees its TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cooperative_groups.h>

#include "sparknet/attention_kernels.cuh"
#include "sparknet/tc_gemm.cuh"

namespace sn {
namespace attn {

namespace cg = cooperative_groups;

// kTcKeys (keys per tile = MMA M of the score product), kTcMaxSpans, tc_tiles() and
// tc_splits() are in attention_kernels.cuh, beside the workspace size they decide.
constexpr int kTcHeads = 16;                  // MMA N: query heads of one KV head, zero-padded
constexpr int kTcThreads = 128;               // warps 0-3 <-> TMEM lanes 0-127
constexpr uint32_t kTcTmemCols = 64;          // scores: 16 per tile (<= 2 tiles), output: 16
constexpr uint32_t kTcOutCol = 32;
constexpr int kHalfBytes = kTcKeys * 128;     // one 64-dim half of a K or V tile: 128 rows x 128 B
constexpr int kTileBytes = 2 * kHalfBytes;    // 32 KB
constexpr int kQHalfBytes = kTcHeads * 128;   // 16 rows x 128 B
constexpr int kPAtomBytes = kTcHeads * 128;   // 16 heads x 64 keys of P (bf16)
constexpr int kErrorSlot = kCounterSlots - 1; // workspace int: nonzero after a wait ran out
constexpr int kTcStamps = 12;                 // phase stamps per CTA (profiling)
constexpr int kClusterMaxSpans = 8;           // spans merged in a (portable) cluster

template <int T>
struct TcLayout {  // byte offsets from the 1024-aligned base of dynamic shared memory
  static constexpr int k = 0;                                  // K[t][half]
  static constexpr int v = k + T * kTileBytes;                 // V[t][half]
  static constexpr int q = v + T * kTileBytes;                 // Q[half]
  static constexpr int p = q + 2 * kQHalfBytes;                // P[t][atom]
  static constexpr int red = p + T * 2 * kPAtomBytes;          // [2][4][16] floats: per-warp max, sum
  static constexpr int stat = red + 2 * 4 * kTcHeads * 4;      // [16][2] floats: span max, sum
  static constexpr int bars = stat + kTcHeads * 2 * 4;         // mbarriers: k_full[T], v_full[T], s_done, o_done, m_full
  static constexpr int misc = bars + (2 * T + 3) * 8;          // tmem slot, error flag, last flag
  static constexpr int end = misc + 16;
  static constexpr int bytes = end + 1024;                     // + alignment slack
};

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(tc::smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(tc::smem_u32(bar))
      : "memory");
}

// Shared-memory descriptor of an MN-major operand in 128-byte-swizzle atoms: 64
// contiguous elements along M (128 B) by 8 rows along K (128 B apart) per 1024-byte
// atom; `lbo` = bytes from one 64-element M block to the next, `sbo` = bytes from one
// 8-row K group to the next.
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(const void* tile, uint32_t lbo, uint32_t sbo) {
  const uint64_t addr = tc::smem_u32(tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version (sm100)
  d |= 2ull << 61;  // 128-byte swizzle
  return d;
}

// bf16 x bf16 -> f32, M = 128, N = 16; A MN-major when `a_mn`, B K-major.
__host__ __device__ constexpr uint32_t idesc_attn(bool a_mn) {
  return tc::idesc_bf16(kTcHeads) | (a_mn ? (1u << 15) : 0u);
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Byte offset of element (row, col) in a 128-byte-swizzled, K-major block whose rows are
// 128 bytes (64 bf16) and whose 8-row groups are 1024 bytes apart.
__device__ __forceinline__ uint32_t sw128_offset(int row, int col) {
  const int chunk = col >> 3;
  return uint32_t(row * 128 + (((chunk ^ (row & 7)) & 7) << 4) + (col & 7) * 2);
}

template <int G, int T>
static __global__ void __launch_bounds__(kTcThreads, 1)
    k_decode_attn_tc(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                     const __nv_bfloat16* __restrict__ q, const int* __restrict__ lengths,
                     __nv_bfloat16* __restrict__ out, int* counters, float* part_o, float* part_ml, int Hkv, int Lmax,
                     float scale_log2, uint64_t* stamps) {
  static_assert(G >= 1 && G <= kTcHeads, "one KV head's query heads must fit the MMA's N");
  // optional phase timing: thread 0 of each CTA records %globaltimer at kTcStamps points
  auto stamp = [&](int i) {
    if (stamps && threadIdx.x == 0) {
      uint64_t now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      stamps[(size_t(blockIdx.y) * gridDim.x + blockIdx.x) * kTcStamps + i] = now;
    }
  };
  stamp(0);  // entry
  using L = TcLayout<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(base + L::red);      // [2][4][16]
  float* stat = reinterpret_cast<float*>(base + L::stat);    // [16][2]
  uint64_t* k_full = reinterpret_cast<uint64_t*>(base + L::bars);
  uint64_t* v_full = k_full + T;
  uint64_t* s_done = v_full + T;
  uint64_t* o_done = s_done + 1;
  uint64_t* m_full = o_done + 1;  // workspace merge: the partial outputs' bulk copy
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + L::misc);
  volatile uint32_t* bad = reinterpret_cast<volatile uint32_t*>(base + L::misc + 4);
  int* last = reinterpret_cast<int*>(base + L::misc + 8);

  // grid (spans, sequences x KV heads); the spans of one (sequence, KV head) are one
  // cluster when the launch asked for it (the merge then runs in distributed shared memory)
  const int bh = blockIdx.y, b = bh / Hkv, h = bh % Hkv, s = blockIdx.x, nsplit = gridDim.x;
  cg::cluster_group cluster = cg::this_cluster();
  const bool cluster_merge = nsplit > 1 && cluster.num_blocks() == unsigned(nsplit);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int Hq = G * Hkv;
  const size_t head0 = size_t(b) * Hq + size_t(h) * G;

  if (t == 0) {
    for (int i = 0; i < T; ++i) {
      tc::mbar_init(&k_full[i], 1);
      tc::mbar_init(&v_full[i], 1);
    }
    tc::mbar_init(s_done, 1);
    tc::mbar_init(o_done, 1);
    tc::mbar_init(m_full, 1);
    *bad = 0u;
    tc::fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, kTcTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  stamp(1);  // barriers and TMEM ready
  const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // Every tile that starts inside this sequence's cache is requested at once, before q
  // is staged (a tile past the length is masked, then drained before exit), so the K/V
  // round trip overlaps the loads of q.  Programmatic dependent launch: the preceding
  // kernel may still be writing q and the newest key / value row (lengths[b] - 1); the
  // lengths and the older rows come from kernels before it.  Tiles wholly below the
  // newest key are therefore requested before griddepcontrol.wait, the rest after it.
  const int chunk = T * kTcKeys;
  const int start = s * chunk;
  const int issued = start < Lmax ? min(T, (Lmax - start + kTcKeys - 1) / kTcKeys) : 0;
  auto issue_tile = [&](int i) {
    const int row = b * Lmax + start + i * kTcKeys;
    tc::mbar_expect_tx(&k_full[i], kTileBytes);
    tma_load_3d(base + L::k + i * kTileBytes, &map_k, 0, h, row, &k_full[i]);
    tma_load_3d(base + L::k + i * kTileBytes + kHalfBytes, &map_k, 64, h, row, &k_full[i]);
    tc::mbar_expect_tx(&v_full[i], kTileBytes);
    tma_load_3d(base + L::v + i * kTileBytes, &map_v, 0, h, row, &v_full[i]);
    tma_load_3d(base + L::v + i * kTileBytes + kHalfBytes, &map_v, 64, h, row, &v_full[i]);
  };
  int early = 0;
  if (t == 0) {
    const int newest = min(lengths[b], Lmax) - 1;
    while (early < issued && start + (early + 1) * kTcKeys <= newest) ++early;
    for (int i = 0; i < early; ++i) issue_tile(i);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (t == 0)
    for (int i = early; i < issued; ++i) issue_tile(i);
  // Q: 16 rows (G real heads, the rest zero) x 128 dims into the swizzled B-operand image
  for (int i = t; i < kTcHeads * 16; i += kTcThreads) {
    const int r = i >> 4, c = i & 15;  // row, 16-byte chunk of the 256-byte row
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < G) v = *reinterpret_cast<const uint4*>(q + (head0 + r) * kHead + c * 8);
    *reinterpret_cast<uint4*>(base + L::q + (c >> 3) * kQHalfBytes + sw128_offset(r, (c & 7) * 8)) = v;
  }
  const int len = min(min(lengths[b], Lmax), nsplit * chunk);
  const int end = min(start + chunk, len);
  const int ntiles = end > start ? (end - start + kTcKeys - 1) / kTcKeys : 0;  // <= issued
  fence_async_smem();
  __syncthreads();
  stamp(2);  // loads issued, Q staged, length known

  float m_span[kTcHeads], l_span[kTcHeads];  // per head: span max (log2 units), sum
#pragma unroll
  for (int g = 0; g < kTcHeads; ++g) {
    m_span[g] = -INFINITY;
    l_span[g] = 0.0f;
  }
  float o[kTcHeads];
#pragma unroll
  for (int g = 0; g < kTcHeads; ++g) o[g] = 0.0f;

  if (ntiles > 0) {
    // S^T = K Q^T, one MMA chain per tile into TMEM columns 16 * tile
    if (t == 0) {
      tc::tc_fence_after();
      for (int i = 0; i < ntiles; ++i) {
        if (!tc::mbar_wait(&k_full[i], 0, bad)) break;
        if (i == 0) stamp(3);  // first K tile landed
        tc::tc_fence_after();
        const uint8_t* kt = base + L::k + i * kTileBytes;
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // 16 dims per MMA: 32 bytes along the swizzled row
          const uint64_t ad = tc::smem_desc_sw128(kt + (j >> 2) * kHalfBytes) + 2 * (j & 3);
          const uint64_t bd = tc::smem_desc_sw128(base + L::q + (j >> 2) * kQHalfBytes) + 2 * (j & 3);
          tc::mma_bf16(tmem + uint32_t(16 * i), ad, bd, idesc_attn(false), j != 0);
        }
      }
      tc::mma_commit(s_done);  // arrives once the issued MMAs retire (also after an early stop)
    }
    __syncwarp();
    bool ok = tc::mbar_wait(s_done, 0, bad);
    stamp(4);  // scores in TMEM
    tc::tc_fence_after();
    // softmax: thread t owns key t of every tile
    float sc[T][kTcHeads];
#pragma unroll
    for (int i = 0; i < T; ++i) {
      if (i < ntiles) tc::tmem_ld16(lane_base + uint32_t(16 * i), sc[i]);
#pragma unroll
      for (int g = 0; g < kTcHeads; ++g) {
        const bool valid = i < ntiles && start + i * kTcKeys + t < end;
        sc[i][g] = valid && ok ? sc[i][g] * scale_log2 : -INFINITY;
        if (g < G) m_span[g] = fmaxf(m_span[g], sc[i][g]);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) m_span[g] = fmaxf(m_span[g], __shfl_xor_sync(0xffffffffu, m_span[g], off));
      if (lane == 0) red[warp * kTcHeads + g] = m_span[g];
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g)
      m_span[g] = fmaxf(fmaxf(red[g], red[kTcHeads + g]), fmaxf(red[2 * kTcHeads + g], red[3 * kTcHeads + g]));
    // P = exp2(S - max), rounded to bf16 into the K-major B-operand image of the second
    // MMA (rows = heads, K = keys); keys past the span and padding heads are zero
#pragma unroll
    for (int i = 0; i < T; ++i) {
      if (i >= ntiles) break;
      uint8_t* pt = base + L::p + i * 2 * kPAtomBytes + (t >> 6) * kPAtomBytes;
#pragma unroll
      for (int g = 0; g < kTcHeads; ++g) {
        float pr = 0.0f;
        if (g < G && sc[i][g] != -INFINITY) pr = exp2f(sc[i][g] - m_span[g]);
        const __nv_bfloat16 pb = __float2bfloat16_rn(pr);
        if (g < G) l_span[g] += __bfloat162float(pb);  // the sum of what the MMA multiplies
        *reinterpret_cast<__nv_bfloat16*>(pt + sw128_offset(g, t & 63)) = pb;
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) l_span[g] += __shfl_xor_sync(0xffffffffu, l_span[g], off);
      if (lane == 0) red[4 * kTcHeads + warp * kTcHeads + g] = l_span[g];
    }
    stamp(5);  // softmax done, P staged
    // V rows past the span may hold anything (another sequence, unwritten cache): zero
    // them, so that 0 * V stays 0 in the second product
    for (int i = 0; i < ntiles; ++i) {
      if (!tc::mbar_wait(&v_full[i], 0, bad)) {
        ok = false;
        break;
      }
      if (start + i * kTcKeys + t >= end) {
        uint8_t* row = base + L::v + i * kTileBytes + t * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          *reinterpret_cast<uint4*>(row + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(row + kHalfBytes + c * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
    }
    fence_async_smem();
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float* rs = red + 4 * kTcHeads;
      l_span[g] = ((rs[g] + rs[kTcHeads + g]) + rs[2 * kTcHeads + g]) + rs[3 * kTcHeads + g];
    }
    // O^T += V^T P^T: A = V as stored (dims contiguous: MN-major), B = P (keys contiguous)
    if (t == 0 && !*bad) {
      tc::tc_fence_after();
      for (int i = 0; i < ntiles; ++i) {
        const uint8_t* vt = base + L::v + i * kTileBytes;
        const uint8_t* pt = base + L::p + i * 2 * kPAtomBytes;
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // 16 keys per MMA: two 8-row groups of V, 32 bytes of P's row
          const uint64_t ad = smem_desc_sw128_mn(vt + j * 2048, kHalfBytes, 1024);
          const uint64_t bd = tc::smem_desc_sw128(pt + (j >> 2) * kPAtomBytes) + 2 * (j & 3);
          tc::mma_bf16(tmem + kTcOutCol, ad, bd, idesc_attn(true), (i | j) != 0);
        }
      }
      tc::mma_commit(o_done);
    }
    __syncwarp();
    if (!*bad && tc::mbar_wait(o_done, 0, bad)) {
      tc::tc_fence_after();
      tc::tmem_ld16(lane_base + kTcOutCol, o);  // thread t: dimension t, one column per head
      stamp(6);  // output accumulator read
    }
  }

  // Let this CTA's own copies land before its shared memory goes away: the tiles past
  // the length (never waited for), and every tile after an error.
  if (t == 0) {
    for (int i = *bad ? 0 : ntiles; i < issued; ++i) {
      tc::mbar_drain(&k_full[i], 0);
      tc::mbar_drain(&v_full[i], 0);
    }
    if (*bad) atomicExch(&counters[kErrorSlot], 1);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, kTcTmemCols);

  if (nsplit == 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float inv = l_span[g] > 0.0f ? 1.0f / l_span[g] : 0.0f;
      out[(head0 + g) * kHead + t] = __float2bfloat16_rn(o[g] * inv);
    }
    return;
  }
  if (cluster_merge) {
    // Each span parks its unnormalised output [G][128] and (max, sum) per head in its own
    // shared memory (the K tiles are free); after a cluster barrier span r finalises heads
    // r, r + nsplit, ...: thread t reads dimension t of every span's partial through
    // distributed shared memory (every load issued before the sum) and merges in span order.
    float* park = reinterpret_cast<float*>(base + L::k);  // [G][128] outputs, then [G][2] (max, sum)
#pragma unroll
    for (int g = 0; g < G; ++g) park[g * kTcThreads + t] = o[g];
    if (t < G) {
      park[G * kTcThreads + 2 * t] = m_span[t];
      park[G * kTcThreads + 2 * t + 1] = l_span[t];
    }
    cluster.sync();
    stamp(7);  // partials parked in the cluster
#pragma unroll 1
    for (int g = s; g < G; g += nsplit) {
      float mx[kClusterMaxSpans], ls[kClusterMaxSpans], ov[kClusterMaxSpans];
#pragma unroll
      for (int r = 0; r < kClusterMaxSpans; ++r) {
        if (r < nsplit) {
          const float* pr = cluster.map_shared_rank(park, r);
          mx[r] = pr[G * kTcThreads + 2 * g];
          ls[r] = pr[G * kTcThreads + 2 * g + 1];
          ov[r] = pr[g * kTcThreads + t];
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < kClusterMaxSpans; ++r)
        if (r < nsplit) M = fmaxf(M, mx[r]);
      float Lt = 0.0f, acc = 0.0f;
#pragma unroll
      for (int r = 0; r < kClusterMaxSpans; ++r) {
        if (r < nsplit) {
          const float w = ls[r] > 0.0f ? exp2f(mx[r] - M) : 0.0f;
          Lt += ls[r] * w;
          acc += ov[r] * w;
        }
      }
      out[(head0 + g) * kHead + t] = __float2bfloat16_rn(Lt > 0.0f ? acc / Lt : 0.0f);
    }
    stamp(11);  // merged
    cluster.sync();  // every span's partial stays readable until the cluster is done
    return;
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const size_t row = (head0 + g) * nsplit + s;
    __stcg(part_o + row * kHead + t, o[g]);
    if (t == 0) {
      __stcg(part_ml + row * 2, m_span[g]);
      __stcg(part_ml + row * 2 + 1, l_span[g]);
    }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) *last = atomicAdd(&counters[bh], 1) == nsplit - 1;
  __syncthreads();
  stamp(7);  // partial stored, counted
  if (!*last) return;
  __threadfence();

  // Merge the spans of each head in span order.  Every (max, sum) pair is loaded in one
  // parallel pass, the weights are formed per head, then each thread (one dimension)
  // sums its partial outputs.  The partial outputs of this KV head's G heads are one
  // contiguous block; when it fits the free K/V tiles, one bulk copy brings it into
  // shared memory while the (max, sum) pairs load and the weights form (measured at 64
  // sequence-head pairs x 9 spans: the L2 loop below took 5 us, three dependent round
  // trips of 32 loads).
  float* ml = reinterpret_cast<float*>(base + L::k);  // [G][nsplit][2]; K tiles are free now
  float* accs = ml + 2 * G * nsplit;                    // [G][kTcThreads] running sums
  const int pairs = G * nsplit;
  const uint32_t po_bytes = uint32_t(pairs) * kHead * 4;
  const uint32_t ps_off = (uint32_t(2 * G * nsplit + G * kTcThreads) * 4 + 15u) & ~15u;
  const float* po_all = part_o + head0 * nsplit * kHead;  // pair i = g * nsplit + sp at [i * kHead]
  const bool staged = ps_off + po_bytes <= uint32_t(L::q - L::k);
  float* ps = reinterpret_cast<float*>(base + L::k + ps_off);
  if (staged && t == 0) {
    asm volatile("fence.proxy.async.global;" ::: "memory");  // the other spans' stores before the copy reads
    tc::mbar_expect_tx(m_full, po_bytes);
    tc::bulk_load(ps, po_all, po_bytes, m_full);
  }
  for (int i = t; i < G * nsplit; i += kTcThreads) {
    const size_t row = (head0 + i / nsplit) * nsplit + i % nsplit;
    const float2 v = __ldcg(reinterpret_cast<const float2*>(part_ml + row * 2));
    ml[2 * i] = v.x;
    ml[2 * i + 1] = v.y;
  }
  __syncthreads();
  stamp(8);  // merge: (max, sum) pairs loaded
  if (t < G) {
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, ml[2 * (t * nsplit + sp)]);
    float Ltot = 0.0f;
    for (int sp = 0; sp < nsplit; ++sp) {
      float* e = ml + 2 * (t * nsplit + sp);
      const float w = e[1] > 0.0f ? exp2f(e[0] - M) : 0.0f;
      Ltot += e[1] * w;
      e[0] = w;
    }
    stat[2 * t] = Ltot;
  }
  __syncthreads();
  stamp(9);  // merge: weights formed
  // Each head's sum goes to a shared-memory column of this thread, spans in order.  The
  // loop is kept compact on purpose: the merge runs once per (sequence, KV head), so its
  // code is always cold in the instruction cache, and a fully unrolled form spent ~29 us
  // fetching instructions.  From L2, kBatch loads are in flight before any is used.
  constexpr int kBatch = 32;
#pragma unroll 1
  for (int g = 0; g < G; ++g) accs[g * kTcThreads + t] = 0.0f;
  if (staged) {
    // a failed wait leaves the partials unread: the error word reports the launch
    if (tc::mbar_wait(m_full, 0, bad)) {
      // per head a register sum over the spans in order (from 0, as the L2 path sums)
#pragma unroll 1
      for (int g = 0; g < G; ++g) {
        const float* pg = ps + size_t(g) * nsplit * kHead + t;
        const float* wg = ml + 2 * g * nsplit;
        float a = 0.0f;
#pragma unroll 4
        for (int sp = 0; sp < nsplit; ++sp) a += pg[sp * kHead] * wg[2 * sp];
        accs[g * kTcThreads + t] = a;
      }
    } else {
      if (t == 0) atomicExch(&counters[kErrorSlot], 1);
      tc::mbar_drain(m_full, 0);  // the copy lands before this CTA's shared memory goes away
    }
  } else {
    const float* po = po_all + t;
#pragma unroll 1
    for (int i0 = 0; i0 < pairs; i0 += kBatch) {
      float v[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) v[j] = i0 + j < pairs ? __ldcg(po + size_t(i0 + j) * kHead) : 0.0f;
      int g = i0 / nsplit, sp = i0 - g * nsplit;
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        if (i0 + j < pairs) accs[g * kTcThreads + t] += v[j] * ml[2 * (i0 + j)];
        if (++sp == nsplit) {
          sp = 0;
          ++g;
        }
      }
    }
  }
  float acc[kTcHeads];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = accs[g * kTcThreads + t];
  stamp(10);  // merge: partial outputs summed
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float Ltot = stat[2 * g], inv = Ltot > 0.0f ? 1.0f / Ltot : 0.0f;
    out[(head0 + g) * kHead + t] = __float2bfloat16_rn(acc[g] * inv);
  }
  stamp(11);  // merged
  if (t == 0) counters[bh] = 0;
}

// --- host side ----------------------------------------------------------------------
using TmapEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no driver library
// handle kept here, nothing allocated); null if the driver does not offer it.
static inline TmapEncodeFn tmap_encode() {
  static TmapEncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return TmapEncodeFn(nullptr);
    return reinterpret_cast<TmapEncodeFn>(p);
  }();
  return fn;
}

// The map of one cache, [B, Lmax, Hkv, 128] bf16, as 3-D (dim, KV head, B * Lmax rows),
// box 64 dims x 1 head x 128 keys, 128-byte swizzle.
static inline bool make_cache_map(CUtensorMap* map, const void* cache, int B, int Lmax, int Hkv) {
  TmapEncodeFn enc = tmap_encode();
  if (!enc) return false;
  cuuint64_t dims[3] = {cuuint64_t(kHead), cuuint64_t(Hkv), cuuint64_t(B) * cuuint64_t(Lmax)};
  cuuint64_t strides[2] = {cuuint64_t(kHead) * 2, cuuint64_t(Hkv) * kHead * 2};
  cuuint32_t box[3] = {64, 1, cuuint32_t(kTcKeys)};
  cuuint32_t elem[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(cache), dims, strides, box, elem,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Whether the tensor-core kernel takes this problem (shapes, alignment, a TMA encoder).
static inline bool tc_eligible(const void* q, const void* k_cache, const void* v_cache, int B, int Hq, int Hkv,
                               int Lmax, int max_len) {
  if (Hkv <= 0 || Hq % Hkv) return false;
  const int G = Hq / Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16) return false;
  if (!tc_tiles(max_len) || size_t(B) * Lmax < size_t(kTcKeys) || B * Hkv > kCounterSlots - 1) return false;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16)
    return false;
  return tmap_encode() != nullptr;
}

template <int G, int T>
static inline cudaError_t launch_tc_gt(const CUtensorMap& mk, const CUtensorMap& mv, const __nv_bfloat16* q,
                                       const int* lengths, __nv_bfloat16* out, int* counters, float* part_o,
                                       float* part_ml, int B, int Hkv, int Lmax, int nsplit, int cluster,
                                       float scale_log2, cudaStream_t st, bool pdl, uint64_t* stamps) {
  auto kernel = k_decode_attn_tc<G, T>;
  static int attr_set[64] = {0};  // function attributes belong to each device's context
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TcLayout<T>::bytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsplit, B * Hkv, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = TcLayout<T>::bytes;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attrs[1].id = cudaLaunchAttributeClusterDimension;
  attrs[1].val.clusterDim.x = cluster;
  attrs[1].val.clusterDim.y = 1;
  attrs[1].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = cluster > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, mk, mv, q, lengths, out, counters, part_o, part_ml, Hkv, Lmax, scale_log2,
                            stamps);
}

// Spans for the cluster merge: up to kClusterMaxSpans spans of T = 1 or 2 tiles cover
// sequences up to 2048 keys; 0 = use the workspace merge (tc_tiles / tc_splits).
static inline void cluster_plan(int max_len, int& T, int& nsplit) {
  T = max_len <= kClusterMaxSpans * kTcKeys ? 1 : 2;
  nsplit = (max_len + T * kTcKeys - 1) / (T * kTcKeys);
  if (nsplit > kClusterMaxSpans) T = nsplit = 0;
}

// Whether the cluster merge applies: a cluster plan exists and the whole grid fits in one
// wave of one CTA per SM.  Clusters of up to 8 CTAs must be co-scheduled on one GPC, and
// with several waves that constraint costs more than the merge saves (measured on one
// B200, 1024 keys, 8 query heads per KV head, graph-timed: batch 64 = 512 CTAs took
// 25.7 us with clusters against 19.7 us with the workspace merge).
static inline bool cluster_merge_fits(int B, int Hkv, int max_len, int sms) {
  int T = 0, nsplit = 0;
  cluster_plan(max_len, T, nsplit);
  return T != 0 && int64_t(B) * Hkv * nsplit <= sms;
}

// Launch over the shared workspace layout [kCounterSlots ints][part_o][part_ml].  With
// `cluster_merge` (only where cluster_merge_fits) the spans of a (sequence, KV head) form
// one cluster and merge in distributed shared memory (the workspace is then used only if
// a tool re-issues the launch without its cluster attribute); otherwise the spans merge
// through the workspace.
static inline cudaError_t launch_decode_attention_tc(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                                                     const __nv_bfloat16* v_cache, const int* lengths,
                                                     __nv_bfloat16* out, float* scratch, int B, int Hq, int Hkv,
                                                     int Lmax, int max_len, float scale, cudaStream_t st, bool pdl,
                                                     bool cluster_merge, uint64_t* stamps = nullptr) {
  CUtensorMap mk, mv;
  if (!make_cache_map(&mk, k_cache, B, Lmax, Hkv) || !make_cache_map(&mv, v_cache, B, Lmax, Hkv))
    return cudaErrorInvalidValue;
  int T = 0, nsplit = 0;
  if (cluster_merge) cluster_plan(max_len, T, nsplit);
  const int cluster = nsplit > 1 ? nsplit : 1;
  if (!T) {
    T = tc_tiles(max_len);
    nsplit = tc_splits(max_len);
  }
  const int G = Hq / Hkv;
  int* counters = reinterpret_cast<int*>(scratch);
  float* part_o = scratch + kCounterSlots;
  float* part_ml = part_o + size_t(B) * Hq * nsplit * kHead;
  const float sl2 = scale * kLog2e;
  const int cl = (cluster > 1 && nsplit == cluster) ? cluster : 1;
#define SN_TC(GG, TT)                                                                                       \
  if (G == GG && T == TT)                                                                                   \
    return launch_tc_gt<GG, TT>(mk, mv, q, lengths, out, counters, part_o, part_ml, B, Hkv, Lmax, nsplit, cl, \
                                sl2, st, pdl, stamps);
  SN_TC(1, 1) SN_TC(2, 1) SN_TC(4, 1) SN_TC(8, 1) SN_TC(16, 1)
  SN_TC(1, 2) SN_TC(2, 2) SN_TC(4, 2) SN_TC(8, 2) SN_TC(16, 2)
#undef SN_TC
  return cudaErrorInvalidValue;
}

// The decode attention entry used by the torch op and the allocation-free C entry
// point.  impl 0 (default): the tensor-core kernel where it is eligible and either its
// cluster merge fits (cluster_merge_fits) or there are at least kTcMinPairs (sequence, KV
// head) pairs, else the CUDA-core kernel; impl 1: the CUDA-core kernel; impl 2: the
// tensor-core kernel, cudaErrorNotSupported where it is not eligible.  Measured on one
// B200, 8 query heads per KV head (graph-timed us, tensor cores / CUDA cores): 1024 keys,
// batch 1: 8.1 / 10.2 and batch 8: 8.5 / 11.4 (cluster merge); batch 64: 19.7 / 28.7
// (workspace merge); 4096 keys, batch 8: 28.4 / 22.6 (workspace merge: 32 spans per pair
// on 8 pairs leave the merge on the critical path).  `stamps` (tensor-core kernel only):
// per-CTA phase timestamps, kTcStamps each, or null.
constexpr int kTcMinPairs = 32;

static inline cudaError_t launch_decode_attention(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                                                  const __nv_bfloat16* v_cache, const int* lengths,
                                                  __nv_bfloat16* out, float* scratch, int B, int Hq, int Hkv,
                                                  int Lmax, int max_len, float scale, int sms, cudaStream_t st,
                                                  bool pdl = false, int impl = 0, uint64_t* stamps = nullptr) {
  const bool fits = cluster_merge_fits(B, Hkv, max_len, sms);
  const bool tc = impl == 2 || (impl == 0 && (fits || B * Hkv >= kTcMinPairs));
  if (tc && tc_eligible(q, k_cache, v_cache, B, Hq, Hkv, Lmax, max_len))
    return launch_decode_attention_tc(q, k_cache, v_cache, lengths, out, scratch, B, Hq, Hkv, Lmax, max_len, scale,
                                      st, pdl, fits, stamps);
  if (impl == 2) return cudaErrorNotSupported;
  return launch_decode_attention_simt(q, k_cache, v_cache, lengths, out, scratch, B, Hq, Hkv, Lmax, max_len, scale,
                                      sms, st, pdl);
}

}  // namespace attn
}  // namespace sn
