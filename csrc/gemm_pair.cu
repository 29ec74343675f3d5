// tcgen05 GEMM over CTA pairs (cta_group::2) for sm_100a:  C[M, N] = A[M, K] B[N, K]^T.
//
// A pair of CTAs (a cluster of 2, fixed at compile time) owns a 256 x BN output tile
// (BN = 256 is the one built).  Each CTA stages 128 rows of A and BN / 2 rows of B per
// K step (32 KB), so a stage costs each SM half the B bytes of a one-CTA
// 128 x 256 tile, and the pair's tensor cores read one 256 x BN x 16 MMA from both CTAs'
// shared memory.  One elected thread of the even CTA issues every MMA; each CTA's TMEM
// holds its own 128 rows of the fp32 accumulator (two BN-column buffers, so the
// epilogue of one tile overlaps the MMAs of the next).
//
// Roles per CTA (192 threads): warp 0 issues the CTA's own TMA loads (one thread),
// warp 1 allocates TMEM for the pair and, in the even CTA, issues the MMAs; warps 2..5
// drain the CTA's accumulator rows and store bf16.
//
// Synchronisation across the pair (all addresses in the even CTA are reached through
// mapa; every wait is bounded and on the waiting CTA's own barrier):
//   full[s]   even CTA only.  The even producer posts the stage's bytes for both CTAs
//             (arrive.expect_tx); both CTAs' TMA loads complete on it.
//   empty[s]  in both CTAs; the MMA thread commits to both once the stage is consumed.
//   tfull[a]  in both CTAs; committed after a tile's last MMA into accumulator a.
//   tempty[a] even CTA only; the epilogue warps of both CTAs arrive once accumulator a
//             is drained (count 8).
// A cluster barrier after set-up and another before TMEM is freed keep each CTA's
// barriers, shared memory and TMEM alive while the other CTA may still use them.
//
// Every TMA load is a plain per-CTA load into the issuing CTA's own shared memory.
//
// Reference: none (the reference has no GEMM; its prefill collectives go to NCCL).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "sparknet/tc_gemm.cuh"

namespace py = pybind11;

namespace sn {
namespace tc {
namespace pair {

constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;
constexpr int kTileM = 256;                 // rows per pair tile
constexpr int kHalf = 128;                  // rows of A per CTA
constexpr int kStages = 6;
constexpr uint32_t kTmemCols = 512;         // two accumulators of up to 256 columns
constexpr int kGroupM = 8;                  // pair row blocks per raster band

// Shared-memory plan and instruction descriptor for a pair tile 256 x BN (BN / 2 rows of
// B per CTA).  The epilogue drains the accumulator in chunks of CW columns.
template <int BN>
struct Plan {
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "pair tile N must be a multiple of 32 in 64..256");
  static constexpr int kBRows = BN / 2;
  static constexpr int kABytes = kHalf * 128;
  static constexpr int kStageBytes = kABytes + kBRows * 128;      // 128-byte rows (64 bf16 of K)
  static constexpr int kCW = BN % 64 == 0 ? 64 : 32;
  static constexpr int kStageRowBytes = kCW * 2 + 16;             // padded staging row
  static constexpr int kEpiBytes = kEpiWarps * 32 * kStageRowBytes;
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024 + 256;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory plan exceeds the per-CTA limit");
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned for the 128-byte swizzle");
  // bf16 x bf16 -> f32, K-major A and B, M = 256 (the pair), N = BN
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) |
                                     (uint32_t(kTileM >> 4) << 24);
};

__device__ __forceinline__ uint32_t rank_in_pair() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t pair_size() {
  uint32_t n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  return n;
}

// shared::cluster address of this CTA's variable `p` as seen in CTA `cta` of the pair
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t cta) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(cta));
  return out;
}

__device__ __forceinline__ void pair_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMA tile into this CTA's shared memory, completing on an mbarrier that may live in
// the other CTA of the pair (`bar` is a shared::cluster address).
__device__ __forceinline__ void tma_load_pair(void* smem_dst, const CUtensorMap* map, int32_t x, int32_t y,
                                              uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void mma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at shared::cluster address `bar` (in either CTA of the pair)
// once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

struct Params {
  int M, N, K;
  __nv_bfloat16* C;
  int ldc;
  uint32_t* err;
};

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    k_gemm_pair(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, Params p) {
  using P = Plan<BN>;
  constexpr int kStageBytes = P::kStageBytes, kEpiBytes = P::kEpiBytes, kStageRowBytes = P::kStageRowBytes;
  constexpr int kTileN = BN, kCW = P::kCW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi = smem + kStages * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi + kEpiBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ uint32_t err_local;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The pair is fixed by __cluster_dims__; a launch that still came without it has
  // nothing to pair with and leaves before it allocates anything.
  if (pair_size() != 2) {
    if (threadIdx.x == 0) atomicExch(p.err, kTcWaitTimeout);
    return;
  }
  const uint32_t cta = rank_in_pair();
  const bool leader = cta == 0;
  volatile uint32_t* err = &err_local;

  if (threadIdx.x == 0) {
    err_local = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, kTmemCols);
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
  }
  tc_fence_before();
  pair_sync();  // both CTAs' barriers initialised and TMEM allocated before any use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int pair_id = int(blockIdx.x) >> 1, npairs = int(gridDim.x) >> 1;
  const int tiles_m = (p.M + kTileM - 1) / kTileM, tiles_n = (p.N + kTileN - 1) / kTileN;
  const int tiles = tiles_m * tiles_n;
  const int kblocks = p.K / kBK;
  // Bands of kGroupM row blocks; inside a band the row block varies fastest, so the
  // tiles in flight share A and B row blocks in L2.
  auto tile_coord = [&](int t, int& m0, int& n0) {
    const int band = t / (kGroupM * tiles_n);
    const int rows_in_band = min(kGroupM, tiles_m - band * kGroupM);
    const int inner = t - band * kGroupM * tiles_n;
    m0 = (band * kGroupM + inner % rows_in_band) * kTileM;
    n0 = (inner / rows_in_band) * kTileN;
  };

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs: their own halves) ----------------
    if (lane == 0) {
      const uint32_t full0 = peer_addr(&full[0], 0);  // the even CTA's full[0]
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair_id; t < tiles && ok; t += npairs) {
        int m0, n0;
        tile_coord(t, m0, n0);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * kStageBytes;
          uint8_t* sb = sa + P::kABytes;
          if (leader) mbar_expect_tx(&full[stage], 2 * kStageBytes);
          const uint32_t fb = full0 + uint32_t(stage * sizeof(uint64_t));
          tma_load_pair(sa, &map_a, kb * kBK, m0 + int(cta) * kHalf, fb);
          tma_load_pair(sb, &map_b, kb * kBK, n0 + int(cta) * P::kBRows, fb);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA) ----------------
    if (leader && lane == 0) {
      uint32_t empty_at[2], tfull_at[2];
      for (uint32_t c = 0; c < 2; ++c) {
        empty_at[c] = peer_addr(&empty[0], c);
        tfull_at[c] = peer_addr(&tfull[0], c);
      }
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair_id; t < tiles && ok; t += npairs) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + uint32_t(acc * kTileN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sa = smem + stage * kStageBytes;
          const uint64_t adesc = smem_desc_sw128(sa), bdesc = smem_desc_sw128(sa + P::kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_pair(d, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), P::kIdesc, (kb | k) ? 1u : 0u);
          const uint32_t off = uint32_t(stage * sizeof(uint64_t));
          commit_pair(empty_at[0] + off);
          commit_pair(empty_at[1] + off);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t off = uint32_t(acc * sizeof(uint64_t));
        commit_pair(tfull_at[0] + off);
        commit_pair(tfull_at[1] + off);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      commit_pair(peer_addr(drain, 0));  // fires once every MMA issued above has completed
      mbar_wait(drain, 0, err);
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs: their own 128 rows) ----------------
    const int quad = warp & 3;  // TMEM lanes 32*quad .. +31
    const uint32_t tempty0 = peer_addr(&tempty[0], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    uint8_t* wst = epi + (warp - 2) * 32 * kStageRowBytes;
    for (int t = pair_id; t < tiles; t += npairs) {
      int m0, n0;
      tile_coord(t, m0, n0);
      if (!mbar_wait(&tfull[acc], acc_phase, err)) break;
      tc_fence_after();
      const int row0 = m0 + int(cta) * kHalf + quad * 32;
      const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * kTileN);
      // kCW columns at a time: TMEM -> registers (this thread's row) -> staging rows ->
      // stores with kCW / 8 lanes per row segment (256 / kCW rows per instruction)
      constexpr int kLanesPerRow = kCW / 8, kRowsPerStore = 32 / kLanesPerRow;
#pragma unroll 1
      for (int c = 0; c < kTileN / kCW; ++c) {
        float v[kCW];
#pragma unroll
        for (int h = 0; h < kCW / 32; ++h) tmem_ld32(taddr + uint32_t(c * kCW + 32 * h), v + 32 * h);
        uint4* my_row = reinterpret_cast<uint4*>(wst + lane * kStageRowBytes);
#pragma unroll
        for (int q = 0; q < kCW / 8; ++q) {
          uint4 pk;
          pk.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
          pk.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
          pk.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
          pk.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
          my_row[q] = pk;
        }
        __syncwarp();
        const int seg = lane % kLanesPerRow;
        const int gn = n0 + c * kCW + seg * 8;
#pragma unroll
        for (int rr = 0; rr < kLanesPerRow; ++rr) {
          const int r = rr * kRowsPerStore + lane / kLanesPerRow;
          const int grow = row0 + r;
          const uint4 pk = *reinterpret_cast<const uint4*>(wst + r * kStageRowBytes + seg * 16);
          if (grow < p.M && gn < p.N) *reinterpret_cast<uint4*>(p.C + size_t(grow) * p.ldc + gn) = pk;
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_remote(tempty0 + uint32_t(acc * sizeof(uint64_t)));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }
  // Every MMA that reads this CTA's shared memory or writes its TMEM has completed
  // before the even CTA's MMA thread gets here (drain); the barrier holds the odd CTA
  // until then.
  tc_fence_before();
  pair_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && err_local) atomicExch(p.err, err_local);
}

}  // namespace pair

// C[M, N] = A[M, K] B[N, K]^T on CTA pairs.  K % 64 == 0, N % 8 == 0.
void gemm_pair(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, at::Tensor& err, int max_pairs) {
  auto check = [](const at::Tensor& t, const char* name) {
    if (!t.is_cuda() || t.scalar_type() != at::kBFloat16 || t.dim() != 2 || t.stride(1) != 1)
      throw std::invalid_argument(std::string(name) + " must be a row-major 2-D CUDA bfloat16 tensor");
  };
  check(A, "A");
  check(B, "B");
  check(C, "C");
  const int M = int(A.size(0)), K = int(A.size(1)), N = int(B.size(0));
  if (B.size(1) != K || C.size(0) != M || C.size(1) != N) throw std::invalid_argument("shape mismatch");
  if (K % kBK || K == 0) throw std::invalid_argument("K must be a positive multiple of 64");
  if (N % 8 || (C.stride(0) * 2) % 16 || reinterpret_cast<uintptr_t>(C.data_ptr()) % 16)
    throw std::invalid_argument("N must be a multiple of 8 and C rows 16-byte aligned");
  if (!err.is_cuda() || err.numel() < 1) throw std::invalid_argument("err must be a CUDA int32 word");
  c10::cuda::CUDAGuard guard(A.device());
  pair::Params p{M, N, K, reinterpret_cast<__nv_bfloat16*>(C.data_ptr()), int(C.stride(0)),
                 reinterpret_cast<uint32_t*>(err.data_ptr())};
  int sms = 0;
  const int dev = A.device().index();
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int pair_slots = sms / 2;
  if (max_pairs > 0) pair_slots = std::min(pair_slots, max_pairs);
  // Pair tile N is 256.  Narrower tiles (224, 192) fill the persistent grid's last round
  // better (8192 x 7168: 13.8 rounds of 74 pairs instead of 12.1) but measured slower at
  // every shape tried (8192 x 7168 x 8192: 1368 / 1238 against 1433 TFLOP/s): each MMA
  // still reads all of A's tile, so A costs more shared-memory bandwidth per FLOP.
  const int tiles_m = (M + pair::kTileM - 1) / pair::kTileM;
  const int bn = 256;
  const int tiles = tiles_m * ((N + bn - 1) / bn);
  const int pairs = std::min(tiles, pair_slots);
  auto s = at::cuda::getCurrentCUDAStream(dev).stream();
  CUtensorMap ma = make_map(A.data_ptr(), M, K, A.stride(0), pair::kHalf);
  CUtensorMap mb = make_map(B.data_ptr(), N, K, B.stride(0), uint32_t(bn / 2));
  using P = pair::Plan<256>;
  static bool attr_done[64] = {};
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(pair::k_gemm_pair<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         P::kSmemBytes);
    if (e != cudaSuccess) throw std::runtime_error(std::string("gemm_pair smem attribute: ") + cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_done[dev] = true;
  }
  pair::k_gemm_pair<256><<<2 * pairs, pair::kThreads, P::kSmemBytes, s>>>(ma, mb, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("gemm_pair launch: ") + cudaGetErrorString(e));
}

}  // namespace tc
}  // namespace sn

void register_gemm_pair(py::module_& m) {
  m.def("gemm_pair", &sn::tc::gemm_pair, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("err"),
        py::arg("max_pairs") = 0,
        "C = A @ B.T on CTA pairs (tcgen05 cta_group::2, 256 x 256 tile per pair; bf16 in, fp32 accumulate)");
}
