// tcgen05 GEMMs for sm_100a: a plain persistent GEMM and the tensor-parallel prefill
// kernels that fuse a collective into it (one launch each):
//
//   gemm      C = A B^T
//   ag_gemm   C = allgather_rows(A_shard) B^T.  Copy CTAs push this rank's rows of A,
//             128-row chunk by chunk, into slot [parity][rank] of every peer's
//             symmetric region and raise a flag per chunk; GEMM CTAs start on their
//             own rows (read in place) and TMA-load a peer's chunk from this GPU's
//             own slot once its flag is up.  Chunk-major tile order: chunk c of every
//             shard is computed while chunk c+1 is in flight.
//   gemm_rs   C_shard = reduce_scatter_rows(A B^T).  Output row blocks are computed
//             in owner-interleaved order; the epilogue stores each bf16 tile straight
//             into slot [parity][rank] of the owner's region (P2P stores) and raises
//             the owner's flag for that tile; after its last tile each CTA's
//             epilogue warps sum, tile by tile as flags arrive, the world's partials
//             of this rank's rows in fixed rank order (fp32), rounding once.
//
// A fused launch is a collective: it reads the device-resident epoch at entry
// (graph-replayable), its flag waits are bounded and report into the runtime's
// status record, and its completion advances the epoch.
//
// Reference: none (the reference has no GEMM; its prefill collectives go to NCCL).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <torch/extension.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "sparknet/dev_mem.cuh"
#include "sparknet/gemm_fused.h"
#include "sparknet/proto.h"
#include "sparknet/tc_gemm.cuh"

namespace py = pybind11;

namespace sn {
namespace tc {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) throw std::runtime_error("libcuda.so.1 not found");
    fn = reinterpret_cast<EncodeFn>(dlsym(lib, "cuTensorMapEncodeTiled"));
    if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled not found");
  }
  return fn;
}

CUtensorMap make_map(const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows, int elem_bytes) {
  if (elem_bytes != 1 && elem_bytes != 2) throw std::invalid_argument("TMA maps are over 1- or 2-byte elements");
  if (reinterpret_cast<uintptr_t>(base) % 16 || (ld * elem_bytes) % 16)
    throw std::invalid_argument("TMA needs 16-byte alignment");
  if (box_rows < 1 || box_rows > 256) throw std::invalid_argument("TMA box rows must be 1..256");
  CUtensorMap map;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * elem_bytes};
  cuuint32_t box[2] = {uint32_t(128 / elem_bytes), box_rows};  // 128 bytes: one swizzle row
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode_fn()(&map, elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                           const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return map;
}

namespace {

constexpr int kThreads = 192;   // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kWarps = kThreads / 32;
constexpr int kEpiWarps = 4;
constexpr int kGroupM = 16;     // row blocks per rasterisation band
constexpr int kCopyPpt = 4;     // all-gather copy CTAs: packs in flight per thread

struct GemmParams {
  int M, N, K;
  __nv_bfloat16* C;  // plain: output; rs: this rank's reduced rows [shard_rows, N]
  int ldc;
  uint32_t* err;
  int mode;          // 0 plain, 1 all-gather -> GEMM, 2 GEMM -> reduce-scatter
  RegionDesc reg;
  int shard_rows;    // rows per rank (ag: of A; rs: of C)
  int slot_rows;     // rows per push slot (ag)
  // ag copy role
  const char* shard;
  int copy_ctas;
  // fp8: UE8M0 scale chunks (512 bytes per 128 rows and 128 K), laid out [row block][K block]
  const uint8_t* sfa;       // A's (ag: this rank's shard's)
  const uint8_t* sfb;
  uint64_t sfa_slot_off;    // ag: byte offset of the pushed shard's scales inside a push slot
};

struct Seq {
  uint32_t seq;
  uint32_t parity;
};

__device__ __forceinline__ Ctrl* ctrl_of(const GemmParams& p) {
  return reinterpret_cast<Ctrl*>(p.reg.base[p.reg.rank] + p.reg.ctrl_off);
}

__device__ __forceinline__ uint32_t* gflag(const GemmParams& p, int owner, int src, int idx) {
  return reinterpret_cast<uint32_t*>(p.reg.base[owner] + p.reg.gflag_off) + size_t(src) * kGFlags + idx;
}

__device__ __forceinline__ char* slot(const GemmParams& p, int owner, uint32_t parity, int src) {
  return p.reg.base[owner] + p.reg.push_off + (uint64_t(parity) * p.reg.world + src) * p.reg.push_cap;
}

// Bounded wait on a flag (in this GPU's memory) until it reaches `want`.
__device__ __forceinline__ bool wait_flag(const uint32_t* f, uint32_t want, const OpCtx& c, uint32_t peer) {
  DevMem m;
  WaitState w;
  while (int32_t(m.ld_acquire_u32(f) - want) < 0) {
    if (!keep_waiting(m, w, c, peer)) return false;
  }
  return true;
}

// F8: A and B are e4m3 with UE8M0 block scales (kind::mxf8f6f4.block_scale); one K
// block is 128 elements instead of 64, the tiles have the same bytes.
template <int BN, int STAGES, bool F8>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
           const __grid_constant__ CUtensorMap map_b, GemmParams p) {
  using S = Smem<BN, STAGES, F8>;
  constexpr int kBKe = F8 ? 128 : kBK;          // K elements per stage
  constexpr int kEsz = F8 ? 1 : 2;              // bytes per element
  constexpr uint32_t kTmemCols = F8 ? 512u : uint32_t(2 * BN);
  constexpr uint32_t kSfaCol = 2 * BN, kSfbCol = 2 * BN + 4;  // fp8 scale columns after the accumulators
  static_assert(!F8 || 2 * BN + 4 + BN / 32 <= 512, "accumulators and scale columns must fit TMEM");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sf_smem = smem + STAGES * S::kStageBytes;             // STAGES x S::kSfBytes
  uint8_t* epi_stage = sf_smem + STAGES * S::kSfBytes;           // S::kEpiStageBytes
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + S::kEpiStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ uint32_t err_local;
  __shared__ uint32_t tile_done[2];  // epilogue warps done with the tile in accumulator 0/1
  __shared__ Seq sq;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile uint32_t* err = &err_local;
  const bool fused = p.mode != 0;
  DevMem m;

  if (threadIdx.x == 0) {
    err_local = 0;
    tile_done[0] = tile_done[1] = 0;
    sq.seq = 0;
    sq.parity = 0;
    if (fused) {
      uint32_t epoch, poison;
      m.ld_volatile_pair(&ctrl_of(p)->epoch, epoch, poison);
      sq.seq = poison ? 0u : next_seq(epoch);
      sq.parity = sq.seq & 1u;
    }
  }
  __syncthreads();
  if (fused && sq.seq == 0) return;  // poisoned: every CTA leaves at entry
  const uint32_t seq = sq.seq, parity = sq.parity;
  const int W = p.reg.world, rank = p.reg.rank;
  OpCtx octx{fused ? ctrl_of(p) : nullptr, p.reg.status, seq, uint32_t(rank), blockIdx.x,
             uint32_t(p.mode == 1 ? kOpAgGemm : kOpGemmRs)};
  const int copy_ctas = p.mode == 1 ? p.copy_ctas : 0;

  // ---- copy CTAs (all-gather): push this rank's shard to every peer, flag per chunk.
  // Work units are chunks, split into `slices` pieces only when there are fewer chunks
  // than copy CTAs (slices = copy_ctas / chunks), taken in chunk order.  An unsplit
  // chunk's CTA raises the chunk's flag at every peer itself (a system-scope release,
  // cumulative over the CTA's stores after the barrier).  For a split chunk, each CTA
  // orders its stores before its count with a system-scope fence, and the CTA that
  // completes the count (a counter in this rank's control words, reset by that CTA)
  // fences again and raises the flags.
  if (int(blockIdx.x) < copy_ctas) {
    const int chunks = p.shard_rows / kBM;
    const int slices = max(1, copy_ctas / max(1, chunks));
    const uint64_t chunk_packs = uint64_t(kBM) * p.K * kEsz / kPack;
    const uint64_t sf_packs = F8 ? uint64_t(p.K / kBKe) * 512 / kPack : 0;  // the chunk's scales
    Ctrl* ctrl = ctrl_of(p);
    for (int u = blockIdx.x; u < chunks * slices; u += copy_ctas) {
      const int c = u / slices, sl = u % slices;
      const uint64_t lo = chunk_packs * sl / slices, hi = chunk_packs * (sl + 1) / slices;
      const uint64_t slo = sf_packs * sl / slices, shi = sf_packs * (sl + 1) / slices;
      const Pack16* src = reinterpret_cast<const Pack16*>(p.shard) + uint64_t(c) * chunk_packs;
      // kCopyPpt packs in flight per thread before the stores
      for (uint64_t i0 = lo + threadIdx.x; i0 < hi; i0 += uint64_t(kCopyPpt) * blockDim.x) {
        Pack16 v[kCopyPpt];
#pragma unroll
        for (int k2 = 0; k2 < kCopyPpt; ++k2) {
          const uint64_t i = i0 + uint64_t(k2) * blockDim.x;
          if (i < hi) v[k2] = m.ld_input(src + i);
        }
#pragma unroll
        for (int k2 = 0; k2 < kCopyPpt; ++k2) {
          const uint64_t i = i0 + uint64_t(k2) * blockDim.x;
          if (i < hi)
            for (int k = 1; k < W; ++k) {
              const int q = (rank + k) % W;
              m.st_remote(reinterpret_cast<Pack16*>(slot(p, q, parity, rank)) + uint64_t(c) * chunk_packs + i,
                          v[k2]);
            }
        }
      }
      if (F8) {
        const Pack16* ssrc = reinterpret_cast<const Pack16*>(p.sfa) + uint64_t(c) * sf_packs;
        for (uint64_t i = slo + threadIdx.x; i < shi; i += blockDim.x) {
          Pack16 v = m.ld_input(ssrc + i);
          for (int k = 1; k < W; ++k) {
            const int q = (rank + k) % W;
            m.st_remote(reinterpret_cast<Pack16*>(slot(p, q, parity, rank) + p.sfa_slot_off) +
                            uint64_t(c) * sf_packs + i, v);
          }
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        bool raise = slices == 1;
        if (!raise) {
          m.fence_sys();
          const uint32_t prev = atomicAdd(&ctrl->chunk_count[c], 1u);
          if (prev == uint32_t(slices) - 1u) {
            m.fence_sys();
            ctrl->chunk_count[c] = 0;  // every slice counted: re-armed for the next collective
            raise = true;
          }
        }
        if (raise)
          for (int k = 1; k < W; ++k) m.st_release_u32(gflag(p, (rank + k) % W, rank, c), seq);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) finish_op(m, ctrl_of(p), seq, gridDim.x);
    return;
  }

  const int cta = blockIdx.x - copy_ctas, ncta = gridDim.x - copy_ctas;
  const int tiles_m = (p.M + kBM - 1) / kBM, tiles_n = (p.N + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int kblocks = p.K / kBKe;
  const int bps = fused ? p.shard_rows / kBM : 1;  // row blocks per shard
  // Tile order.  Tiles go in bands of kGroupM row blocks; inside a band the row block
  // varies fastest, so the ~148 tiles in flight cover a compact 16 x 9 block whose A
  // and B tiles stay in L2 (raster along N re-reads all of B for every row block).
  // Logical row block i maps to a physical one by mode.  ag: chunk-major over shards
  // starting at this rank (own rows are ready first, chunk c of every shard before
  // chunk c+1).  rs: owner-interleaved starting with the next rank, so every link
  // carries traffic all along and each owner's tiles arrive progressively.
  auto tile_coord = [&](int t, int& m0, int& n0) {
    const int band = t / (kGroupM * tiles_n);
    const int rows_in_band = min(kGroupM, tiles_m - band * kGroupM);
    const int inner = t - band * kGroupM * tiles_n;
    const int i = band * kGroupM + inner % rows_in_band, nb = inner / rows_in_band;
    int mb = i;
    if (p.mode == 1) mb = ((rank + i % W) % W) * bps + i / W;
    else if (p.mode == 2) mb = ((rank + 1 + i % W) % W) * bps + i / W;
    m0 = mb * kBM;
    n0 = nb * BN;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
    if (p.mode == 1) prefetch_tmap(&map_a2);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = cta; t < tiles && ok; t += ncta) {
        int m0, n0;
        tile_coord(t, m0, n0);
        const CUtensorMap* amap = &map_a;
        int arow = m0;
        const uint8_t* sfa_src = F8 ? p.sfa + size_t(m0 / kBM) * kblocks * 512 : nullptr;
        if (p.mode == 1) {
          const int shard = m0 / p.shard_rows, r_in = m0 % p.shard_rows;
          if (shard == rank) {
            arow = r_in;
            if (F8) sfa_src = p.sfa + size_t(r_in / kBM) * kblocks * 512;
          } else {
            if (!wait_flag(gflag(p, rank, shard, r_in / kBM), seq, octx, uint32_t(shard))) {
              *err = kTcFlagTimeout;
              ok = false;
              break;
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");  // peer's stores before TMA reads
            amap = &map_a2;
            arow = int((parity * W + shard) * p.slot_rows) + r_in;
            if (F8)
              sfa_src = reinterpret_cast<const uint8_t*>(slot(p, rank, parity, shard) + p.sfa_slot_off) +
                        size_t(r_in / kBM) * kblocks * 512;
          }
        }
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_expect_tx(&full[stage], S::kStageBytes + S::kSfBytes);
          tma_load_2d(sa, amap, kb * kBKe, arow, &full[stage]);
          tma_load_2d(sb, &map_b, kb * kBKe, n0, &full[stage]);
          if (F8) {
            uint8_t* sfs = sf_smem + stage * S::kSfBytes;
            bulk_load(sfs, sfa_src + size_t(kb) * 512, 512, &full[stage]);
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              bulk_load(sfs + 512 * (1 + j), p.sfb + (size_t(n0 / 128 + j) * kblocks + kb) * 512, 512, &full[stage]);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = F8 ? idesc_mxf8(BN) : idesc_bf16(BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cta; t < tiles && ok; t += ncta) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + uint32_t(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          const uint64_t adesc = smem_desc_sw128(sa), bdesc = smem_desc_sw128(sb);
          if (F8) {
            // scales of this K block -> TMEM (ordered before the MMAs below by the
            // tcgen05 pipeline of this thread), then four K=32 steps
            uint8_t* sfs = sf_smem + stage * S::kSfBytes;
            tmem_cp_sf(tmem_base + kSfaCol, smem_desc_sf(sfs));
#pragma unroll
            for (int j = 0; j < BN / 128; ++j) tmem_cp_sf(tmem_base + kSfbCol + 4 * j, smem_desc_sf(sfs + 512 * (1 + j)));
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_mxf8(d, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc, tmem_base + kSfaCol,
                       tmem_base + kSfbCol, uint32_t(k), (kb | k) ? 1u : 0u);
          } else {
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              // +32 bytes per 16-element K step inside the 128-byte swizzle atom
              mma_bf16(d, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc, (kb | k) ? 1u : 0u);
            }
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      mma_commit(drain);  // fires once every MMA this thread issued has completed
      mbar_wait(drain, 0, err);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;  // TMEM lanes 32*quad .. +31
    const int row = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cta; t < tiles; t += ncta) {
      int m0, n0;
      tile_coord(t, m0, n0);
      if (!mbar_wait(&tfull[acc], acc_phase, err)) break;
      tc_fence_after();
      const int gm = m0 + row;
      const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * BN);
      const int owner = p.mode == 2 ? m0 / p.shard_rows : 0;
      (void)gm;
      // 64 columns at a time: TMEM -> registers (this thread's row) -> staging rows ->
      // coalesced stores, 8 lanes per 128-byte row segment (4 rows per instruction).
      uint8_t* wst = epi_stage + (warp - 2) * 32 * S::kStageRowBytes;
#pragma unroll 1
      for (int c = 0; c < BN / 64; ++c) {
        float v[64];
        tmem_ld32(taddr + uint32_t(c * 64), v);
        tmem_ld32(taddr + uint32_t(c * 64 + 32), v + 32);
        uint4* my_row = reinterpret_cast<uint4*>(wst + lane * S::kStageRowBytes);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint4 pk;
          pk.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
          pk.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
          pk.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
          pk.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
          my_row[q] = pk;
        }
        __syncwarp();
        const int gn = n0 + c * 64 + (lane & 7) * 8;
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          const int r = rr * 4 + (lane >> 3);            // row within this warp's 32
          const int grow = m0 + quad * 32 + r;
          const uint4 pk = *reinterpret_cast<const uint4*>(wst + r * S::kStageRowBytes + (lane & 7) * 16);
          if (grow < p.M && gn < p.N) {
            Pack16 v16;
            v16.w[0] = pk.x;
            v16.w[1] = pk.y;
            v16.w[2] = pk.z;
            v16.w[3] = pk.w;
            if (p.mode == 2) {
              const int owner_r = grow - owner * p.shard_rows;
              m.st_remote(reinterpret_cast<Pack16*>(reinterpret_cast<__nv_bfloat16*>(slot(p, owner, parity, rank)) +
                                                    size_t(owner_r) * p.N + gn), v16);
            } else {
              m.st_local(reinterpret_cast<Pack16*>(p.C + size_t(grow) * p.ldc + gn), v16);
            }
          }
        }
        __syncwarp();
      }
      __syncwarp();  // the warp's stores are ordered before lane 0's count below
      if (p.mode == 2 && lane == 0) {
        // Publish the tile to its owner once all four epilogue warps stored their rows.
        // Each warp counts in with a CTA-scope release; the fourth raises the owner's
        // flag with a system-scope release, which is cumulative over the stores the
        // counts ordered before it.  Counting happens before the accumulator is
        // released, so no warp can run two tiles ahead and count for the wrong tile.
        // No CTA barrier: a warp that gave up on a wait cannot strand the others.
        uint32_t prev;
        asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "r"(smem_u32(&tile_done[acc]))
                     : "memory");
        if (prev % kEpiWarps == kEpiWarps - 1) {
          const int tile_in = ((m0 - owner * p.shard_rows) / kBM) * tiles_n + n0 / BN;
          m.st_release_u32(gflag(p, owner, rank, tile_in), seq);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (p.mode == 2 && !*err) {
      // ---- reduce this rank's rows: item = (row block, BN columns); warp takes 32 rows
      const int items = bps * tiles_n;
      const char* mine = p.reg.base[rank];
      for (int it = cta; it < items; it += ncta) {
        bool ok = true;
        if (lane < W) ok = wait_flag(gflag(p, rank, lane, it), seq, octx, uint32_t(lane));
        if (!__all_sync(0xffffffffu, ok)) {
          *err = kTcFlagTimeout;
          break;
        }
        const int r0 = (it / tiles_n) * kBM + quad * 32, c0 = (it % tiles_n) * BN;
        for (int e = lane; e < 32 * (BN / 8); e += 32) {
          const int r = r0 + e / (BN / 8), c = c0 + (e % (BN / 8)) * 8;
          if (r >= p.shard_rows || c >= p.N) continue;
          Acc a;
          acc_zero<kBF16>(a);
          for (int s = 0; s < W; ++s) {
            const Pack16* src = reinterpret_cast<const Pack16*>(
                mine + p.reg.push_off + (uint64_t(parity) * W + s) * p.reg.push_cap) + (size_t(r) * p.N + c) / 8;
            acc_add<kBF16>(a, m.ld_peer_data(src));
          }
          m.st_output(reinterpret_cast<Pack16*>(p.C + size_t(r) * p.ldc + c), acc_round<kBF16>(a));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) {
    if (err_local) atomicExch(p.err, err_local);
    if (fused) finish_op(m, ctrl_of(p), seq, gridDim.x);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <int BN, int STAGES, bool F8 = false>
void launch(const CUtensorMap& a, const CUtensorMap& a2, const CUtensorMap& b, const GemmParams& p, int grid,
            cudaStream_t s) {
  using S = Smem<BN, STAGES, F8>;
  static_assert(S::kBytes <= 227 * 1024, "shared memory plan exceeds the per-CTA limit");
  auto kern = k_gemm<BN, STAGES, F8>;
  // function attributes belong to each device's context: set once per device
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
    if (e != cudaSuccess) throw std::runtime_error(std::string("gemm smem attribute: ") + cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_done[dev] = true;
  }
  kern<<<grid, kThreads, S::kBytes, s>>>(a, a2, b, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("gemm launch: ") + cudaGetErrorString(e));
}

void check_mat(const at::Tensor& t, const char* name) {
  if (!t.is_cuda() || t.scalar_type() != at::kBFloat16 || t.dim() != 2 || t.stride(1) != 1)
    throw std::invalid_argument(std::string(name) + " must be a row-major 2-D CUDA bfloat16 tensor");
}

int sm_count(int device) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  return n;
}

GemmParams base_params(int M, int N, int K, at::Tensor& C, at::Tensor& err) {
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = reinterpret_cast<__nv_bfloat16*>(C.data_ptr());
  p.ldc = int(C.stride(0));
  p.err = reinterpret_cast<uint32_t*>(err.data_ptr());
  return p;
}

}  // namespace

// C[M,N] = A[M,K] B[N,K]^T
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, at::Tensor& err, int bn, int max_ctas) {
  check_mat(A, "A");
  check_mat(B, "B");
  check_mat(C, "C");
  const int M = int(A.size(0)), K = int(A.size(1)), N = int(B.size(0));
  if (B.size(1) != K || C.size(0) != M || C.size(1) != N) throw std::invalid_argument("shape mismatch");
  if (K % kBK) throw std::invalid_argument("K must be a multiple of 64");
  if (N % 32) throw std::invalid_argument("N must be a multiple of 32");
  c10::cuda::CUDAGuard guard(A.device());
  GemmParams p = base_params(M, N, K, C, err);
  CUtensorMap ma = make_map(A.data_ptr(), M, K, A.stride(0), kBM);
  auto s = at::cuda::getCurrentCUDAStream(A.device().index()).stream();
  int sms = max_ctas > 0 ? max_ctas : sm_count(A.device().index());
  if (bn == 128) {
    CUtensorMap mb = make_map(B.data_ptr(), N, K, B.stride(0), 128);
    int tiles = ((M + 127) / 128) * ((N + 127) / 128);
    launch<128, 6>(ma, ma, mb, p, std::min(tiles, sms), s);
  } else {
    CUtensorMap mb = make_map(B.data_ptr(), N, K, B.stride(0), 256);
    int tiles = ((M + 127) / 128) * ((N + 255) / 256);
    launch<256, 4>(ma, ma, mb, p, std::min(tiles, sms), s);
  }
}

void ag_gemm(const RegionDesc& reg, const at::Tensor& x_shard, const at::Tensor& B, at::Tensor& C, at::Tensor& err,
             int copy_ctas, int max_ctas) {
  check_mat(x_shard, "x_shard");
  check_mat(B, "B");
  check_mat(C, "C");
  const int W = reg.world;
  const int shard_rows = int(x_shard.size(0)), K = int(x_shard.size(1)), N = int(B.size(0));
  const int M = shard_rows * W;
  if (!x_shard.is_contiguous() || B.size(1) != K || C.size(0) != M || C.size(1) != N)
    throw std::invalid_argument("ag_gemm shapes: x_shard [T/W, K], B [N, K], C [T, N]");
  if (shard_rows % kBM || K % kBK || N % 32) throw std::invalid_argument("ag_gemm needs T/W % 128, K % 64, N % 32");
  const uint64_t row_bytes = uint64_t(K) * 2;
  if (reg.push_cap % row_bytes || reg.push_cap / row_bytes < uint64_t(shard_rows))
    throw std::invalid_argument("the shard does not fit a push slot (raise max_gather_bytes)");
  if (shard_rows / kBM > kChunkCounters) throw std::invalid_argument("too many 128-row chunks per shard");
  c10::cuda::CUDAGuard guard(x_shard.device());
  GemmParams p = base_params(M, N, K, C, err);
  p.mode = 1;
  p.reg = reg;
  p.shard_rows = shard_rows;
  p.slot_rows = int(reg.push_cap / row_bytes);
  p.shard = static_cast<const char*>(x_shard.data_ptr());
  p.copy_ctas = W > 1 ? std::max(1, copy_ctas) : 0;
  CUtensorMap ma = make_map(x_shard.data_ptr(), shard_rows, K, K, kBM);
  // every push slot of this rank's region, both parities, as one [2*W*slot_rows, K] matrix
  CUtensorMap ma2 = make_map(reg.base[reg.rank] + reg.push_off, uint64_t(2) * W * p.slot_rows, K, K, kBM);
  CUtensorMap mb = make_map(B.data_ptr(), N, K, B.stride(0), 256);
  auto s = at::cuda::getCurrentCUDAStream(x_shard.device().index()).stream();
  int sms = max_ctas > 0 ? max_ctas : sm_count(x_shard.device().index());
  const int tiles = (M / kBM) * ((N + 255) / 256);
  launch<256, 4>(ma, ma2, mb, p, std::min(tiles, sms - p.copy_ctas) + p.copy_ctas, s);
}

void gemm_rs(const RegionDesc& reg, const at::Tensor& A, const at::Tensor& B, at::Tensor& C_shard, at::Tensor& err,
             int max_ctas) {
  check_mat(A, "A");
  check_mat(B, "B");
  check_mat(C_shard, "C_shard");
  const int W = reg.world;
  const int M = int(A.size(0)), K = int(A.size(1)), N = int(B.size(0));
  if (B.size(1) != K || M % W || C_shard.size(0) != M / W || C_shard.size(1) != N)
    throw std::invalid_argument("gemm_rs shapes: A [T, K], B [N, K], C_shard [T/W, N]");
  const int shard_rows = M / W;
  if (shard_rows % kBM || K % kBK || N % 256) throw std::invalid_argument("gemm_rs needs T/W % 128, K % 64, N % 256");
  if (uint64_t(shard_rows) * N * 2 > reg.push_cap) throw std::invalid_argument("the partial does not fit a push slot");
  if ((shard_rows / kBM) * (N / 256) > kGFlags) throw std::invalid_argument("too many tiles per shard");
  c10::cuda::CUDAGuard guard(A.device());
  GemmParams p = base_params(M, N, K, C_shard, err);
  p.mode = 2;
  p.reg = reg;
  p.shard_rows = shard_rows;
  CUtensorMap ma = make_map(A.data_ptr(), M, K, A.stride(0), kBM);
  CUtensorMap mb = make_map(B.data_ptr(), N, K, B.stride(0), 256);
  auto s = at::cuda::getCurrentCUDAStream(A.device().index()).stream();
  int sms = max_ctas > 0 ? max_ctas : sm_count(A.device().index());
  const int tiles = (M / kBM) * (N / 256);
  launch<256, 4>(ma, ma, mb, p, std::min(tiles, sms), s);
}

// ---------------------------------------------------------------------------
// Block-scaled fp8 (e4m3 operands, UE8M0 scales per 128 rows and 128 K of each operand
// -- 1 x 128 for activations, 128 x 128 for weights, both expanded to per-row chunks;
// layout in fp8_quant.cu).  BN = 128: two 128-column accumulators plus the scale
// columns fit TMEM's 512 columns.
// ---------------------------------------------------------------------------
namespace {

void check_fp8_mat(const at::Tensor& t, const char* name) {
  if (!t.is_cuda() || t.element_size() != 1 || t.dim() != 2 || t.stride(1) != 1)
    throw std::invalid_argument(std::string(name) + " must be a row-major 2-D CUDA tensor of 1-byte (e4m3) elements");
}

void check_sf(const at::Tensor& sf, int rows, int K, const char* name) {
  const int64_t need = int64_t((rows + 127) / 128) * (K / 128) * 512;
  if (!sf.is_cuda() || sf.element_size() != 1 || !sf.is_contiguous() || sf.numel() < need ||
      reinterpret_cast<uintptr_t>(sf.data_ptr()) % 16)
    throw std::invalid_argument(std::string(name) + ": scales must be a contiguous 16-byte aligned CUDA byte tensor of " +
                                std::to_string(need) + " bytes");
}

constexpr int kF8BN = 128, kF8Stages = 6;

}  // namespace

void gemm_fp8(const at::Tensor& A, const at::Tensor& sfa, const at::Tensor& B, const at::Tensor& sfb, at::Tensor& C,
              at::Tensor& err, int max_ctas) {
  check_fp8_mat(A, "A");
  check_fp8_mat(B, "B");
  check_mat(C, "C");
  const int M = int(A.size(0)), K = int(A.size(1)), N = int(B.size(0));
  if (B.size(1) != K || C.size(0) != M || C.size(1) != N) throw std::invalid_argument("shape mismatch");
  if (K % 128 || N % 128) throw std::invalid_argument("fp8 GEMM needs K and N multiples of 128");
  check_sf(sfa, M, K, "sfa");
  check_sf(sfb, N, K, "sfb");
  c10::cuda::CUDAGuard guard(A.device());
  GemmParams p = base_params(M, N, K, C, err);
  p.sfa = static_cast<const uint8_t*>(sfa.data_ptr());
  p.sfb = static_cast<const uint8_t*>(sfb.data_ptr());
  CUtensorMap ma = make_map(A.data_ptr(), M, K, A.stride(0), kBM, 1);
  CUtensorMap mb = make_map(B.data_ptr(), N, K, B.stride(0), kF8BN, 1);
  auto s = at::cuda::getCurrentCUDAStream(A.device().index()).stream();
  int sms = max_ctas > 0 ? max_ctas : sm_count(A.device().index());
  const int tiles = ((M + 127) / 128) * (N / kF8BN);
  launch<kF8BN, kF8Stages, true>(ma, ma, mb, p, std::min(tiles, sms), s);
}

void ag_gemm_fp8(const RegionDesc& reg, const at::Tensor& xq_shard, const at::Tensor& sfa_shard, const at::Tensor& B,
                 const at::Tensor& sfb, at::Tensor& C, at::Tensor& err, int copy_ctas, int max_ctas) {
  check_fp8_mat(xq_shard, "xq_shard");
  check_fp8_mat(B, "B");
  check_mat(C, "C");
  const int W = reg.world;
  const int shard_rows = int(xq_shard.size(0)), K = int(xq_shard.size(1)), N = int(B.size(0));
  const int M = shard_rows * W;
  if (!xq_shard.is_contiguous() || B.size(1) != K || C.size(0) != M || C.size(1) != N)
    throw std::invalid_argument("ag_gemm_fp8 shapes: xq_shard [T/W, K], B [N, K], C [T, N]");
  if (shard_rows % kBM || K % 128 || N % kF8BN) throw std::invalid_argument("ag_gemm_fp8 needs T/W % 128, K % 128, N % 128");
  check_sf(sfa_shard, shard_rows, K, "sfa_shard");
  check_sf(sfb, N, K, "sfb");
  const uint64_t data_bytes = uint64_t(shard_rows) * K;
  const uint64_t sf_bytes = uint64_t(shard_rows / 128) * (K / 128) * 512;
  if (reg.push_cap % uint64_t(K) || reg.push_cap < data_bytes + sf_bytes)
    throw std::invalid_argument("the fp8 shard and its scales do not fit a push slot (raise max_gather_bytes)");
  if (shard_rows / kBM > kChunkCounters) throw std::invalid_argument("too many 128-row chunks per shard");
  c10::cuda::CUDAGuard guard(xq_shard.device());
  GemmParams p = base_params(M, N, K, C, err);
  p.mode = 1;
  p.reg = reg;
  p.shard_rows = shard_rows;
  p.slot_rows = int(reg.push_cap / uint64_t(K));
  p.shard = static_cast<const char*>(xq_shard.data_ptr());
  p.copy_ctas = W > 1 ? std::max(1, copy_ctas) : 0;
  p.sfa = static_cast<const uint8_t*>(sfa_shard.data_ptr());
  p.sfb = static_cast<const uint8_t*>(sfb.data_ptr());
  p.sfa_slot_off = data_bytes;
  CUtensorMap ma = make_map(xq_shard.data_ptr(), shard_rows, K, K, kBM, 1);
  CUtensorMap ma2 = make_map(reg.base[reg.rank] + reg.push_off, uint64_t(2) * W * p.slot_rows, K, K, kBM, 1);
  CUtensorMap mb = make_map(B.data_ptr(), N, K, B.stride(0), kF8BN, 1);
  auto s = at::cuda::getCurrentCUDAStream(xq_shard.device().index()).stream();
  int sms = max_ctas > 0 ? max_ctas : sm_count(xq_shard.device().index());
  const int tiles = (M / kBM) * (N / kF8BN);
  launch<kF8BN, kF8Stages, true>(ma, ma2, mb, p, std::min(tiles, sms - p.copy_ctas) + p.copy_ctas, s);
}

void gemm_rs_fp8(const RegionDesc& reg, const at::Tensor& A, const at::Tensor& sfa, const at::Tensor& B,
                 const at::Tensor& sfb, at::Tensor& C_shard, at::Tensor& err, int max_ctas) {
  check_fp8_mat(A, "A");
  check_fp8_mat(B, "B");
  check_mat(C_shard, "C_shard");
  const int W = reg.world;
  const int M = int(A.size(0)), K = int(A.size(1)), N = int(B.size(0));
  if (B.size(1) != K || M % W || C_shard.size(0) != M / W || C_shard.size(1) != N)
    throw std::invalid_argument("gemm_rs_fp8 shapes: A [T, K], B [N, K], C_shard [T/W, N]");
  const int shard_rows = M / W;
  if (shard_rows % kBM || K % 128 || N % kF8BN) throw std::invalid_argument("gemm_rs_fp8 needs T/W % 128, K % 128, N % 128");
  check_sf(sfa, M, K, "sfa");
  check_sf(sfb, N, K, "sfb");
  if (uint64_t(shard_rows) * N * 2 > reg.push_cap) throw std::invalid_argument("the partial does not fit a push slot");
  if ((shard_rows / kBM) * (N / kF8BN) > kGFlags) throw std::invalid_argument("too many tiles per shard");
  c10::cuda::CUDAGuard guard(A.device());
  GemmParams p = base_params(M, N, K, C_shard, err);
  p.mode = 2;
  p.reg = reg;
  p.shard_rows = shard_rows;
  p.sfa = static_cast<const uint8_t*>(sfa.data_ptr());
  p.sfb = static_cast<const uint8_t*>(sfb.data_ptr());
  CUtensorMap ma = make_map(A.data_ptr(), M, K, A.stride(0), kBM, 1);
  CUtensorMap mb = make_map(B.data_ptr(), N, K, B.stride(0), kF8BN, 1);
  auto s = at::cuda::getCurrentCUDAStream(A.device().index()).stream();
  int sms = max_ctas > 0 ? max_ctas : sm_count(A.device().index());
  const int tiles = (M / kBM) * (N / kF8BN);
  launch<kF8BN, kF8Stages, true>(ma, ma, mb, p, std::min(tiles, sms), s);
}

}  // namespace tc
}  // namespace sn

void register_gemm(py::module_& m) {
  m.def("gemm", &sn::tc::gemm, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("err"), py::arg("bn") = 256,
        py::arg("max_ctas") = 0, "C = A @ B.T on tcgen05 tensor cores (bf16 in, fp32 accumulate)");
  m.def("gemm_fp8", &sn::tc::gemm_fp8, py::arg("A"), py::arg("sfa"), py::arg("B"), py::arg("sfb"), py::arg("C"),
        py::arg("err"), py::arg("max_ctas") = 0,
        "C = (A * sfa) @ (B * sfb).T: e4m3 operands with UE8M0 block scales (kind::mxf8f6f4), bf16 out");
}
