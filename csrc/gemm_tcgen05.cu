// tcgen05 GEMMs for sm_100a: a plain persistent GEMM and the tensor-parallel prefill
// kernels that fuse a collective into it:
//
//   gemm            C = A B^T
//   ag_gemm         C = allgather_rows(A_shard) B^T : copy CTAs push this rank's rows
//                   of A into every peer's symmetric slot and raise a flag per 128-row
//                   chunk; GEMM CTAs start on their own rows and load a peer's chunk
//                   (from local memory) once its flag is up.
//   gemm_rs         C_shard = reduce_scatter_rows(A B^T) : every output tile is sent,
//                   in bf16, to the rank that owns its rows (P2P stores from the
//                   epilogue, a flag per tile); each rank then sums the world's
//                   partials of its rows in fixed rank order (fp32) as they arrive.
//
// Reference: none (the reference has no GEMM; its prefill collectives go to NCCL).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <torch/extension.h>

#include <stdexcept>
#include <string>

#include "sparknet/dev_mem.cuh"
#include "sparknet/proto.h"
#include "sparknet/tc_gemm.cuh"

namespace py = pybind11;

namespace sn {
namespace tc {
namespace {

constexpr int kThreads = 192;   // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kEpiWarps = 4;

// ---------------------------------------------------------------------------
// Fusion hooks
// ---------------------------------------------------------------------------
struct AgFusion {
  // Rows of A are grouped in shards of `shard_rows` rows, shard s = rank s's rows.
  // The own shard is read through `map_local`, the others through `map_gather`
  // (this rank's symmetric slots), row = s * slot_rows + r.  A chunk of 128 rows of
  // shard s may be read once gflags[s * chunks_per_shard + chunk] >= seq.
  int world, rank, shard_rows, slot_rows, chunks_per_shard;
  const uint32_t* gflags;
  uint32_t seq;
};

struct RsFusion {
  // Output rows are owned in shards of `shard_rows` rows; a tile of owner c is sent
  // to peers[c] + slot_off(parity, this rank) and flagged at
  // peer_flags[c] + this_rank * tiles_per_shard + tile_in_shard.
  int world, rank, shard_rows, tiles_per_shard, tiles_n;
  char* peer_base[kMaxRanks];   // every rank's region (this rank's mapping)
  uint64_t slot_off[kMaxRanks]; // offset of slot [parity][src] for src = 0..W-1
  uint64_t gflag_off;
  uint32_t seq;
  int ldp;                       // elements per row of a partial slot (= N)
};

struct GemmParams {
  int M, N, K;
  __nv_bfloat16* C;
  int ldc;
  uint32_t* err;
  int mode;  // 0 plain, 1 ag, 2 rs
  AgFusion ag;
  RsFusion rs;
  // copy role (ag): this rank's shard, pushed to every peer
  const char* shard;
  uint64_t shard_bytes;
  char* peer_slot[kMaxRanks];       // peers' slot [parity][rank] (this rank's data lands there)
  uint32_t* peer_gflags[kMaxRanks]; // peers' gflags + rank * chunks_per_shard
  int copy_ctas;
  // completion bookkeeping of the symmetric region (ag / rs)
  Ctrl* ctrl;
  Status* status;
};


// Bounded wait on a flag in this GPU's memory written by a peer.
__device__ __forceinline__ bool wait_flag(const uint32_t* f, uint32_t want, volatile uint32_t* err) {
  DevMem m;
  for (uint32_t i = 0;; ++i) {
    if (int32_t(m.ld_acquire_u32(f) - want) >= 0) return true;
    if ((i & 255u) == 255u) {
      if (*err) return false;
      if (i > (1u << 26)) {
        *err = kTcFlagTimeout;
        return false;
      }
    }
  }
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
           const __grid_constant__ CUtensorMap map_b, GemmParams p) {
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ uint32_t err_local;
  __shared__ uint32_t tile_done[2];  // epilogue warps done with the tile in accumulator 0/1

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile uint32_t* err = &err_local;
  const int copy_ctas = p.mode == 1 ? p.copy_ctas : 0;

  // ---- copy CTAs (all-gather): push this rank's shard to every peer, flag per chunk
  if (int(blockIdx.x) < copy_ctas) {
    DevMem m;
    const uint64_t packs = p.shard_bytes / kPack;
    const uint64_t chunk_packs = packs / p.ag.chunks_per_shard;
    const int W = p.ag.world, r = p.ag.rank;
    for (int c = blockIdx.x; c < p.ag.chunks_per_shard; c += copy_ctas) {
      const Pack16* src = reinterpret_cast<const Pack16*>(p.shard) + uint64_t(c) * chunk_packs;
      for (uint64_t i = threadIdx.x; i < chunk_packs; i += blockDim.x) {
        Pack16 v = m.ld_input(src + i);
        for (int k = 1; k < W; ++k) {
          int q = (r + k) % W;
          m.st_remote(reinterpret_cast<Pack16*>(p.peer_slot[q]) + uint64_t(c) * chunk_packs + i, v);
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        m.fence_sys();
        for (int k = 1; k < W; ++k) {
          int q = (r + k) % W;
          m.st_release_u32(p.peer_gflags[q] + c, p.ag.seq);
        }
      }
      __syncthreads();
    }
    return;
  }

  const int cta = blockIdx.x - copy_ctas, ncta = gridDim.x - copy_ctas;
  const int tiles_m = (p.M + kBM - 1) / kBM, tiles_n = (p.N + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int kblocks = p.K / kBK;
  // the row-block order: all-gather starts on this rank's own shard, reduce-scatter
  // sends to the next owners first and finishes with its own rows
  auto tile_coord = [&](int t, int& m0, int& n0) {
    int mb = t / tiles_n, nb = t % tiles_n;
    if (p.mode == 1) {
      const int per = p.ag.shard_rows / kBM;
      mb = (mb + p.ag.rank * per) % tiles_m;
    } else if (p.mode == 2) {
      const int per = p.rs.shard_rows / kBM;
      mb = (mb + (p.rs.rank + 1) * per) % tiles_m;
    }
    m0 = mb * kBM;
    n0 = nb * BN;
  };

  if (threadIdx.x == 0) {
    err_local = 0;
    tile_done[0] = tile_done[1] = 0;
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
  if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
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
        if (p.mode == 1) {
          const int shard = m0 / p.ag.shard_rows, r_in = m0 % p.ag.shard_rows;
          if (shard == p.ag.rank) {
            arow = r_in;
          } else {
            if (!wait_flag(p.ag.gflags + shard * p.ag.chunks_per_shard + r_in / kBM, p.ag.seq, err)) {
              ok = false;
              break;
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");  // peer's stores -> TMA reads
            amap = &map_a2;
            arow = shard * p.ag.slot_rows + r_in;
          }
        }
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_expect_tx(&full[stage], S::kStageBytes);
          tma_load_2d(sa, amap, kb * kBK, arow, &full[stage]);
          tma_load_2d(sb, &map_b, kb * kBK, n0, &full[stage]);
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
      const uint32_t idesc = idesc_bf16(BN);
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
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // +32 bytes per 16-element K step inside the 128-byte swizzle atom
            mma_bf16(d, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc, (kb | k) ? 1u : 0u);
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
      // every MMA this thread issued has completed once `drain` fires
      mma_commit(drain);
      mbar_wait(drain, 0, err);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;               // TMEM lanes 32*quad .. +31
    const int row = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    DevMem m;
    for (int t = cta; t < tiles; t += ncta) {
      int m0, n0;
      tile_coord(t, m0, n0);
      if (!mbar_wait(&tfull[acc], acc_phase, err)) break;
      tc_fence_after();
      const int gm = m0 + row;
      const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * BN);
      // destination of this row of the tile
      __nv_bfloat16* dst_row = nullptr;
      if (p.mode == 2) {
        const int owner = m0 / p.rs.shard_rows;
        const int r_in = gm - owner * p.rs.shard_rows;
        char* base = p.rs.peer_base[owner] + p.rs.slot_off[p.rs.rank];
        dst_row = reinterpret_cast<__nv_bfloat16*>(base) + size_t(r_in) * p.rs.ldp;
      } else if (gm < p.M) {
        dst_row = p.C + size_t(gm) * p.ldc;
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(taddr + uint32_t(c * 32), v);
        const int gn = n0 + c * 32;
        if (dst_row != nullptr && gm < p.M && gn < p.N) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
          Pack16* out = reinterpret_cast<Pack16*>(dst_row + gn);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            Pack16 pk;
            pk.w[0] = w[4 * q];
            pk.w[1] = w[4 * q + 1];
            pk.w[2] = w[4 * q + 2];
            pk.w[3] = w[4 * q + 3];
            if (p.mode == 2) m.st_remote(out + q, pk);
            else m.st_local(out + q, pk);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (p.mode == 2 && lane == 0) {
        // Publish the tile to its owner once all four epilogue warps stored their rows.
        // No CTA barrier (a warp that gave up on a wait must not strand the others):
        // each warp fences its own stores at system scope, then counts in; the fourth
        // warp to count in raises the owner's flag.
        m.fence_sys();
        uint32_t prev;
        asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                     : "=r"(prev) : "r"(smem_u32(&tile_done[acc])) : "memory");
        if (prev % kEpiWarps == kEpiWarps - 1) {
          const int owner = m0 / p.rs.shard_rows;
          const int tile_in = ((m0 % p.rs.shard_rows) / kBM) * p.rs.tiles_n + n0 / BN;
          uint32_t* f = reinterpret_cast<uint32_t*>(p.rs.peer_base[owner] + p.rs.gflag_off) +
                        p.rs.rank * p.rs.tiles_per_shard + tile_in;
          m.st_release_u32(f, p.rs.seq);
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
  if (threadIdx.x == 0 && err_local) atomicExch(p.err, err_local);
}

// Reduce-scatter finish: sum the world's bf16 partials of this rank's rows in rank
// order (fp32), round once.  Work items are 128 x 256 tiles of the owned rows; each
// waits for the W flags of its tile.
__global__ void __launch_bounds__(256) k_rs_reduce(GemmParams p, __nv_bfloat16* out, int ldo) {
  DevMem m;
  const RsFusion& rs = p.rs;
  const int tiles_n = rs.tiles_n;
  const int items = rs.tiles_per_shard;
  __shared__ uint32_t err_local;
  if (threadIdx.x == 0) err_local = 0;
  __syncthreads();
  volatile uint32_t* err = &err_local;
  char* mine = rs.peer_base[rs.rank];
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(mine + rs.gflag_off);
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    if (threadIdx.x < uint32_t(rs.world)) {
      if (!wait_flag(flags + threadIdx.x * rs.tiles_per_shard + it, rs.seq, err)) {
      }
    }
    __syncthreads();
    if (*err) break;
    const int r0 = (it / tiles_n) * kBM, c0 = (it % tiles_n) * 256;
    // 128 rows x 256 cols = 4096 packs of 8 bf16
    for (int i = threadIdx.x; i < kBM * 32; i += blockDim.x) {
      const int r = r0 + i / 32, c = c0 + (i % 32) * 8;
      if (r >= rs.shard_rows || c >= rs.ldp) continue;
      Acc a;
      acc_zero<kBF16>(a);
      for (int s = 0; s < rs.world; ++s) {
        const Pack16* src =
            reinterpret_cast<const Pack16*>(mine + rs.slot_off[s]) + (size_t(r) * rs.ldp + c) / 8;
        acc_add<kBF16>(a, m.ld_peer_data(src));
      }
      m.st_output(reinterpret_cast<Pack16*>(out + size_t(r) * ldo + c), acc_round<kBF16>(a));
    }
    __syncthreads();
  }
  if (threadIdx.x == 0 && err_local) atomicExch(p.err, err_local);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) throw std::runtime_error("libcuda.so.1 not found");
    fn = reinterpret_cast<EncodeFn>(dlsym(lib, "cuTensorMapEncodeTiled"));
    if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled not found");
  }
  return fn;
}

// 2-D bf16 map over `rows` x `cols` (row-major, row pitch `ld` elements), box
// `box_rows` x 64 with 128-byte swizzle.
CUtensorMap make_map(const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || (ld * 2) % 16) throw std::invalid_argument("TMA needs 16-byte alignment");
  CUtensorMap map;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {uint32_t(kBK), box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return map;
}

template <int BN, int STAGES>
void launch_gemm(const CUtensorMap& a, const CUtensorMap& a2, const CUtensorMap& b, const GemmParams& p, int grid,
                 cudaStream_t s) {
  using S = Smem<BN, STAGES>;
  auto kern = k_gemm<BN, STAGES>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
    attr = true;
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
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = reinterpret_cast<__nv_bfloat16*>(C.data_ptr());
  p.ldc = int(C.stride(0));
  p.err = reinterpret_cast<uint32_t*>(err.data_ptr());
  p.mode = 0;
  CUtensorMap ma = make_map(A.data_ptr(), M, K, A.stride(0), kBM);
  auto s = at::cuda::getCurrentCUDAStream(A.device().index()).stream();
  int sms = max_ctas > 0 ? max_ctas : sm_count(A.device().index());
  if (bn == 128) {
    CUtensorMap mb = make_map(B.data_ptr(), N, K, B.stride(0), 128);
    int tiles = ((M + 127) / 128) * ((N + 127) / 128);
    launch_gemm<128, 6>(ma, ma, mb, p, std::min(tiles, sms), s);
  } else {
    CUtensorMap mb = make_map(B.data_ptr(), N, K, B.stride(0), 256);
    int tiles = ((M + 127) / 128) * ((N + 255) / 256);
    launch_gemm<256, 4>(ma, ma, mb, p, std::min(tiles, sms), s);
  }
}

}  // namespace

// -- fused prefill kernels, called by the communicator (comm.cpp) ----------------
struct PrefillDesc {
  // region views
  char* base[kMaxRanks];
  int world, rank;
  uint64_t slot_off[2][kMaxRanks];  // push slots: [parity][src]
  uint64_t gflag_off;
  uint64_t slot_bytes;
  Ctrl* ctrl;
};

}  // namespace tc
}  // namespace sn

void register_gemm(py::module_& m) {
  m.def("gemm", &sn::tc::gemm, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("err"), py::arg("bn") = 256,
        py::arg("max_ctas") = 0, "C = A @ B.T on tcgen05 tensor cores (bf16 in, fp32 accumulate)");
}
