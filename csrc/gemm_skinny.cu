// Decode GEMM for few tokens on tcgen05 tensor cores:
//
//   Y[M, N] = X[M, K] W[N, K]^T          M = tokens (1..256), W in nn.Linear layout
//
// With M this small the tensor cores idle and the job is streaming W from HBM, so
// the roles of the operands are swapped: 128 weight rows are the MMA's M side and
// the tokens, padded to a multiple of 16, its N side (D^T = W X^T, accumulated in
// TMEM as 128 lanes x tokens).  The grid is (ceil(N / 128) weight tiles) x (K
// splits), sized so one wave covers every SM with several 16 KB weight stages in
// flight per CTA.  Warp 0 issues the TMA loads (one elected thread), warp 1 the MMAs;
// after the last K block all four warps drain TMEM.  With several K splits each CTA
// stores its fp32 partial tile, and the last CTA of a weight tile to finish (an
// atomic counter per tile) sums the partials in split order, so results do not
// depend on which CTA finished last.
//
// Epilogues: mode 0 writes Y; mode 1 is SwiGLU over a gate/up weight whose 128-row
// tiles are [64 gate rows; 64 up rows] of the same 64 features, and writes
// Y[m, f] = silu(gate) * up for the N/2 features (no intermediate tensor); mode 2 is the
// QKV projection with RoPE (rotate-half, fp32) and the KV-cache write, one 128-row
// tile per head (no qkv tensor, no separate RoPE kernel).
//
// Every mbarrier wait is bounded (sets the error word and unwinds).
// Reference: none (the reference has no model GEMMs).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <algorithm>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "sparknet/dev_mem.cuh"
#include "sparknet/gemm_fused.h"
#include "sparknet/tc_gemm.cuh"

namespace py = pybind11;
namespace cg = cooperative_groups;

namespace sn {
namespace tc {
namespace {

constexpr int kSkThreads = 128;
constexpr int kWRows = 128;                      // weight rows per tile (MMA M)
constexpr int kWStage = kWRows * kBK * 2;        // 16 KB of weights per stage
constexpr int kMaxTokens = 256;
constexpr int kMaxSplits = 16;                   // cluster size (non-portable above 8)

struct SkinnyParams {
  int M, N, K;        // tokens, weight rows, reduction
  int mp;             // MMA N: tokens rounded up to 16
  int stages;
  int kb_per_split;   // K blocks (64) per split
  int splits;
  int tiles;          // weight tiles
  int mode;           // 0 plain, 1 SwiGLU over interleaved gate/up tiles, 2 QKV + RoPE + KV cache
  __nv_bfloat16* Y;
  int ldy;
  uint32_t* err;
  // mode 2: tile h < hq is query head h, then hkv key heads, then hkv value heads (128 rows
  // = head_dim each); q and k are rotated (rotate-half RoPE, pair (d, d + 64)) with
  // cos/sin[pos][d] and written to q_out [M, hq, 128] and k_cache / v_cache
  // [M, lmax, hkv, 128] at position positions[m]
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  const float* cos_t;
  const float* sin_t;
  const int* positions;
  int hq, hkv, lmax;
  uint64_t* stamps;   // optional: kStamps %globaltimer values per CTA (phase timing), or null
};

constexpr int kStamps = 8;

__device__ __forceinline__ void stamp(const SkinnyParams& p, int i) {
  if (p.stamps) {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    p.stamps[(size_t(blockIdx.y) * gridDim.x + blockIdx.x) * kStamps + i] = t;
  }
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// grid (splits, tiles), cluster (splits, 1, 1): the K splits of one weight tile are one
// thread-block cluster.  After the main loop each CTA parks its fp32 partial tile in
// its own shared memory; after a cluster barrier, CTA r sums its contiguous block of the
// tile's rows over the S partials through distributed shared memory, in split order, and
// writes them; a second cluster barrier keeps every partial alive until all reads are
// done.  No global scratch, no atomics.
//
// Programmatic dependent launch: the weight tiles of the first stages are requested
// before griddepcontrol.wait (weights do not depend on the previous kernel); the
// activation tiles and everything after come after it.
__global__ void __launch_bounds__(kSkThreads) k_skinny(const __grid_constant__ CUtensorMap map_w,
                                                       const __grid_constant__ CUtensorMap map_x,
                                                       SkinnyParams p) {
  extern __shared__ uint8_t raw_smem[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~uintptr_t(1023));
  const int x_stage = p.mp * kBK * 2;
  const int stage_bytes = kWStage + x_stage;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + p.stages * stage_bytes);
  uint64_t* empty = full + p.stages;
  uint64_t* done = empty + p.stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  float* part = reinterpret_cast<float*>(base);  // [mp][128] fp32 (token-major), over the idle stage buffers

  cg::cluster_group cluster = cg::this_cluster();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.y;
  const int S = int(cluster.num_blocks());  // == splits, as planned
  // A launch re-issued without its cluster attribute (a profiler may do that) has
  // clusters smaller than the split count.  The first cluster then covers the whole
  // K range, split S ways, and every other CTA exits before it holds any resource, so
  // each output is still written (or pushed) exactly once.
  const bool reshaped = S != int(gridDim.x);
  if (reshaped && blockIdx.x >= unsigned(S)) return;
  const int split = int(cluster.block_rank());
  const int kbps = reshaped ? (p.K / kBK + S - 1) / S : p.kb_per_split;
  const int kb0 = split * kbps;
  const int nkb = max(0, min(kbps, p.K / kBK - kb0));
  volatile uint32_t* err = p.err;
  const uint32_t ncols = p.mp <= 32 ? 32u : (p.mp <= 64 ? 64u : (p.mp <= 128 ? 128u : 256u));

  if (threadIdx.x == 0) {
    stamp(p, 0);  // entry
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    stamp(p, 1);  // set-up done (barriers, TMEM)
    prefetch_tmap(&map_w);
    prefetch_tmap(&map_x);
    const int pre = min(nkb, p.stages);
    for (int i = 0; i < pre; ++i) {  // weights first: independent of the previous kernel
      mbar_expect_tx(&full[i], stage_bytes);
      tma_load_2d(base + i * stage_bytes, &map_w, (kb0 + i) * kBK, tile * kWRows, &full[i]);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    stamp(p, 2);  // previous kernel complete
    for (int i = 0; i < pre; ++i) tma_load_2d(base + i * stage_bytes + kWStage, &map_x, (kb0 + i) * kBK, 0, &full[i]);
    for (int i = pre; i < nkb; ++i) {
      const int s = i % p.stages;
      const uint32_t ph = (i / p.stages) & 1;
      if (!mbar_wait(&empty[s], ph ^ 1, err)) break;
      uint8_t* st = base + s * stage_bytes;
      mbar_expect_tx(&full[s], stage_bytes);
      tma_load_2d(st, &map_w, (kb0 + i) * kBK, tile * kWRows, &full[s]);
      tma_load_2d(st + kWStage, &map_x, (kb0 + i) * kBK, 0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = idesc_bf16(p.mp);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % p.stages;
      const uint32_t ph = (i / p.stages) & 1;
      if (!mbar_wait(&full[s], ph, err)) break;
      if (i == 0) stamp(p, 3);  // first stage landed
      tc_fence_after();
      uint8_t* st = base + s * stage_bytes;
      const uint64_t adesc = smem_desc_sw128(st), bdesc = smem_desc_sw128(st + kWStage);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k)  // 16 bf16 = 32 bytes = +2 in descriptor units
        mma_bf16(tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (i | k) != 0);
      mma_commit(&empty[s]);
    }
    stamp(p, 4);  // last stage landed, last MMA issued
    mma_commit(done);  // also after an early exit: arrives once issued MMAs retire
  }
  __syncwarp();
  mbar_wait(done, 0, err);
  tc_fence_after();
  if (threadIdx.x == 64) stamp(p, 5);  // accumulator complete
  // a PDL-launched successor may launch now: it still waits for this grid to finish
  // before it reads anything this kernel writes
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // TMEM lane = weight row within the tile; warp w may read lanes 32w..32w+31.  Park
  // the partial (all stage reads and MMAs are complete: `done` fired).
  const int row = warp * 32 + lane;
  const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);
  const int chunks = p.mp / 16;
  for (int c = 0; c < chunks; ++c) {
    float v[16];
    tmem_ld16(lane_addr + c * 16, v);
    if (nkb == 0) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) part[(c * 16 + j) * kWRows + row] = v[j];  // a warp: 32 consecutive words
  }
  tc_fence_before();
  cluster.sync();  // every split's partial is parked
  if (threadIdx.x == 64) stamp(p, 6);

  // CTA `split` writes a contiguous block of the tile's rows (mode 0) or row pairs
  // (modes 1 and 2: gate/up halves, RoPE pairs).  The partials are parked token-major
  // and neighbouring lanes take neighbouring rows, so a warp reads consecutive words of
  // each partial (distributed shared memory is served in sectors, like global memory;
  // the row-major layout read with rows across lanes took 2x longer) and stores
  // neighbouring outputs of one token.  Loads are issued before the sums and stores
  // they feed (the stores could alias them as far as the compiler knows); each sum runs
  // over the splits in split order.
  constexpr int kWarps = kSkThreads / 32;
  auto partial = [&](int s, int r, int m) -> float {
    return cluster.map_shared_rank(part, s)[m * kWRows + r];
  };
  // Rounding and writing one output (row r of the tile, or pair r, r + 64) for token m.
  auto emit = [&](int r, int m, float x1, float x2) {
    if (p.mode == 0) {
      const int n = tile * kWRows + r;
      if (n < p.N) p.Y[size_t(m) * p.ldy + n] = __float2bfloat16_rn(x1);
      return;
    }
    if (p.mode == 1) {  // rows 0..63 gate, 64..127 up of the same 64 features
      p.Y[size_t(m) * p.ldy + tile * 64 + r] = __float2bfloat16_rn(silu(x1) * x2);
      return;
    }
    const int pos = p.positions[m];
    __nv_bfloat16* dst;
    if (tile < p.hq + p.hkv) {  // q or k: rotate
      const float cs = p.cos_t[size_t(pos) * 64 + r], sn = p.sin_t[size_t(pos) * 64 + r];
      const float y1 = x1 * cs - x2 * sn, y2 = x2 * cs + x1 * sn;
      x1 = y1;
      x2 = y2;
    }
    if (tile < p.hq) dst = p.q_out + (size_t(m) * p.hq + tile) * kWRows;
    else if (tile < p.hq + p.hkv)
      dst = p.k_cache + ((size_t(m) * p.lmax + pos) * p.hkv + (tile - p.hq)) * kWRows;
    else dst = p.v_cache + ((size_t(m) * p.lmax + pos) * p.hkv + (tile - p.hq - p.hkv)) * kWRows;
    dst[r] = __float2bfloat16_rn(x1);
    dst[r + 64] = __float2bfloat16_rn(x2);
  };
  const bool pairs = p.mode != 0;
  const int span = pairs ? 64 : kWRows;  // rows (mode 0) or row pairs (modes 1, 2) of a tile
  const int rb = (span + S - 1) / S, r0 = min(span, split * rb), r1 = min(span, r0 + rb);
  if (S > 1) {
    // Split K: a small block of rows per CTA, so all threads share its (row, token)
    // elements, row-fastest, a batch at a time (4 single rows or 2 row pairs).
    // Measured at 64 tokens against one warp per token: 39 against 54 us for
    // 5120 x 8192, 23.7 against 30.9 us for 8192 x 4096.
    const int nr = r1 - r0, total = max(0, nr) * p.M;
    auto run = [&](auto batch_tag, auto pair_tag) {
      constexpr int kBatch = decltype(batch_tag)::value;
      constexpr bool kPairs = decltype(pair_tag)::value;
      for (int e0 = threadIdx.x; e0 < total; e0 += kBatch * blockDim.x) {
        float va[kBatch][kMaxSplits], vb[kBatch][kPairs ? kMaxSplits : 1];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int e = e0 + b * int(blockDim.x);
          const bool in = e < total;
          const int r = r0 + (in ? e % nr : 0), m = in ? e / nr : 0;
#pragma unroll
          for (int q = 0; q < kMaxSplits; ++q) {
            va[b][q] = (in && q < S) ? partial(q, r, m) : 0.0f;
            if constexpr (kPairs) vb[b][q] = (in && q < S) ? partial(q, r + 64, m) : 0.0f;
          }
        }
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int e = e0 + b * int(blockDim.x);
          if (e >= total) break;
          float x1 = 0.0f, x2 = 0.0f;
#pragma unroll
          for (int q = 0; q < kMaxSplits; ++q) {
            x1 += va[b][q];
            if constexpr (kPairs) x2 += vb[b][q];
          }
          emit(r0 + e % nr, e / nr, x1, x2);
        }
      }
    };
    if (pairs) run(std::integral_constant<int, 2>{}, std::true_type{});
    else run(std::integral_constant<int, 4>{}, std::false_type{});
  } else {
    // One split: the whole tile is this CTA's own partial.  Warp w takes tokens w, w + 4,
    // ...; its lanes take the rows (no division per element) and read the partial from
    // their own shared memory.  Measured at 64 tokens, 28672 x 8192: 98.8 us against
    // 109.4 us with the element loop above.  The sum starts from 0.0f as in the split
    // path, so both round the same value.
    constexpr int kChunks = kWRows / 32;
    for (int m = warp; m < p.M; m += kWarps) {
      float v[kChunks];
#pragma unroll
      for (int c = 0; c < kChunks; ++c) v[c] = 0.0f + part[m * kWRows + c * 32 + lane];
      if (!pairs) {
#pragma unroll
        for (int c = 0; c < kChunks; ++c) emit(c * 32 + lane, m, v[c], 0.0f);
      } else {
#pragma unroll
        for (int c = 0; c < kChunks / 2; ++c) emit(c * 32 + lane, m, v[c], v[c + kChunks / 2]);
      }
    }
  }
  cluster.sync();  // partials stay readable until every CTA of the cluster is done
  if (threadIdx.x == 64) stamp(p, 7);  // exit
  if (warp == 1) tmem_dealloc(tmem, ncols);
}

struct Plan {
  int mp, stages, splits, kb_per_split, tiles, smem;
};

// Tuning (process-wide): CTAs per SM (0: by token count) and the split cap.
int g_cps = 0;

Plan plan(int M, int N, int K, int sms, int max_splits) {
  Plan pl;
  pl.mp = std::max(16, (M + 15) / 16 * 16);
  pl.tiles = (N + kWRows - 1) / kWRows;
  const int x_stage = pl.mp * kBK * 2;
  const int stage = kWStage + x_stage;
  // two CTAs per SM while the token tile is small, one beyond
  const int ctas_per_sm = g_cps > 0 ? g_cps : (pl.mp <= 64 ? 2 : 1);
  const int budget = (224 / ctas_per_sm) * 1024 - 1024 /*align*/ - 1024 /*barriers*/;
  pl.stages = std::max(2, std::min(12, budget / stage));
  pl.smem = 1024 + pl.stages * stage + 1024;
  const int kbs = K / kBK;
  int splits = std::max(1, sms * ctas_per_sm / pl.tiles);  // one wave
  splits = std::min({splits, kbs, max_splits > 0 ? std::min(max_splits, kMaxSplits) : kMaxSplits});
  pl.kb_per_split = (kbs + splits - 1) / splits;
  pl.splits = (kbs + pl.kb_per_split - 1) / pl.kb_per_split;
  return pl;
}

void check_mat(const at::Tensor& t, const char* name) {
  if (!t.is_cuda() || t.scalar_type() != at::kBFloat16 || t.dim() != 2 || t.stride(1) != 1)
    throw std::invalid_argument(std::string(name) + " must be a row-major 2-D CUDA bfloat16 tensor");
}

void launch_skinny(const at::Tensor& W, const at::Tensor& X, const SkinnyParams& p, const Plan& pl, int dev, bool pdl) {
  if (size_t(kWRows) * pl.mp * 4 > size_t(pl.stages) * (kWStage + pl.mp * kBK * 2))
    throw std::logic_error("decode GEMM: the parked partial does not fit the stage buffers");
  CUtensorMap mw = make_map(W.data_ptr(), p.N, p.K, W.stride(0), kWRows);
  CUtensorMap mx = make_map(X.data_ptr(), p.M, p.K, X.stride(0), pl.mp);
  static int attr_done[64] = {0};
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {  // function attributes belong to each device's context
    cudaError_t e = cudaFuncSetAttribute(k_skinny, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_skinny, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) throw std::runtime_error(std::string("decode GEMM attributes: ") + cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_done[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.splits, pl.tiles, 1);
  cfg.blockDim = dim3(kSkThreads, 1, 1);
  cfg.dynamicSmemBytes = size_t(pl.smem);
  cfg.stream = at::cuda::getCurrentCUDAStream(dev).stream();
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = pl.splits;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_skinny, mw, mx, p);
  if (e != cudaSuccess) throw std::runtime_error(std::string("decode GEMM launch: ") + cudaGetErrorString(e));
}

}  // namespace

void skinny_gemm(const at::Tensor& X, const at::Tensor& W, at::Tensor& Y, at::Tensor& err, int mode, int max_splits,
                 bool pdl, const c10::optional<at::Tensor>& stamps) {
  check_mat(X, "X");
  check_mat(W, "W");
  check_mat(Y, "Y");
  const int M = int(X.size(0)), K = int(X.size(1)), N = int(W.size(0));
  if (W.size(1) != K) throw std::invalid_argument("X and W must share K");
  if (M < 1 || M > kMaxTokens) throw std::invalid_argument("skinny_gemm takes 1..256 token rows");
  if (K % kBK) throw std::invalid_argument("K must be a multiple of 64");
  if (mode == 0 && (Y.size(0) != M || Y.size(1) != N)) throw std::invalid_argument("Y must be [M, N]");
  if (mode == 1 && (N % kWRows || Y.size(0) != M || Y.size(1) != N / 2))
    throw std::invalid_argument("SwiGLU mode: W rows a multiple of 128 and Y [M, N/2]");
  if (mode != 0 && mode != 1) throw std::invalid_argument("mode must be 0 or 1");
  const int dev = X.device().index();
  c10::cuda::CUDAGuard guard(X.device());
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  Plan pl = plan(M, N, K, sms, max_splits);
  SkinnyParams p;
  memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.mp = pl.mp;
  p.stages = pl.stages;
  p.kb_per_split = pl.kb_per_split;
  p.splits = pl.splits;
  p.tiles = pl.tiles;
  p.mode = mode;
  p.Y = reinterpret_cast<__nv_bfloat16*>(Y.data_ptr());
  p.ldy = int(Y.stride(0));
  p.err = reinterpret_cast<uint32_t*>(err.data_ptr());
  p.stamps = nullptr;
  if (stamps) {
    if (!stamps->is_cuda() || stamps->element_size() != 8 || stamps->numel() < int64_t(pl.splits) * pl.tiles * kStamps)
      throw std::invalid_argument("stamps must be a CUDA 8-byte tensor of splits * tiles * 8 entries");
    p.stamps = reinterpret_cast<uint64_t*>(stamps->data_ptr());
  }
  launch_skinny(W, X, p, pl, dev, pdl);
}

// QKV projection for decode with RoPE and the KV-cache write in the epilogue:
// X [M, K] x W [(hq + 2 hkv) * 128, K]^T; q -> q_out [M, hq, 128] (rotated), k (rotated)
// and v -> k_cache / v_cache [M, lmax, hkv, 128] at positions[m].
void skinny_qkv_rope(const at::Tensor& X, const at::Tensor& W, const at::Tensor& cos_t, const at::Tensor& sin_t,
                     const at::Tensor& positions, at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache,
                     at::Tensor& err, int hq, int hkv, bool pdl) {
  check_mat(X, "X");
  check_mat(W, "W");
  const int M = int(X.size(0)), K = int(X.size(1)), N = int(W.size(0));
  if (W.size(1) != K) throw std::invalid_argument("X and W must share K");
  if (N != (hq + 2 * hkv) * kWRows) throw std::invalid_argument("W must have (hq + 2 hkv) * 128 rows");
  if (M < 1 || M > kMaxTokens || K % kBK) throw std::invalid_argument("1..256 tokens and K a multiple of 64");
  auto bf16c = [](const at::Tensor& t) {
    return t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous();
  };
  if (!bf16c(q_out) || q_out.numel() != int64_t(M) * hq * kWRows) throw std::invalid_argument("q_out [M, hq, 128] bf16");
  if (!bf16c(k_cache) || !bf16c(v_cache) || k_cache.dim() != 4 || k_cache.size(0) != M || k_cache.size(2) != hkv ||
      k_cache.size(3) != kWRows || !k_cache.sizes().equals(v_cache.sizes()))
    throw std::invalid_argument("k_cache / v_cache [M, lmax, hkv, 128] bf16");
  if (!cos_t.is_cuda() || cos_t.scalar_type() != at::kFloat || !cos_t.is_contiguous() || cos_t.size(1) != 64 ||
      !sin_t.sizes().equals(cos_t.sizes()) || sin_t.scalar_type() != at::kFloat)
    throw std::invalid_argument("cos/sin tables [lmax, 64] float32");
  if (!positions.is_cuda() || positions.scalar_type() != at::kInt || positions.numel() != M)
    throw std::invalid_argument("positions [M] int32");
  const int dev = X.device().index();
  c10::cuda::CUDAGuard guard(X.device());
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  Plan pl = plan(M, N, K, sms, 0);
  SkinnyParams p;
  memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.mp = pl.mp;
  p.stages = pl.stages;
  p.kb_per_split = pl.kb_per_split;
  p.splits = pl.splits;
  p.tiles = pl.tiles;
  p.mode = 2;
  p.err = reinterpret_cast<uint32_t*>(err.data_ptr());
  p.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  p.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  p.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  p.cos_t = cos_t.data_ptr<float>();
  p.sin_t = sin_t.data_ptr<float>();
  p.positions = positions.data_ptr<int>();
  p.hq = hq;
  p.hkv = hkv;
  p.lmax = int(k_cache.size(1));
  launch_skinny(W, X, p, pl, dev, pdl);
}

void skinny_tune(int ctas_per_sm) { g_cps = ctas_per_sm; }

std::vector<int> skinny_plan(int M, int N, int K, int sms, int max_splits) {
  Plan pl = plan(M, N, K, sms, max_splits);
  return {pl.mp, pl.stages, pl.splits, pl.kb_per_split, pl.tiles, pl.smem};
}

}  // namespace tc
}  // namespace sn

void register_skinny(py::module_& m) {
  m.def("skinny_gemm", &sn::tc::skinny_gemm, py::arg("X"), py::arg("W"), py::arg("Y"), py::arg("err"),
        py::arg("mode") = 0, py::arg("max_splits") = 0, py::arg("pdl") = false, py::arg("stamps") = py::none(),
        "Y = X @ W.T for few token rows (tcgen05, split-K reduced in a cluster, optional SwiGLU epilogue)");
  m.def("skinny_qkv_rope", &sn::tc::skinny_qkv_rope, py::arg("X"), py::arg("W"), py::arg("cos"), py::arg("sin"),
        py::arg("positions"), py::arg("q_out"), py::arg("k_cache"), py::arg("v_cache"), py::arg("err"),
        py::arg("hq"), py::arg("hkv"), py::arg("pdl") = false,
        "decode QKV projection with RoPE and the KV-cache write fused into the epilogue");
  m.def("skinny_tune", &sn::tc::skinny_tune, py::arg("ctas_per_sm") = 0,
        "process-wide decode GEMM tuning: CTAs per SM (0 = by token count)");
  m.def("skinny_plan", &sn::tc::skinny_plan, py::arg("M"), py::arg("N"), py::arg("K"), py::arg("sms"),
        py::arg("max_splits") = 0);
}
