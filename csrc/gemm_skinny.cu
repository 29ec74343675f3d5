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
// Y[m, f] = silu(gate) * up for the N/2 features (no intermediate tensor).
//
// Every mbarrier wait is bounded (sets the error word and unwinds).
// Reference: none (the reference has no model GEMMs).
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
namespace {

constexpr int kSkThreads = 128;
constexpr int kWRows = 128;                      // weight rows per tile (MMA M)
constexpr int kWStage = kWRows * kBK * 2;        // 16 KB of weights per stage
constexpr int kMaxTokens = 256;
constexpr int kRedBatch = 8;                     // split partials loaded at once by the last CTA

struct SkinnyParams {
  int M, N, K;        // tokens, weight rows, reduction
  int mp;             // MMA N: tokens rounded up to 16
  int stages;
  int kb_per_split;   // K blocks (64) per split
  int splits;
  int tiles;          // weight tiles
  int mode;           // 0 plain, 1 SwiGLU over interleaved gate/up tiles
  int rot;            // K-block rotation per weight tile (spreads concurrent reads over channels)
  __nv_bfloat16* Y;
  int ldy;
  float* ws;          // [splits][tiles][mp / 16][128][16] fp32 partials
  int* counters;      // [tiles], zero between launches (the last CTA resets its tile)
  uint32_t* err;
};

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

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
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* xchg = reinterpret_cast<float*>(base + p.stages * stage_bytes + 1024);  // [64][17] SwiGLU exchange

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int kb0 = split * p.kb_per_split;
  const int nkb = min(p.kb_per_split, p.K / kBK - kb0);
  volatile uint32_t* err = p.err;
  const uint32_t ncols = p.mp <= 32 ? 32u : (p.mp <= 64 ? 64u : (p.mp <= 128 ? 128u : 256u));

  if (threadIdx.x == 0) {
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
    prefetch_tmap(&map_w);
    prefetch_tmap(&map_x);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % p.stages;
      const uint32_t ph = (i / p.stages) & 1;
      if (i >= p.stages && !mbar_wait(&empty[s], ph ^ 1, err)) break;
      uint8_t* st = base + s * stage_bytes;
      const int kb = kb0 + (i + tile * p.rot) % nkb;
      mbar_expect_tx(&full[s], stage_bytes);
      tma_load_2d(st, &map_w, kb * kBK, tile * kWRows, &full[s]);
      tma_load_2d(st + kWStage, &map_x, kb * kBK, 0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = idesc_bf16(p.mp);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % p.stages;
      const uint32_t ph = (i / p.stages) & 1;
      if (!mbar_wait(&full[s], ph, err)) break;
      tc_fence_after();
      uint8_t* st = base + s * stage_bytes;
      const uint64_t adesc = smem_desc_sw128(st), bdesc = smem_desc_sw128(st + kWStage);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k)  // 16 bf16 = 32 bytes = +2 in descriptor units
        mma_bf16(tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (i | k) != 0);
      mma_commit(&empty[s]);
    }
    mma_commit(done);  // also after an early exit: arrives once issued MMAs retire
  }
  __syncwarp();
  const bool ok = mbar_wait(done, 0, err);
  tc_fence_after();

  // TMEM lane = weight row within the tile; warp w may read lanes 32w..32w+31.
  const int row = warp * 32 + lane;
  const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);
  const int chunks = p.mp / 16;
  auto final_store = [&](int c, const float* v) {
    if (p.mode == 0) {
      const int n = tile * kWRows + row;
      if (n < p.N) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c * 16 + j < p.M) p.Y[size_t(c * 16 + j) * p.ldy + n] = __float2bfloat16_rn(v[j]);
      }
    } else {
      // rows 64..127 (warps 2, 3) hold `up`, rows 0..63 `gate` of the same features
      if (row >= 64) {
#pragma unroll
        for (int j = 0; j < 16; ++j) xchg[(row - 64) * 17 + j] = v[j];
      }
      __syncthreads();
      if (row < 64) {
        const int f = tile * 64 + row;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c * 16 + j < p.M)
            p.Y[size_t(c * 16 + j) * p.ldy + f] = __float2bfloat16_rn(silu(v[j]) * xchg[row * 17 + j]);
      }
      __syncthreads();
    }
  };

  if (p.splits == 1) {
    for (int c = 0; c < chunks; ++c) {
      float v[16];
      tmem_ld16(lane_addr + c * 16, v);
      final_store(c, v);
    }
  } else {
    float* mine = p.ws + (size_t(split) * p.tiles + tile) * chunks * kWRows * 16;
    for (int c = 0; c < chunks; ++c) {
      float v[16];
      tmem_ld16(lane_addr + c * 16, v);
      float4* dst = reinterpret_cast<float4*>(mine + (size_t(c) * kWRows + row) * 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) __stcg(dst + j, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *last_flag = atomicAdd(&p.counters[tile], 1) == p.splits - 1;
    __syncthreads();
    if (*last_flag) {
      __threadfence();
      for (int c = 0; c < chunks; ++c) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.0f;
        // fixed split order; kRedBatch splits' loads in flight before any add
        for (int s0 = 0; s0 < p.splits; s0 += kRedBatch) {
          float4 t[kRedBatch][4];
#pragma unroll
          for (int b = 0; b < kRedBatch; ++b) {
            const float4* src = reinterpret_cast<const float4*>(
                p.ws + ((size_t(s0 + b) * p.tiles + tile) * chunks * kWRows + size_t(c) * kWRows + row) * 16);
#pragma unroll
            for (int j = 0; j < 4; ++j) t[b][j] = s0 + b < p.splits ? __ldcg(src + j) : make_float4(0, 0, 0, 0);
          }
#pragma unroll
          for (int b = 0; b < kRedBatch; ++b) {
            if (s0 + b < p.splits) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                v[4 * j] += t[b][j].x;
                v[4 * j + 1] += t[b][j].y;
                v[4 * j + 2] += t[b][j].z;
                v[4 * j + 3] += t[b][j].w;
              }
            }
          }
        }
        final_store(c, v);
      }
      if (threadIdx.x == 0) p.counters[tile] = 0;
    }
  }
  (void)ok;
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, ncols);
}

struct Plan {
  int mp, stages, splits, kb_per_split, tiles, smem;
};

// Tuning (process-wide): CTAs per SM (0: by token count) and K-block rotation.
int g_cps = 0;
int g_rot = 0;

Plan plan(int M, int N, int K, int sms, int max_splits) {
  Plan pl;
  pl.mp = std::max(16, (M + 15) / 16 * 16);
  pl.tiles = (N + kWRows - 1) / kWRows;
  const int x_stage = pl.mp * kBK * 2;
  const int stage = kWStage + x_stage;
  // two CTAs per SM while the token tile is small, one beyond
  const int ctas_per_sm = g_cps > 0 ? g_cps : (pl.mp <= 64 ? 2 : 1);
  const int budget = (224 / ctas_per_sm) * 1024 - 1024 /*align*/ - 1024 /*barriers*/ - 64 * 17 * 4;
  pl.stages = std::max(2, std::min(12, budget / stage));
  pl.smem = 1024 + pl.stages * stage + 1024 + 64 * 17 * 4;
  const int kbs = K / kBK;
  int splits = std::max(1, sms * ctas_per_sm / pl.tiles);  // one wave
  splits = std::min({splits, kbs, max_splits > 0 ? max_splits : 16});
  pl.kb_per_split = (kbs + splits - 1) / splits;
  pl.splits = (kbs + pl.kb_per_split - 1) / pl.kb_per_split;
  return pl;
}

void check_mat(const at::Tensor& t, const char* name) {
  if (!t.is_cuda() || t.scalar_type() != at::kBFloat16 || t.dim() != 2 || t.stride(1) != 1)
    throw std::invalid_argument(std::string(name) + " must be a row-major 2-D CUDA bfloat16 tensor");
}

}  // namespace

// Floats of fp32 workspace and ints of counters a call with these shapes needs.
std::pair<int64_t, int64_t> skinny_workspace(int M, int N, int K, int sms, int max_splits) {
  Plan pl = plan(M, N, K, sms, max_splits);
  if (pl.splits == 1) return {0, pl.tiles};
  return {int64_t(pl.splits) * pl.tiles * pl.mp * kWRows, pl.tiles};
}

void skinny_gemm(const at::Tensor& X, const at::Tensor& W, at::Tensor& Y, at::Tensor& ws, at::Tensor& counters,
                 at::Tensor& err, int mode, int max_splits) {
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
  if (ws.scalar_type() != at::kFloat || counters.scalar_type() != at::kInt || !ws.is_cuda() || !counters.is_cuda())
    throw std::invalid_argument("workspace must be CUDA float32 and counters CUDA int32");
  const int dev = X.device().index();
  c10::cuda::CUDAGuard guard(X.device());
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  Plan pl = plan(M, N, K, sms, max_splits);
  const int64_t need_ws = pl.splits == 1 ? 0 : int64_t(pl.splits) * pl.tiles * pl.mp * kWRows;
  if (ws.numel() < need_ws || counters.numel() < pl.tiles)
    throw std::invalid_argument("workspace or counters too small (see skinny_workspace)");

  SkinnyParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.mp = pl.mp;
  p.stages = pl.stages;
  p.kb_per_split = pl.kb_per_split;
  p.splits = pl.splits;
  p.tiles = pl.tiles;
  p.mode = mode;
  p.rot = g_rot;
  p.Y = reinterpret_cast<__nv_bfloat16*>(Y.data_ptr());
  p.ldy = int(Y.stride(0));
  p.ws = ws.data_ptr<float>();
  p.counters = counters.data_ptr<int>();
  p.err = reinterpret_cast<uint32_t*>(err.data_ptr());
  CUtensorMap mw = make_map(W.data_ptr(), N, K, W.stride(0), kWRows);
  CUtensorMap mx = make_map(X.data_ptr(), M, K, X.stride(0), pl.mp);
  static int attr_done[64] = {0};
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaFuncSetAttribute(k_skinny, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr_done[dev] = 1;
  }
  auto s = at::cuda::getCurrentCUDAStream(dev).stream();
  k_skinny<<<dim3(pl.tiles, pl.splits), kSkThreads, pl.smem, s>>>(mw, mx, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("skinny_gemm launch: ") + cudaGetErrorString(e));
}

void skinny_tune(int ctas_per_sm, int rotation) {
  g_cps = ctas_per_sm;
  g_rot = rotation;
}

std::vector<int> skinny_plan(int M, int N, int K, int sms, int max_splits) {
  Plan pl = plan(M, N, K, sms, max_splits);
  return {pl.mp, pl.stages, pl.splits, pl.kb_per_split, pl.tiles, pl.smem};
}

}  // namespace tc
}  // namespace sn

void register_skinny(py::module_& m) {
  m.def("skinny_gemm", &sn::tc::skinny_gemm, py::arg("X"), py::arg("W"), py::arg("Y"), py::arg("ws"),
        py::arg("counters"), py::arg("err"), py::arg("mode") = 0, py::arg("max_splits") = 0,
        "Y = X @ W.T for few token rows (tcgen05, split-K, optional SwiGLU epilogue)");
  m.def("skinny_workspace", &sn::tc::skinny_workspace, py::arg("M"), py::arg("N"), py::arg("K"), py::arg("sms"),
        py::arg("max_splits") = 0);
  m.def("skinny_tune", &sn::tc::skinny_tune, py::arg("ctas_per_sm") = 0, py::arg("rotation") = 0,
        "process-wide decode GEMM tuning: CTAs per SM (0 = by token count) and K-block rotation per tile");
  m.def("skinny_plan", &sn::tc::skinny_plan, py::arg("M"), py::arg("N"), py::arg("K"), py::arg("sms"),
        py::arg("max_splits") = 0);
}
