// NVLink data-movement microbenchmark kernels (sm_100a): what a collective's data
// phase can do over NVSwitch, one mechanism at a time.
//
//   store        this GPU reads its buffer and stores 16-byte packs into a peer's buffer
//                (the one-shot "push")
//   load         this GPU loads 16-byte packs from a peer's buffer and stores them locally
//                (the "pull")
//   mc_store     multimem.st through the NVLS multicast alias: one store, every GPU of
//                the multicast group receives it
//   mc_reduce    multimem.ld_reduce.add (bf16x2, fp32 accumulation) through the alias:
//                one load returns the sum over every GPU's copy
//   bulk         one thread per CTA: bulk copy local -> shared memory, then one bulk
//                store per destination (the copy engine of the SM does the moving)
//
// Each kernel is a grid-stride loop over `bytes` (a multiple of 16) with `ppt` packs in
// flight per thread before the first store, so grid size, block size and loads in
// flight can be swept independently.  No waits, no flags: a launch cannot hang.
// Reference: the data-phase sweeps of evidence/2026-10-20-wide-read/sweep.cu (k_pack,
// k_multi, k_gather) measured the same questions for the GB10 host-staged path.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "sparknet/tc_gemm.cuh"

namespace py = pybind11;

namespace {

constexpr int kMaxPpt = 8;

__device__ __forceinline__ uint4 ld_nc(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
// peer data that another GPU may have written: bypass L1
__device__ __forceinline__ uint4 ld_peer(const uint4* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_plain(uint4* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ void mc_st(uint4* p, uint4 v) {
  asm volatile("multimem.st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 mc_ld_reduce_bf16(const uint4* p) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// mode 0 store (src local -> dst peer), 1 load (src peer -> dst local), 2 mc_store (src
// local -> dst multicast), 3 mc_reduce (src multicast -> dst local)
template <int MODE>
__global__ void __launch_bounds__(1024) k_move(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t packs,
                                                int ppt) {
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  for (size_t base = size_t(blockIdx.x) * blockDim.x + threadIdx.x; base < packs; base += stride * ppt) {
    uint4 v[kMaxPpt];
#pragma unroll
    for (int j = 0; j < kMaxPpt; ++j) {
      const size_t i = base + j * stride;
      if (j < ppt && i < packs) {
        if (MODE == 0 || MODE == 2) v[j] = ld_nc(src + i);
        else if (MODE == 1) v[j] = ld_peer(src + i);
        else v[j] = mc_ld_reduce_bf16(src + i);
      }
    }
#pragma unroll
    for (int j = 0; j < kMaxPpt; ++j) {
      const size_t i = base + j * stride;
      if (j < ppt && i < packs) {
        if (MODE == 2) mc_st(dst + i, v[j]);
        else st_plain(dst + i, v[j]);
      }
    }
  }
}

// mode 4, bulk fan-out: one thread per CTA moves `piece`-byte pieces (CTA b takes pieces
// b, b + grid, ...) from local memory into shared memory with a bulk copy, then stores
// each piece to every destination in `dst` (1..8 addresses: peers' mappings) with one
// bulk store apiece: the TMA engine moves the data, no thread touches it.  Two stage
// buffers: the load of piece i+1 overlaps the stores of piece i.  A load that does not
// complete within the poll bound ends the loop with `err` set (no hang).
struct BulkDsts {
  char* d[8];
  int n;
};

__global__ void __launch_bounds__(32) k_bulk_fanout(const char* __restrict__ src, BulkDsts dsts, size_t bytes,
                                                   int piece, int* err) {
  extern __shared__ __align__(128) char stage[];  // 2 x piece
  __shared__ __align__(8) uint64_t bar[2];
  __shared__ uint32_t wait_err;
  if (threadIdx.x != 0) return;
  wait_err = 0;
  for (int i = 0; i < 2; ++i) sn::tc::mbar_init(&bar[i], 1);
  sn::tc::fence_barrier_init();
  int iter = 0;
  for (size_t off = size_t(blockIdx.x) * piece; off < bytes; off += size_t(gridDim.x) * piece, ++iter) {
    const int b = iter & 1;
    const uint32_t n = uint32_t(min(size_t(piece), bytes - off));
    char* buf = stage + b * piece;
    // the stores issued from this buffer two pieces ago must have read it
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    sn::tc::mbar_expect_tx(&bar[b], n);
    sn::tc::bulk_load(buf, src + off, n, &bar[b]);
    if (!sn::tc::mbar_wait(&bar[b], uint32_t((iter >> 1) & 1), &wait_err)) {
      atomicExch(err, 1);
      break;
    }
    for (int q = 0; q < dsts.n; ++q)
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dsts.d[q] + off),
                   "r"(sn::tc::smem_u32(buf)), "r"(n)
                   : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

}  // namespace

// Bulk fan-out (mode 4 of the microbenchmark): `bytes` from `src` to every address in
// `dsts`, `piece` bytes per bulk copy, `blocks` CTAs of one working thread each.
void nvlink_bulk_fanout(int64_t src, std::vector<int64_t> dsts, int64_t bytes, int blocks, int piece,
                        at::Tensor err, int device) {
  if (bytes <= 0 || bytes % 16 || src % 16 || piece < 16 || piece % 16 || piece > 96 * 1024)
    throw std::invalid_argument("16-byte aligned sizes, piece 16 B .. 96 KB");
  if (dsts.empty() || dsts.size() > 8) throw std::invalid_argument("1 to 8 destinations");
  BulkDsts d{};
  d.n = int(dsts.size());
  for (size_t i = 0; i < dsts.size(); ++i) {
    if (dsts[i] % 16) throw std::invalid_argument("16-byte aligned destinations");
    d.d[i] = reinterpret_cast<char*>(dsts[i]);
  }
  if (err.scalar_type() != at::kInt || !err.is_cuda()) throw std::invalid_argument("err: int32 CUDA tensor");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  auto st = at::cuda::getCurrentCUDAStream(device).stream();
  const size_t smem = 2 * size_t(piece);
  cudaError_t e = cudaFuncSetAttribute(k_bulk_fanout, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) throw std::runtime_error(std::string("bulk fan-out attributes: ") + cudaGetErrorString(e));
  k_bulk_fanout<<<blocks, 32, smem, st>>>(reinterpret_cast<const char*>(src), d, size_t(bytes), piece,
                                          err.data_ptr<int>());
  e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("bulk fan-out launch: ") + cudaGetErrorString(e));
}

// Move `bytes` from address `src` to address `dst` (raw device addresses: local, a
// peer's mapping, or a multicast alias, by mode) with `blocks` x `threads` and `ppt`
// packs in flight per thread, on the current stream.
void nvlink_move(int64_t src, int64_t dst, int64_t bytes, int mode, int blocks, int threads, int ppt, int device) {
  if (bytes <= 0 || bytes % 16 || src % 16 || dst % 16) throw std::invalid_argument("16-byte aligned sizes only");
  if (blocks < 1 || threads < 32 || threads > 1024 || threads % 32 || ppt < 1 || ppt > kMaxPpt)
    throw std::invalid_argument("blocks >= 1, threads a multiple of 32 up to 1024, 1 <= ppt <= 8");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  auto st = at::cuda::getCurrentCUDAStream(device).stream();
  const auto* s = reinterpret_cast<const uint4*>(src);
  auto* d = reinterpret_cast<uint4*>(dst);
  const size_t packs = size_t(bytes) / 16;
  switch (mode) {
    case 0: k_move<0><<<blocks, threads, 0, st>>>(s, d, packs, ppt); break;
    case 1: k_move<1><<<blocks, threads, 0, st>>>(s, d, packs, ppt); break;
    case 2: k_move<2><<<blocks, threads, 0, st>>>(s, d, packs, ppt); break;
    case 3: k_move<3><<<blocks, threads, 0, st>>>(s, d, packs, ppt); break;
    default: throw std::invalid_argument("mode: 0 store, 1 load, 2 mc_store, 3 mc_reduce");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("nvlink_move launch: ") + cudaGetErrorString(e));
}

void register_microbench(py::module_& m) {
  m.def("nvlink_move", &nvlink_move, py::arg("src"), py::arg("dst"), py::arg("bytes"), py::arg("mode"),
        py::arg("blocks"), py::arg("threads") = 512, py::arg("ppt") = 1, py::arg("device") = 0,
        "data-phase microbenchmark: 0 P2P store, 1 P2P load, 2 multimem.st, 3 multimem.ld_reduce (bf16)");
  m.def("nvlink_bulk_fanout", &nvlink_bulk_fanout, py::arg("src"), py::arg("dsts"), py::arg("bytes"),
        py::arg("blocks"), py::arg("piece"), py::arg("err"), py::arg("device") = 0,
        "data-phase microbenchmark: bulk (TMA engine) copies local -> shared -> every destination");
}
