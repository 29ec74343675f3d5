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

}  // namespace

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
}
