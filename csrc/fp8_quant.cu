// fp8 (e4m3) quantisation with power-of-two (UE8M0) block scales, in the layout the
// block-scaled tcgen05 GEMM reads.
//
//   rows     activations [M, K]: one scale per row and 128-column block (1 x 128)
//   blocks   weights     [N, K]: one scale per 128 x 128 block
//
// A scale is 2^(e - 127) with e the smallest exponent for which |x| / scale <= 448
// (the e4m3 maximum) over the block; values are scaled by the exact power of two and
// rounded to e4m3 with saturation.
//
// Scale layout (both kinds): chunk (rb, kb) of 512 bytes for row block rb (128 rows)
// and K block kb (128 columns) at byte ((rb * K/128) + kb) * 512; inside it, the
// scale of row rb*128 + 32*g + i (i < 32, g < 4) for MMA K-step j (j < 4, 32 columns
// each) at byte 16*i + 4*g + j.  Each 16-byte line is one TMEM lane's four 32-bit
// columns after tcgen05.cp.32x128b.warpx4, so one copy stages a chunk.  The MMA scales
// every 32 columns; the four K-steps of a 128-column block carry the same exponent.
// Reference: none (the reference has no GEMMs or fp8 path).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <torch/extension.h>

#include <stdexcept>

namespace py = pybind11;

namespace {

// UE8M0 exponent of the smallest power of two s with amax / s <= 448, exactly: with
// amax = m * 2^E (1 <= m < 2) and 448 = 1.75 * 2^8, amax <= 448 * 2^k holds from
// k = E - 8 when m <= 1.75 (mantissa field <= 0x600000), else from k = E - 7.
__device__ __forceinline__ uint32_t ue8m0_for(float amax) {
  if (!(amax > 0.0f)) return 127u;  // zero (or NaN) block: scale 1
  const uint32_t bits = __float_as_uint(amax);
  const int exp_field = int((bits >> 23) & 0xFFu);
  if (exp_field == 0) return 1u;                                   // subnormal amax: smallest scale
  int e = exp_field - 8 + ((bits & 0x7FFFFFu) > 0x600000u ? 1 : 0);  // 127 + k
  return uint32_t(e < 1 ? 1 : (e > 254 ? 254 : e));
}

// 2^(127 - e): multiplying by it divides by the scale exactly.
__device__ __forceinline__ float inv_scale(uint32_t e) { return __uint_as_float((254u - e) << 23); }

__device__ __forceinline__ uint32_t pack_fp8x4(float a, float b, float c, float d) {
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return uint32_t(lo) | (uint32_t(hi) << 16);
}

__device__ __forceinline__ size_t sf_byte(int row, int kb, int kblocks) {
  const int rb = row >> 7, r = row & 127;
  return (size_t(rb) * kblocks + kb) * 512 + (r & 31) * 16 + (r >> 5) * 4;
}

// One warp per (row, 128-column block): lane holds 4 values.
__global__ void k_quant_rows(const __nv_bfloat16* __restrict__ x, int M, int K, int ldx, uint8_t* __restrict__ q,
                             uint8_t* __restrict__ sf) {
  const int kblocks = K / 128;
  const int warps = (blockDim.x >> 5) * gridDim.x;
  const int lane = threadIdx.x & 31;
  for (int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < M * kblocks; w += warps) {
    const int row = w / kblocks, kb = w % kblocks;
    const __nv_bfloat16* src = x + size_t(row) * ldx + kb * 128 + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    float amax = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const uint32_t e = ue8m0_for(amax);
    const float s = inv_scale(e);
    *reinterpret_cast<uint32_t*>(q + size_t(row) * K + kb * 128 + lane * 4) =
        pack_fp8x4(a.x * s, a.y * s, b.x * s, b.y * s);
    if (lane == 0) *reinterpret_cast<uint32_t*>(sf + sf_byte(row, kb, kblocks)) = e * 0x01010101u;
  }
}

// One block of 256 threads per 128 x 128 block.
__global__ void __launch_bounds__(256) k_quant_blocks(const __nv_bfloat16* __restrict__ w, int N, int K, int ldw,
                                                      uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  __shared__ float red[8];
  const int kblocks = K / 128;
  const int rb = blockIdx.x / kblocks, kb = blockIdx.x % kblocks;
  const int t = threadIdx.x;
  const int r0 = rb * 128;
  // thread t: rows r0 + t/2 (128 rows, 2 threads per row), 64 columns each, as 8 vectors of 8
  const int r = r0 + (t >> 1);
  const int c0 = kb * 128 + (t & 1) * 64;
  uint4 v[8];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = r < N ? *reinterpret_cast<const uint4*>(w + size_t(r) * ldw + c0 + i * 8) : make_uint4(0, 0, 0, 0);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((t & 31) == 0) red[t >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  const uint32_t e = ue8m0_for(amax);
  const float s = inv_scale(e);
  if (r < N) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
      const float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
      const float2 f2 = __bfloat1622float2(h[2]), f3 = __bfloat1622float2(h[3]);
      uint2 o;
      o.x = pack_fp8x4(f0.x * s, f0.y * s, f1.x * s, f1.y * s);
      o.y = pack_fp8x4(f2.x * s, f2.y * s, f3.x * s, f3.y * s);
      *reinterpret_cast<uint2*>(q + size_t(r) * K + c0 + i * 8) = o;
    }
  }
  // the chunk: 512 bytes, all this block's exponent
  if (t < 128) reinterpret_cast<uint32_t*>(sf + (size_t(rb) * kblocks + kb) * 512)[t] = e * 0x01010101u;
}

void check_in(const at::Tensor& x, const at::Tensor& q, const at::Tensor& sf, int rows, int K) {
  if (!x.is_cuda() || x.scalar_type() != at::kBFloat16 || x.dim() != 2 || x.stride(1) != 1)
    throw std::invalid_argument("input must be a row-major 2-D CUDA bfloat16 tensor");
  if (K % 128) throw std::invalid_argument("K must be a multiple of 128");
  if (x.stride(0) % 8) throw std::invalid_argument("input row pitch must be a multiple of 8 elements");
  if (!q.is_cuda() || !q.is_contiguous() || q.element_size() != 1 || q.numel() != int64_t(rows) * K)
    throw std::invalid_argument("q must be a contiguous 1-byte CUDA tensor of the input's shape");
  const int64_t need = int64_t((rows + 127) / 128) * (K / 128) * 512;
  if (!sf.is_cuda() || !sf.is_contiguous() || sf.element_size() != 1 || sf.numel() < need)
    throw std::invalid_argument("sf must be a contiguous 1-byte CUDA tensor of scale_bytes(rows, K) bytes");
}

}  // namespace

int64_t fp8_scale_bytes(int rows, int K) { return int64_t((rows + 127) / 128) * (K / 128) * 512; }

void fp8_quantize_rows(const at::Tensor& x, at::Tensor& q, at::Tensor& sf) {
  const int M = int(x.size(0)), K = int(x.size(1));
  check_in(x, q, sf, M, K);
  c10::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream(x.device().index()).stream();
  const int64_t warps = int64_t(M) * (K / 128);
  const int blocks = int(std::min<int64_t>((warps + 7) / 8, 148 * 16));
  if (warps)
    k_quant_rows<<<blocks, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), M, K,
                                         int(x.stride(0)), static_cast<uint8_t*>(q.data_ptr()),
                                         static_cast<uint8_t*>(sf.data_ptr()));
}

void fp8_quantize_blocks(const at::Tensor& w, at::Tensor& q, at::Tensor& sf) {
  const int N = int(w.size(0)), K = int(w.size(1));
  check_in(w, q, sf, N, K);
  c10::cuda::CUDAGuard guard(w.device());
  auto st = at::cuda::getCurrentCUDAStream(w.device().index()).stream();
  const int blocks = ((N + 127) / 128) * (K / 128);
  if (blocks)
    k_quant_blocks<<<blocks, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), N, K,
                                           int(w.stride(0)), static_cast<uint8_t*>(q.data_ptr()),
                                           static_cast<uint8_t*>(sf.data_ptr()));
}

void register_fp8(py::module_& m) {
  m.def("fp8_scale_bytes", &fp8_scale_bytes, py::arg("rows"), py::arg("K"));
  m.def("fp8_quantize_rows", &fp8_quantize_rows, py::arg("x"), py::arg("q"), py::arg("sf"),
        "e4m3 + UE8M0 scales per row and 128 columns (activations)");
  m.def("fp8_quantize_blocks", &fp8_quantize_blocks, py::arg("w"), py::arg("q"), py::arg("sf"),
        "e4m3 + UE8M0 scales per 128 x 128 block (weights)");
}
