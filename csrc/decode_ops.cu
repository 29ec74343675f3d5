// Decode-step kernels for the tensor-parallel Llama harness (sm_100a):
//
//   rope_qkv_cache : split the fused QKV projection, rotate q and k (RoPE, rotate-half
//                    form, cos/sin from a table), write k and v into the KV cache at
//                    each sequence's position, emit the rotated q.
//   decode_attention : split-KV flash decoding for grouped-query attention, one query
//                    token per sequence, one launch.  Each block takes one (sequence,
//                    KV head) and one span of the cache, keeps the group's G query
//                    heads in shared memory, and writes unnormalised partial outputs
//                    and (max, sum) pairs into a workspace; the last block of each
//                    (sequence, KV head) merges the spans with their log-sum-exp
//                    weights (kernels in attention_kernels.cuh).
//   add_rmsnorm    : residual add + RMSNorm of rows (the unfused epilogue, used by the
//                    NCCL arm and the first layer), same rounding points as the fused
//                    all-reduce kernel.
//   silu_mul       : SwiGLU activation on the fused gate/up projection.
//   row_argmax     : (max, index) of each row of the logits shard.
//
// The reference has no model code (inference engine is vLLM); these exist so the
// collectives can be measured inside a Llama-3-70B-shaped decode step.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <algorithm>
#include <stdexcept>

#include "sparknet/attention_kernels.cuh"
#include "sparknet/attention_tc.cuh"

namespace py = pybind11;

namespace {

using sn::attn::bf;
using sn::attn::kHead;

// ---------------------------------------------------------------------------
// RoPE + KV cache write.  qkv: [B, (Hq + 2*Hkv) * 128]; cos/sin: [Lmax, 64] fp32;
// positions: [B] int32 (index of the new token); caches: [B, Lmax, Hkv, 128].
// grid (B, Hq + 2*Hkv), block 64: thread i rotates the pair (i, i + 64).
// ---------------------------------------------------------------------------
__global__ void k_rope_qkv_cache(const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ cos_t,
                                 const float* __restrict__ sin_t, const int* __restrict__ positions,
                                 __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                 __nv_bfloat16* __restrict__ v_cache, int Hq, int Hkv, int Lmax) {
  const int b = blockIdx.x, h = blockIdx.y, i = threadIdx.x;
  const int heads = Hq + 2 * Hkv;
  const int pos = positions[b];
  const __nv_bfloat16* src = qkv + (size_t(b) * heads + h) * kHead;
  float x1 = bf(src[i]), x2 = bf(src[i + 64]);
  if (h < Hq + Hkv) {  // q or k: rotate
    float c = cos_t[size_t(pos) * 64 + i], s = sin_t[size_t(pos) * 64 + i];
    float y1 = x1 * c - x2 * s;
    float y2 = x2 * c + x1 * s;
    x1 = y1;
    x2 = y2;
  }
  __nv_bfloat16* dst;
  if (h < Hq) {
    dst = q_out + (size_t(b) * Hq + h) * kHead;
  } else if (h < Hq + Hkv) {
    dst = k_cache + ((size_t(b) * Lmax + pos) * Hkv + (h - Hq)) * kHead;
  } else {
    dst = v_cache + ((size_t(b) * Lmax + pos) * Hkv + (h - Hq - Hkv)) * kHead;
  }
  dst[i] = __float2bfloat16_rn(x1);
  dst[i + 64] = __float2bfloat16_rn(x2);
}

// ---------------------------------------------------------------------------
// residual add + RMSNorm.  One block per row, each thread holding VPT vectors of 8
// bf16 in registers (every load of the row is in flight at once); rounds after the
// add, like the fused all-reduce epilogue.  residual_out may alias residual.
// ---------------------------------------------------------------------------
template <int VPT>
__global__ void __launch_bounds__(1024) k_add_rmsnorm(const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* residual, __nv_bfloat16* residual_out,
                                                      const __nv_bfloat16* __restrict__ gamma,
                                                      __nv_bfloat16* __restrict__ out, int H, float eps) {
  __shared__ float warp_sums[32];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // a PDL-launched successor may start early
  const size_t row = blockIdx.x;
  float v[VPT][8];
  float sq = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = (j * blockDim.x + threadIdx.x) * 8;
    if (i < H) {
      uint4 xv = *reinterpret_cast<const uint4*>(x + row * H + i);
      uint4 rv = make_uint4(0, 0, 0, 0);
      if (residual) rv = *reinterpret_cast<const uint4*>(residual + row * H + i);
      const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 a = __bfloat1622float2(x2[e]);
        if (residual) {
          float2 r = __bfloat1622float2(r2[e]);
          a.x = bf(__float2bfloat16_rn(a.x + r.x));
          a.y = bf(__float2bfloat16_rn(a.y + r.y));
        }
        v[j][2 * e] = a.x;
        v[j][2 * e + 1] = a.y;
        sq += a.x * a.x + a.y * a.y;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = sq;
  __syncthreads();
  float total = 0.0f;
  for (int w = 0; w < int(blockDim.x + 31) / 32; ++w) total += warp_sums[w];
  const float scale = rsqrtf(total / float(H) + eps);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = (j * blockDim.x + threadIdx.x) * 8;
    if (i < H) {
      uint4 gv = *reinterpret_cast<const uint4*>(gamma + i);
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
      uint4 ov, rv;
      uint32_t* o32 = reinterpret_cast<uint32_t*>(&ov);
      uint32_t* r32 = reinterpret_cast<uint32_t*>(&rv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 g = __bfloat1622float2(g2[e]);
        __nv_bfloat162 o = __floats2bfloat162_rn(v[j][2 * e] * scale * g.x, v[j][2 * e + 1] * scale * g.y);
        __nv_bfloat162 r = __floats2bfloat162_rn(v[j][2 * e], v[j][2 * e + 1]);
        o32[e] = *reinterpret_cast<uint32_t*>(&o);
        r32[e] = *reinterpret_cast<uint32_t*>(&r);
      }
      *reinterpret_cast<uint4*>(out + row * H + i) = ov;
      if (residual_out) *reinterpret_cast<uint4*>(residual_out + row * H + i) = rv;
    }
  }
}

// out[b, i] = silu(gate_i) * up_i.  block == 0: gu[b] = [gate | up]; block > 0: gu[b]
// is made of [block gate | block up] column groups (the decode GEMM's SwiGLU layout).
__global__ void k_silu_mul(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int F,
                           size_t total, int block) {
  for (size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    size_t b = idx / F, i = idx % F;
    size_t gi = block ? (i / block) * 2 * block + i % block : i;
    size_t ui = block ? gi + block : F + i;
    float g = bf(gu[b * 2 * F + gi]), u = bf(gu[b * 2 * F + ui]);
    out[idx] = __float2bfloat16_rn(g / (1.0f + expf(-g)) * u);
  }
}

// (max, argmax) of each row; ties take the lowest index.  One block of 1024 threads
// per row; each thread first loads its vectors of 8 (all in flight), then scans them.
__device__ __forceinline__ void better(float& best, int& bi, float v, int i) {
  if (v > best || (v == best && i < bi)) {
    best = v;
    bi = i;
  }
}

template <int VPT>
__global__ void __launch_bounds__(1024) k_row_argmax(const __nv_bfloat16* __restrict__ logits, int V,
                                                     int index_offset, float* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const size_t row = blockIdx.x;
  const __nv_bfloat16* base = logits + row * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  uint4 vec[VPT];
  const bool aligned = (reinterpret_cast<uintptr_t>(base) & 15) == 0;
  const int nvec = aligned ? V / 8 : 0;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int w = j * blockDim.x + threadIdx.x;
    vec[j] = w < nvec ? *reinterpret_cast<const uint4*>(base + size_t(w) * 8) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int w = j * blockDim.x + threadIdx.x;
    if (w < nvec) {
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&vec[j]);
#pragma unroll
      for (int k = 0; k < 8; ++k) better(best, bi, bf(e[k]), w * 8 + k);
    }
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) better(best, bi, bf(base[i]), i);  // tail
  // rows longer than the vectors held in registers
  for (int w = VPT * blockDim.x + threadIdx.x; w < nvec; w += blockDim.x) {
    uint4 q = *reinterpret_cast<const uint4*>(base + size_t(w) * 8);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&q);
    for (int k = 0; k < 8; ++k) better(best, bi, bf(e[k]), w * 8 + k);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(best, bi, ov, oi);
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x + 31) / 32; ++w) better(best, bi, sv[w], si[w]);
    out[row * 2] = best;
    out[row * 2 + 1] = float(bi + index_offset);
  }
}

void check_bf16(const at::Tensor& t, const char* name) {
  if (!t.is_cuda() || t.scalar_type() != at::kBFloat16 || !t.is_contiguous())
    throw std::invalid_argument(std::string(name) + " must be a contiguous CUDA bfloat16 tensor");
}

cudaStream_t stream_of(const at::Tensor& t) { return at::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

void rope_qkv_cache(const at::Tensor& qkv, const at::Tensor& cos_t, const at::Tensor& sin_t,
                    const at::Tensor& positions, at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache, int Hq,
                    int Hkv) {
  check_bf16(qkv, "qkv");
  check_bf16(k_cache, "k_cache");
  int B = int(qkv.size(0)), Lmax = int(k_cache.size(1));
  if (qkv.size(1) != int64_t(Hq + 2 * Hkv) * kHead) throw std::invalid_argument("qkv width mismatch");
  c10::cuda::CUDAGuard guard(qkv.device());
  k_rope_qkv_cache<<<dim3(B, Hq + 2 * Hkv), 64, 0, stream_of(qkv)>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
      positions.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), Hq,
      Hkv, Lmax);
}

// workspace: float32, sn::attn::scratch_floats() long, its first kCounterSlots ints zero
// before the first call (every completed call leaves them zero).
void decode_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                      const at::Tensor& lengths, at::Tensor& out, at::Tensor& workspace, int max_len, double scale,
                      bool pdl, int impl, const c10::optional<at::Tensor>& stamps) {
  check_bf16(q, "q");
  check_bf16(out, "out");
  int B = int(q.size(0)), Hq = int(q.size(1)), Hkv = int(k_cache.size(2)), Lmax = int(k_cache.size(1));
  if (q.size(2) != kHead) throw std::invalid_argument("head_dim must be 128");
  if (Hq % Hkv) throw std::invalid_argument("query heads must be a multiple of KV heads");
  int G = Hq / Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16) throw std::invalid_argument("unsupported GQA group size");
  if (B * Hkv > sn::attn::kCounterSlots) throw std::invalid_argument("too many (sequence, KV head) pairs");
  if (max_len > Lmax) throw std::invalid_argument("max_len exceeds the cache length");
  c10::cuda::CUDAGuard guard(q.device());
  int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  size_t need = sn::attn::scratch_floats(B, Hq, Hkv, max_len, sms);
  if (workspace.scalar_type() != at::kFloat || !workspace.is_contiguous() || size_t(workspace.numel()) < need)
    throw std::invalid_argument("workspace too small for the attention partials");
  if (stamps.has_value() &&
      (impl != 2 || stamps->scalar_type() != at::kLong || !stamps->is_contiguous() ||
       size_t(stamps->numel()) < size_t(B) * Hkv * std::max(1, sn::attn::tc_splits(max_len)) * sn::attn::kTcStamps))
    throw std::invalid_argument("stamps: impl 2 and a contiguous int64 tensor of (grid CTAs x 12) entries");
  cudaError_t e = sn::attn::launch_decode_attention(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr()), lengths.data_ptr<int>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), workspace.data_ptr<float>(), B, Hq, Hkv, Lmax, max_len,
      float(scale), sms, stream_of(q), pdl, impl,
      stamps.has_value() ? reinterpret_cast<uint64_t*>(stamps->data_ptr<int64_t>()) : nullptr);
  if (e != cudaSuccess) throw std::runtime_error(std::string("decode_attention launch: ") + cudaGetErrorString(e));
}

size_t attention_workspace_floats(int B, int Hq, int Hkv, int max_len, int sms) {
  return sn::attn::scratch_floats(B, Hq, Hkv, max_len, sms);
}

void add_rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual,
                 const c10::optional<at::Tensor>& residual_out, const at::Tensor& gamma, at::Tensor& out, double eps) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  check_bf16(gamma, "gamma");
  if (residual) check_bf16(*residual, "residual");
  if (residual_out) check_bf16(*residual_out, "residual_out");
  int rows = int(x.size(0)), H = int(x.size(1));
  if (H % 8 || H > 1024 * 8 * 8) throw std::invalid_argument("add_rmsnorm needs H a multiple of 8, at most 65536");
  c10::cuda::CUDAGuard guard(x.device());
  const int vecs = H / 8;
  const int threads = std::min(1024, (vecs + 31) / 32 * 32);
  const int vpt = (vecs + threads - 1) / threads;
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto rp = residual ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  auto rop = residual_out ? reinterpret_cast<__nv_bfloat16*>(residual_out->data_ptr()) : nullptr;
  auto gp = reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr());
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  auto st = stream_of(x);
  if (vpt == 1) k_add_rmsnorm<1><<<rows, threads, 0, st>>>(xp, rp, rop, gp, op, H, float(eps));
  else if (vpt == 2) k_add_rmsnorm<2><<<rows, threads, 0, st>>>(xp, rp, rop, gp, op, H, float(eps));
  else if (vpt <= 4) k_add_rmsnorm<4><<<rows, threads, 0, st>>>(xp, rp, rop, gp, op, H, float(eps));
  else k_add_rmsnorm<8><<<rows, threads, 0, st>>>(xp, rp, rop, gp, op, H, float(eps));
}

void silu_mul(const at::Tensor& gu, at::Tensor& out, int block) {
  check_bf16(gu, "gate_up");
  int F = int(gu.size(1) / 2);
  if (block < 0 || (block && F % block)) throw std::invalid_argument("silu_mul block must divide the feature count");
  size_t total = size_t(gu.size(0)) * F;
  c10::cuda::CUDAGuard guard(gu.device());
  int blocks = int(std::min<size_t>((total + 255) / 256, 148 * 8));
  k_silu_mul<<<blocks, 256, 0, stream_of(gu)>>>(reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
                                                 reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), F, total, block);
}

void row_argmax(const at::Tensor& logits, int index_offset, at::Tensor& out) {
  check_bf16(logits, "logits");
  c10::cuda::CUDAGuard guard(logits.device());
  const int V = int(logits.size(1));
  auto lp = reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr());
  auto st = stream_of(logits);
  const int rows = int(logits.size(0));
  if (V <= 1024 * 8 * 2) k_row_argmax<2><<<rows, 1024, 0, st>>>(lp, V, index_offset, out.data_ptr<float>());
  else k_row_argmax<4><<<rows, 1024, 0, st>>>(lp, V, index_offset, out.data_ptr<float>());
}

}  // namespace

void register_decode(py::module_& m) {
  m.def("rope_qkv_cache", &rope_qkv_cache);
  m.def("decode_attention", &decode_attention, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("lengths"),
        py::arg("out"), py::arg("workspace"), py::arg("max_len"), py::arg("scale"), py::arg("pdl") = false,
        py::arg("impl") = 0, py::arg("stamps") = py::none(),
        "split-KV decode attention; pdl: programmatic dependent launch (the kernel waits for the previous one "
        "before it reads q, K/V or lengths); impl: 0 tensor cores for 32 or more (sequence, KV head) pairs where "
        "eligible, else CUDA cores; 1 CUDA cores; 2 tensor cores (or an error where not eligible); stamps (impl 2): "
        "int64 tensor of grid x 12 phase timestamps");
  m.def("attention_workspace_floats", &attention_workspace_floats);
  m.def("add_rmsnorm", &add_rmsnorm, py::arg("x"), py::arg("residual"), py::arg("residual_out"), py::arg("gamma"),
        py::arg("out"), py::arg("eps"));
  m.def("silu_mul", &silu_mul, py::arg("gate_up"), py::arg("out"), py::arg("block") = 0);
  m.def("row_argmax", &row_argmax);
}
