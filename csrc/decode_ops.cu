// Decode-step kernels for the tensor-parallel Llama harness (sm_100a):
//
//   rope_qkv_cache : split the fused QKV projection, rotate q and k (RoPE, rotate-half
//                    form, cos/sin from a table), write k and v into the KV cache at
//                    each sequence's position, emit the rotated q.
//   decode_attention (+ combine): split-KV flash decoding for grouped-query attention
//                    (one query token per sequence).  Each block takes one (sequence,
//                    KV head) and one span of the cache, keeps the group's G query
//                    heads in shared memory, and writes unnormalised partial outputs
//                    and (max, sum) pairs into a workspace; the combine kernel merges
//                    the spans with their log-sum-exp weights.
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

namespace py = pybind11;

namespace {

using sn::attn::bf;
using sn::attn::k_decode_attn;
using sn::attn::k_decode_combine;
using sn::attn::kHead;
using sn::attn::kLog2e;
using sn::attn::kTile;

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
// residual add + RMSNorm.  One block per row; rounds after the add, like the fused
// all-reduce epilogue.  residual_out may alias residual.
// ---------------------------------------------------------------------------
__global__ void k_add_rmsnorm(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* residual,
                              __nv_bfloat16* residual_out, const __nv_bfloat16* __restrict__ gamma,
                              __nv_bfloat16* __restrict__ out, int H, float eps) {
  extern __shared__ float rowbuf[];
  __shared__ float warp_sums[32];
  const size_t row = blockIdx.x;
  float sq = 0.0f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = bf(x[row * H + i]);
    if (residual) v = bf(__float2bfloat16_rn(v + bf(residual[row * H + i])));
    rowbuf[i] = v;
    sq += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = sq;
  __syncthreads();
  float total = 0.0f;
  for (int w = 0; w < int(blockDim.x + 31) / 32; ++w) total += warp_sums[w];
  const float scale = rsqrtf(total / float(H) + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = rowbuf[i];
    if (residual_out) residual_out[row * H + i] = __float2bfloat16_rn(v);
    out[row * H + i] = __float2bfloat16_rn(v * scale * bf(gamma[i]));
  }
}

// out[b, i] = silu(gu[b, i]) * gu[b, F + i]
__global__ void k_silu_mul(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int F,
                           size_t total) {
  for (size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    size_t b = idx / F, i = idx % F;
    float g = bf(gu[b * 2 * F + i]), u = bf(gu[b * 2 * F + F + i]);
    out[idx] = __float2bfloat16_rn(g / (1.0f + expf(-g)) * u);
  }
}

// (max, argmax) of each row; ties take the lowest index.  One block per row.
__global__ void k_row_argmax(const __nv_bfloat16* __restrict__ logits, int V, int index_offset,
                             float* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const size_t row = blockIdx.x;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float v = bf(logits[row * V + i]);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x + 31) / 32; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
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

int attn_splits(int B, int Hkv, int max_len, int sms) { return sn::attn::splits(B, Hkv, max_len, sms); }

void decode_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                      const at::Tensor& lengths, at::Tensor& out, at::Tensor& workspace, int max_len, double scale) {
  check_bf16(q, "q");
  check_bf16(out, "out");
  int B = int(q.size(0)), Hq = int(q.size(1)), Hkv = int(k_cache.size(2)), Lmax = int(k_cache.size(1));
  if (q.size(2) != kHead) throw std::invalid_argument("head_dim must be 128");
  if (Hq % Hkv) throw std::invalid_argument("query heads must be a multiple of KV heads");
  int G = Hq / Hkv;
  c10::cuda::CUDAGuard guard(q.device());
  int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  int nsplit = attn_splits(B, Hkv, max_len, sms);
  int chunk = ((max_len + nsplit - 1) / nsplit + kTile - 1) / kTile * kTile;
  size_t need = size_t(B) * Hq * nsplit * (kHead + 2);
  if (workspace.scalar_type() != at::kFloat || size_t(workspace.numel()) < need)
    throw std::invalid_argument("workspace too small for the attention partials");
  float* part_o = workspace.data_ptr<float>();
  float* part_ml = part_o + size_t(B) * Hq * nsplit * kHead;
  auto st = stream_of(q);
  float scale_log2 = float(scale) * kLog2e;
  dim3 grid(B * Hkv, nsplit);
#define SN_ATT(GG)                                                                                          \
  case GG:                                                                                                  \
    k_decode_attn<GG><<<grid, 128, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()),           \
                                            reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr()),     \
                                            reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr()),     \
                                            lengths.data_ptr<int>(), part_o, part_ml, Hkv, Lmax, chunk,     \
                                            scale_log2);                                                    \
    break;
  switch (G) {
    SN_ATT(1)
    SN_ATT(2)
    SN_ATT(4)
    SN_ATT(8)
    SN_ATT(16)
    default:
      throw std::invalid_argument("unsupported GQA group size");
  }
#undef SN_ATT
  k_decode_combine<<<B * Hq, kHead, 0, st>>>(part_o, part_ml, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                              nsplit);
}

size_t attention_workspace_floats(int B, int Hq, int Hkv, int max_len, int sms) {
  return size_t(B) * Hq * attn_splits(B, Hkv, max_len, sms) * (kHead + 2);
}

void add_rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual,
                 const c10::optional<at::Tensor>& residual_out, const at::Tensor& gamma, at::Tensor& out, double eps) {
  check_bf16(x, "x");
  int rows = int(x.size(0)), H = int(x.size(1));
  c10::cuda::CUDAGuard guard(x.device());
  k_add_rmsnorm<<<rows, 256, H * sizeof(float), stream_of(x)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      residual ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr,
      residual_out ? reinterpret_cast<__nv_bfloat16*>(residual_out->data_ptr()) : nullptr,
      reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), H,
      float(eps));
}

void silu_mul(const at::Tensor& gu, at::Tensor& out) {
  check_bf16(gu, "gate_up");
  int F = int(gu.size(1) / 2);
  size_t total = size_t(gu.size(0)) * F;
  c10::cuda::CUDAGuard guard(gu.device());
  int blocks = int(std::min<size_t>((total + 255) / 256, 148 * 8));
  k_silu_mul<<<blocks, 256, 0, stream_of(gu)>>>(reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
                                                 reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), F, total);
}

void row_argmax(const at::Tensor& logits, int index_offset, at::Tensor& out) {
  check_bf16(logits, "logits");
  c10::cuda::CUDAGuard guard(logits.device());
  k_row_argmax<<<int(logits.size(0)), 512, 0, stream_of(logits)>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), int(logits.size(1)), index_offset,
      out.data_ptr<float>());
}

}  // namespace

void register_decode(py::module_& m) {
  m.def("rope_qkv_cache", &rope_qkv_cache);
  m.def("decode_attention", &decode_attention);
  m.def("attention_workspace_floats", &attention_workspace_floats);
  m.def("add_rmsnorm", &add_rmsnorm, py::arg("x"), py::arg("residual"), py::arg("residual_out"), py::arg("gamma"),
        py::arg("out"), py::arg("eps"));
  m.def("silu_mul", &silu_mul);
  m.def("row_argmax", &row_argmax);
}
