// Host-side interface of the fused prefill GEMMs (gemm_tcgen05.cu), used by comm.cpp.
#pragma once

#include <torch/extension.h>

#include "proto.h"

namespace sn {

// What a fused GEMM needs to know about the communicator's symmetric region.
struct RegionDesc {
  char* base[kMaxRanks];   // this rank's mapping of every rank's region
  int world, rank;
  uint64_t ctrl_off, gflag_off, push_off, push_cap;
  Status* status;          // device pointer of the pinned status record
};

namespace tc {
// The copy CTAs spread the shard's chunks (or slices of them) among themselves.
void ag_gemm(const RegionDesc& reg, const at::Tensor& x_shard, const at::Tensor& B, at::Tensor& C, at::Tensor& err,
             int copy_ctas, int max_ctas);
void ag_gemm_fp8(const RegionDesc& reg, const at::Tensor& xq_shard, const at::Tensor& sfa_shard, const at::Tensor& B,
                 const at::Tensor& sfb, at::Tensor& C, at::Tensor& err, int copy_ctas, int max_ctas);
void gemm_rs_fp8(const RegionDesc& reg, const at::Tensor& A, const at::Tensor& sfa, const at::Tensor& B,
                 const at::Tensor& sfb, at::Tensor& C_shard, at::Tensor& err, int max_ctas);
void gemm_rs(const RegionDesc& reg, const at::Tensor& A, const at::Tensor& B, at::Tensor& C_shard, at::Tensor& err,
             int max_ctas);
}  // namespace tc

}  // namespace sn
