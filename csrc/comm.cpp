// Communicator object and Python bindings (sparknet._C).
//
// `Comm` owns the launch-side state of one rank: its view of every peer's
// symmetric region, the region layout, the pinned status record and the launch
// geometry rules.  Python builds the mappings (symm_mem.cpp) and the policy; every
// collective is then one call here that launches one kernel on the caller's current
// CUDA stream, which makes it capturable into CUDA graphs.
//
// An "emulated" communicator holds `world` regions on one GPU and launches every
// rank of a collective in one cooperative grid (rank = blockIdx.y), so the full
// protocol is testable on a single device.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <algorithm>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "sparknet/collectives.h"
#include "sparknet/gemm_fused.h"
#include "sparknet/symm_mem.h"

namespace py = pybind11;

namespace sn {

void ck_rt(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kHalf: return kF16;
    case at::kBFloat16: return kBF16;
    case at::kFloat: return kF32;
    default: throw std::invalid_argument("dtype must be float16, bfloat16 or float32");
  }
}

const char* ptr_of(const at::Tensor& t) { return static_cast<const char*>(t.data_ptr()); }

void require_aligned(const at::Tensor& t, const char* name) {
  if (!t.is_cuda() || !t.is_contiguous()) throw std::invalid_argument(std::string(name) + " must be contiguous CUDA");
  if (reinterpret_cast<uintptr_t>(t.data_ptr()) % kPack)
    throw std::invalid_argument(std::string(name) + " must be 16-byte aligned");
}

class Comm {
 public:
  Comm(int rank, int world, int device, uint64_t lam_cap, uint64_t ll_cap, uint64_t push_cap,
       std::vector<uint64_t> bases, uint64_t mc, uint64_t mc_uc, uint64_t mc_cap, bool emulate)
      : rank_(rank), world_(world), device_(device), emulate_(emulate) {
    if (world < 1 || world > kMaxRanks) throw std::invalid_argument("world must be 1..8");
    if (rank < 0 || rank >= world) throw std::invalid_argument("rank out of range");
    if (!emulate && int(bases.size()) != world) throw std::invalid_argument("need one base address per rank");
    L_ = Layout::make(uint32_t(world), lam_cap, ll_cap, push_cap);
    c10::cuda::CUDAGuard guard(device);
    cudaDeviceProp prop;
    ck_rt(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    sms_ = prop.multiProcessorCount;
    int nstatus = emulate ? world : 1;
    ck_rt(cudaHostAlloc(reinterpret_cast<void**>(&status_h_), sizeof(Status) * nstatus,
                        cudaHostAllocMapped | cudaHostAllocPortable),
          "cudaHostAlloc(status)");
    memset(status_h_, 0, sizeof(Status) * nstatus);
    const cudaError_t pe = cudaHostGetDevicePointer(reinterpret_cast<void**>(&status_d_), status_h_, 0);
    if (pe != cudaSuccess) {  // a constructor that throws runs no destructor
      cudaFreeHost(status_h_);
      status_h_ = nullptr;
      ck_rt(pe, "cudaHostGetDevicePointer(status)");
    }
    for (int i = 0; i < nstatus; ++i) status_h_[i].timeout_us = 10u * 1000u * 1000u;
    if (emulate) {
      // world regions in one device allocation, each rank seeing all of them
      const cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&emu_blob_), L_.total * world);
      if (e != cudaSuccess) {  // a constructor that throws runs no destructor
        cudaFreeHost(status_h_);
        status_h_ = nullptr;
        emu_blob_ = nullptr;
        ck_rt(e, "cudaMalloc(emulated regions)");
      }
      for (int w = 0; w < world; ++w) {
        View& v = emu_.v[w];
        memset(&v, 0, sizeof(v));
        for (int q = 0; q < world; ++q) v.base[q] = emu_blob_ + L_.total * q;
        v.status = status_d_ + w;
      }
      view_ = emu_.v[0];
    } else {
      memset(&view_, 0, sizeof(view_));
      for (int q = 0; q < world; ++q) view_.base[q] = reinterpret_cast<char*>(bases[q]);
      view_.status = status_d_;
      view_.mc = reinterpret_cast<char*>(mc);
      view_.mc_uc = reinterpret_cast<char*>(mc_uc);
      view_.mc_cap = mc_cap;
    }
  }

  ~Comm() {
    if (trace_host_) cudaHostUnregister(trace_host_);
    if (emu_blob_) cudaFree(emu_blob_);
    if (status_h_) cudaFreeHost(status_h_);
  }

  // Zero control words and flags, fill Lamport slots with the sentinel.  Local
  // region only (emulated: all regions).  Callers barrier across ranks afterwards.
  void init_region() {
    c10::cuda::CUDAGuard guard(device_);
    int n = emulate_ ? world_ : 1;
    for (int w = 0; w < n; ++w) {
      char* base = emulate_ ? emu_.v[w].base[w] : view_.base[rank_];
      ck_rt(cudaMemset(base, 0, L_.lam_off), "memset ctrl");
      ck_rt(cudaMemset(base + L_.lam_off, 0xff, L_.ll_off - L_.lam_off), "memset lamport");
      ck_rt(cudaMemset(base + L_.ll_off, 0, L_.total - L_.ll_off), "memset ll/push");
      status_h_[w].failed_seq = 0;
      status_h_[w].kind = 0;
    }
    ck_rt(cudaDeviceSynchronize(), "init_region sync");
  }

  // -- geometry (rank-invariant: depends on sizes and world only) ---------------
  LaunchGeom geom(uint64_t items, int threads, int max_blocks) const {
    if (threads < 32 || threads > kMaxThreads || threads % 32)
      throw std::invalid_argument("threads must be a multiple of 32 between 32 and " + std::to_string(kMaxThreads));
    LaunchGeom g;
    g.threads = threads;
    int cap = max_blocks > 0 ? max_blocks : sms_;
    if (emulate_) {
      // every emulated rank's blocks must be co-resident in one cooperative grid
      cap = std::max(1, std::min(cap, (sms_ * 2) / world_));
    }
    cap = std::min(cap, kMaxBlocks);
    uint64_t want = (items + threads - 1) / threads;
    g.blocks = int(std::max<uint64_t>(1, std::min<uint64_t>(want, uint64_t(cap))));
    g.ranks = world_;
    g.emulate = emulate_;
    g.cluster = 1;
    g.pdl = pdl_ && !emulate_;
    return g;
  }

  Job job(uint64_t nbytes) const {
    Job j;
    memset(&j, 0, sizeof(j));
    j.v = view_;
    j.L = L_;
    j.rank = uint32_t(rank_);
    j.world = uint32_t(world_);
    j.nbytes = nbytes;
    j.valid_out_bytes = -1;
    j.skip_rank = skip_rank_;
    j.pdl = (pdl_ && !emulate_) ? 1u : 0u;
    j.trace = trace_d_;
    return j;
  }

  EmuViews emu_views(const std::vector<at::Tensor>& ins, const std::vector<at::Tensor>& outs,
                     const std::vector<at::Tensor>* res = nullptr,
                     const std::vector<at::Tensor>* res_out = nullptr) const {
    EmuViews e = emu_;
    if (int(ins.size()) != world_ || int(outs.size()) != world_)
      throw std::invalid_argument("emulated collectives take one input and one output per rank");
    for (int w = 0; w < world_; ++w) {
      e.in[w] = ptr_of(ins[w]);
      e.out[w] = static_cast<char*>(outs[w].data_ptr());
      e.residual[w] = res ? ptr_of((*res)[w]) : nullptr;
      e.residual_out[w] = res_out ? static_cast<char*>((*res_out)[w].data_ptr()) : nullptr;
    }
    return e;
  }

  void check_views(const std::vector<at::Tensor>& ins, const std::vector<at::Tensor>& outs) const {
    size_t want = emulate_ ? size_t(world_) : 1u;
    if (ins.size() != want || outs.size() != want) throw std::invalid_argument("wrong number of tensors");
    for (auto& t : ins) require_aligned(t, "input");
    for (auto& t : outs) require_aligned(t, "output");
  }

  // -- collectives ----------------------------------------------------------------
  void all_reduce(const std::vector<at::Tensor>& ins, const std::vector<at::Tensor>& outs, int algo, int threads,
                  int max_blocks) {
    check_views(ins, outs);
    const at::Tensor& in = ins[0];
    uint64_t nbytes = uint64_t(in.numel()) * in.element_size();
    if (nbytes % kPack) throw std::invalid_argument("all-reduce size must be a multiple of 16 bytes");
    if (algo == kLocal) {
      if (world_ != 1 || emulate_) throw std::invalid_argument("the local all-reduce is the one-rank case");
      if (in.data_ptr() == outs[0].data_ptr()) return;  // in place: the input already is the sum
      launch_copy_local(ptr_of(in), static_cast<char*>(outs[0].data_ptr()), nbytes, threads ? threads : 512,
                        max_blocks > 0 ? max_blocks : 2 * sms_, at::cuda::getCurrentCUDAStream(device_).stream());
      return;
    }
    if (algo == kNvls && !view_.mc) throw std::invalid_argument("NVLS is not available on this communicator");
    if (algo == kNvls && nbytes > view_.mc_cap) throw std::invalid_argument("message exceeds the NVLS buffer");
    if (algo == kOneShot && nbytes > L_.lam_cap) throw std::invalid_argument("message exceeds one-shot capacity");
    if (algo == kTwoShot && (nbytes + kPack * world_) / world_ > L_.lam_cap / 2)
      throw std::invalid_argument("message exceeds two-shot capacity");
    uint64_t packs = nbytes / kPack;
    uint64_t items = (algo == kOneShot || world_ == 1) ? packs : (packs + world_ - 1) / world_;
    LaunchGeom g = geom(items, threads ? threads : 512, max_blocks);
    Job j = job(nbytes);
    j.in = ptr_of(in);
    j.out = static_cast<char*>(outs[0].data_ptr());
    auto stream = at::cuda::getCurrentCUDAStream(device_).stream();
    if (emulate_) {
      EmuViews e = emu_views(ins, outs);
      launch_allreduce(j, &e, dtype_code(in), algo, g, stream);
    } else {
      launch_allreduce(j, nullptr, dtype_code(in), algo, g, stream);
    }
  }

  void reduce_scatter(const std::vector<at::Tensor>& ins, const std::vector<at::Tensor>& outs, uint64_t chunk_bytes,
                      uint64_t src_peer_stride, int threads, int max_blocks) {
    check_views(ins, outs);
    if (chunk_bytes % kPack || src_peer_stride % kPack) throw std::invalid_argument("16-byte chunks required");
    if (chunk_bytes > L_.lam_cap) throw std::invalid_argument("chunk exceeds reduce-scatter capacity");
    LaunchGeom g = geom(chunk_bytes / kPack, threads ? threads : 512, max_blocks);
    Job j = job(chunk_bytes);
    j.in = ptr_of(ins[0]);
    j.out = static_cast<char*>(outs[0].data_ptr());
    j.src_peer_stride = src_peer_stride;
    auto stream = at::cuda::getCurrentCUDAStream(device_).stream();
    if (emulate_) {
      EmuViews e = emu_views(ins, outs);
      launch_reducescatter(j, &e, dtype_code(ins[0]), g, stream);
    } else {
      launch_reducescatter(j, nullptr, dtype_code(ins[0]), g, stream);
    }
  }

  void all_gather(const std::vector<at::Tensor>& ins, const std::vector<at::Tensor>& outs, uint64_t shard_bytes,
                  uint64_t row_bytes, uint64_t dst_row_stride, uint64_t dst_src_stride, int algo, int threads,
                  int max_blocks) {
    check_views(ins, outs);
    uint64_t items;
    if (algo == kGatherLL) {
      if (shard_bytes % 8 || (row_bytes && row_bytes % 8)) throw std::invalid_argument("LL gather needs 8-byte rows");
      if (shard_bytes > L_.ll_cap) throw std::invalid_argument("shard exceeds LL capacity");
      items = shard_bytes / 8;
    } else {
      if (shard_bytes % kPack || (row_bytes && row_bytes % kPack))
        throw std::invalid_argument("bulk gather needs 16-byte rows");
      if (algo == kGatherNvls) {
        if (!view_.mc) throw std::invalid_argument("NVLS is not available on this communicator");
        if (shard_bytes * world_ > view_.mc_cap) throw std::invalid_argument("gather exceeds the NVLS buffer");
      } else if (shard_bytes > L_.push_cap) {
        throw std::invalid_argument("shard exceeds push capacity");
      }
      items = shard_bytes / kPack;
    }
    LaunchGeom g = geom(items, threads ? threads : 512, max_blocks);
    Job j = job(shard_bytes);
    j.in = ptr_of(ins[0]);
    j.out = static_cast<char*>(outs[0].data_ptr());
    j.row_bytes = row_bytes;
    j.dst_row_stride = dst_row_stride;
    j.dst_src_stride = dst_src_stride;
    auto stream = at::cuda::getCurrentCUDAStream(device_).stream();
    if (emulate_) {
      EmuViews e = emu_views(ins, outs);
      launch_gather(j, &e, algo, kOpAllGather, g, stream);
    } else {
      launch_gather(j, nullptr, algo, kOpAllGather, g, stream);
    }
  }

  void exchange(const std::vector<at::Tensor>& ins, const std::vector<at::Tensor>& outs, uint64_t chunk_bytes,
                uint64_t src_peer_stride, uint64_t dst_peer_stride, uint64_t total_src_bytes, int64_t valid_out_bytes,
                bool copy_self, int threads, int max_blocks) {
    size_t want = emulate_ ? size_t(world_) : 1u;
    if (ins.size() != want || outs.size() != want) throw std::invalid_argument("wrong number of tensors");
    // chunks are addressed by byte strides from the first element: strided slices are fine
    for (auto* v : {&ins, &outs})
      for (auto& t : *v)
        if (!t.is_cuda() || reinterpret_cast<uintptr_t>(t.data_ptr()) % kPack)
          throw std::invalid_argument("exchange tensors must be 16-byte aligned CUDA tensors");
    if (chunk_bytes % kPack || src_peer_stride % kPack || dst_peer_stride % kPack)
      throw std::invalid_argument("exchange needs 16-byte chunks and strides");
    if (chunk_bytes > L_.push_cap) throw std::invalid_argument("chunk exceeds push capacity");
    LaunchGeom g = geom(chunk_bytes / kPack, threads ? threads : 512, max_blocks);
    Job j = job(chunk_bytes);
    j.in = ptr_of(ins[0]);
    j.out = static_cast<char*>(outs[0].data_ptr());
    j.src_peer_stride = src_peer_stride;
    j.dst_src_stride = dst_peer_stride;
    j.total_src_bytes = total_src_bytes;
    j.valid_out_bytes = valid_out_bytes;
    j.copy_self = copy_self ? 1u : 0u;
    auto stream = at::cuda::getCurrentCUDAStream(device_).stream();
    if (emulate_) {
      EmuViews e = emu_views(ins, outs);
      launch_gather(j, &e, kGatherPush, kOpExchange, g, stream);
    } else {
      launch_gather(j, nullptr, kGatherPush, kOpExchange, g, stream);
    }
  }

  void barrier(int blocks) {
    LaunchGeom g = geom(uint64_t(blocks) * 32, 32, blocks);
    Job j = job(0);
    auto stream = at::cuda::getCurrentCUDAStream(device_).stream();
    if (emulate_) {
      EmuViews e = emu_;
      launch_gather(j, &e, kGatherPush, kOpBarrier, g, stream);
    } else {
      launch_gather(j, nullptr, kGatherPush, kOpBarrier, g, stream);
    }
  }

  struct FusedPlan {
    Job j;
    LaunchGeom g;
    int dtype;
  };

  // Every check of the fused norm, and its launch description; launches nothing (so a
  // caller can validate before it launches anything that writes into peers' slots).
  FusedPlan plan_fused_norm(const std::vector<at::Tensor>& ins, const std::vector<at::Tensor>& residuals,
                            const at::Tensor& gamma, double eps, const std::vector<at::Tensor>& outs,
                            const std::vector<at::Tensor>& residual_outs, int algo, int cluster, int max_clusters,
                            int threads = 0) const {
    check_views(ins, outs);
    check_views(residuals, residual_outs);
    require_aligned(gamma, "gamma");
    const at::Tensor& x = ins[0];
    if (x.dim() != 2) throw std::invalid_argument("fused norm takes [tokens, hidden]");
    int64_t T = x.size(0), H = x.size(1);
    int elems = 16 / int(x.element_size());
    if (H % (elems * cluster)) throw std::invalid_argument("hidden must split into 16-byte packs per cluster CTA");
    uint64_t nbytes = uint64_t(T) * H * x.element_size();
    if (algo == kTwoShot && world_ > 1) {
      uint64_t rows_per_owner = (uint64_t(T) + world_ - 1) / world_;
      if (rows_per_owner * H * x.element_size() > L_.lam_cap / 2)
        throw std::invalid_argument("tokens exceed fused two-shot capacity");
    } else if (nbytes > L_.lam_cap) {
      throw std::invalid_argument("tokens exceed fused one-shot capacity");
    }
    // One 16-byte pack per thread when it fits in a block; otherwise each thread takes
    // every blockDim-th pack of its CTA's share (the kernel follows the launch it got).
    int cta_packs = int(H / elems / cluster);
    if (threads < 0 || threads % 32 || threads > kMaxThreads)
      throw std::invalid_argument("fused norm threads must be 0 (auto) or a multiple of 32 up to " +
                                  std::to_string(kMaxThreads));
    LaunchGeom g;
    g.threads = threads ? threads : std::min(kMaxThreads, std::max(32, (cta_packs + 31) / 32 * 32));
    int nclusters = int(std::min<int64_t>(T, max_clusters > 0 ? max_clusters : 64));
    if (emulate_) nclusters = std::max(1, std::min(nclusters, (sms_ * 4) / (cluster * world_)));
    g.blocks = nclusters * cluster;
    g.cluster = cluster;
    g.ranks = world_;
    g.emulate = emulate_;
    g.pdl = pdl_ && !emulate_;
    Job j = job(nbytes);
    j.in = ptr_of(x);
    j.out = static_cast<char*>(outs[0].data_ptr());
    j.residual = ptr_of(residuals[0]);
    j.residual_out = static_cast<char*>(residual_outs[0].data_ptr());
    j.gamma = ptr_of(gamma);
    j.eps = float(eps);
    j.hidden = uint32_t(H);
    return FusedPlan{j, g, dtype_code(x)};
  }

  void fused_norm(const std::vector<at::Tensor>& ins, const std::vector<at::Tensor>& residuals,
                  const at::Tensor& gamma, double eps, const std::vector<at::Tensor>& outs,
                  const std::vector<at::Tensor>& residual_outs, int algo, int cluster, int max_clusters,
                  int threads = 0) {
    FusedPlan p = plan_fused_norm(ins, residuals, gamma, eps, outs, residual_outs, algo, cluster, max_clusters,
                                  threads);
    auto stream = at::cuda::getCurrentCUDAStream(device_).stream();
    if (emulate_) {
      EmuViews e = emu_views(ins, outs, &residuals, &residual_outs);
      launch_fused_norm(p.j, &e, p.dtype, algo, p.g, stream);
    } else {
      launch_fused_norm(p.j, nullptr, p.dtype, algo, p.g, stream);
    }
  }



  // -- fused prefill GEMMs (tcgen05) ----------------------------------------------
  RegionDesc region() const {
    if (emulate_) throw std::invalid_argument("the fused GEMMs run on real ranks (one GPU each)");
    RegionDesc r;
    memset(&r, 0, sizeof(r));
    for (int q = 0; q < world_; ++q) r.base[q] = view_.base[q];
    r.world = world_;
    r.rank = rank_;
    r.ctrl_off = L_.ctrl_off;
    r.gflag_off = L_.gflag_off;
    r.push_off = L_.push_off;
    r.push_cap = L_.push_cap;
    r.status = status_d_;
    return r;
  }

  void ag_gemm(const at::Tensor& x_shard, const at::Tensor& w, at::Tensor& out, at::Tensor& err, int copy_ctas,
               int max_ctas) {
    tc::ag_gemm(region(), x_shard, w, out, err, copy_ctas, max_ctas);
  }

  void ag_gemm_fp8(const at::Tensor& xq_shard, const at::Tensor& sfa_shard, const at::Tensor& w,
                   const at::Tensor& sfw, at::Tensor& out, at::Tensor& err, int copy_ctas, int max_ctas) {
    tc::ag_gemm_fp8(region(), xq_shard, sfa_shard, w, sfw, out, err, copy_ctas, max_ctas);
  }
  void gemm_rs_fp8(const at::Tensor& a, const at::Tensor& sfa, const at::Tensor& w, const at::Tensor& sfw,
                   at::Tensor& out, at::Tensor& err, int max_ctas) {
    tc::gemm_rs_fp8(region(), a, sfa, w, sfw, out, err, max_ctas);
  }
  void gemm_rs(const at::Tensor& a, const at::Tensor& w, at::Tensor& out, at::Tensor& err, int max_ctas) {
    tc::gemm_rs(region(), a, w, out, err, max_ctas);
  }

  // -- health ---------------------------------------------------------------------
  py::dict status(int which) const {
    const Status& s = status_h_[which];
    py::dict d;
    d["timeout_us"] = s.timeout_us;
    d["failed_seq"] = s.failed_seq;
    d["kind"] = s.kind;
    d["peer"] = s.peer;
    d["block"] = s.block;
    d["waited_us"] = s.waited_us;
    d["op"] = s.op;
    return d;
  }
  uint32_t failed_seq(int which) const { return status_h_[which].failed_seq; }
  void set_timeout_us(uint32_t us) {
    int n = emulate_ ? world_ : 1;
    for (int i = 0; i < n; ++i) status_h_[i].timeout_us = us;
  }
  uint64_t status_address() const { return reinterpret_cast<uint64_t>(status_h_); }

  // Device control words (synchronous read; diagnostics only).
  py::dict ctrl(int which) const {
    c10::cuda::CUDAGuard guard(device_);
    Ctrl c;
    const char* base = emulate_ ? emu_.v[which].base[which] : view_.base[rank_];
    ck_rt(cudaMemcpy(&c, base + L_.ctrl_off, sizeof(Ctrl), cudaMemcpyDeviceToHost), "read ctrl");
    py::dict d;
    d["epoch"] = c.epoch;
    d["done"] = c.done;
    d["poison"] = c.poison;
    d["ops"] = c.ops;
    return d;
  }

  py::dict layout() const {
    py::dict d;
    d["world"] = L_.world;
    d["lam_cap"] = L_.lam_cap;
    d["ll_cap"] = L_.ll_cap;
    d["push_cap"] = L_.push_cap;
    d["lam_off"] = L_.lam_off;
    d["ll_off"] = L_.ll_off;
    d["push_off"] = L_.push_off;
    d["total"] = L_.total;
    d["abi"] = kAbiVersion;
    return d;
  }

  // Trace file: pin the host mapping [addr, addr + bytes) and stamp collectives into
  // its records (after a header of kTraceHeaderBytes).  addr 0 turns tracing off.
  void set_trace(uint64_t addr, uint64_t bytes) {
    if (trace_host_) {
      cudaHostUnregister(trace_host_);
      trace_host_ = nullptr;
      trace_d_ = nullptr;
    }
    if (!addr) return;
    if (bytes < kTraceHeaderBytes + uint64_t(kTraceRecords) * kTraceWords * 8)
      throw std::invalid_argument("trace mapping too small");
    c10::cuda::CUDAGuard guard(device_);
    void* h = reinterpret_cast<void*>(addr);
    ck_rt(cudaHostRegister(h, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable), "cudaHostRegister(trace)");
    void* d = nullptr;
    ck_rt(cudaHostGetDevicePointer(&d, h, 0), "cudaHostGetDevicePointer(trace)");
    trace_host_ = h;
    trace_d_ = reinterpret_cast<uint64_t*>(static_cast<char*>(d) + kTraceHeaderBytes);
  }

  // Test hook: in an emulated group, rank `r` skips every following launch (-1: none).
  void set_skip_rank(int r) {
    if (!emulate_ && r >= 0) throw std::invalid_argument("skip_rank is a test hook of emulated groups");
    skip_rank_ = r;
  }

  // Launch the collective kernels with programmatic stream serialisation (each waits
  // for its predecessor on the stream before touching anything, then lets its own
  // successor be scheduled).  Emulated groups always launch cooperatively, never so.
  void set_pdl(bool on) { pdl_ = on; }
  bool pdl() const { return pdl_ && !emulate_; }

  int rank() const { return rank_; }
  int world() const { return world_; }
  bool emulated() const { return emulate_; }
  bool has_multicast() const { return view_.mc != nullptr; }
  int sms() const { return sms_; }

 private:
  int rank_, world_, device_;
  bool emulate_;
  int sms_ = 148;
  Layout L_;
  View view_;
  EmuViews emu_{};
  char* emu_blob_ = nullptr;
  Status* status_h_ = nullptr;
  Status* status_d_ = nullptr;
  int skip_rank_ = -1;
  bool pdl_ = false;
  void* trace_host_ = nullptr;
  uint64_t* trace_d_ = nullptr;
};

uint64_t layout_total(int world, uint64_t lam_cap, uint64_t ll_cap, uint64_t push_cap) {
  return Layout::make(uint32_t(world), lam_cap, ll_cap, push_cap).total;
}

}  // namespace sn

void register_trace(py::module_& m);
void register_gemm(py::module_& m);
void register_gemm_pair(py::module_& m);
void register_decode(py::module_& m);
void register_skinny(py::module_& m);
void register_fp8(py::module_& m);
void register_microbench(py::module_& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace sn;
  m.doc() = "sparknet native core: symmetric memory over NVLink and sm_100a collective kernels";
  m.attr("ABI_VERSION") = kAbiVersion;
  m.attr("MAX_RANKS") = kMaxRanks;
  m.attr("MAX_BLOCKS") = kMaxBlocks;
  m.attr("TRACE_WORDS") = kTraceWords;
  m.attr("TRACE_RECORDS") = kTraceRecords;
  m.attr("TRACE_HEADER_BYTES") = kTraceHeaderBytes;
  m.def("layout_total", &layout_total);
  m.def("fd_listen", &fd_listen);
  m.def("fd_serve", &fd_serve, py::call_guard<py::gil_scoped_release>());
  m.def("fd_fetch", &fd_fetch, py::call_guard<py::gil_scoped_release>());
  m.def("fd_close", &fd_close);
  m.def("vmm_granularity", &vmm_granularity);
  m.def("device_attribute", &device_attribute);
  m.def("multicast_supported", &multicast_supported);

  py::class_<LocalRegion, std::shared_ptr<LocalRegion>>(m, "LocalRegion")
      .def(py::init<int, size_t, size_t>(), py::arg("device"), py::arg("bytes"), py::arg("align") = 0)
      .def_property_readonly("ptr", &LocalRegion::ptr)
      .def_property_readonly("bytes", &LocalRegion::bytes)
      .def("export_fd", &LocalRegion::export_fd)
      .def("map_peer", &LocalRegion::map_peer);

  py::class_<Multicast, std::shared_ptr<Multicast>>(m, "Multicast")
      .def(py::init<int, size_t, int>())
      .def("create_and_export", &Multicast::create_and_export)
      .def("import_handle", &Multicast::import_handle)
      .def("add_device", &Multicast::add_device)
      .def("bind_and_map", &Multicast::bind_and_map)
      .def_property_readonly("mc_ptr", &Multicast::mc_ptr)
      .def_property_readonly("uc_ptr", &Multicast::uc_ptr)
      .def_property_readonly("bytes", &Multicast::bytes);

  py::class_<Comm, std::shared_ptr<Comm>>(m, "Comm")
      .def(py::init<int, int, int, uint64_t, uint64_t, uint64_t, std::vector<uint64_t>, uint64_t, uint64_t, uint64_t,
                    bool>(),
           py::arg("rank"), py::arg("world"), py::arg("device"), py::arg("lam_cap"), py::arg("ll_cap"),
           py::arg("push_cap"), py::arg("bases"), py::arg("mc") = 0, py::arg("mc_uc") = 0, py::arg("mc_cap") = 0,
           py::arg("emulate") = false)
      .def("init_region", &Comm::init_region)
      .def("all_reduce", &Comm::all_reduce, py::arg("ins"), py::arg("outs"), py::arg("algo"),
           py::arg("threads") = 0, py::arg("max_blocks") = 0)
      .def("reduce_scatter", &Comm::reduce_scatter, py::arg("ins"), py::arg("outs"), py::arg("chunk_bytes"),
           py::arg("src_peer_stride"), py::arg("threads") = 0, py::arg("max_blocks") = 0)
      .def("all_gather", &Comm::all_gather, py::arg("ins"), py::arg("outs"), py::arg("shard_bytes"),
           py::arg("row_bytes"), py::arg("dst_row_stride"), py::arg("dst_src_stride"), py::arg("algo"),
           py::arg("threads") = 0, py::arg("max_blocks") = 0)
      .def("exchange", &Comm::exchange, py::arg("ins"), py::arg("outs"), py::arg("chunk_bytes"),
           py::arg("src_peer_stride"), py::arg("dst_peer_stride"), py::arg("total_src_bytes"),
           py::arg("valid_out_bytes"), py::arg("copy_self"), py::arg("threads") = 0, py::arg("max_blocks") = 0)
      .def("barrier", &Comm::barrier, py::arg("blocks") = 1)
      .def("ag_gemm", &Comm::ag_gemm, py::arg("x_shard"), py::arg("w"), py::arg("out"), py::arg("err"),
           py::arg("copy_ctas") = 16, py::arg("max_ctas") = 0)
      .def("gemm_rs", &Comm::gemm_rs, py::arg("a"), py::arg("w"), py::arg("out"), py::arg("err"),
           py::arg("max_ctas") = 0)
      .def("ag_gemm_fp8", &Comm::ag_gemm_fp8, py::arg("xq_shard"), py::arg("sfa_shard"), py::arg("w"),
           py::arg("sfw"), py::arg("out"), py::arg("err"), py::arg("copy_ctas") = 8, py::arg("max_ctas") = 0)
      .def("gemm_rs_fp8", &Comm::gemm_rs_fp8, py::arg("a"), py::arg("sfa"), py::arg("w"), py::arg("sfw"),
           py::arg("out"), py::arg("err"), py::arg("max_ctas") = 0)
      .def("fused_norm", &Comm::fused_norm, py::arg("ins"), py::arg("residuals"), py::arg("gamma"), py::arg("eps"),
           py::arg("outs"), py::arg("residual_outs"), py::arg("algo"), py::arg("cluster") = 8,
           py::arg("max_clusters") = 0, py::arg("threads") = 0)
      .def("status", &Comm::status, py::arg("which") = 0)
      .def("failed_seq", &Comm::failed_seq, py::arg("which") = 0)
      .def("set_timeout_us", &Comm::set_timeout_us)
      .def("set_skip_rank", &Comm::set_skip_rank)
      .def("set_pdl", &Comm::set_pdl)
      .def_property_readonly("pdl", &Comm::pdl)
      .def("set_trace", &Comm::set_trace)
      .def("status_address", &Comm::status_address)
      .def("ctrl", &Comm::ctrl, py::arg("which") = 0)
      .def("layout", &Comm::layout)
      .def_property_readonly("rank", &Comm::rank)
      .def_property_readonly("world", &Comm::world)
      .def_property_readonly("emulated", &Comm::emulated)
      .def_property_readonly("has_multicast", &Comm::has_multicast)
      .def_property_readonly("sms", &Comm::sms);

  register_trace(m);
  register_gemm(m);
  register_gemm_pair(m);
  register_decode(m);
  register_skinny(m);
  register_fp8(m);
  register_microbench(m);
}
