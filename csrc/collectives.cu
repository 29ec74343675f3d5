// sm_100a collective kernels: one-shot / two-shot / NVLS all-reduce, all-gather
// (LL8, bulk push, NVLS broadcast), reduce-scatter, exchange and a barrier.
//
// Each kernel is one launch that moves data over NVLink with device stores into
// peers' symmetric regions (no host in the loop) and reads the device-resident
// epoch at entry, so it replays inside CUDA graphs.  Reference kernels these
// replace: sparknet/oneshot/_oneshot_tilelang.py:68-184 (all-reduce),
// _allgather_tilelang.py:29-113, _reducescatter_tilelang.py:33-203,
// _exchange_tilelang.py:27-203.
//
// Every kernel has an "emulated" twin (grid.y = world, rank = blockIdx.y) that runs
// all ranks of a collective inside one cooperative launch on one GPU: the protocol
// is exercised end to end without two processes spinning on one device.
#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "sparknet/collectives.h"
#include "sparknet/dev_mem.cuh"

namespace sn {

namespace {

SN_DEV Ctrl* ctrl_of(const Job& j) { return reinterpret_cast<Ctrl*>(j.v.base[j.rank] + j.L.ctrl_off); }

// Programmatic dependent launch (Job::pdl): wait until the previous kernel on the
// stream has finished and its writes are visible (the epoch it published included),
// then let the next programmatically serialised launch be scheduled.  The trigger
// comes from blocks that are already running, so a successor can only take SM slots
// once this whole grid is resident: no block of a collective waits on peers while
// one of its own blocks is kept off the GPU.
SN_DEV void pdl_enter(const Job& j) {
  if (!j.pdl) return;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Returns the sequence number of this collective, or 0 if the rank is poisoned.
SN_DEV uint32_t enter(const Job& j) {
  DevMem m;
  Ctrl* ctrl = ctrl_of(j);
  if (int32_t(j.rank) == j.skip_rank) return 0u;
  uint32_t epoch, poison;
  m.ld_volatile_pair(&ctrl->epoch, epoch, poison);
  if (poison) return 0u;
  return next_seq(epoch);  // 0 stays "poisoned"; the wrap keeps the parity alternating
}

SN_DEV void leave(const Job& j, uint32_t seq) {
  __syncthreads();
  if (threadIdx.x == 0) {
    DevMem m;
    finish_op(m, ctrl_of(j), seq, gridDim.x);
  }
}

// Trace stamps: thread 0 of block 0 owns the collective's record (ring of records,
// indexed by sequence); emulated launches do not trace.
SN_DEV void trace_begin(const Job& j, OpCtx& c, uint32_t op) {
  if (!j.trace || blockIdx.x != 0 || threadIdx.x != 0 || gridDim.y != 1) return;
  DevMem m;
  uint64_t* rec = j.trace + uint64_t(c.seq % kTraceRecords) * kTraceWords;
  rec[0] = uint64_t(c.seq) | (uint64_t(op) << 32);
  rec[1] = j.nbytes;
  rec[2] = m.now_ns();
  rec[4 + j.rank] = rec[2];
  c.trace = rec;
}

SN_DEV void trace_end(const OpCtx& c) {
  if (!c.trace) return;
  DevMem m;
  c.trace[3] = m.now_ns();
}

SN_DEV Job emulated(const Job& j0, const EmuViews& e) {
  Job j = j0;
  j.rank = blockIdx.y;
  j.v = e.v[blockIdx.y];
  j.in = e.in[blockIdx.y];
  j.out = e.out[blockIdx.y];
  j.residual = e.residual[blockIdx.y];
  j.residual_out = e.residual_out[blockIdx.y];
  return j;
}

// Block-wide barrier over peer flags, led by thread 0; every thread learns the verdict.
SN_DEV bool block_barrier(const Job& j, const OpCtx& c) {
  __shared__ int ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    DevMem m;
    fence_proxy_alias();
    ok = block_barrier_leader(m, j, c, blockIdx.x) ? 1 : 0;
    fence_proxy_alias();
  }
  __syncthreads();
  return ok != 0;
}

// ---------------------------------------------------------------------------
// all-reduce
// ---------------------------------------------------------------------------
template <int D>
SN_DEV void nvls_allreduce(const Job& j, const OpCtx& c, uint64_t gtid, uint64_t gstride) {
  const uint64_t packs = j.nbytes / kPack;
  const uint32_t W = j.world, r = j.rank;
  const uint64_t chunk = (packs + W - 1) / W;
  const Pack16* in = reinterpret_cast<const Pack16*>(j.in);
  Pack16* uc = reinterpret_cast<Pack16*>(j.v.mc_uc);
  Pack16* mc = reinterpret_cast<Pack16*>(j.v.mc);
  Pack16* out = reinterpret_cast<Pack16*>(j.out);
  DevMem m;
  // Pack p of every chunk is staged, reduced and copied out by the same block on
  // every rank, so per-block barriers order exactly the packs each block touches.
  for (uint64_t p = gtid; p < chunk; p += gstride) {
    for (uint32_t k = 0; k < W; ++k) {
      uint64_t i = uint64_t(k) * chunk + p;
      if (i < packs) m.st_local(uc + i, m.ld_input(in + i));
    }
  }
  if (!block_barrier(j, c)) return;
  for (uint64_t p = gtid; p < chunk; p += gstride) {
    uint64_t i = uint64_t(r) * chunk + p;
    if (i < packs) mm_st(mc + i, mm_ld_reduce<D>(mc + i));
  }
  if (!block_barrier(j, c)) return;
  for (uint64_t p = gtid; p < chunk; p += gstride) {
    for (uint32_t k = 0; k < W; ++k) {
      uint64_t i = uint64_t(k) * chunk + p;
      if (i < packs) m.st_output(out + i, m.ld_peer_data(uc + i));
    }
  }
}

// A one-rank collective is a copy: no peers, no sequence, no completion count.
SN_DEV void copy_body(const Job& j) {
  DevMem m;
  const Pack16* in = reinterpret_cast<const Pack16*>(j.in);
  Pack16* out = reinterpret_cast<Pack16*>(j.out);
  const uint64_t packs = j.nbytes / kPack;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < packs; i += uint64_t(gridDim.x) * blockDim.x)
    m.st_output(out + i, m.ld_input(in + i));
}

template <int D>
SN_DEV void allreduce_body(const Job& j, int algo) {
  pdl_enter(j);
  if (j.world == 1) {
    if (j.in != j.out) copy_body(j);
    return;
  }
  uint32_t seq = enter(j);
  if (!seq) return;
  DevMem m;
  OpCtx c{ctrl_of(j), j.v.status, seq, j.rank, blockIdx.x, kOpAllReduce};
  trace_begin(j, c, kOpAllReduce);
  const uint64_t gtid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t gstride = uint64_t(gridDim.x) * blockDim.x;
  if (algo == kOneShot) {
    oneshot_allreduce<DevMem, D>(m, j, c, gtid, gstride);
  } else if (algo == kTwoShot) {
    twoshot_allreduce<DevMem, D>(m, j, c, gtid, gstride);
  } else {
    nvls_allreduce<D>(j, c, gtid, gstride);
  }
  trace_end(c);
  leave(j, seq);
}

template <int D>
__global__ void __launch_bounds__(kMaxThreads) k_allreduce(Job j, int algo) {
  allreduce_body<D>(j, algo);
}

// The one-rank all-reduce (kLocal): the sum over one rank is the input itself, so
// the call is a copy with three arguments instead of the collective's Job.  It is
// launched with programmatic stream serialisation: in a chain of calls (a graph of
// back-to-back all-reduces) each launch is scheduled while the previous kernel
// runs, and griddepcontrol.wait holds this grid's first access until that kernel
// has finished and its writes are visible.  The trigger comes after the wait, so
// at most two copies are resident at a time.  No peers, no waits: it cannot hang.
constexpr int kCopyPpt = 4;  // packs in flight per thread
__global__ void __launch_bounds__(kMaxThreads) k_copy_local(const Pack16* __restrict__ in,
                                                             Pack16* __restrict__ out, uint64_t packs) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  DevMem m;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t base = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; base < packs; base += stride * kCopyPpt) {
    Pack16 v[kCopyPpt];
    SN_UNROLL
    for (int k = 0; k < kCopyPpt; ++k) {
      const uint64_t i = base + uint64_t(k) * stride;
      if (i < packs) v[k] = m.ld_input(in + i);
    }
    SN_UNROLL
    for (int k = 0; k < kCopyPpt; ++k) {
      const uint64_t i = base + uint64_t(k) * stride;
      if (i < packs) m.st_output(out + i, v[k]);
    }
  }
}
template <int D>
__global__ void __launch_bounds__(kMaxThreads) k_allreduce_emu(Job j, EmuViews e, int algo) {
  allreduce_body<D>(emulated(j, e), algo);
}

// ---------------------------------------------------------------------------
// reduce-scatter
// ---------------------------------------------------------------------------
template <int D>
SN_DEV void reducescatter_body(const Job& j) {
  pdl_enter(j);
  uint32_t seq = enter(j);
  if (!seq) return;
  DevMem m;
  OpCtx c{ctrl_of(j), j.v.status, seq, j.rank, blockIdx.x, kOpReduceScatter};
  const uint64_t gtid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t gstride = uint64_t(gridDim.x) * blockDim.x;
  if (j.world == 1) {
    const Pack16* in = reinterpret_cast<const Pack16*>(j.in);
    Pack16* out = reinterpret_cast<Pack16*>(j.out);
    for (uint64_t i = gtid; i < j.nbytes / kPack; i += gstride) m.st_output(out + i, m.ld_input(in + i));
  } else {
    reduce_scatter<DevMem, D>(m, j, c, gtid, gstride);
  }
  leave(j, seq);
}
template <int D>
__global__ void __launch_bounds__(kMaxThreads) k_reducescatter(Job j) { reducescatter_body<D>(j); }
template <int D>
__global__ void __launch_bounds__(kMaxThreads) k_reducescatter_emu(Job j, EmuViews e) {
  reducescatter_body<D>(emulated(j, e));
}

// ---------------------------------------------------------------------------
// all-gather and exchange
// ---------------------------------------------------------------------------
SN_DEV void nvls_allgather(const Job& j, const OpCtx& c, uint64_t gtid, uint64_t gstride) {
  const uint64_t packs = j.nbytes / kPack;
  const uint32_t W = j.world, r = j.rank;
  const Pack16* in = reinterpret_cast<const Pack16*>(j.in);
  Pack16* uc = reinterpret_cast<Pack16*>(j.v.mc_uc);
  Pack16* mc = reinterpret_cast<Pack16*>(j.v.mc);
  DevMem m;
  for (uint64_t i = gtid; i < packs; i += gstride) {
    Pack16 v = m.ld_input(in + i);
    mm_st(mc + uint64_t(r) * packs + i, v);
  }
  if (!block_barrier(j, c)) return;
  for (uint64_t i = gtid; i < packs; i += gstride) {
    for (uint32_t s = 0; s < W; ++s) {
      Pack16 v = m.ld_peer_data(uc + uint64_t(s) * packs + i);
      m.st_output(reinterpret_cast<Pack16*>(j.out + gather_dst(j, s, i * kPack)), v);
    }
  }
  // second barrier: nobody may overwrite the buffer before every rank copied out
  block_barrier(j, c);
}

SN_DEV void gather_body(const Job& j, int algo, int op) {
  pdl_enter(j);
  uint32_t seq = enter(j);
  if (!seq) return;
  DevMem m;
  OpCtx c{ctrl_of(j), j.v.status, seq, j.rank, blockIdx.x, uint32_t(op)};
  const bool exchange = (op == kOpExchange);
  const uint64_t gtid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t gstride = uint64_t(gridDim.x) * blockDim.x;
  if (op == kOpBarrier) {
    block_barrier(j, c);
  } else if (!exchange && algo == kGatherLL) {
    allgather_ll(m, j, c, gtid, gstride);
  } else if (!exchange && algo == kGatherNvls) {
    nvls_allgather(j, c, gtid, gstride);
  } else {
    push_send(m, j, c, exchange, gtid, gstride);
    if (block_barrier(j, c)) push_receive(m, j, c, exchange, gtid, gstride);
  }
  leave(j, seq);
}

__global__ void __launch_bounds__(kMaxThreads) k_gather(Job j, int algo, int op) { gather_body(j, algo, op); }
__global__ void __launch_bounds__(kMaxThreads) k_gather_emu(Job j, EmuViews e, int algo, int op) {
  gather_body(emulated(j, e), algo, op);
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename... KArgs, typename... Args>
void launch(void (*kernel)(KArgs...), const LaunchGeom& g, cudaStream_t stream, Args... args) {
  if (g.emulate) {
    // every emulated rank's blocks must be co-resident: cap the blocks per rank by the
    // kernel's occupancy at this block size (the kernels stride over gridDim.x, and all
    // emulated ranks share the grid, so they see the same block count)
    int dev = 0, sms = 0, per_sm = 0;
    check(cudaGetDevice(&dev), "cudaGetDevice");
    check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
    check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, g.threads, 0), "occupancy");
    const int blocks = std::max(1, std::min(g.blocks, (per_sm * sms) / std::max(1, g.ranks)));
    void* argv[] = {static_cast<void*>(&args)...};
    check(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kernel), dim3(blocks, g.ranks),
                                      dim3(g.threads), argv, 0, stream),
          "cooperative launch");
  } else if (g.pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(g.blocks);
    cfg.blockDim = dim3(g.threads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    check(cudaLaunchKernelEx(&cfg, kernel, args...), "collective launch (PDL)");
  } else {
    kernel<<<dim3(g.blocks), dim3(g.threads), 0, stream>>>(args...);
    check(cudaGetLastError(), "collective launch");
  }
}

}  // namespace

void launch_allreduce(const Job& j, const EmuViews* e, int dtype, int algo, const LaunchGeom& g,
                      cudaStream_t s) {
  switch (dtype) {
#define SN_AR(DT)                                                             \
  case DT:                                                                    \
    if (e) launch(k_allreduce_emu<DT>, g, s, j, *e, algo);                    \
    else launch(k_allreduce<DT>, g, s, j, algo);                              \
    break;
    SN_AR(kF16)
    SN_AR(kBF16)
    SN_AR(kF32)
#undef SN_AR
    default:
      throw std::invalid_argument("unsupported all-reduce dtype");
  }
}

void launch_copy_local(const char* in, char* out, uint64_t nbytes, int threads, int max_blocks, cudaStream_t s) {
  if (nbytes % kPack || reinterpret_cast<uintptr_t>(in) % kPack || reinterpret_cast<uintptr_t>(out) % kPack)
    throw std::invalid_argument("the one-rank all-reduce copies 16-byte aligned packs");
  if (threads < 32 || threads > kMaxThreads || threads % 32 || max_blocks < 1)
    throw std::invalid_argument("local copy: bad launch geometry");
  const uint64_t packs = nbytes / kPack;
  if (packs == 0) return;
  // two packs per thread before the grid reaches its cap, up to kCopyPpt after it
  const uint64_t per_block = uint64_t(threads) * 2;
  const int blocks = int(std::max<uint64_t>(1, std::min<uint64_t>((packs + per_block - 1) / per_block,
                                                                   uint64_t(max_blocks))));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  check(cudaLaunchKernelEx(&cfg, k_copy_local, reinterpret_cast<const Pack16*>(in), reinterpret_cast<Pack16*>(out),
                           packs),
        "local copy launch");
}

void launch_reducescatter(const Job& j, const EmuViews* e, int dtype, const LaunchGeom& g, cudaStream_t s) {
  switch (dtype) {
#define SN_RS(DT)                                                             \
  case DT:                                                                    \
    if (e) launch(k_reducescatter_emu<DT>, g, s, j, *e);                      \
    else launch(k_reducescatter<DT>, g, s, j);                                \
    break;
    SN_RS(kF16)
    SN_RS(kBF16)
    SN_RS(kF32)
#undef SN_RS
    default:
      throw std::invalid_argument("unsupported reduce-scatter dtype");
  }
}

void launch_gather(const Job& j, const EmuViews* e, int algo, int op, const LaunchGeom& g, cudaStream_t s) {
  if (e) launch(k_gather_emu, g, s, j, *e, algo, op);
  else launch(k_gather, g, s, j, algo, op);
}

}  // namespace sn
