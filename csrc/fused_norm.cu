// Fused decode all-reduce + residual add + RMSNorm (K8), sm_100a.
//
//   s   = round( sum_r x_r )            fixed rank order, fp32 accumulation (= all_reduce)
//   res = round( s + residual )          -> residual_out
//   out = round( res * rsqrt(mean(res^2) + eps) * gamma )
//
// The reference has no fused path (sparknet/integration/vllm/roce_all_reduce.py:260-261
// reports supports_fused_add_rms_norm() == False); this kernel replaces the unfused
// sequence all_reduce -> add -> rms_norm of a tensor-parallel decoder layer.
//
// Layout of work: one thread-block cluster of `CL` CTAs per token row, each CTA owning
// H/CL contiguous elements (one 16-byte pack per thread).  The all-reduce is the
// Lamport push protocol of proto.h (one-shot: every rank pushes every row; two-shot:
// row t is reduced by rank t % W and the rounded sum is pushed back to all).  The sum
// of squares is reduced per CTA with a fixed shuffle tree, then across the cluster by
// reading every CTA's partial through distributed shared memory in CTA order, so all
// ranks and all CTAs of a row compute the same scale bit for bit.  Clusters loop over
// rows (persistent), so the grid never exceeds what is resident.
#include <algorithm>
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "sparknet/collectives.h"
#include "sparknet/dev_mem.cuh"

namespace cg = cooperative_groups;

namespace sn {
namespace {

SN_DEV Ctrl* ctrl_of(const Job& j) { return reinterpret_cast<Ctrl*>(j.v.base[j.rank] + j.L.ctrl_off); }

SN_DEV Job emulated(const Job& j0, const EmuViews& e, uint32_t rank) {
  Job j = j0;
  j.rank = rank;
  j.v = e.v[rank];
  j.in = e.in[rank];
  j.out = e.out[rank];
  j.residual = e.residual[rank];
  j.residual_out = e.residual_out[rank];
  return j;
}

// Poll one Lamport slot pack until it arrived; consume it (sentinel back).
template <int D>
SN_DEV bool take(DevMem& m, Pack16* slot, Pack16& x, const OpCtx& c, uint32_t peer) {
  WaitState w;
  for (;;) {
    x = m.ld_poll(slot);
    if (pack_arrived<D>(x)) break;
    if (!keep_waiting(m, w, c, peer)) return false;
  }
  m.st_local(slot, pack_fill(kSentinel));
  return true;
}

// Sum of squares of this thread's lanes, reduced over the CTA then the cluster in a
// fixed order.  `part` is this CTA's shared partial; returns the row's total.
SN_DEV float row_sumsq(float mine, float* warp_part, float* part, cg::cluster_group& cluster) {
  const unsigned lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
  if (lane == 0) warp_part[warp] = mine;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (unsigned w = 0; w < (blockDim.x + 31u) / 32u; ++w) t += warp_part[w];
    *part = t;
  }
  cluster.sync();
  float total = 0.0f;
  for (unsigned k = 0; k < cluster.num_blocks(); ++k) total += *cluster.map_shared_rank(part, k);
  return total;
}

template <int D>
SN_DEV void fused_body(const Job& j, int algo) {
  DevMem m;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float warp_part[32];
  __shared__ float part;

  Ctrl* ctrl = ctrl_of(j);
  if (int32_t(j.rank) == j.skip_rank) return;
  uint32_t epoch, poison;
  m.ld_volatile_pair(&ctrl->epoch, epoch, poison);
  if (poison) return;
  const uint32_t seq = next_seq(epoch);
  OpCtx c{ctrl, j.v.status, seq, j.rank, blockIdx.x, kOpFusedNorm};

  constexpr int kElems = 16 / (Codec<D>::kLanes == 2 ? 2 : 4);   // elements per pack
  const uint32_t W = j.world, r = j.rank;
  const uint32_t parity = seq & 1u;
  // Geometry from the launch as it actually ran: the cluster size and the block size
  // are read here, not assumed from the host's plan.  A tool that re-issues the launch
  // without its cluster attribute (a profiler) then still gets a correct result:
  // every CTA covers row_packs / CL packs, each thread as many strided packs as that
  // takes; the row's sum of squares is still reduced in a fixed order.
  const uint32_t CL = cluster.num_blocks();
  const uint32_t cta = cluster.block_rank();
  const uint64_t row_packs = j.hidden / kElems;
  const uint64_t cta_packs = row_packs / CL;
  const uint32_t per_thread = uint32_t((cta_packs + blockDim.x - 1) / blockDim.x);
  const uint64_t T = j.nbytes / (row_packs * kPack);
  const uint32_t nclusters = gridDim.x / CL;
  const uint32_t cid = blockIdx.x / CL;
  const uint64_t half = j.L.lam_cap / 2 / kPack;

  const Pack16* x = reinterpret_cast<const Pack16*>(j.in);
  const Pack16* res = reinterpret_cast<const Pack16*>(j.residual);
  const Pack16* gamma = reinterpret_cast<const Pack16*>(j.gamma);
  Pack16* out = reinterpret_cast<Pack16*>(j.out);
  Pack16* res_out = reinterpret_cast<Pack16*>(j.residual_out);
  const bool twoshot = (algo == kTwoShot) && W > 1;
  bool ok = row_packs % CL == 0;  // always true for a cluster size the host accepts
  if (!ok) record_failure(m, c, kFailGeometry, r, 0);

  // pack index within the row of this thread's k-th pack, or ~0 when it has none
  auto row_pack = [&](uint32_t k) -> uint64_t {
    const uint64_t within = uint64_t(threadIdx.x) + uint64_t(k) * blockDim.x;
    return within < cta_packs ? uint64_t(cta) * cta_packs + within : ~0ull;
  };

  // 1. push: one-shot sends every row to every peer; two-shot sends row t to its owner.
  if (ok && W > 1) {
    for (uint64_t t = cid; t < T; t += nclusters) {
      for (uint32_t k = 0; k < per_thread; ++k) {
        const uint64_t tpack = row_pack(k);
        if (tpack == ~0ull) break;
        const uint64_t i = t * row_packs + tpack;
        Pack16 v = pack_canon<D>(m.ld_input(x + i));
        if (twoshot) {
          uint32_t q = uint32_t(t % W);
          if (q != r) m.st_remote(lam_pack(j, q, parity, r, (t / W) * row_packs + tpack), v);
        } else {
          for (uint32_t s = 1; s < W; ++s) m.st_remote(lam_pack(j, (r + s) % W, parity, r, i), v);
        }
      }
    }
  }

  // 2. two-shot: reduce the rows this rank owns and push the rounded sums back.
  if (twoshot && ok) {
    for (uint64_t t = cid; t < T && ok; t += nclusters) {
      if (t % W != r) continue;
      for (uint32_t k = 0; k < per_thread && ok; ++k) {
        const uint64_t tpack = row_pack(k);
        if (tpack == ~0ull) break;
        const uint64_t i = t * row_packs + tpack;
        const uint64_t slot_pack = (t / W) * row_packs + tpack;
        Pack16 xs[kMaxRanks];
        const Pack16 own = pack_canon<D>(m.ld_input(x + i));
        ok = take_all<DevMem, D>(m, j, c, parity, slot_pack, peers_mask(W, r), xs, 1, 1);
        if (!ok) break;
        Pack16 y = pack_canon<D>(sum_rank_order<D>(own, xs, W, r));
        for (uint32_t s = 1; s < W; ++s) m.st_remote(lam_pack(j, (r + s) % W, parity, r, half + slot_pack), y);
        // keep the own sum for step 3 in the output buffer (overwritten there)
        m.st_local(out + i, y);
      }
    }
  }

  // 3. per row: the all-reduced sum, + residual, RMSNorm over the cluster.  Pass A
  //    writes the new residual and sums its squares; pass B scales it.  The first
  //    pack stays in registers; any further pack (only when the launch ran with fewer
  //    CTAs per row than planned) is read back from residual_out, which this thread
  //    wrote itself.
  for (uint64_t t = cid; t < T; t += nclusters) {
    float sq = 0.0f;
    Pack16 first = pack_fill(0u);
    for (uint32_t k = 0; k < per_thread && ok; ++k) {
      const uint64_t tpack = row_pack(k);
      if (tpack == ~0ull) break;
      const uint64_t i = t * row_packs + tpack;
      Pack16 sum = pack_fill(0u);
      if (W == 1) {
        sum = m.ld_input(x + i);
      } else if (twoshot) {
        uint32_t owner = uint32_t(t % W);
        if (owner == r) {
          sum = m.ld_peer_data(out + i);
        } else {
          ok = take<D>(m, lam_pack(j, r, parity, owner, half + (t / W) * row_packs + tpack), sum, c, owner);
        }
      } else {
        Pack16 xs[kMaxRanks];
        const Pack16 own = pack_canon<D>(m.ld_input(x + i));
        ok = take_all<DevMem, D>(m, j, c, parity, i, peers_mask(W, r), xs, 1, 1);
        if (ok) sum = sum_rank_order<D>(own, xs, W, r);
      }
      if (!ok) break;
      // residual add (rounded once, as the unfused add would be)
      Acc a;
      acc_zero<D>(a);
      acc_add<D>(a, sum);
      acc_add<D>(a, m.ld_peer_data(res + i));  // coherent: residual_out may alias residual
      const Pack16 newres = acc_round<D>(a);
      Acc rr;
      acc_zero<D>(rr);
      acc_add<D>(rr, newres);
      for (int e = 0; e < kElems; ++e) sq += rr.v[e] * rr.v[e];
      if (k == 0) first = newres;
      m.st_output(res_out + i, newres);
    }
    // every thread of every CTA of the cluster takes part in the reduction
    float total = row_sumsq(sq, warp_part, &part, cluster);
    float scale = rsqrtf(total / float(j.hidden) + j.eps);
    for (uint32_t k = 0; k < per_thread && ok; ++k) {
      const uint64_t tpack = row_pack(k);
      if (tpack == ~0ull) break;
      const uint64_t i = t * row_packs + tpack;
      Acc rr, g;
      acc_zero<D>(rr);
      acc_zero<D>(g);
      acc_add<D>(rr, k == 0 ? first : m.ld_peer_data(res_out + i));
      acc_add<D>(g, m.ld_input(gamma + tpack));
      Acc o;
      for (int e = 0; e < kElems; ++e) o.v[e] = (rr.v[e] * scale) * g.v[e];
      m.st_output(out + i, acc_round<D>(o));
    }
    cluster.sync();  // partials are rewritten by the next row
  }

  __syncthreads();
  if (threadIdx.x == 0) finish_op(m, ctrl, seq, gridDim.x);
}

template <int D>
__global__ void __launch_bounds__(kMaxThreads) k_fused(Job j, int algo) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // a PDL-launched successor may start early
  // launched with PDL itself: nothing (the epoch included) is read before the previous
  // kernel on the stream has finished
  if (j.pdl) asm volatile("griddepcontrol.wait;" ::: "memory");
  fused_body<D>(j, algo);
}

template <int D>
__global__ void __launch_bounds__(kMaxThreads) k_fused_emu(Job j, EmuViews e, int algo) {
  fused_body<D>(emulated(j, e, blockIdx.y), algo);
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename... KArgs, typename... Args>
void launch_cluster(void (*kernel)(KArgs...), const LaunchGeom& g, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g.blocks, g.emulate ? g.ranks : 1);
  cfg.blockDim = dim3(g.threads);
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = g.cluster;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  int n = 1;
  if (g.pdl && !g.emulate) {
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    n = 2;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  if (g.emulate) {
    // every emulated rank's clusters must be co-resident: cap by the clusters that fit
    int fit = 0;
    check(cudaOccupancyMaxActiveClusters(&fit, kernel, &cfg), "cluster occupancy");
    const int per_rank = std::max(1, std::min(int(g.blocks / g.cluster), fit / std::max(1, g.ranks)));
    cfg.gridDim = dim3(per_rank * g.cluster, g.ranks);
    attrs[1].id = cudaLaunchAttributeCooperative;
    attrs[1].val.cooperative = 1;
    cfg.numAttrs = 2;
  }
  check(cudaLaunchKernelEx(&cfg, kernel, args...), "fused norm launch");
}

}  // namespace

void launch_fused_norm(const Job& j, const EmuViews* e, int dtype, int algo, const LaunchGeom& g, cudaStream_t s) {
  switch (dtype) {
#define SN_FN(DT)                                                   \
  case DT:                                                          \
    if (e) launch_cluster(k_fused_emu<DT>, g, s, j, *e, algo);      \
    else launch_cluster(k_fused<DT>, g, s, j, algo);                \
    break;
    SN_FN(kF16)
    SN_FN(kBF16)
    SN_FN(kF32)
#undef SN_FN
    default:
      throw std::invalid_argument("unsupported fused-norm dtype");
  }
}

}  // namespace sn
