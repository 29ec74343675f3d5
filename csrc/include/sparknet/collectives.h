// Host-side declarations of the collective launchers (collectives.cu, fused.cu).
#pragma once

#include <cuda_runtime.h>

#include "proto.h"

namespace sn {

enum GatherAlgo : int { kGatherLL = 0, kGatherPush = 1, kGatherNvls = 2 };

// Per-rank pointers for an emulated launch (all ranks inside one cooperative grid).
struct EmuViews {
  View v[kMaxRanks];
  const char* in[kMaxRanks];
  char* out[kMaxRanks];
  const char* residual[kMaxRanks];
  char* residual_out[kMaxRanks];
};

struct LaunchGeom {
  int blocks = 1;
  int threads = 32;
  int ranks = 1;        // grid.y for emulated launches
  bool emulate = false;
  int cluster = 1;      // thread-block cluster size (fused kernels), 1 = none
  bool pdl = false;     // programmatic stream serialisation (never for emulated launches)
};

void launch_allreduce(const Job& j, const EmuViews* e, int dtype, int algo, const LaunchGeom& g, cudaStream_t s);
// One-rank all-reduce (kLocal): `nbytes` from `in` to `out` in one kernel launched
// with programmatic stream serialisation; grid capped at `max_blocks`.
void launch_copy_local(const char* in, char* out, uint64_t nbytes, int threads, int max_blocks, cudaStream_t s);
void launch_reducescatter(const Job& j, const EmuViews* e, int dtype, const LaunchGeom& g, cudaStream_t s);
void launch_gather(const Job& j, const EmuViews* e, int algo, int op, const LaunchGeom& g, cudaStream_t s);
void launch_fused_norm(const Job& j, const EmuViews* e, int dtype, int algo, const LaunchGeom& g, cudaStream_t s);

}  // namespace sn
