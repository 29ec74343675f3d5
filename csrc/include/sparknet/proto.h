// sparknet protocol core: region layout, control records, element codecs and the
// per-thread bodies of every collective.  Compiles as CUDA (device kernels) and as
// plain C++ (the host simulator), so the code the simulator checks is the code the
// GPU runs.  Memory accesses go through a `Mem` policy: `DevMem` (PTX, dev_mem.cuh)
// or `HostMem` (C++ atomics, tests/sim/host_mem.h).
//
// Reference behaviour this replaces (pinned-host staging + RDMA writes posted by a
// host proxy): sparknet/oneshot/_device.py:27-595 and _roce_proxy.c:949-1019.  The
// B200 design keeps the fixed rank-order fp32 reduction (bit-identical ranks) and the
// device-resident sequence number, but the data crosses NVLink as device stores.
#pragma once

#include <stdint.h>
#include <stddef.h>

#if defined(__CUDACC__)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#endif

#if defined(__CUDACC__)
#define SN_HD __host__ __device__ __forceinline__
#define SN_DEV __device__ __forceinline__
#if defined(__CUDA_ARCH__)  // the device pass; the host pass of a .cu file has no such pragma
#define SN_UNROLL _Pragma("unroll")
#else
#define SN_UNROLL
#endif
#else
#define SN_HD inline
#define SN_DEV inline
#define SN_UNROLL
#endif

namespace sn {

// ---------------------------------------------------------------------------
// Limits and ABI
// ---------------------------------------------------------------------------
constexpr int kAbiVersion = 8;       // bumped when Layout/Ctrl/Status/Job change
constexpr int kMaxRanks = 8;         // one NVSwitch box
constexpr int kMaxBlocks = 256;      // per launch (grid.x)
constexpr int kChunkCounters = 1024; // fused all-gather->GEMM: 128-row chunks per shard
constexpr int kMaxThreads = 512;     // per block of the collective kernels: a thread may hold
                                     // every peer's pack at once (128 registers available)
constexpr int kPack = 16;            // bytes moved per vector access
constexpr int kGFlags = 4096;        // per-source chunk/tile flags of the fused GEMMs
constexpr size_t kPage = 4096;
constexpr uint32_t kSentinel = 0xFFFFFFFFu;  // "not yet written" in Lamport slots

enum DType : int { kF16 = 0, kBF16 = 1, kF32 = 2 };
// kLocal: the one-rank all-reduce, a copy (no protocol)
enum Algo : int { kOneShot = 0, kTwoShot = 1, kNvls = 2, kLocal = 3 };
// kFailBounds: a slot access outside its area (builds with SN_BOUNDS_CHECK only)
// kFailGeometry: a kernel found a launch shape it cannot serve (the work was skipped)
enum FailKind : int {
  kFailNone = 0, kFailTimeout = 1, kFailPoisoned = 2, kFailIterations = 3, kFailBounds = 4, kFailGeometry = 5
};

SN_HD size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Pack16 {
  uint32_t w[4];
};

// ---------------------------------------------------------------------------
// Device-resident control words (page 0 of every rank's symmetric region).  Only
// the owning rank's kernels touch them, so they need no peer-scope ordering.
// ---------------------------------------------------------------------------
struct Ctrl {
  // epoch and poison are adjacent so one 8-byte load at kernel entry reads both
  uint32_t epoch;                  // sequence of the last completed collective
  uint32_t poison;                 // nonzero after a failed wait: every kernel exits at entry
  uint32_t done;                   // blocks of the current collective that finished
  uint32_t ops;                    // collectives completed (stats)
  uint32_t bar_count[kMaxBlocks];  // per-block barrier generation (push/flag protocols)
  uint32_t mc_count[kMaxBlocks];   // per-block multicast barrier target
  uint32_t chunk_count[kChunkCounters];  // fused all-gather->GEMM: copy CTAs done with a chunk
  alignas(16) uint32_t sink[8];    // bounds-checked builds: where a rejected slot access goes
};
static_assert(sizeof(Ctrl) <= kPage * 3, "ctrl must fit its pages");

// Pinned host record, written by a kernel that gives up and read by the host's
// health check without a device synchronisation.  `timeout_us` is host-written and
// read by kernels at run time, so it also applies to replayed CUDA graphs.
struct Status {
  volatile uint32_t timeout_us;
  volatile uint32_t failed_seq;    // 0 = healthy
  volatile uint32_t kind;          // FailKind
  volatile uint32_t peer;          // the rank waited for
  volatile uint32_t block;         // the block that gave up
  volatile uint32_t waited_us;
  volatile uint32_t op;            // which collective (OpCode)
  volatile uint32_t reserved;
};

enum OpCode : int {
  kOpAllReduce = 1, kOpAllGather = 2, kOpReduceScatter = 3, kOpExchange = 4,
  kOpBarrier = 5, kOpFusedNorm = 6, kOpAgGemm = 7, kOpGemmRs = 8
};

// ---------------------------------------------------------------------------
// Region layout.  Every rank maps every peer's region at the same offsets.
//   ctrl    : Ctrl (local use)
//   flags   : u32 [kMaxBlocks][kMaxRanks]   per-block barrier flags written by peers
//   gflags  : u32 [kMaxRanks][kGFlags]      chunk/tile flags of the fused GEMMs, by source
//   lamport : 2 parities x W sources x lam_cap     (Lamport slots, all-ones when free)
//   ll      : 2 parities x W sources x 2*ll_cap    (8-byte data+flag units)
//   push    : 2 parities x W sources x push_cap    (flagged bulk slots)
// ---------------------------------------------------------------------------
struct Layout {
  uint32_t world;
  uint64_t lam_cap, ll_cap, push_cap;
  uint64_t ctrl_off, flag_off, gflag_off, lam_off, ll_off, push_off, total;

  SN_HD static Layout make(uint32_t world, uint64_t lam_cap, uint64_t ll_cap, uint64_t push_cap) {
    Layout l;
    l.world = world;
    l.lam_cap = align_up(lam_cap, kPage);
    l.ll_cap = align_up(ll_cap, kPage);
    l.push_cap = align_up(push_cap, kPage);
    l.ctrl_off = 0;
    l.flag_off = kPage * 3;
    l.gflag_off = align_up(l.flag_off + sizeof(uint32_t) * kMaxBlocks * kMaxRanks, kPage);
    l.lam_off = align_up(l.gflag_off + sizeof(uint32_t) * kMaxRanks * kGFlags, kPage);
    l.ll_off = l.lam_off + 2ull * world * l.lam_cap;
    l.push_off = l.ll_off + 2ull * world * 2ull * l.ll_cap;
    l.total = l.push_off + 2ull * world * l.push_cap;
    return l;
  }
  SN_HD uint64_t lam(uint32_t parity, uint32_t src) const {
    return lam_off + (uint64_t(parity) * world + src) * lam_cap;
  }
  SN_HD uint64_t ll(uint32_t parity, uint32_t src) const {
    return ll_off + (uint64_t(parity) * world + src) * 2ull * ll_cap;
  }
  SN_HD uint64_t push(uint32_t parity, uint32_t src) const {
    return push_off + (uint64_t(parity) * world + src) * push_cap;
  }
  SN_HD uint64_t flag(uint32_t block, uint32_t src) const {
    return flag_off + sizeof(uint32_t) * (uint64_t(block) * kMaxRanks + src);
  }
};

// What one rank sees: its own region, every peer's region mapped locally, and
// (optionally) the multicast alias of the NVLS buffer.
struct View {
  char* base[kMaxRanks];
  Status* status;          // device pointer of the pinned host status record
  char* mc;                // multicast alias (NVLS) or null
  char* mc_uc;             // this rank's unicast alias of the multicast-bound buffer
  uint64_t mc_cap;         // bytes of data in the multicast buffer (flags follow)
};

// ---------------------------------------------------------------------------
// Element codecs: the reduction accumulates in fp32 and rounds once to nearest-even.
// Device builds call CUDA's conversion intrinsics; host builds use the IEEE-754
// definitions below (round-to-nearest-even on the dropped bits), which tests check
// against torch's conversions.
// ---------------------------------------------------------------------------
SN_HD float bits_to_f32(uint32_t b) {
  union { uint32_t u; float f; } c;
  c.u = b;
  return c.f;
}
SN_HD uint32_t f32_to_bits(float f) {
  union { uint32_t u; float f; } c;
  c.f = f;
  return c.u;
}

// bf16 <- f32, round to nearest, ties to even; NaN stays NaN (quiet bit set).
SN_HD uint16_t host_f32_to_bf16(float f) {
  uint32_t u = f32_to_bits(f);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return uint16_t((u >> 16) | 0x0040u);
  uint32_t lsb = (u >> 16) & 1u;
  return uint16_t((u + 0x7fffu + lsb) >> 16);
}
SN_HD float host_bf16_to_f32(uint16_t h) { return bits_to_f32(uint32_t(h) << 16); }

// binary16 -> binary32 (exact).
SN_HD float host_f16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0x1f) return bits_to_f32(sign | 0x7f800000u | (man << 13));
  if (exp == 0) {
    if (man == 0) return bits_to_f32(sign);
    // subnormal: value = man * 2^-24
    float v = float(man) * (1.0f / 16777216.0f);
    return sign ? -v : v;
  }
  return bits_to_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

// binary32 -> binary16, round to nearest, ties to even (IEEE 754-2008 §4.3.1).
SN_HD uint16_t host_f32_to_f16(float f) {
  uint32_t u = f32_to_bits(f);
  uint32_t sign = (u >> 16) & 0x8000u;
  uint32_t exp = (u >> 23) & 0xffu;
  uint32_t man = u & 0x7fffffu;
  if (exp == 0xff) return uint16_t(sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0u));
  int e = int(exp) - 127 + 15;
  if (e >= 0x1f) return uint16_t(sign | 0x7c00u);            // overflow -> inf
  if (e <= 0) {                                               // subnormal or zero
    if (e < -10) return uint16_t(sign);
    uint32_t m = man | 0x800000u;                             // implicit bit
    uint32_t shift = uint32_t(14 - e);                        // 24-bit mantissa -> 10 bits at 2^-24
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return uint16_t(sign | q);
  }
  uint32_t q = (uint32_t(e) << 10) | (man >> 13);
  uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;      // may carry into exponent: correct
  return uint16_t(sign | q);
}

// Codec per dtype: how many lanes a 32-bit word holds and how to widen/narrow them.
template <int D> struct Codec;

template <> struct Codec<kF32> {
  static constexpr int kLanes = 1;
  SN_HD static void widen(uint32_t w, float* o) { o[0] = bits_to_f32(w); }
  SN_HD static uint32_t narrow(const float* v) { return f32_to_bits(v[0]); }
  SN_HD static bool free_word(uint32_t w) { return w == kSentinel; }
  // A real value equal to the sentinel (one particular NaN) is re-encoded as another NaN.
  SN_HD static uint32_t canon(uint32_t w) { return w == kSentinel ? (w ^ 1u) : w; }
};

template <> struct Codec<kBF16> {
  static constexpr int kLanes = 2;
#if defined(__CUDA_ARCH__)
  SN_HD static void widen(uint32_t w, float* o) {
    o[0] = __uint_as_float(w << 16);
    o[1] = __uint_as_float(w & 0xffff0000u);
  }
  SN_HD static uint32_t narrow(const float* v) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[0], v[1]);
    return *reinterpret_cast<uint32_t*>(&h);
  }
#else
  SN_HD static void widen(uint32_t w, float* o) {
    o[0] = host_bf16_to_f32(uint16_t(w & 0xffffu));
    o[1] = host_bf16_to_f32(uint16_t(w >> 16));
  }
  SN_HD static uint32_t narrow(const float* v) {
    return uint32_t(host_f32_to_bf16(v[0])) | (uint32_t(host_f32_to_bf16(v[1])) << 16);
  }
#endif
  SN_HD static bool free_word(uint32_t w) { return (w & 0xffffu) == 0xffffu || (w >> 16) == 0xffffu; }
  SN_HD static uint32_t canon(uint32_t w) {
    if ((w & 0xffffu) == 0xffffu) w ^= 1u;
    if ((w >> 16) == 0xffffu) w ^= 0x10000u;
    return w;
  }
};

template <> struct Codec<kF16> {
  static constexpr int kLanes = 2;
#if defined(__CUDA_ARCH__)
  SN_HD static void widen(uint32_t w, float* o) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    float2 f = __half22float2(h);
    o[0] = f.x;
    o[1] = f.y;
  }
  SN_HD static uint32_t narrow(const float* v) {
    __half2 h = __floats2half2_rn(v[0], v[1]);
    return *reinterpret_cast<uint32_t*>(&h);
  }
#else
  SN_HD static void widen(uint32_t w, float* o) {
    o[0] = host_f16_to_f32(uint16_t(w & 0xffffu));
    o[1] = host_f16_to_f32(uint16_t(w >> 16));
  }
  SN_HD static uint32_t narrow(const float* v) {
    return uint32_t(host_f32_to_f16(v[0])) | (uint32_t(host_f32_to_f16(v[1])) << 16);
  }
#endif
  SN_HD static bool free_word(uint32_t w) { return Codec<kBF16>::free_word(w); }
  SN_HD static uint32_t canon(uint32_t w) { return Codec<kBF16>::canon(w); }
};

template <int D> SN_HD bool pack_arrived(const Pack16& p) {
  return !(Codec<D>::free_word(p.w[0]) || Codec<D>::free_word(p.w[1]) ||
           Codec<D>::free_word(p.w[2]) || Codec<D>::free_word(p.w[3]));
}
template <int D> SN_HD Pack16 pack_canon(Pack16 p) {
  for (int i = 0; i < 4; ++i) p.w[i] = Codec<D>::canon(p.w[i]);
  return p;
}
SN_HD Pack16 pack_fill(uint32_t v) {
  Pack16 p;
  p.w[0] = p.w[1] = p.w[2] = p.w[3] = v;
  return p;
}

// fp32 accumulator for one 16-byte pack (8 lanes at most).
struct Acc {
  float v[8];
};
template <int D> SN_HD void acc_zero(Acc& a) {
  for (int i = 0; i < 8; ++i) a.v[i] = 0.0f;  // +0: an all -0 sum yields +0, as sequential fp32 from 0 does
}
template <int D> SN_HD void acc_add(Acc& a, const Pack16& p) {
  constexpr int L = Codec<D>::kLanes;
  for (int i = 0; i < 4; ++i) {
    float f[2];
    Codec<D>::widen(p.w[i], f);
    for (int l = 0; l < L; ++l) a.v[i * L + l] = a.v[i * L + l] + f[l];
  }
}
template <int D> SN_HD Pack16 acc_round(const Acc& a) {
  constexpr int L = Codec<D>::kLanes;
  Pack16 p;
  for (int i = 0; i < 4; ++i) p.w[i] = Codec<D>::narrow(&a.v[i * L]);
  return p;
}

// ---------------------------------------------------------------------------
// Bounded waits.  A wait checks the clock every `kSpinCheck` polls; after
// `kGraceNs` it starts watching the poison word and the host-set timeout.  A wait
// that runs out records the failure and returns false: nothing traps, so the GPU
// context stays usable and the host learns of it from `Status`.
// ---------------------------------------------------------------------------
constexpr uint32_t kSpinCheck = 64;
constexpr uint64_t kGraceNs = 20000;          // 20 us before the slow-path checks
constexpr uint64_t kMaxSpins = 4000000000ull; // absolute iteration cap, independent of the clock

struct WaitState {
  uint64_t t0 = 0;
  uint64_t limit_ns = 0;
  uint64_t spins = 0;
};

struct OpCtx {
  Ctrl* ctrl;          // this rank's control words
  Status* status;      // pinned host record
  uint32_t seq;
  uint32_t rank;
  uint32_t block;
  uint32_t op;
  uint64_t* trace = nullptr;  // this collective's trace record (thread 0 of block 0 only), or null
};

// Trace record (u64 words), written by thread 0 of block 0 when tracing is on:
//   [0] seq | op << 32   [1] bytes   [2] entry ns   [3] exit ns
//   [4 + s] time pack 0 from source s arrived (this rank's own entry for s == rank)
constexpr int kTraceWords = 32;
constexpr int kTraceRecords = 65536;
constexpr int kTraceHeaderBytes = 4096;

template <class M>
SN_HD void trace_arrival(M& m, const OpCtx& c, uint64_t gtid, uint64_t i, uint32_t s) {
  if (c.trace && gtid == 0 && i == 0) c.trace[4 + s] = m.now_ns();
}

// Records the failure once per rank (first writer wins) and poisons the rank.
template <class M>
SN_HD void record_failure(M& m, const OpCtx& c, uint32_t kind, uint32_t peer, uint64_t waited_ns) {
  if (m.cas_u32(&c.ctrl->poison, 0u, 1u) == 0u) {
    c.status->kind = kind;
    c.status->peer = peer;
    c.status->block = c.block;
    c.status->waited_us = uint32_t(waited_ns / 1000u);
    c.status->op = c.op;
    m.fence_sys();
    c.status->failed_seq = c.seq ? c.seq : 1u;
    m.fence_sys();
  }
}

// One step of a bounded wait; true = keep polling.
template <class M>
SN_HD bool keep_waiting(M& m, WaitState& w, const OpCtx& c, uint32_t peer) {
  ++w.spins;
  if (w.spins % kSpinCheck) return true;
  if (w.spins > kMaxSpins) {
    record_failure(m, c, kFailIterations, peer, 0);
    return false;
  }
  uint64_t now = m.now_ns();
  if (!w.t0) {
    w.t0 = now;
    return true;
  }
  uint64_t waited = now - w.t0;
  if (waited < kGraceNs) return true;
  if (m.ld_volatile_u32(&c.ctrl->poison)) return false;  // another block gave up already
  if (!w.limit_ns) {
    uint32_t us = m.ld_volatile_u32(&c.status->timeout_us);
    w.limit_ns = uint64_t(us ? us : 1u) * 1000ull;
  }
  if (waited >= w.limit_ns) {
    record_failure(m, c, kFailTimeout, peer, waited);
    return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Job descriptions (plain data, passed by value to kernels).
// ---------------------------------------------------------------------------
struct Job {
  View v;
  Layout L;
  uint32_t rank;
  uint32_t world;
  const char* in;
  char* out;
  uint64_t nbytes;        // all-reduce: message; reduce-scatter: chunk; all-gather: shard
  // all-gather / exchange addressing (in 16-byte packs or 8-byte units as stated)
  uint64_t row_bytes;     // bytes per source row (all-gather: shard row; 0 = whole shard is one row)
  uint64_t dst_row_stride;   // bytes between output rows
  uint64_t dst_src_stride;   // bytes between sources' blocks in the output
  uint64_t src_peer_stride;  // exchange: bytes between chunks[p] in the input
  uint64_t total_src_bytes;  // exchange(all_to_all_rows): valid input bytes (rows beyond are absent)
  int64_t valid_out_bytes;   // exchange(all_to_all_rows): own rows that exist (-1 = all)
  uint32_t copy_self;
  // fused residual + RMSNorm (kOpFusedNorm)
  const char* residual;
  char* residual_out;
  const char* gamma;
  float eps;
  uint32_t hidden;        // elements per row
  // Test hook (emulated groups only): this rank's blocks return at entry, as if
  // the rank never launched the collective.  -1 = none.
  int32_t skip_rank;
  // 1: launched with programmatic stream serialisation.  The kernel waits for the
  // previous kernel on its stream (griddepcontrol.wait) before its first access and
  // then lets the next such launch be scheduled (launch_dependents): the successor
  // can only start once every block of this grid is resident.
  uint32_t pdl;
  // Trace ring (device pointer of the pinned trace file's records), or null.
  uint64_t* trace;
};

// Slot accessors: every access of the protocols to a peer-written area (Lamport, LL
// and bulk-push slots, per-block flags) takes its address from one of these.  Builds
// with SN_BOUNDS_CHECK check the owner and source ranks (< world), the parity (< 2)
// and that the whole pack (or flag) lies inside its slot.  A violation is recorded in
// the pinned status (kind kFailBounds, `peer` = which check, `block` = the offending
// pack index, low 32 bits), poisons the rank, and redirects the access to a sink in
// the control page: the collective then ends poisoned, and no neighbouring slot is
// touched.  Without the macro the accessors are plain address arithmetic.
enum BoundsCheck : uint32_t { kBoundsLam = 1, kBoundsLL = 2, kBoundsPush = 3, kBoundsFlag = 4 };

#if defined(SN_BOUNDS_CHECK)
SN_HD uint32_t* bounds_violation(const Job& j, uint32_t owner, uint32_t which, uint64_t index) {
  Status* st = j.v.status;
  if (st && st->failed_seq == 0u) {
    st->kind = kFailBounds;
    st->peer = which;
    st->block = uint32_t(index);
    st->waited_us = 0u;
    st->op = 0u;
    st->failed_seq = 0xFFFFFFFFu;  // the sequence is not known at the access
  }
  volatile uint32_t* poison = &reinterpret_cast<Ctrl*>(j.v.base[j.rank] + j.L.ctrl_off)->poison;
  *poison = 1u;
  char* base = owner < j.world ? j.v.base[owner] : j.v.base[j.rank];
  return reinterpret_cast<Ctrl*>(base + j.L.ctrl_off)->sink;
}
#define SN_SLOT_CHECK(ok, j, owner, which, index, T) \
  if (!(ok)) return reinterpret_cast<T*>(bounds_violation(j, owner, which, index))
#else
#define SN_SLOT_CHECK(ok, j, owner, which, index, T) (void)0
#endif

// Pack `pack` of Lamport slot [parity][src] in `owner`'s region.
SN_HD Pack16* lam_pack(const Job& j, uint32_t owner, uint32_t parity, uint32_t src, uint64_t pack) {
  SN_SLOT_CHECK(owner < j.world && src < j.world && parity < 2u && (pack + 1u) * kPack <= j.L.lam_cap, j, owner,
                kBoundsLam, pack, Pack16);
  return reinterpret_cast<Pack16*>(j.v.base[owner] + j.L.lam(parity, src)) + pack;
}
// 16-byte unit `unit` of LL slot [parity][src] (2 x ll_cap bytes) in `owner`'s region.
SN_HD Pack16* ll_pack(const Job& j, uint32_t owner, uint32_t parity, uint32_t src, uint64_t unit) {
  SN_SLOT_CHECK(owner < j.world && src < j.world && parity < 2u && (unit + 1u) * kPack <= 2u * j.L.ll_cap, j, owner,
                kBoundsLL, unit, Pack16);
  return reinterpret_cast<Pack16*>(j.v.base[owner] + j.L.ll(parity, src)) + unit;
}
// Pack `pack` of bulk-push slot [parity][src] in `owner`'s region.
SN_HD Pack16* push_pack(const Job& j, uint32_t owner, uint32_t parity, uint32_t src, uint64_t pack) {
  SN_SLOT_CHECK(owner < j.world && src < j.world && parity < 2u && (pack + 1u) * kPack <= j.L.push_cap, j, owner,
                kBoundsPush, pack, Pack16);
  return reinterpret_cast<Pack16*>(j.v.base[owner] + j.L.push(parity, src)) + pack;
}
// Barrier flag [block][src] in `owner`'s region.
SN_HD uint32_t* flag_word(const Job& j, uint32_t owner, uint32_t block, uint32_t src) {
  SN_SLOT_CHECK(owner < j.world && src < j.world && block < uint32_t(kMaxBlocks), j, owner, kBoundsFlag, block,
                uint32_t);
  return reinterpret_cast<uint32_t*>(j.v.base[owner] + j.L.flag(block, src));
}

// ---------------------------------------------------------------------------
// One-shot all-reduce (Lamport push).  Every thread owns packs i = gtid, gtid +
// gstride, ...: it pushes its (canonicalised) input pack into slot [parity][rank]
// of every peer, then polls its own slots [parity][src] until each peer's pack has
// arrived (no sentinel lane left), sums the W packs in rank order in fp32, rounds
// once, and writes the sentinel back over the slots it consumed so the slot
// parity is clean for reuse two collectives later.
//
// Reuse proof (two parities suffice): a peer writes parity p for collective s+2
// only after it completed collective s+1, which needed this rank's pushes for s+1,
// which this rank issues only after its kernel for s (reads and clears) finished.
// ---------------------------------------------------------------------------
// Lowest set bit of a non-zero mask (portable between host and device).
SN_HD uint32_t lowest_bit(uint32_t mask) {
  uint32_t s = 0;
  while (!((mask >> s) & 1u)) ++s;
  return s;
}

// Consume pack `off` of this rank's Lamport slots [parity][s] for every source s in
// `mask`: each sweep issues one load per outstanding source before testing any of
// them, so all sources cost one memory round trip together instead of one each; each
// slot is re-armed with the sentinel once every source's data is in hand.  xs[s]
// receives source s's pack.  False if a wait ran out (the failure names the lowest
// source still outstanding).
template <class M, int D>
SN_HD bool take_all(M& m, const Job& j, const OpCtx& c, uint32_t parity, uint64_t off, uint32_t mask,
                    Pack16 (&xs)[kMaxRanks], uint64_t gtid, uint64_t ti) {
  const uint32_t r = j.rank;
  uint32_t pending = mask;
  WaitState w;
  while (pending) {
SN_UNROLL
    for (uint32_t s = 0; s < uint32_t(kMaxRanks); ++s)
      if ((pending >> s) & 1u) xs[s] = m.ld_poll(lam_pack(j, r, parity, s, off));
SN_UNROLL
    for (uint32_t s = 0; s < uint32_t(kMaxRanks); ++s)
      if (((pending >> s) & 1u) && pack_arrived<D>(xs[s])) {
        pending &= ~(1u << s);
        trace_arrival(m, c, gtid, ti, s);
      }
    if (pending && !keep_waiting(m, w, c, lowest_bit(pending))) return false;
  }
SN_UNROLL
  for (uint32_t s = 0; s < uint32_t(kMaxRanks); ++s)
    if ((mask >> s) & 1u) m.st_local(lam_pack(j, r, parity, s, off), pack_fill(kSentinel));
  return true;
}

SN_HD uint32_t peers_mask(uint32_t W, uint32_t r) { return ((W >= 32u ? 0u : (1u << W)) - 1u) & ~(1u << r); }

// Rank-order fp32 sum of the own pack and the peers' packs from take_all.  The loop
// index is a constant after unrolling, so xs stays in registers.
template <int D>
SN_HD Pack16 sum_rank_order(const Pack16& own, const Pack16 (&xs)[kMaxRanks], uint32_t W, uint32_t r) {
  Acc a;
  acc_zero<D>(a);
SN_UNROLL
  for (uint32_t s = 0; s < uint32_t(kMaxRanks); ++s)
    if (s < W) acc_add<D>(a, s == r ? own : xs[s]);
  return acc_round<D>(a);
}

template <class M, int D>
SN_HD bool oneshot_allreduce(M& m, const Job& j, const OpCtx& c, uint64_t gtid, uint64_t gstride) {
  const uint64_t packs = j.nbytes / kPack;
  const uint32_t parity = c.seq & 1u;
  const uint32_t W = j.world, r = j.rank;
  const Pack16* in = reinterpret_cast<const Pack16*>(j.in);
  Pack16* out = reinterpret_cast<Pack16*>(j.out);
  for (uint64_t i = gtid; i < packs; i += gstride) {
    Pack16 v = pack_canon<D>(m.ld_input(in + i));
    for (uint32_t k = 1; k < W; ++k) {
      uint32_t q = (r + k) % W;
      m.st_remote(lam_pack(j, q, parity, r, i), v);
    }
  }
  const uint32_t peers = peers_mask(W, r);
  for (uint64_t i = gtid; i < packs; i += gstride) {
    Pack16 xs[kMaxRanks];
    const Pack16 own = pack_canon<D>(m.ld_input(in + i));
    if (!take_all<M, D>(m, j, c, parity, i, peers, xs, gtid, i)) return false;
    m.st_output(out + i, sum_rank_order<D>(own, xs, W, r));
  }
  return true;
}

// ---------------------------------------------------------------------------
// Two-shot all-reduce (Lamport push, reduce-scatter then all-gather).  Chunk c of
// the message is reduced by rank c: every rank pushes chunk c's pack j to rank c's
// slot [parity][rank] at pack j (first half of the slot); rank c sums the W packs in
// rank order, rounds once, canonicalises, writes its output and pushes the result
// to every peer's slot [parity][c] at pack j of the slot's second half; every rank
// then copies the other chunks out of its slots.  Each rank sends 2(W-1)/W of the
// message instead of W-1 times it.
// ---------------------------------------------------------------------------
template <class M, int D>
SN_HD bool twoshot_allreduce(M& m, const Job& j, const OpCtx& c, uint64_t gtid, uint64_t gstride) {
  const uint64_t packs = j.nbytes / kPack;
  const uint32_t W = j.world, r = j.rank;
  const uint64_t chunk = (packs + W - 1) / W;
  const uint32_t parity = c.seq & 1u;
  const uint64_t half = j.L.lam_cap / 2 / kPack;   // second-half offset in packs
  const Pack16* in = reinterpret_cast<const Pack16*>(j.in);
  Pack16* out = reinterpret_cast<Pack16*>(j.out);
  // scatter: pack j of every chunk to its owner
  for (uint64_t p = gtid; p < chunk; p += gstride) {
    for (uint32_t k = 1; k < W; ++k) {
      uint32_t q = (r + k) % W;
      uint64_t i = uint64_t(q) * chunk + p;
      if (i >= packs) continue;
      Pack16 v = pack_canon<D>(m.ld_input(in + i));
      m.st_remote(lam_pack(j, q, parity, r, p), v);
    }
  }
  // reduce the own chunk, broadcast the result
  for (uint64_t p = gtid; p < chunk; p += gstride) {
    uint64_t i = uint64_t(r) * chunk + p;
    if (i >= packs) continue;
    Pack16 xs[kMaxRanks];
    const Pack16 own = pack_canon<D>(m.ld_input(in + i));
    if (!take_all<M, D>(m, j, c, parity, p, peers_mask(W, r), xs, gtid, p)) return false;
    Pack16 y = pack_canon<D>(sum_rank_order<D>(own, xs, W, r));
    m.st_output(out + i, y);
    for (uint32_t k = 1; k < W; ++k) {
      uint32_t q = (r + k) % W;
      m.st_remote(lam_pack(j, q, parity, r, half + p), y);
    }
  }
  // gather the other owners' results
  for (uint64_t p = gtid; p < chunk; p += gstride) {
    uint32_t mask = 0;
SN_UNROLL
    for (uint32_t s = 0; s < uint32_t(kMaxRanks); ++s)
      if (s < W && s != r && uint64_t(s) * chunk + p < packs) mask |= 1u << s;
    if (!mask) continue;
    Pack16 xs[kMaxRanks];
    if (!take_all<M, D>(m, j, c, parity, half + p, mask, xs, gtid, ~0ull)) return false;
SN_UNROLL
    for (uint32_t s = 0; s < uint32_t(kMaxRanks); ++s)
      if ((mask >> s) & 1u) m.st_output(out + uint64_t(s) * chunk + p, xs[s]);
  }
  return true;
}

// ---------------------------------------------------------------------------
// Reduce-scatter (Lamport push): the input holds W chunks of `nbytes`; chunk c is
// summed in rank order on rank c.
// ---------------------------------------------------------------------------
template <class M, int D>
SN_HD bool reduce_scatter(M& m, const Job& j, const OpCtx& c, uint64_t gtid, uint64_t gstride) {
  const uint64_t chunk = j.nbytes / kPack;
  const uint32_t W = j.world, r = j.rank;
  const uint32_t parity = c.seq & 1u;
  const Pack16* in = reinterpret_cast<const Pack16*>(j.in);
  const uint64_t peer_stride = j.src_peer_stride ? j.src_peer_stride / kPack : chunk;
  Pack16* out = reinterpret_cast<Pack16*>(j.out);
  for (uint64_t p = gtid; p < chunk; p += gstride) {
    for (uint32_t k = 1; k < W; ++k) {
      uint32_t q = (r + k) % W;
      Pack16 v = pack_canon<D>(m.ld_input(in + uint64_t(q) * peer_stride + p));
      m.st_remote(lam_pack(j, q, parity, r, p), v);
    }
  }
  const uint32_t peers = peers_mask(W, r);
  for (uint64_t p = gtid; p < chunk; p += gstride) {
    Pack16 xs[kMaxRanks];
    const Pack16 own = pack_canon<D>(m.ld_input(in + uint64_t(r) * peer_stride + p));
    if (!take_all<M, D>(m, j, c, parity, p, peers, xs, gtid, ~0ull)) return false;
    m.st_output(out + p, sum_rank_order<D>(own, xs, W, r));
  }
  return true;
}

// ---------------------------------------------------------------------------
// All-gather, LL8 form: every 8 bytes of payload travel with a 4-byte copy of the
// collective's flag next to each 4-byte word ({d0, f, d1, f} per 16-byte store), so
// a receiver knows the unit arrived without a separate flag and for any dtype.
// The flag is 2*seq+1 (odd, never 0) and slots hold the previous parity's flag,
// so no clearing is needed.
// Output address of (src, byte offset o in the shard):
//   (o / row) * dst_row_stride + src * dst_src_stride + (o % row)
// ---------------------------------------------------------------------------
SN_HD uint64_t gather_dst(const Job& j, uint32_t src, uint64_t o) {
  const uint64_t row = j.row_bytes ? j.row_bytes : j.nbytes;
  return (o / row) * j.dst_row_stride + uint64_t(src) * j.dst_src_stride + (o % row);
}

template <class M>
SN_HD bool allgather_ll(M& m, const Job& j, const OpCtx& c, uint64_t gtid, uint64_t gstride) {
  const uint64_t units = j.nbytes / 8;
  const uint32_t W = j.world, r = j.rank;
  const uint32_t parity = c.seq & 1u;
  const uint32_t flag = c.seq * 2u + 1u;
  for (uint64_t u = gtid; u < units; u += gstride) {
    uint32_t d[2];
    m.ld_input8(j.in + u * 8, d);
    Pack16 p;
    p.w[0] = d[0];
    p.w[1] = flag;
    p.w[2] = d[1];
    p.w[3] = flag;
    for (uint32_t k = 1; k < W; ++k) {
      uint32_t q = (r + k) % W;
      m.st_remote(ll_pack(j, q, parity, r, u), p);
    }
    m.st_output8(j.out + gather_dst(j, r, u * 8), d);
  }
  const uint32_t peers = peers_mask(W, r);
  for (uint64_t u = gtid; u < units; u += gstride) {
    // every outstanding source polled per sweep (one round trip for all of them)
    uint32_t pending = peers;
    WaitState w;
    while (pending) {
      Pack16 xs[kMaxRanks];
SN_UNROLL
      for (uint32_t s = 0; s < uint32_t(kMaxRanks); ++s)
        if ((pending >> s) & 1u) xs[s] = m.ld_poll(ll_pack(j, r, parity, s, u));
SN_UNROLL
      for (uint32_t s = 0; s < uint32_t(kMaxRanks); ++s)
        if (((pending >> s) & 1u) && xs[s].w[1] == flag && xs[s].w[3] == flag) {
          pending &= ~(1u << s);
          uint32_t d[2] = {xs[s].w[0], xs[s].w[2]};
          m.st_output8(j.out + gather_dst(j, s, u * 8), d);
        }
      if (pending && !keep_waiting(m, w, c, lowest_bit(pending))) return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// Per-block barrier over peer flags.  Block b of every rank keeps a generation
// count; it releases (system scope) the new count into slot [b][rank] of every
// peer and waits until every peer's slot [b][src] reached it.  Used after bulk
// pushes: a block's data is published by the flag that follows it.
// ---------------------------------------------------------------------------
template <class M>
SN_HD bool block_barrier_leader(M& m, const Job& j, const OpCtx& c, uint32_t block) {
  const uint32_t W = j.world, r = j.rank;
  uint32_t gen = c.ctrl->bar_count[block] + 1u;
  c.ctrl->bar_count[block] = gen;
  // The system-scope release of each flag orders this block's pushes before it (the
  // caller synchronised the block first; release is cumulative): no separate fence.
  for (uint32_t k = 1; k < W; ++k) {
    uint32_t q = (r + k) % W;
    m.st_release_u32(flag_word(j, q, block, r), gen);
  }
  uint32_t pending = peers_mask(W, r);
  WaitState w;
  while (pending) {
    uint32_t seen[kMaxRanks];
SN_UNROLL
    for (uint32_t s = 0; s < uint32_t(kMaxRanks); ++s)
      if ((pending >> s) & 1u) seen[s] = m.ld_acquire_u32(flag_word(j, r, block, s));
SN_UNROLL
    for (uint32_t s = 0; s < uint32_t(kMaxRanks); ++s)
      if (((pending >> s) & 1u) && int32_t(seen[s] - gen) >= 0) pending &= ~(1u << s);
    if (pending && !keep_waiting(m, w, c, lowest_bit(pending))) return false;
  }
  return true;
}

// Bulk push (large all-gather and exchange): every block pushes its share of the
// payload into slot [parity][rank] of each destination peer; after the block
// barrier it copies its share of every source's slot to the output.  All-gather
// sends the whole shard to every peer; exchange sends chunks[q] to peer q, where
// chunks[q] starts at q * src_peer_stride.  For all_to_all_rows, input bytes at or
// beyond total_src_bytes do not exist (not sent) and only the first
// valid_out_bytes of each received chunk are written (the rank-invariant row count
// of this rank's block).
template <class M>
SN_HD void push_send(M& m, const Job& j, const OpCtx& c, bool exchange, uint64_t gtid, uint64_t gstride) {
  const uint32_t W = j.world, r = j.rank;
  const uint32_t parity = c.seq & 1u;
  const uint64_t packs = j.nbytes / kPack;
  for (uint64_t i = gtid; i < packs; i += gstride) {
    if (!exchange) {
      Pack16 v = m.ld_input(reinterpret_cast<const Pack16*>(j.in) + i);
      for (uint32_t k = 1; k < W; ++k) {
        uint32_t q = (r + k) % W;
        m.st_remote(push_pack(j, q, parity, r, i), v);
      }
      m.st_output(reinterpret_cast<Pack16*>(j.out + gather_dst(j, r, i * kPack)), v);
      continue;
    }
    for (uint32_t k = 1; k < W; ++k) {
      uint32_t q = (r + k) % W;
      uint64_t src_off = uint64_t(q) * j.src_peer_stride + i * kPack;
      if (j.total_src_bytes && src_off >= j.total_src_bytes) continue;
      Pack16 v = m.ld_input(reinterpret_cast<const Pack16*>(j.in + src_off));
      m.st_remote(push_pack(j, q, parity, r, i), v);
    }
    if (j.copy_self && (j.valid_out_bytes < 0 || int64_t(i * kPack) < j.valid_out_bytes)) {
      uint64_t src_off = uint64_t(r) * j.src_peer_stride + i * kPack;
      if (!(j.total_src_bytes && src_off >= j.total_src_bytes)) {
        Pack16 v = m.ld_input(reinterpret_cast<const Pack16*>(j.in + src_off));
        m.st_output(reinterpret_cast<Pack16*>(j.out + uint64_t(r) * j.dst_src_stride + i * kPack), v);
      }
    }
  }
}

template <class M>
SN_HD void push_receive(M& m, const Job& j, const OpCtx& c, bool exchange, uint64_t gtid, uint64_t gstride) {
  const uint32_t W = j.world, r = j.rank;
  const uint32_t parity = c.seq & 1u;
  const uint64_t packs = j.nbytes / kPack;
  for (uint64_t i = gtid; i < packs; i += gstride) {
    if (exchange && j.valid_out_bytes >= 0 && int64_t(i * kPack) >= j.valid_out_bytes) continue;
    for (uint32_t k = 1; k < W; ++k) {
      uint32_t s = (r + W - k) % W;
      Pack16 v = m.ld_peer_data(push_pack(j, r, parity, s, i));
      uint64_t dst = exchange ? uint64_t(s) * j.dst_src_stride + i * kPack : gather_dst(j, s, i * kPack);
      m.st_output(reinterpret_cast<Pack16*>(j.out + dst), v);
    }
  }
}

// Completion: the last block to finish publishes the sequence as the new epoch.
// Every block consumed its entry read of the epoch (it computed `seq` from it)
// before its increment of `done`, so no block can read the new value early, and the
// next collective on this rank starts only after this kernel completes.  No fence is
// needed: the kernel boundary publishes the new epoch to the next launch.
// Sequence number of the collective after `epoch`.  0 is reserved (a poisoned rank's
// kernels leave with it), so the wrap after 0xFFFFFFFF goes to 2, not 1: consecutive
// collectives keep alternating their slot parity (seq & 1) across the wrap, which the
// two-parity reuse argument of the Lamport and LL slots needs.
SN_HD uint32_t next_seq(uint32_t epoch) {
  const uint32_t s = epoch + 1u;
  return s ? s : 2u;
}

template <class M>
SN_HD void finish_op(M& m, Ctrl* ctrl, uint32_t seq, uint32_t nblocks) {
  uint32_t old = m.atomic_add_u32(&ctrl->done, 1u);
  if (old == nblocks - 1u) {
    ctrl->done = 0u;
    ctrl->ops = ctrl->ops + 1u;
    m.st_volatile_u32(&ctrl->epoch, seq);
  }
}

}  // namespace sn
