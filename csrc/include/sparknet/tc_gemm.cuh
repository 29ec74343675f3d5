// sm_100a GEMM building blocks: TMA tile loads, mbarriers, tcgen05.mma with TMEM
// accumulators, and a persistent warp-specialised tile loop shared by the plain GEMM
// and the fused all-gather->GEMM / GEMM->reduce-scatter kernels.
//
//   C[M, N] = A[M, K] * B[N, K]^T      (bf16 in, fp32 accumulate in TMEM, both K-major)
//
// CTA tile 128 x BN (BN = 256 or 128), K step 64 (one 128-byte swizzle atom per row),
// STAGES-deep shared-memory ring.  Warp 0 issues TMA loads (one elected thread),
// warp 1 allocates TMEM and issues tcgen05.mma (one elected thread), warps 2..5 drain
// the accumulator with tcgen05.ld and run the epilogue; the accumulator is double
// buffered in TMEM so the epilogue of tile i overlaps the MMAs of tile i+1.
//
// Every TMA load is a plain per-CTA load (the fused kernels run on several GPUs).  Every
// mbarrier wait is bounded: a wait that runs out sets the kernel's error word and the
// roles unwind, free TMEM and return.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace sn {
namespace tc {

constexpr int kBM = 128;
constexpr int kBK = 64;                 // bf16 elements per 128-byte swizzled row
constexpr uint32_t kWaitLimit = 1u << 27;  // try_wait polls before giving up

enum TcError : uint32_t { kTcOk = 0, kTcWaitTimeout = 1, kTcFlagTimeout = 2 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait for the phase with parity `parity` to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* err) {
  uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 1023u) == 1023u && *err) return false;  // another role already gave up
  }
  *err = kTcWaitTimeout;
  return false;
}

// Bounded wait that ignores other roles' failures: lets a CTA's own copies land before
// it exits after an error (or before it exits with copies it never needed).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return;
  }
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// --- tcgen05 ---------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* tile) {
  uint64_t addr = smem_u32(tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;          // start address (16-byte units)
  d |= 1ull << 16;                        // leading byte offset (unused for swizzled K-major)
  d |= (1024ull >> 4) << 32;              // stride byte offset: next 8-row group
  d |= 1ull << 46;                        // descriptor version (sm100)
  d |= 2ull << 61;                        // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor: bf16 x bf16 -> f32, A and B K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4)                        // D format f32
         | (1u << 7)                      // A bf16
         | (1u << 10)                     // B bf16
         | (uint32_t(n >> 3) << 17)       // N / 8
         | (uint32_t(kBM >> 4) << 24);    // M / 16
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1), "r"(mask2),
      "r"(mask3)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// --- block-scaled fp8 (kind::mxf8f6f4, e4m3 x e4m3, UE8M0 scales every 32 K) -----
// One K block is 128 fp8 = one 128-byte swizzle row, like 64 bf16: the tile shapes and
// descriptors of the bf16 path carry over; each K block adds a 512-byte scale chunk per
// 128 rows of A and of B (layout in fp8_quant.cu), staged into TMEM by tcgen05.cp.

// Bulk (non-tensor) copy global -> this CTA's shared memory, completing on `bar`.
// 16-byte aligned addresses, size a multiple of 16.  Per-CTA destination only.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Descriptor of a 512-byte scale chunk for tcgen05.cp: K-major, no swizzle, 32 rows of
// 16 bytes, 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sf(const void* chunk) {
  uint64_t d = 0;
  d |= (uint64_t(smem_u32(chunk)) >> 4) & 0x3FFFull;
  d |= 1ull << 16;                // leading byte offset (one core matrix along K)
  d |= (128ull >> 4) << 32;       // stride byte offset: next 8 rows
  d |= 1ull << 46;                // descriptor version (sm100)
  return d;                       // layout 0: no swizzle
}

// 32 TMEM lanes x 128 bits from shared memory, replicated into all four lane quarters.
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Instruction descriptor: e4m3 x e4m3 -> f32, K-major, UE8M0 scales, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_mxf8(int n) {
  return (0u << 7) | (0u << 10)           // A, B e4m3
         | (uint32_t(n >> 3) << 17)       // N / 8
         | (1u << 23)                     // scale format UE8M0
         | (uint32_t(kBM >> 4) << 24);    // M / 16
}

// One K=32 step; `sf_id` (instruction descriptor) selects the scale byte of this step
// in the TMEM columns.  The scale addresses are plain column addresses.  (With 1 x 128
// and 128 x 128 scales all four bytes of a column hold the same exponent, so the step's
// byte choice cannot change the result.)
__device__ __forceinline__ void mma_mxf8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t tsfa, uint32_t tsfb, uint32_t sf_id, uint32_t accumulate) {
  const uint32_t id = idesc | (sf_id << 29) | (sf_id << 4);
  const uint32_t sa = tsfa, sb = tsfb;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(id), "r"(accumulate), "r"(sa), "r"(sb)
      : "memory");
}

// Shared-memory plan of the tile loop.
template <int BN, int STAGES, bool F8 = false>
struct Smem {
  static constexpr int kABytes = kBM * 128;        // 128 rows x 128 bytes (64 bf16 or 128 fp8)
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kSfBytes = F8 ? 512 * (1 + BN / 128) : 0;  // scale chunks of A and B per stage
  // epilogue staging: per epilogue warp, 32 rows x 64 bf16 columns, rows padded to
  // 144 bytes so row-per-thread writes and 16-byte-per-lane reads avoid bank conflicts
  static constexpr int kStageRowBytes = 144;
  static constexpr int kEpiStageBytes = 4 * 32 * kStageRowBytes;
  static constexpr int kBytes =
      STAGES * (kStageBytes + kSfBytes) + kEpiStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// Host: 2-D tensor map over `rows` x `cols` (row pitch `ld` elements) of 2-byte
// (bf16) or 1-byte (fp8) elements, box `box_rows` x 128 bytes, 128-byte swizzle, zero
// fill out of bounds.
CUtensorMap make_map(const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                     int elem_bytes = 2);

struct TileCoord {
  int m0, n0;
};

// Tile order: CTAs walk tiles blockIdx.x, +gridDim.x, ...; consecutive tiles share
// the A row block, so A stays in L2 while the CTAs sweep N.  `remap` lets a fused
// kernel start each rank on different rows (its own shard first).
struct Schedule {
  int tiles_m, tiles_n;
  __device__ __forceinline__ int count() const { return tiles_m * tiles_n; }
};

}  // namespace tc
}  // namespace sn
