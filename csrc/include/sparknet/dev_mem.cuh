// Device memory policy for the protocol bodies in proto.h: inline PTX for the
// NVLink peer scope.  Peer data stores and polls are volatile 16-byte accesses
// (never cached in L1, performed in program order per thread); flags use
// release/acquire at system scope; multimem (NVLS) accesses go through the
// multicast alias.  Replaces the reference's pinned-host protocol helpers
// (sparknet/oneshot/_device.py:62-595).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "proto.h"

namespace sn {

struct DevMem {
  SN_DEV Pack16 ld_input(const Pack16* p) const {
    Pack16 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
                 : "l"(p));
    return v;
  }
  SN_DEV void ld_input8(const char* p, uint32_t* d) const {
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(d[0]), "=r"(d[1]) : "l"(p));
  }
  // A slot a peer writes into: bypass L1, observe the latest value.
  SN_DEV Pack16 ld_poll(const Pack16* p) const {
    Pack16 v;
    asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
                 : "l"(p)
                 : "memory");
    return v;
  }
  // Data published by a flag this thread's block already acquired.
  SN_DEV Pack16 ld_peer_data(const Pack16* p) const {
    Pack16 v;
    asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
                 : "l"(p)
                 : "memory");
    return v;
  }
  SN_DEV void st_remote(Pack16* p, const Pack16& v) const {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.w[0]), "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3])
                 : "memory");
  }
  SN_DEV void st_local(Pack16* p, const Pack16& v) const {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.w[0]), "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3])
                 : "memory");
  }
  SN_DEV void st_output(Pack16* p, const Pack16& v) const { st_local(p, v); }
  SN_DEV void st_output8(char* p, const uint32_t* d) const {
    asm volatile("st.global.v2.u32 [%0], {%1,%2};" :: "l"(p), "r"(d[0]), "r"(d[1]) : "memory");
  }
  SN_DEV uint32_t ld_acquire_u32(const uint32_t* p) const {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
  }
  SN_DEV uint32_t ld_volatile_u32(const volatile uint32_t* p) const {
    uint32_t v;
    asm volatile("ld.volatile.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
  }
  // epoch and poison words of Ctrl in one access
  SN_DEV void ld_volatile_pair(const uint32_t* p, uint32_t& a, uint32_t& b) const {
    asm volatile("ld.volatile.global.v2.u32 {%0,%1}, [%2];" : "=r"(a), "=r"(b) : "l"(p) : "memory");
  }
  SN_DEV void st_release_u32(uint32_t* p, uint32_t v) const {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
  }
  SN_DEV void st_volatile_u32(uint32_t* p, uint32_t v) const {
    asm volatile("st.volatile.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
  }
  SN_DEV uint32_t atomic_add_u32(uint32_t* p, uint32_t v) const { return atomicAdd(p, v); }
  SN_DEV uint32_t cas_u32(uint32_t* p, uint32_t expect, uint32_t v) const { return atomicCAS(p, expect, v); }
  SN_DEV void fence_sys() const { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
  SN_DEV void fence_device() const { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
  SN_DEV uint64_t now_ns() const {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
  }
};

// ---------------------------------------------------------------------------
// NVLS (multimem) primitives.  `mc` addresses are the multicast alias: a load-
// reduce returns the switch's sum over every bound rank's copy; a store writes
// every rank's copy.  The switch's summation order is not the rank order, so these
// paths are rank-identical (one rank computes, every rank receives the same bits)
// but not equal to the sequential fp32 reference: they are opt-in.
// ---------------------------------------------------------------------------
template <int D> SN_DEV Pack16 mm_ld_reduce(const Pack16* mc);

template <> SN_DEV Pack16 mm_ld_reduce<kBF16>(const Pack16* mc) {
  Pack16 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
               : "l"(mc)
               : "memory");
  return v;
}
template <> SN_DEV Pack16 mm_ld_reduce<kF16>(const Pack16* mc) {
  Pack16 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
               : "l"(mc)
               : "memory");
  return v;
}
template <> SN_DEV Pack16 mm_ld_reduce<kF32>(const Pack16* mc) {
  Pack16 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
               : "l"(mc)
               : "memory");
  return v;
}
SN_DEV void mm_st(Pack16* mc, const Pack16& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};"
               :: "l"(mc), "r"(v.w[0]), "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3])
               : "memory");
}
SN_DEV void mm_red_add_release(uint32_t* mc, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" :: "l"(mc), "r"(v) : "memory");
}
SN_DEV void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

}  // namespace sn
