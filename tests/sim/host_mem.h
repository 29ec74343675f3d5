// Host memory policy for the protocol bodies in csrc/include/sparknet/proto.h.
//
// Ranks are threads and "peer memory" is plain memory; every access the device does
// with volatile/relaxed/acquire/release PTX is a C++ atomic here, so the sanitizers
// see the protocol's real synchronisation.  A remote 16-byte store is split into its
// two 8-byte halves, written in random order with random pauses between them: the
// protocols may assume 8-byte single-copy atomicity (as NVLink stores give) but not
// 16-byte atomicity.  A simulated clock lets bounded waits time out without waiting.
#pragma once

#include <sched.h>
#include <stdint.h>
#include <time.h>

#include <atomic>
#include <random>

#include "sparknet/proto.h"

namespace sim {

struct Chaos {
  uint32_t permille_pause;  // chance (per mille) of a pause around a remote store
  uint32_t max_spin;        // pause length bound (yields)
  uint32_t far_penalty;     // extra yields for "far" peers (ring4-like mode)
  int world;
  int ring4;                // 1: ranks two apart are far
};

struct HostMem {
  std::mt19937 rng;
  const Chaos* chaos;
  int rank;

  HostMem(uint32_t seed, const Chaos* c, int r) : rng(seed), chaos(c), rank(r) {}

  void maybe_pause(uint32_t extra = 0) {
    if (!chaos) return;
    if (rng() % 1000 < chaos->permille_pause) {
      uint32_t n = chaos->max_spin ? rng() % chaos->max_spin : 0;
      for (uint32_t i = 0; i < n + extra; ++i) sched_yield();
    }
  }

  static uint64_t ld64(const void* p) { return __atomic_load_n(reinterpret_cast<const uint64_t*>(p), __ATOMIC_RELAXED); }
  static void st64(void* p, uint64_t v) { __atomic_store_n(reinterpret_cast<uint64_t*>(p), v, __ATOMIC_RELAXED); }

  sn::Pack16 ld_input(const sn::Pack16* p) {
    sn::Pack16 v;
    for (int i = 0; i < 4; ++i) v.w[i] = __atomic_load_n(&p->w[i], __ATOMIC_RELAXED);
    return v;
  }
  void ld_input8(const char* p, uint32_t* d) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(p);
    d[0] = __atomic_load_n(w, __ATOMIC_RELAXED);
    d[1] = __atomic_load_n(w + 1, __ATOMIC_RELAXED);
  }
  sn::Pack16 ld_poll(const sn::Pack16* p) {
    sn::Pack16 v;
    uint64_t a = ld64(p), b = ld64(reinterpret_cast<const char*>(p) + 8);
    v.w[0] = uint32_t(a);
    v.w[1] = uint32_t(a >> 32);
    v.w[2] = uint32_t(b);
    v.w[3] = uint32_t(b >> 32);
    sched_yield();
    return v;
  }
  sn::Pack16 ld_peer_data(const sn::Pack16* p) { return ld_poll(p); }
  void st_remote(sn::Pack16* p, const sn::Pack16& v) {
    // ring4-like mode: odd ranks deliver late, as relayed (two-hop) peers would
    maybe_pause(chaos && chaos->ring4 && (rank & 1) ? chaos->far_penalty : 0);
    uint64_t lo = uint64_t(v.w[0]) | (uint64_t(v.w[1]) << 32);
    uint64_t hi = uint64_t(v.w[2]) | (uint64_t(v.w[3]) << 32);
    char* c = reinterpret_cast<char*>(p);
    if (rng() & 1) {
      st64(c, lo);
      maybe_pause();
      st64(c + 8, hi);
    } else {
      st64(c + 8, hi);
      maybe_pause();
      st64(c, lo);
    }
  }
  void st_local(sn::Pack16* p, const sn::Pack16& v) {
    char* c = reinterpret_cast<char*>(p);
    st64(c, uint64_t(v.w[0]) | (uint64_t(v.w[1]) << 32));
    st64(c + 8, uint64_t(v.w[2]) | (uint64_t(v.w[3]) << 32));
  }
  void st_output(sn::Pack16* p, const sn::Pack16& v) { st_local(p, v); }
  void st_output8(char* p, const uint32_t* d) {
    uint32_t* w = reinterpret_cast<uint32_t*>(p);
    __atomic_store_n(w, d[0], __ATOMIC_RELAXED);
    __atomic_store_n(w + 1, d[1], __ATOMIC_RELAXED);
  }
  uint32_t ld_acquire_u32(const uint32_t* p) {
    sched_yield();
    return __atomic_load_n(p, __ATOMIC_ACQUIRE);
  }
  uint32_t ld_volatile_u32(const volatile uint32_t* p) {
    return __atomic_load_n(const_cast<const uint32_t*>(p), __ATOMIC_RELAXED);
  }
  void st_release_u32(uint32_t* p, uint32_t v) {
    maybe_pause();
    __atomic_store_n(p, v, __ATOMIC_RELEASE);
  }
  void st_volatile_u32(uint32_t* p, uint32_t v) { __atomic_store_n(p, v, __ATOMIC_RELAXED); }
  uint32_t atomic_add_u32(uint32_t* p, uint32_t v) { return __atomic_fetch_add(p, v, __ATOMIC_ACQ_REL); }
  uint32_t cas_u32(uint32_t* p, uint32_t expect, uint32_t v) {
    __atomic_compare_exchange_n(p, &expect, v, false, __ATOMIC_ACQ_REL, __ATOMIC_ACQUIRE);
    return expect;
  }
  // A sequentially consistent RMW on a shared word stands in for a fence: it orders
  // like one and, unlike a bare fence, ThreadSanitizer understands it.
  static uint32_t* fence_word() {
    static uint32_t w = 0;
    return &w;
  }
  void fence_sys() { __atomic_fetch_add(fence_word(), 0u, __ATOMIC_SEQ_CST); }
  void fence_device() { fence_sys(); }
  uint64_t now_ns() {
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return uint64_t(t.tv_sec) * 1000000000ull + uint64_t(t.tv_nsec);
  }
};

}  // namespace sim
