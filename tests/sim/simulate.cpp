// Host simulator of the NVLink collective protocols.
//
// Compiles the production protocol bodies (csrc/include/sparknet/proto.h) against
// HostMem and runs `world` ranks x `blocks` blocks as threads over plain memory:
// every rank's symmetric region is an ordinary allocation that every "peer" thread
// writes into.  A group keeps its regions across calls, so sequences of collectives
// exercise epoch advance, parity slots and slot cleaning exactly as the GPU does
// (each call joins all threads before returning: the kernel boundary).  Exposed with
// a C ABI for the Python tests (ctypes); built with ASan/UBSan or TSan by the tests.
//
// This mirrors the reference's approach of testing its transport with simulated
// endpoints (reference tests/oneshot_sim/simulate.c), for a device-initiated design.
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <thread>
#include <vector>

#include "host_mem.h"

namespace {

struct Group {
  int world;
  sn::Layout L;
  std::vector<char*> regions;
  std::vector<sn::Status> status;
  sim::Chaos chaos;
};

sn::Ctrl* ctrl_of(Group* g, int r) { return reinterpret_cast<sn::Ctrl*>(g->regions[r] + g->L.ctrl_off); }

void init_region(Group* g, int r) {
  char* base = g->regions[r];
  memset(base, 0, g->L.lam_off);
  memset(base + g->L.lam_off, 0xff, g->L.ll_off - g->L.lam_off);
  memset(base + g->L.ll_off, 0, g->L.total - g->L.ll_off);
  memset(&g->status[r], 0, sizeof(sn::Status));
}

}  // namespace

extern "C" {

void* sim_group_create(int world, uint64_t lam_cap, uint64_t ll_cap, uint64_t push_cap) {
  if (world < 1 || world > sn::kMaxRanks) return nullptr;
  Group* g = new Group();
  g->world = world;
  g->L = sn::Layout::make(uint32_t(world), lam_cap, ll_cap, push_cap);
  g->status.resize(world);
  for (int r = 0; r < world; ++r) {
    g->regions.push_back(static_cast<char*>(aligned_alloc(4096, g->L.total)));
    init_region(g, r);
  }
  g->chaos = {0, 0, 0, world, 0};
  return g;
}

void sim_group_destroy(void* handle) {
  Group* g = static_cast<Group*>(handle);
  for (char* p : g->regions) free(p);
  delete g;
}

void sim_group_reset(void* handle) {
  Group* g = static_cast<Group*>(handle);
  for (int r = 0; r < g->world; ++r) init_region(g, r);
}

void sim_group_chaos(void* handle, uint32_t permille, uint32_t max_spin, uint32_t far_penalty, int ring4) {
  Group* g = static_cast<Group*>(handle);
  g->chaos = {permille, max_spin, far_penalty, g->world, ring4};
}

uint32_t sim_failed_seq(void* handle, int rank) { return static_cast<Group*>(handle)->status[rank].failed_seq; }
uint32_t sim_failed_peer(void* handle, int rank) { return static_cast<Group*>(handle)->status[rank].peer; }
uint32_t sim_failed_kind(void* handle, int rank) { return static_cast<Group*>(handle)->status[rank].kind; }
// Region inspection for tests: offsets of the layout's areas and a byte copy.
uint64_t sim_lam_offset(void* handle, uint32_t parity, uint32_t src) {
  return static_cast<Group*>(handle)->L.lam(parity, src);
}
uint64_t sim_ll_offset(void* handle) { return static_cast<Group*>(handle)->L.ll_off; }
void sim_read(void* handle, int rank, uint64_t offset, void* dst, uint64_t n) {
  memcpy(dst, static_cast<Group*>(handle)->regions[rank] + offset, n);
}
uint32_t sim_epoch(void* handle, int rank) { return ctrl_of(static_cast<Group*>(handle), rank)->epoch; }
void sim_set_epoch(void* handle, uint32_t epoch) {
  Group* g = static_cast<Group*>(handle);
  for (int r = 0; r < g->world; ++r) ctrl_of(g, r)->epoch = epoch;
}
uint32_t sim_poison(void* handle, int rank) { return ctrl_of(static_cast<Group*>(handle), rank)->poison; }

// op: 1 all-reduce, 2 all-gather, 3 reduce-scatter, 4 exchange, 5 barrier
// algo: all-reduce 0 one-shot / 1 two-shot; all-gather 0 LL / 1 push
int sim_collective(void* handle, int op, int algo, int dtype, int blocks, uint32_t seed, uint64_t nbytes,
                   const void* const* inputs, void* const* outputs, uint64_t row_bytes, uint64_t dst_row_stride,
                   uint64_t dst_src_stride, uint64_t src_peer_stride, int skip_rank, uint32_t timeout_us) {
  Group* g = static_cast<Group*>(handle);
  if (blocks < 1 || blocks > sn::kMaxBlocks) return -1;
  std::vector<std::thread> threads;
  for (int r = 0; r < g->world; ++r) g->status[r].timeout_us = timeout_us;
  for (int r = 0; r < g->world; ++r) {
    for (int b = 0; b < blocks; ++b) {
      threads.emplace_back([=]() {
        if (r == skip_rank) return;
        sim::HostMem m(seed * 7919u + uint32_t(r) * 131u + uint32_t(b), &g->chaos, r);
        sn::Job j;
        memset(&j, 0, sizeof(j));
        for (int q = 0; q < g->world; ++q) j.v.base[q] = g->regions[q];
        j.v.status = &g->status[r];
        j.L = g->L;
        j.rank = uint32_t(r);
        j.world = uint32_t(g->world);
        j.in = static_cast<const char*>(inputs ? inputs[r] : nullptr);
        j.out = static_cast<char*>(outputs ? outputs[r] : nullptr);
        j.nbytes = nbytes;
        j.row_bytes = row_bytes;
        j.dst_row_stride = dst_row_stride;
        j.dst_src_stride = dst_src_stride;
        j.src_peer_stride = src_peer_stride;
        j.valid_out_bytes = -1;
        j.skip_rank = skip_rank;
        sn::Ctrl* ctrl = ctrl_of(g, r);
        if (m.ld_volatile_u32(&ctrl->poison)) return;
        const uint32_t seq = sn::next_seq(m.ld_volatile_u32(&ctrl->epoch));
        sn::OpCtx c{ctrl, j.v.status, seq, uint32_t(r), uint32_t(b), uint32_t(op)};
        const uint64_t gtid = uint64_t(b), gstride = uint64_t(blocks);
        if (g->world == 1) {
          // a one-rank collective is a copy (no sequence): mirrors copy_body on the device
          if (op == 1 || op == 3) {
            const sn::Pack16* in = reinterpret_cast<const sn::Pack16*>(j.in);
            sn::Pack16* out = reinterpret_cast<sn::Pack16*>(j.out);
            for (uint64_t i = gtid; i < nbytes / sn::kPack; i += gstride) m.st_output(out + i, m.ld_input(in + i));
            return;
          }
        }
        switch (op) {
          case 1:
            if (algo == 0) {
              if (dtype == sn::kBF16) sn::oneshot_allreduce<sim::HostMem, sn::kBF16>(m, j, c, gtid, gstride);
              else if (dtype == sn::kF16) sn::oneshot_allreduce<sim::HostMem, sn::kF16>(m, j, c, gtid, gstride);
              else sn::oneshot_allreduce<sim::HostMem, sn::kF32>(m, j, c, gtid, gstride);
            } else {
              if (dtype == sn::kBF16) sn::twoshot_allreduce<sim::HostMem, sn::kBF16>(m, j, c, gtid, gstride);
              else if (dtype == sn::kF16) sn::twoshot_allreduce<sim::HostMem, sn::kF16>(m, j, c, gtid, gstride);
              else sn::twoshot_allreduce<sim::HostMem, sn::kF32>(m, j, c, gtid, gstride);
            }
            break;
          case 3:
            if (dtype == sn::kBF16) sn::reduce_scatter<sim::HostMem, sn::kBF16>(m, j, c, gtid, gstride);
            else if (dtype == sn::kF16) sn::reduce_scatter<sim::HostMem, sn::kF16>(m, j, c, gtid, gstride);
            else sn::reduce_scatter<sim::HostMem, sn::kF32>(m, j, c, gtid, gstride);
            break;
          case 2:
            if (algo == 0) {
              sn::allgather_ll(m, j, c, gtid, gstride);
            } else {
              sn::push_send(m, j, c, false, gtid, gstride);
              if (sn::block_barrier_leader(m, j, c, uint32_t(b))) sn::push_receive(m, j, c, false, gtid, gstride);
            }
            break;
          case 4:
            j.copy_self = 1;
            sn::push_send(m, j, c, true, gtid, gstride);
            if (sn::block_barrier_leader(m, j, c, uint32_t(b))) sn::push_receive(m, j, c, true, gtid, gstride);
            break;
          case 5:
            sn::block_barrier_leader(m, j, c, uint32_t(b));
            break;
          default:
            return;
        }
        sn::finish_op(m, ctrl, seq, uint32_t(blocks));
      });
    }
  }
  for (auto& t : threads) t.join();
  int failed = 0;
  for (int r = 0; r < g->world; ++r) failed += g->status[r].failed_seq != 0;
  return failed;
}

// Host conversions, exported so the tests can check them against torch.
uint16_t sim_f32_to_bf16(float f) { return sn::host_f32_to_bf16(f); }
uint16_t sim_f32_to_f16(float f) { return sn::host_f32_to_f16(f); }
float sim_f16_to_f32(uint16_t h) { return sn::host_f16_to_f32(h); }

}  // extern "C"

// ---------------------------------------------------------------------------
// Self-checking driver (the sanitizer builds run this as an executable).
//   simulate check <world> <blocks> <ops> <seed> <chaos_permille> <ring4>
//   simulate timeout <world>
// ---------------------------------------------------------------------------
#ifdef SIM_MAIN
#include <stdio.h>

#include <random>

namespace {

uint32_t to_bits(int dtype, float v) {
  if (dtype == sn::kF32) return sn::f32_to_bits(v);
  return dtype == sn::kBF16 ? sn::host_f32_to_bf16(v) : sn::host_f32_to_f16(v);
}
float from_bits(int dtype, uint32_t b) {
  if (dtype == sn::kF32) return sn::bits_to_f32(b);
  return dtype == sn::kBF16 ? sn::host_bf16_to_f32(uint16_t(b)) : sn::host_f16_to_f32(uint16_t(b));
}
size_t esize(int dtype) { return dtype == sn::kF32 ? 4 : 2; }
uint32_t get(const std::vector<char>& buf, int dtype, size_t i) {
  uint32_t v = 0;
  memcpy(&v, buf.data() + i * esize(dtype), esize(dtype));
  return v;
}
void put(std::vector<char>& buf, int dtype, size_t i, uint32_t v) { memcpy(buf.data() + i * esize(dtype), &v, esize(dtype)); }

// The sentinel's bit pattern is re-encoded on send (a NaN stays a NaN); the oracle
// does the same before summing.
uint32_t canon(int dtype, uint32_t b) {
  if (dtype == sn::kF32) return b == 0xffffffffu ? (b ^ 1u) : b;
  return b == 0xffffu ? (b ^ 1u) : b;
}

int check(int world, int blocks, int ops, uint32_t seed, uint32_t chaos, int ring4, uint32_t start_epoch = 0) {
  const uint64_t cap = 256 * 1024;
  void* g = sim_group_create(world, cap, cap, cap);
  sim_group_chaos(g, chaos, 8, 4, ring4);
  sim_set_epoch(g, start_epoch);
  std::mt19937 rng(seed);
  std::normal_distribution<float> normal(0.0f, 1.0f);
  int bad = 0;
  for (int k = 0; k < ops; ++k) {
    int op = int(rng() % 5) + 1;
    int dtype = int(rng() % 3);
    int algo = int(rng() % 2);
    size_t packs = 1 + rng() % 512;
    if (op == 5) {
      int f = sim_collective(g, 5, 0, 0, blocks, seed + k, 0, nullptr, nullptr, 0, 0, 0, 0, -1, 5000000);
      if (f) { printf("op %d barrier failed\n", k); ++bad; }
      continue;
    }
    size_t nbytes = packs * sn::kPack;
    if (op == 1 && algo == 1) nbytes = std::min<size_t>(nbytes, cap / 4);
    size_t ne = nbytes / esize(dtype);
    size_t in_bytes = op == 3 || op == 4 ? nbytes * world : nbytes;
    size_t out_bytes = op == 2 || op == 4 ? nbytes * world : nbytes;
    std::vector<std::vector<char>> in(world, std::vector<char>(in_bytes)), out(world, std::vector<char>(out_bytes));
    for (int r = 0; r < world; ++r)
      for (size_t i = 0; i < in_bytes / esize(dtype); ++i) {
        uint32_t v = to_bits(dtype, normal(rng));
        if (rng() % 97 == 0) v = dtype == sn::kF32 ? 0xffffffffu : 0xffffu;  // the sentinel pattern itself
        put(in[r], dtype, i, v);
      }
    std::vector<const void*> ip(world);
    std::vector<void*> op_(world);
    for (int r = 0; r < world; ++r) { ip[r] = in[r].data(); op_[r] = out[r].data(); }
    const uint32_t before = sim_epoch(g, 0);
    int f = sim_collective(g, op, algo, dtype, blocks, seed + k, nbytes, ip.data(), op_.data(), 0, 0, nbytes, nbytes,
                           -1, 5000000);
    if (f) { printf("op %d (kind %d) reported a failure\n", k, op); ++bad; continue; }
    const uint32_t after = sim_epoch(g, 0);
    if (world > 1 && (after == 0 || ((after ^ before) & 1u) == 0u)) {
      printf("op %d: sequence %u after %u does not alternate parity\n", k, after, before);
      ++bad;
      break;
    }
    // oracle
    for (int r = 0; r < world && !bad; ++r) {
      if (op == 1 || op == 3) {
        size_t base = op == 3 ? size_t(r) * ne : 0;
        for (size_t i = 0; i < ne; ++i) {
          float acc = 0.0f;
          for (int s = 0; s < world; ++s) acc = acc + from_bits(dtype, canon(dtype, get(in[s], dtype, base + i)));
          uint32_t want = to_bits(dtype, acc), got = get(out[r], dtype, i);
          bool both_nan = acc != acc && from_bits(dtype, got) != from_bits(dtype, got);
          if (got != want && !both_nan) {
            printf("op %d kind %d algo %d dtype %d rank %d elem %zu: got %08x want %08x\n", k, op, algo, dtype, r, i,
                   got, want);
            ++bad;
            break;
          }
        }
      } else {
        for (int s = 0; s < world; ++s) {
          const char* src = op == 2 ? in[s].data() : in[s].data() + size_t(r) * nbytes;
          if (memcmp(out[r].data() + size_t(s) * nbytes, src, nbytes) != 0) {
            printf("op %d kind %d rank %d: block from %d differs\n", k, op, r, s);
            ++bad;
            break;
          }
        }
      }
    }
    if (bad) break;
  }
  for (int r = 0; r < world; ++r)
    if (sim_epoch(g, r) != sim_epoch(g, 0)) { printf("epochs diverged\n"); ++bad; }
  printf("%s: world %d blocks %d ops %d epoch %u\n", bad ? "FAILED" : "passed", world, blocks, ops, sim_epoch(g, 0));
  sim_group_destroy(g);
  return bad ? 1 : 0;
}

int timeout_case(int world) {
  void* g = sim_group_create(world, 65536, 65536, 65536);
  std::vector<std::vector<char>> in(world, std::vector<char>(4096, 0)), out(world, std::vector<char>(4096));
  std::vector<const void*> ip(world);
  std::vector<void*> op(world);
  for (int r = 0; r < world; ++r) { ip[r] = in[r].data(); op[r] = out[r].data(); }
  int f = sim_collective(g, 1, 0, sn::kBF16, 2, 1, 4096, ip.data(), op.data(), 0, 0, 0, 0, world - 1, 50000);
  int ok = f == world - 1;
  for (int r = 0; r < world - 1; ++r) ok = ok && sim_failed_peer(g, r) == uint32_t(world - 1) && sim_poison(g, r);
  sim_group_reset(g);
  f = sim_collective(g, 1, 0, sn::kBF16, 2, 2, 4096, ip.data(), op.data(), 0, 0, 0, 0, -1, 50000);
  ok = ok && f == 0;
  printf("%s: timeout world %d\n", ok ? "passed" : "FAILED", world);
  sim_group_destroy(g);
  return ok ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc >= 2 && !strcmp(argv[1], "check") && argc >= 8)
    return check(atoi(argv[2]), atoi(argv[3]), atoi(argv[4]), uint32_t(atoi(argv[5])), uint32_t(atoi(argv[6])),
                 atoi(argv[7]), argc >= 9 ? uint32_t(strtoul(argv[8], nullptr, 0)) : 0u);
  if (argc >= 3 && !strcmp(argv[1], "timeout")) return timeout_case(atoi(argv[2]));
  fprintf(stderr, "usage: simulate check <world> <blocks> <ops> <seed> <chaos> <ring4> [start_epoch] | timeout <world>\n");
  return 2;
}
#endif
