// GPU/host clock calibration (K12) for the per-collective trace.
//
// One GPU thread answers host pings through pinned memory with %globaltimer; the
// host brackets each ping with CLOCK_MONOTONIC_RAW and keeps the round with the
// smallest round trip, NTP style: offset = gpu - (t_send + t_recv) / 2, uncertainty
// = half the round trip.  Both sides give up after a bounded number of polls, so a
// lost ping cannot hang the device.  Replaces sparknet/oneshot/_trace_clock.py:24-91.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <time.h>
#include <torch/extension.h>

#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

namespace py = pybind11;

namespace {

struct PingPage {
  volatile unsigned int request;   // host -> device round number (0 = none yet)
  volatile unsigned int reply;     // device -> host round number
  volatile unsigned long long gpu_ns;
  volatile unsigned int stop;
};

__global__ void k_clock_probe(PingPage* page, unsigned int rounds, unsigned long long max_polls) {
  if (threadIdx.x != 0) return;
  unsigned long long polls = 0;
  for (unsigned int r = 1; r <= rounds; ++r) {
    unsigned int seen;
    do {
      asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(seen) : "l"(&page->request) : "memory");
      if (++polls > max_polls || page->stop) return;
    } while (seen < r);
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    page->gpu_ns = t;
    __threadfence_system();
    page->reply = r;
    __threadfence_system();
  }
}

unsigned long long host_ns() {
  timespec t;
  clock_gettime(CLOCK_MONOTONIC_RAW, &t);
  return (unsigned long long)t.tv_sec * 1000000000ull + t.tv_nsec;
}

// Returns [(host_send_ns, gpu_ns, host_recv_ns), ...] for every answered round.
std::vector<std::tuple<unsigned long long, unsigned long long, unsigned long long>> clock_probe(int device,
                                                                                                   int rounds) {
  c10::cuda::CUDAGuard guard(device);
  PingPage* page = nullptr;
  if (cudaHostAlloc(reinterpret_cast<void**>(&page), sizeof(PingPage), cudaHostAllocMapped) != cudaSuccess)
    throw std::runtime_error("cudaHostAlloc(ping page) failed");
  memset(page, 0, sizeof(PingPage));
  PingPage* dpage = nullptr;
  cudaStream_t s = nullptr;
  cudaError_t e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&dpage), page, 0);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e == cudaSuccess) {
    k_clock_probe<<<1, 32, 0, s>>>(dpage, unsigned(rounds), 400000000ull);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {  // nothing was launched (or the launch failed): release and report why
    if (s) cudaStreamDestroy(s);
    cudaFreeHost(page);
    throw std::runtime_error(std::string("clock probe set-up: ") + cudaGetErrorString(e));
  }
  std::vector<std::tuple<unsigned long long, unsigned long long, unsigned long long>> out;
  bool lost = false;
  for (int r = 1; r <= rounds && !lost; ++r) {
    unsigned long long t0 = host_ns();
    __atomic_store_n(&page->request, unsigned(r), __ATOMIC_SEQ_CST);
    for (;;) {
      if (__atomic_load_n(&page->reply, __ATOMIC_ACQUIRE) >= unsigned(r)) break;
      if (host_ns() - t0 > 2000000000ull) {  // 2 s: the kernel is not answering
        lost = true;
        break;
      }
    }
    if (lost) break;
    unsigned long long t1 = host_ns();
    out.emplace_back(t0, page->gpu_ns, t1);
  }
  page->stop = 1;
  cudaStreamSynchronize(s);
  cudaStreamDestroy(s);
  cudaFreeHost(page);
  if (lost) throw std::runtime_error("clock probe kernel did not answer");
  return out;
}

}  // namespace

void register_trace(py::module_& m) {
  m.def("clock_probe", &clock_probe, py::arg("device"), py::arg("rounds") = 200,
        py::call_guard<py::gil_scoped_release>());
}
