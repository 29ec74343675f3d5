// Allocation-free decode attention (see sparknet/noalloc.h for who needs it and the
// contract).  Same kernels as the torch entry point (attention_kernels.cuh); the only
// difference is where the per-split partials live: a file-scope device array of fixed
// size instead of a caller- or torch-allocated workspace.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <functional>
#include <mutex>
#include <stdexcept>
#include <string>

#include "sparknet/attention_kernels.cuh"
#include "sparknet/attention_tc.cuh"
#include "sparknet/noalloc.h"

namespace {

constexpr size_t kScratchFloats = SPARKNET_NOALLOC_SCRATCH_BYTES / sizeof(float);
constexpr int kMaxDevices = 64;

// The scratch.  In host code this name is only a host-side stand-in for the symbol:
// its device address comes from cudaGetSymbolAddress, per device.
static __device__ __align__(256) float g_attention_scratch[kScratchFloats];

// Per device: the scratch's device address and the SM count, looked up once.  The
// once-flags make concurrent first calls from several host threads safe; a lookup that
// failed throws out of call_once, so the next call on that device tries again.
struct DeviceSetup {
  std::once_flag once;
  float* scratch = nullptr;
  int sms = 0;
};
DeviceSetup g_setup[kMaxDevices];
thread_local std::string g_error;

int fail(int code, const std::string& what) {
  g_error = what;
  return code;
}

void lookup(int device, DeviceSetup& d) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_attention_scratch);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  int n = 0;
  e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
  d.sms = n;
  d.scratch = static_cast<float*>(p);
}

// With `device` current: the scratch's device address and the SM count used to split
// sequences.
int setup(int device, float** scratch, int* sms) {
  if (device < 0 || device >= kMaxDevices) return fail(1, "device ordinal out of range");
  DeviceSetup& d = g_setup[device];
  try {
    std::call_once(d.once, lookup, device, std::ref(d));
  } catch (const std::exception& ex) {
    return fail(3, ex.what());
  }
  *scratch = d.scratch;
  *sms = d.sms;
  return 0;
}

}  // namespace

extern "C" size_t sparknet_decode_attention_scratch_bytes(int B, int Hq, int Hkv, int max_len) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || max_len <= 0 || Hq % Hkv) return 0;
  // the split count depends on the SM count: that of the current device, as a call uses
  int device = 0, sms = 0;
  if (cudaGetDevice(&device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0)
    return 0;
  return sn::attn::scratch_floats(B, Hq, Hkv, max_len, sms) * sizeof(float);
}

extern "C" const char* sparknet_noalloc_last_error(void) { return g_error.c_str(); }

extern "C" int sparknet_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                                 const int32_t* lengths, void* out, int B, int Hq, int Hkv, int Lmax,
                                                 int max_len, float scale, cudaStream_t stream) {
  g_error.clear();
  if (!q || !k_cache || !v_cache || !lengths || !out) return fail(1, "null pointer argument");
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Lmax <= 0 || max_len <= 0 || max_len > Lmax)
    return fail(1, "sizes must be positive and max_len <= Lmax");
  if (Hq % Hkv) return fail(1, "query heads must be a multiple of KV heads");
  const int G = Hq / Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16) return fail(1, "unsupported GQA group size");
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return fail(3, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  float* scratch = nullptr;
  int sms = 0;
  if (int rc = setup(device, &scratch, &sms)) return rc;
  if (B * Hkv > sn::attn::kCounterSlots) return fail(1, "too many (sequence, KV head) pairs");
  const size_t need = sn::attn::scratch_floats(B, Hq, Hkv, max_len, sms);
  if (need > kScratchFloats)
    return fail(2, "problem needs " + std::to_string(need * sizeof(float)) + " bytes of scratch; the built-in scratch is " +
                       std::to_string(SPARKNET_NOALLOC_SCRATCH_BYTES) + " bytes (use the allocating entry point)");
  // the counters this call uses must be zero when its kernel starts: clear them on the
  // caller's stream (a device memset: nothing is allocated)
  e = cudaMemsetAsync(scratch, 0, size_t(B) * Hkv * sizeof(int), stream);
  if (e != cudaSuccess) return fail(3, std::string("clearing the counters: ") + cudaGetErrorString(e));
  e = sn::attn::launch_decode_attention(static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k_cache),
                                        static_cast<const __nv_bfloat16*>(v_cache), lengths,
                                        static_cast<__nv_bfloat16*>(out), scratch, B, Hq, Hkv, Lmax, max_len, scale, sms,
                                        stream);
  if (e != cudaSuccess) return fail(3, std::string("launch: ") + cudaGetErrorString(e));
  return 0;
}
