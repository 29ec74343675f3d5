// Allocation-free decode attention (see sparknet/noalloc.h for who needs it and the
// contract).  Same kernels as the torch entry point (attention_kernels.cuh); the only
// difference is where the per-split partials live: a file-scope device array of fixed
// size instead of a caller- or torch-allocated workspace.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <string>

#include "sparknet/attention_kernels.cuh"
#include "sparknet/noalloc.h"

namespace {

constexpr size_t kScratchFloats = SPARKNET_NOALLOC_SCRATCH_BYTES / sizeof(float);
constexpr int kMaxDevices = 64;

// The scratch.  In host code this name is only a host-side stand-in for the symbol:
// its device address comes from cudaGetSymbolAddress, per device.
static __device__ __align__(256) float g_attention_scratch[kScratchFloats];

float* g_scratch_ptr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
thread_local std::string g_error;

int fail(int code, const std::string& what) {
  g_error = what;
  return code;
}

// Once per device, with that device current: the scratch's device address and the SM
// count used to split sequences.
int setup(int device, float** scratch, int* sms) {
  if (device < 0 || device >= kMaxDevices) return fail(1, "device ordinal out of range");
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_attention_scratch);
    if (e != cudaSuccess) return fail(3, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return fail(3, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
    g_sms[device] = n;
    g_scratch_ptr[device] = static_cast<float*>(p);
  }
  *scratch = g_scratch_ptr[device];
  *sms = g_sms[device];
  return 0;
}

}  // namespace

extern "C" size_t sparknet_decode_attention_scratch_bytes(int B, int Hq, int Hkv, int max_len) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || max_len <= 0 || Hq % Hkv) return 0;
  // the split count depends on the SM count; 148 SMs on B200 (queried per device at run time)
  return sn::attn::scratch_floats(B, Hq, Hkv, max_len, 148) * sizeof(float);
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
