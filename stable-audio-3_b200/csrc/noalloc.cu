// Allocation-free FP8 linear: sa3_fp8_linear_noalloc.
//
// Some callers of this library cannot call cudaMalloc. A TensorRT plugin's
// enqueue runs on memory TensorRT planned ahead of time and must not allocate.
// A host with a fixed device-memory budget (several models sharing one GPU) is
// in the same position, and so is an engine that must never hit the implicit
// device synchronisation cudaMalloc can cause in the middle of a stream.
// The regular FP8 path needs scratch for the dynamic activation scale and for
// the e4m3 copy of the activation, which its caller allocates. This entry point
// keeps that scratch in a file-scope __device__ array instead. The array is
// sized once for the whole process (every GPU that loads the library holds
// it until exit), so a call allocates nothing.
//
// Scratch layout (kNoAllocScratchBytes = 16 MiB):
//   [0, 4)    max|x| of the current call (cleared at the start of every call)
//   [4, 8)    s_x = max(max|x|, 1e-12) / 448
//   [256, ..) e4m3 copy of x, M * K bytes, so M * K <= 16 MiB - 256
//
// Every call shares the array and leaves its contents behind. Two calls that
// overlap on the GPU (for example on two streams) race on it; serialise them.
#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace sa3 {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr size_t kNoAllocHeaderBytes = 256;

static __device__ __align__(256) unsigned char g_fp8_linear_scratch[kNoAllocScratchBytes];

// Device address of g_fp8_linear_scratch for the current device. In host code
// the symbol is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
static int noalloc_scratch(unsigned char** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SA3_ERR_LAUNCH;
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fp8_linear_scratch) != cudaSuccess || !p) return SA3_ERR_LAUNCH;
    addr[dev] = p;
  }
  *out = static_cast<unsigned char*>(addr[dev]);
  return SA3_OK;
}

}  // namespace sa3

using namespace sa3;

extern "C" int sa3_fp8_linear_noalloc(const void* x, const void* w, const float* w_scale, const float* bias, void* out,
                                      int M, int N, int K, long long ldx, long long ldw, long long ldo,
                                      void* stream) {
  if (!x || !w || !out || M <= 0 || N <= 0 || K <= 0) return SA3_ERR_ARG;
  if (K % 16) return SA3_ERR_ALIGN;  // the e4m3 copy's rows feed TMA: 16-byte multiples
  // Everything the three launches below would refuse is refused here, before the shared scratch is
  // touched: a call that fails leaves the scratch (which an earlier call on the GPU may still be
  // reading) alone. Activation (sa3_quantize_e4m3): bf16 rows, 16-byte aligned, stride >= K, multiple
  // of 8. Weight (sa3_gemm, e4m3): 16-byte aligned rows, stride >= K, multiple of 16. Output: stride >= N.
  if (ldx < K || ldw < K || ldo < N) return SA3_ERR_ARG;
  if (!aligned16(x) || (ldx % 8) || !aligned16(w) || (ldw % 16)) return SA3_ERR_ALIGN;
  static_assert(SA3_FP8_NOALLOC_MAX_ELEMS == (long long)(kNoAllocScratchBytes - kNoAllocHeaderBytes),
                "header limit and scratch size disagree");
  if ((unsigned long long)M * (unsigned long long)K > (unsigned long long)SA3_FP8_NOALLOC_MAX_ELEMS)
    return SA3_ERR_UNSUPPORTED;  // activation larger than the fixed scratch
  unsigned char* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  float* amax = reinterpret_cast<float*>(scratch);
  float* scale = amax + 1;
  unsigned char* xq = scratch + kNoAllocHeaderBytes;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // The reduction accumulates with atomic max, so its slot must start at zero.
  if (cudaMemsetAsync(amax, 0, sizeof(float), st) != cudaSuccess) return SA3_ERR_LAUNCH;
  if ((rc = sa3_quantize_e4m3(x, nullptr, M, K, ldx, 0, nullptr, nullptr, amax, stream))) return rc;
  if ((rc = sa3_quantize_e4m3(x, xq, M, K, ldx, K, amax, scale, nullptr, stream))) return rc;
  sa3_epilogue e{};
  e.kind = SA3_EPI_STORE;
  e.bias = bias;
  return sa3_gemm(xq, w, out, M, N, K, K, ldw, ldo, SA3_DT_E4M3, scale, w_scale, &e, stream);
}
