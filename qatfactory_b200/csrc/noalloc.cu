// qatf_nvfp4_fake_quant_noalloc: NVFP4 fake quantization with an implicit tensor amax for
// callers that cannot allocate device memory.
//
// qatf_nvfp4_fake_quant needs one caller-owned FP32 word of scratch for the tensor amax.
// Some callers have no way to provide it: a C, cgo or JNI host that binds only this library
// and has no device allocator of its own, or a runtime whose memory pool is sized up front
// and must not see cudaMalloc/cudaFree (which synchronise the device) inside a step.  This
// variant keeps its scratch in a file-scope __device__ array instead, so the caller passes
// only its input and output buffers.
//
// The amax pass here is a two-level reduction: each CTA reduces a fixed chunk of
// kChunk elements into one partial maximum in the static array, and the last CTA to finish
// (a ticket counter in the same array) folds the partials into the final amax, which the
// existing NVFP4 QDQ kernel then reads from device memory.  The array therefore bounds the
// tensor size: at most kMaxPartials chunks, QATF_NOALLOC_MAX_ELEMENTS elements.
//
// Shared-state rules:
//   * the array (about 33 KB) lives on every GPU that loads the library until the process
//     exits;
//   * every call reuses it and it keeps the previous call's contents; the ticket counter
//     is cleared on the call's stream before the reduction starts, and the partials are
//     always written before they are read;
//   * two calls that overlap on the GPU (different streams, or different host threads on
//     one device) race on the array; callers must serialise them;
//   * every call resolves the array's device address with cudaGetSymbolAddress for the
//     current device, so the stream passed must belong to the current device; the first
//     call on a device also loads the module there, so make it before any stream capture.
#include "qatf.h"
#include "qatf_common.cuh"

namespace qatf {
namespace {

constexpr int kNoAllocThreads = 256;
constexpr int64_t kChunk = 65536;      // elements per CTA of the amax pass
constexpr int kMaxPartials = 8192;     // partial maxima the array holds
constexpr int kHeaderWords = 32;       // [0] final amax bits, [1] ticket, rest padding

static_assert((int64_t)kMaxPartials * kChunk == QATF_NOALLOC_MAX_ELEMENTS, "limit mismatch");

__device__ __align__(256) uint32_t g_noalloc_scratch[kHeaderWords + kMaxPartials];

// Device address of the static array on the current device.  Resolved on every call rather
// than cached: a host that resets the device (cudaDeviceReset) or destroys and re-creates its
// primary context gets a new module instance, and a cached address would then be stale.
int scratch_address(uint32_t** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return QATF_ERR_LAUNCH;
  *out = static_cast<uint32_t*>(p);
  return QATF_OK;
}

// One partial max per CTA over elements [blockIdx.x * kChunk, +kChunk); the last CTA folds
// the partials into g_noalloc_scratch[0].  Max over |x| bits: NaN-propagating like torch.amax.
template <typename T>
__global__ void __launch_bounds__(kNoAllocThreads) amax_partials_kernel(const T* __restrict__ x, int64_t n,
                                                                        int vec_ok) {
  using VT = VecTraits<T>;
  constexpr int VEC = VT::kVec;
  const int64_t begin = (int64_t)blockIdx.x * kChunk;
  const int64_t end = begin + kChunk < n ? begin + kChunk : n;
  uint32_t m = 0u;
  if (vec_ok) {
    const int64_t vb = begin / VEC, ve = end / VEC;  // begin is a multiple of VEC
    for (int64_t v = vb + threadIdx.x; v < ve; v += kNoAllocThreads) {
      float f[VEC];
      VT::to_float(ld_stream(x + v * VEC), f);
#pragma unroll
      for (int i = 0; i < VEC; ++i) m = max(m, abs_bits(f[i]));
    }
    for (int64_t e = ve * VEC + threadIdx.x; e < end; e += kNoAllocThreads) m = max(m, abs_bits(VT::load1(x + e)));
  } else {
    for (int64_t e = begin + threadIdx.x; e < end; e += kNoAllocThreads) m = max(m, abs_bits(VT::load1(x + e)));
  }
  m = __reduce_max_sync(0xffffffffu, m);
  __shared__ uint32_t warp_max[kNoAllocThreads / 32];
  __shared__ bool last;
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t b = 0u;
    for (int w = 0; w < kNoAllocThreads / 32; ++w) b = max(b, warp_max[w]);
    g_noalloc_scratch[kHeaderWords + blockIdx.x] = b;
    __threadfence();
    const uint32_t ticket = atomicAdd(&g_noalloc_scratch[1], 1u);
    last = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  uint32_t r = 0u;
  for (uint32_t i = threadIdx.x; i < gridDim.x; i += kNoAllocThreads)
    r = max(r, __ldcg(&g_noalloc_scratch[kHeaderWords + i]));
  r = __reduce_max_sync(0xffffffffu, r);
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = r;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t b = 0u;
    for (int w = 0; w < kNoAllocThreads / 32; ++w) b = max(b, warp_max[w]);
    g_noalloc_scratch[0] = b;
    g_noalloc_scratch[1] = 0u;  // ticket back to zero for the next call
  }
}

}  // namespace
}  // namespace qatf

using namespace qatf;

extern "C" int qatf_nvfp4_fake_quant_noalloc(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, void* y,
                                             uint8_t* mask_bits, void* stream) {
  if (rows < 0 || cols < 0 || ld < cols) return QATF_ERR_INVALID;
  if (rows > 0 && cols > 0 && ld != cols) return QATF_ERR_UNSUPPORTED;  // the amax pass reads a dense tensor
  if (cols > 0 && rows > QATF_NOALLOC_MAX_ELEMENTS / cols) return QATF_ERR_UNSUPPORTED;  // beyond the static scratch
  if (dtype != kF32 && dtype != kF16 && dtype != kBF16) return QATF_ERR_DTYPE;
  const int64_t n = rows * cols;
  if (n == 0) return QATF_OK;
  if (x == nullptr || y == nullptr) return QATF_ERR_INVALID;
  uint32_t* scratch = nullptr;
  int st = scratch_address(&scratch);
  if (st != QATF_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch + 1, 0, sizeof(uint32_t), s) != cudaSuccess) return QATF_ERR_LAUNCH;
  const unsigned grid = (unsigned)((n + kChunk - 1) / kChunk);
  const int vec_ok = aligned16(x) ? 1 : 0;
  switch (dtype) {
    case kF32:
      amax_partials_kernel<float><<<grid, kNoAllocThreads, 0, s>>>(static_cast<const float*>(x), n, vec_ok);
      break;
    case kF16:
      amax_partials_kernel<__half><<<grid, kNoAllocThreads, 0, s>>>(static_cast<const __half*>(x), n, vec_ok);
      break;
    default:
      amax_partials_kernel<__nv_bfloat16><<<grid, kNoAllocThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n,
                                                                          vec_ok);
      break;
  }
  if (launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH) != QATF_OK) return QATF_ERR_LAUNCH;
  return qatf_nvfp4_qdq(x, dtype, rows, cols, ld, reinterpret_cast<const float*>(scratch), y, mask_bits, stream);
}
