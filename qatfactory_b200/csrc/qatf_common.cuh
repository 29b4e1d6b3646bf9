// Shared device helpers for the fake-quantization kernels (sm_100a).
//
// Numerics contract: every helper reproduces, bit for bit, one PyTorch CPU expression of
// the reference quantizers (qatfactory/quant/formats/*.py).  Division-free shortcuts are
// used only where they are provably identical to the IEEE operation they replace:
//   * x / 2^k is computed as x * 2^-k (both round the same real number once);
//   * a / b for a per-block divisor b uses Markstein's correction
//         y = RN(1/b), q0 = RN(a*y), r = fma(-q0, b, a), q = fma(r, y, q0)
//     which returns RN(a/b) whenever no intermediate over/underflows (P. Markstein,
//     "IA-64 and Elementary Functions", 2000, Thm. 8.10); outside the guarded range the
//     kernels call __fdiv_rn.
//   * E2M1 round-half-to-even of a clamped value |v| <= 6 is rint(v * s) / s with
//     s = 2, 1, 1/2 on the binades [0,2), [2,4), [4,6]: the E2M1 grid is uniform with
//     step 1/s there and its midpoints are exactly the reference's tie boundaries
//     (exhaustively checked against the bucketize rule for every float32).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <unordered_map>

namespace qatf {

enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

// ------------------------------------------------------------------ 16-byte vectors
template <typename T>
struct VecTraits;

template <>
struct VecTraits<float> {
  static constexpr int kVec = 4;
  __device__ __forceinline__ static void to_float(const uint4& raw, float* f) {
    f[0] = __uint_as_float(raw.x);
    f[1] = __uint_as_float(raw.y);
    f[2] = __uint_as_float(raw.z);
    f[3] = __uint_as_float(raw.w);
  }
  __device__ __forceinline__ static uint4 from_float(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
  __device__ __forceinline__ static float load1(const float* p) { return *p; }
  __device__ __forceinline__ static void store1(float* p, float v) { *p = v; }
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);  // cvt.rn.bf16x2.f32, RNE like c10::BFloat16
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);  // RNE, overflow to inf like c10::Half
  return *reinterpret_cast<uint32_t*>(&h);
}

template <>
struct VecTraits<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static void unpack2(uint32_t w, float* f) {
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xFFFF0000u);
  }
  __device__ __forceinline__ static void to_float(const uint4& raw, float* f) {
    unpack2(raw.x, f + 0);
    unpack2(raw.y, f + 2);
    unpack2(raw.z, f + 4);
    unpack2(raw.w, f + 6);
  }
  __device__ __forceinline__ static uint4 from_float(const float* f) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                      pack_bf16x2(f[6], f[7]));
  }
  __device__ __forceinline__ static float load1(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  __device__ __forceinline__ static void store1(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

template <>
struct VecTraits<__half> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static void unpack2(uint32_t w, float* f) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    float2 v = __half22float2(h);
    f[0] = v.x;
    f[1] = v.y;
  }
  __device__ __forceinline__ static void to_float(const uint4& raw, float* f) {
    unpack2(raw.x, f + 0);
    unpack2(raw.y, f + 2);
    unpack2(raw.z, f + 4);
    unpack2(raw.w, f + 6);
  }
  __device__ __forceinline__ static uint4 from_float(const float* f) {
    return make_uint4(pack_f16x2(f[0], f[1]), pack_f16x2(f[2], f[3]), pack_f16x2(f[4], f[5]), pack_f16x2(f[6], f[7]));
  }
  __device__ __forceinline__ static float load1(const __half* p) { return __half2float(*p); }
  __device__ __forceinline__ static void store1(__half* p, float v) { *p = __float2half_rn(v); }
};

// Streaming 16-byte load that does not allocate in L1 (each byte is read once).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// 256-bit streaming load and plain 256-bit store (sm_100).
__device__ __forceinline__ void ld_stream256(const void* p, uint32_t* w) {
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
               : "l"(p));
}

__device__ __forceinline__ void st256(void* p, const uint32_t* w) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]),
               "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

__device__ __forceinline__ void st_v4(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// |x| as raw bits: ordering of non-negative floats matches their bit patterns and every
// NaN sorts above +inf, so an integer max over these bits is torch.amax (NaN-propagating).
__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7FFFFFFFu; }

// ------------------------------------------------------------------------ E4M3 / E2M1

// torch: values.clamp(0, 448).to(float8_e4m3fn).float() (nvfp4.py:55-58).  RNE with
// subnormals in units of 2^-9.  NaN stays NaN.  Also returns the stored byte.
__device__ __forceinline__ float e4m3_rne(float v, uint32_t* byte_out) {
  if (!(v == v)) {
    *byte_out = 0x7Fu;
    return v;
  }
  v = fminf(fmaxf(v, 0.0f), 448.0f);
  if (v < 0.015625f) {
    float units = rintf(__fmul_rn(v, 512.0f));
    *byte_out = (uint32_t)units;  // 0..8; 8 also encodes 2^-6 as a normal
    return __fmul_rn(units, 0.001953125f);
  }
  uint32_t bits = __float_as_uint(v);
  uint32_t rounded = (bits + 0x7FFFFu + ((bits >> 20) & 1u)) & 0xFFF00000u;
  uint32_t e = ((rounded >> 23) & 0xFFu) - 120u;  // (exp - 127) + 7
  *byte_out = (e << 3) | ((rounded >> 20) & 7u);
  return __uint_as_float(rounded);
}

// Magnitude index (0..7) of an E2M1 code magnitude c in {0,.5,1,1.5,2,3,4,6}.
__device__ __forceinline__ uint32_t e2m1_index(float c) {
  // c < 2: 2c ; 2 <= c < 4: c + 2 ; c >= 4: c/2 + 4   (all exact)
  float idx = c < 2.0f ? c * 2.0f : (c < 4.0f ? c + 2.0f : __fmaf_rn(c, 0.5f, 4.0f));
  return (uint32_t)idx;
}

// _round_to_e2m1(clamp(n, -6, 6)) (nvfp4.py:44-52, :496-497): returns the signed code
// value.  NaN maps to +0 (torch.sign(NaN) == 0) and so does a zero of either sign; a
// nonzero value that rounds to zero keeps its sign (-0 for a tiny negative).
__device__ __forceinline__ float e2m1_round(float n) {
  if (!(n == n)) return 0.0f;
  float c = fminf(fmaxf(n, -6.0f), 6.0f);
  float a = fabsf(c);
  float s = a < 2.0f ? 2.0f : (a < 4.0f ? 1.0f : 0.5f);
  float si = a < 2.0f ? 0.5f : (a < 4.0f ? 1.0f : 2.0f);
  float r = __fmul_rn(rintf(__fmul_rn(c, s)), si);
  return c == 0.0f ? 0.0f : r;
}

// Divisor state for a / b with one b per quantization block.  `fast` holds when the
// Markstein sequence is exact for every element a of the block that is zero or has
// |a| >= 2^-100: b in [2^-100, 2^26] keeps RN(a*y) normal and the residual representable,
// a finite block amax rules out infinite a, and amax < 2^126 * b rules out overflow.
struct BlockDivisor {
  float b, y;
  bool fast;
};

__device__ __forceinline__ BlockDivisor make_divisor(float b, uint32_t block_amax_bits) {
  BlockDivisor d;
  d.b = b;
  uint32_t bb = __float_as_uint(b);
  int exp_gap = (int)(block_amax_bits >> 23) - (int)(bb >> 23);
  d.fast = bb >= 0x0D800000u && bb <= 0x4C800000u && block_amax_bits < 0x7F800000u && exp_gap <= 125;
  d.y = __frcp_rn(b);
  return d;
}

// IEEE a / b (== __fdiv_rn(a, b)).
__device__ __forceinline__ float divide(const BlockDivisor& d, float a) {
  uint32_t abits = __float_as_uint(a) & 0x7FFFFFFFu;
  bool tiny = (abits - 1u) < 0x0D7FFFFFu;  // 0 < |a| < 2^-100
  if (d.fast && !tiny) {
    float q0 = __fmul_rn(a, d.y);
    float r = __fmaf_rn(-q0, d.b, a);
    return __fmaf_rn(r, d.y, q0);
  }
  return __fdiv_rn(a, d.b);
}

// 2^k for integer k in [-127, 127], built exactly from bits (2^-127 is subnormal).
__device__ __forceinline__ float pow2i(int k) {
  return k == -127 ? __uint_as_float(0x00400000u) : __uint_as_float((uint32_t)(k + 127) << 23);
}

// _e8m0_exponent_even (mxfp4.py:48-60) from the raw bits of a non-negative block amax.
__device__ __forceinline__ int e8m0_exponent_even(uint32_t amax_bits) {
  uint32_t rounded = (amax_bits + 0x200000u) & 0x7F800000u;
  int e = (int)(rounded >> 23);
  if (e == 0) return -127;   // 2^-126 -> -128 -> clamp
  if (e == 255) return 127;  // +inf -> clamp
  int k = e - 129;
  return k < -127 ? -127 : (k > 127 ? 127 : k);
}

// _e8m0_exponent_ceil (mxfp4.py:73-98): returns the biased exponent in [0, 254]; 0 marks
// a zero block.
__device__ __forceinline__ int e8m0_biased_ceil(float amax) {
  float q = __fmul_rn(amax, 0.16666667163372039794921875f);
  uint32_t bits = __float_as_uint(q);
  int e = (int)((bits >> 23) & 0xFFu);
  uint32_t man = bits & 0x7FFFFFu;
  bool tiny = (e == 0) && (man <= 0x400000u);
  int biased = e + ((man != 0u && !tiny) ? 1 : 0);
  return biased > 254 ? 254 : biased;
}

// ------------------------------------------------------------------- launch helpers
// Counts one kernel launch when `status` is QATF_OK and returns `status` (capi.cu).
int launched(int status);

// Programmatic dependent launch.  A kernel launched by launch_pdl may be scheduled while the
// previous kernel on its stream is still finishing: it calls pdl_wait() before it touches any
// global memory (the wait returns once the previous grid has completed and its writes are
// visible), then pdl_launch_dependents() so that the next such kernel can be scheduled into
// the SM slots its own CTAs leave.  Back-to-back quantizer launches (one layer's weights after
// another) then overlap one kernel's launch and tail with the next one's start.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
#ifdef QATF_DISABLE_PDL
  cfg.numAttrs = 0;
#else
  cfg.numAttrs = 1;
#endif
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

inline int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

// Resident blocks per SM of `kernel` at `block` threads, queried once per (device, kernel).
inline int blocks_per_sm(const void* kernel, int block) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t key = (reinterpret_cast<uintptr_t>(kernel) << 8) ^ (uint64_t)dev ^ ((uint64_t)block << 48);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, block, 0) != cudaSuccess || occ <= 0) occ = 1;
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = occ;
  return occ;
}

// Grid for a grid-stride kernel: enough blocks for `threads_needed`, at most one full wave
// (of at most `max_per_sm` blocks per SM when that is positive).
inline int64_t persistent_grid(int64_t threads_needed, const void* kernel, int block, int max_per_sm = 0) {
  int per_sm = blocks_per_sm(kernel, block);
  if (max_per_sm > 0 && per_sm > max_per_sm) per_sm = max_per_sm;
  const int64_t full = (int64_t)num_sms() * per_sm;
  const int64_t need = (threads_needed + block - 1) / block;
  return need < full ? (need > 0 ? need : 1) : full;
}

}  // namespace qatf
