// Exhaustive check of the hardware FP4/FP8 converters the bf16 fast path relies on,
// against the library's own exact software rounding (which the CPU tests pin to the
// reference):
//   * cvt.rn.satfinite.e2m1x2.f32 + cvt.rn.f16x2.e2m1x2 on every float32 in [0, 8]
//     versus e2m1_round (RNE to {0,.5,1,1.5,2,3,4,6}, saturating at 6);
//   * cvt.rn.satfinite.e4m3x2.f32 + cvt.rn.f16x2.e4m3x2 on every float32 in [0, 1024]
//     versus e4m3_rne (RNE with subnormals, saturating at 448), value and byte.
// Prints the mismatch counts; exits non-zero on any mismatch.
#include <cstdio>

#include "qatf_common.cuh"

using namespace qatf;

__global__ void check_e2m1(uint32_t lo, uint32_t hi, unsigned long long* bad) {
  unsigned long long local = 0;
  for (uint64_t u = lo + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u <= hi;
       u += (uint64_t)gridDim.x * blockDim.x) {
    const float v = __uint_as_float((uint32_t)u);
    uint32_t h;
    asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
        : "=r"(h)
        : "f"(v), "f"(0.0f));
    const float hw = __half2float(__ushort_as_half((uint16_t)(h & 0xFFFFu)));
    const float sw = e2m1_round(v);
    if (__float_as_uint(hw) != __float_as_uint(sw)) ++local;
  }
  if (local) atomicAdd(bad, local);
}

__global__ void check_e4m3(uint32_t lo, uint32_t hi, unsigned long long* bad) {
  unsigned long long local = 0;
  for (uint64_t u = lo + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u <= hi;
       u += (uint64_t)gridDim.x * blockDim.x) {
    const float v = __uint_as_float((uint32_t)u);
    uint16_t b;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(b) : "f"(v), "f"(0.0f));
    uint32_t h;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(b));
    const float hw = __half2float(__ushort_as_half((uint16_t)(h & 0xFFFFu)));
    uint32_t sw_byte;
    const float sw = e4m3_rne(v, &sw_byte);
    if (__float_as_uint(hw) != __float_as_uint(sw) || (b & 0xFFu) != sw_byte) ++local;
  }
  if (local) atomicAdd(bad, local);
}

int main() {
  unsigned long long* bad = nullptr;
  if (cudaMalloc(&bad, 2 * sizeof(unsigned long long)) != cudaSuccess) return 2;
  cudaMemset(bad, 0, 2 * sizeof(unsigned long long));
  check_e2m1<<<1184, 256>>>(0u, 0x41000000u, bad);       // [0, 8]
  check_e4m3<<<1184, 256>>>(0u, 0x44800000u, bad + 1);   // [0, 1024]
  unsigned long long h[2] = {0, 0};
  if (cudaMemcpy(h, bad, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess) return 2;
  cudaFree(bad);
  printf("e2m1 mismatches %llu\ne4m3 mismatches %llu\n", h[0], h[1]);
  return (h[0] == 0 && h[1] == 0) ? 0 : 1;
}
