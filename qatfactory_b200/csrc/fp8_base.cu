// Dequantization of block-scaled FP8 frozen bases (sm_100a).
//
// Pre-quantized checkpoints keep their weights as float8 codes (E4M3 or E5M2) plus a grid of
// FP32 `scale_inv` values, one per (rows / scale_rows) x (cols / scale_cols) block; LoRA-QAD
// keeps the codes as the frozen base and dequantizes one weight (or one fused expert tensor)
// at a time (qatfactory/quant/formats/fp8_base.py:27-52):
//     out = (float(code) * scale_inv[block]).to(dtype)
// The code widens exactly, the product is one FP32 multiply rounded to nearest even and the
// cast to BF16 / FP16 rounds to nearest even, so the output equals the reference's torch
// expression bit for bit.  One thread widens 16 codes (a 16-byte load) of one block row and
// writes them with one or two vector stores.
#include <cuda_fp8.h>

#include <type_traits>

#include "qatf.h"
#include "qatf_common.cuh"

namespace qatf {

constexpr int kFp8Threads = 256;

template <int FMT>
__device__ __forceinline__ void fp8x2_to_float2(uint16_t pair, float* f) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(pair, FMT == QATF_FP8_E4M3 ? __NV_E4M3 : __NV_E5M2);
  const __half2 v = *reinterpret_cast<const __half2*>(&h);
  f[0] = __low2float(v);
  f[1] = __high2float(v);
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float* f) {
  using VT = VecTraits<T>;
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int v = 0; v < 4; ++v) st_v4(p + 4 * v, VT::from_float(f + 4 * v));
  } else {
    st_v4(p, VT::from_float(f));
    st_v4(p + 8, VT::from_float(f + 8));
  }
}

// Vector path: cols % 16 == 0 and the block width a multiple of 16, so 16 consecutive codes
// of a row share one scale.
template <int FMT, typename T>
__global__ void __launch_bounds__(kFp8Threads) fp8_block_dequant_vec_kernel(
    const uint8_t* __restrict__ codes, int64_t n16, int64_t rows, int64_t cols16, int64_t block_rows,
    int64_t block_cols16, int64_t scale_rows, int64_t scale_cols, const float* __restrict__ scale_inv,
    T* __restrict__ out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n16; v += stride) {
    const int64_t row_all = v / cols16;  // row over all batches
    const int64_t c16 = v - row_all * cols16;
    const int64_t b = row_all / rows;
    const int64_t r = row_all - b * rows;
    const float s = __ldg(scale_inv + (b * scale_rows + r / block_rows) * scale_cols + c16 / block_cols16);
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(codes) + v);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    float f[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      fp8x2_to_float2<FMT>((uint16_t)(w[i] & 0xFFFFu), f + 4 * i);
      fp8x2_to_float2<FMT>((uint16_t)(w[i] >> 16), f + 4 * i + 2);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) f[i] = __fmul_rn(f[i], s);
    store16(out + v * 16, f);
  }
}

// Any shape: one element per thread.
template <int FMT, typename T>
__global__ void __launch_bounds__(kFp8Threads) fp8_block_dequant_kernel(
    const uint8_t* __restrict__ codes, int64_t n, int64_t rows, int64_t cols, int64_t block_rows, int64_t block_cols,
    int64_t scale_rows, int64_t scale_cols, const float* __restrict__ scale_inv, T* __restrict__ out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
    const int64_t row_all = e / cols;
    const int64_t c = e - row_all * cols;
    const int64_t b = row_all / rows;
    const int64_t r = row_all - b * rows;
    const float s = __ldg(scale_inv + (b * scale_rows + r / block_rows) * scale_cols + c / block_cols);
    float f[2];
    fp8x2_to_float2<FMT>((uint16_t)codes[e], f);
    VecTraits<T>::store1(out + e, __fmul_rn(f[0], s));
  }
}

}  // namespace qatf

using namespace qatf;

extern "C" int qatf_fp8_block_dequant(const uint8_t* codes, int fp8_format, int64_t batches, int64_t rows,
                                      int64_t cols, const float* scale_inv, int64_t scale_rows, int64_t scale_cols,
                                      void* out, int out_dtype, void* stream) {
  if (batches < 0 || rows < 0 || cols < 0 || scale_rows <= 0 || scale_cols <= 0) return QATF_ERR_INVALID;
  if (fp8_format != QATF_FP8_E4M3 && fp8_format != QATF_FP8_E5M2) return QATF_ERR_INVALID;
  if (rows % scale_rows != 0 || cols % scale_cols != 0) return QATF_ERR_INVALID;
  if (batches == 0 || rows == 0 || cols == 0) return QATF_OK;
  if (codes == nullptr || scale_inv == nullptr || out == nullptr) return QATF_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t block_rows = rows / scale_rows, block_cols = cols / scale_cols;
  const int64_t n = batches * rows * cols;
  auto run = [&](auto fmt_tag, auto out_tag) -> int {
    constexpr int FMT = decltype(fmt_tag)::value;
    using T = decltype(out_tag);
    T* o = static_cast<T*>(out);
    if (cols % 16 == 0 && block_cols % 16 == 0 && aligned16(codes) && aligned16(out)) {
      auto k = fp8_block_dequant_vec_kernel<FMT, T>;
      const int64_t n16 = n / 16;
      k<<<persistent_grid(n16, (const void*)k, kFp8Threads), kFp8Threads, 0, s>>>(
          codes, n16, rows, cols / 16, block_rows, block_cols / 16, scale_rows, scale_cols, scale_inv, o);
    } else {
      auto k = fp8_block_dequant_kernel<FMT, T>;
      k<<<persistent_grid(n, (const void*)k, kFp8Threads), kFp8Threads, 0, s>>>(
          codes, n, rows, cols, block_rows, block_cols, scale_rows, scale_cols, scale_inv, o);
    }
    return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH);
  };
  auto by_out = [&](auto fmt_tag) -> int {
    switch (out_dtype) {
      case QATF_F32:
        return run(fmt_tag, float{});
      case QATF_F16:
        return run(fmt_tag, __half{});
      case QATF_BF16:
        return run(fmt_tag, __nv_bfloat16{});
      default:
        return QATF_ERR_DTYPE;
    }
  };
  return fp8_format == QATF_FP8_E4M3 ? by_out(std::integral_constant<int, QATF_FP8_E4M3>{})
                                     : by_out(std::integral_constant<int, QATF_FP8_E5M2>{});
}
