// Fused forward-KL distillation loss over a vocabulary (sm_100a).
//
// Semantics: distill_loss (qatfactory/distill/kd_loss.py:147-195) with hard_label_weight 0:
// per supervised token, KL(softmax(t/T) || softmax(s/T)) * T^2 over the vocabulary, computed by
// the reference as FP32 log_softmax / softmax / kl_div(reduction="sum") on chunks of rows.
//
// One CTA per row.  Pass 1 streams the row once with online softmax statistics for both
// logit sets (running max m, z = sum exp(x - m), and a = sum exp(t - m_t) * (t - s)), merged
// across threads; then KL = a / z_t - lse_t + lse_s (sum p_t = 1).  Pass 2, when a gradient is
// wanted, writes d/ds = T * (softmax(s/T) - softmax(t/T)) * grad_scale; its reads of the row
// (2 x 300 KB at vocabulary 151936) mostly hit L2.  exp is __expf (ex2.approx based).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "qatf.h"
#include "qatf_common.cuh"

namespace qatf {
namespace {

constexpr int kKdThreads = 512;

struct Online {
  float m, z;
};

// -inf logits contribute nothing (and never produce inf - inf).
__device__ __forceinline__ void online_add(Online& o, float x) {
  if (x > o.m) {
    o.z = o.z * __expf(o.m - x) + 1.0f;
    o.m = x;
  } else if (x > -INFINITY) {
    o.z += __expf(x - o.m);
  }
}

__device__ __forceinline__ Online online_merge(Online a, Online b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return a;
  return {m, a.z * __expf(a.m - m) + b.z * __expf(b.m - m)};
}

template <typename T>
__device__ __forceinline__ float ld1(const T* p) {
  return VecTraits<T>::load1(p);
}

template <typename T>
__global__ void __launch_bounds__(kKdThreads) kd_forward_kl_kernel(const T* __restrict__ s, const T* __restrict__ t,
                                                                  int64_t vocab, int64_t ld_s, int64_t ld_t,
                                                                  float inv_temp, float temp,
                                                                  const uint8_t* __restrict__ row_valid,
                                                                  float* __restrict__ row_loss,
                                                                  T* __restrict__ grad, float grad_scale) {
  const int64_t row = blockIdx.x;
  const T* sr = s + row * ld_s;
  const T* tr = t + row * ld_t;
  const bool valid = row_valid == nullptr || row_valid[row] != 0;
  __shared__ float red[5][kKdThreads / 32];
  __shared__ float stats[4];

  // ---------------------------------------------------------------------- pass 1
  Online os{-INFINITY, 0.0f}, ot{-INFINITY, 0.0f};
  float a = 0.0f;  // sum exp(t - m_t) * (t - s), rescaled with m_t
  for (int64_t j = threadIdx.x; j < vocab; j += kKdThreads) {
    const float xs = ld1(sr + j) * inv_temp;
    const float xt = ld1(tr + j) * inv_temp;
    online_add(os, xs);
    if (xt > ot.m) {
      const float r = __expf(ot.m - xt);
      ot.z = ot.z * r + 1.0f;
      a = a * r + (xt - xs);
      ot.m = xt;
    } else if (xt > -INFINITY) {  // a zero teacher probability adds nothing (kl_div's xlogy rule)
      const float e = __expf(xt - ot.m);
      ot.z += e;
      a += e * (xt - xs);
    }
  }
  // warp merge
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Online os2{__shfl_xor_sync(0xffffffffu, os.m, o), __shfl_xor_sync(0xffffffffu, os.z, o)};
    Online ot2{__shfl_xor_sync(0xffffffffu, ot.m, o), __shfl_xor_sync(0xffffffffu, ot.z, o)};
    const float a2 = __shfl_xor_sync(0xffffffffu, a, o);
    os = online_merge(os, os2);
    const float m = fmaxf(ot.m, ot2.m);
    if (m != -INFINITY) {
      const float r1 = __expf(ot.m - m), r2 = __expf(ot2.m - m);
      a = a * r1 + a2 * r2;
      ot = {m, ot.z * r1 + ot2.z * r2};
    }
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red[0][w] = os.m;
    red[1][w] = os.z;
    red[2][w] = ot.m;
    red[3][w] = ot.z;
    red[4][w] = a;
  }
  __syncthreads();
  if (w == 0) {
    constexpr int kW = kKdThreads / 32;
    os = lane < kW ? Online{red[0][lane], red[1][lane]} : Online{-INFINITY, 0.0f};
    ot = lane < kW ? Online{red[2][lane], red[3][lane]} : Online{-INFINITY, 0.0f};
    a = lane < kW ? red[4][lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Online os2{__shfl_xor_sync(0xffffffffu, os.m, o), __shfl_xor_sync(0xffffffffu, os.z, o)};
      Online ot2{__shfl_xor_sync(0xffffffffu, ot.m, o), __shfl_xor_sync(0xffffffffu, ot.z, o)};
      const float a2 = __shfl_xor_sync(0xffffffffu, a, o);
      os = online_merge(os, os2);
      const float m = fmaxf(ot.m, ot2.m);
      if (m != -INFINITY) {
        const float r1 = __expf(ot.m - m), r2 = __expf(ot2.m - m);
        a = a * r1 + a2 * r2;
        ot = {m, ot.z * r1 + ot2.z * r2};
      }
    }
    if (lane == 0) {
      const float lse_s = os.m + logf(os.z);
      const float lse_t = ot.m + logf(ot.z);
      stats[0] = lse_s;
      stats[1] = lse_t;
      row_loss[row] = valid ? (a / ot.z - lse_t + lse_s) * temp * temp : 0.0f;
    }
  }
  if (grad == nullptr) return;
  __syncthreads();

  // ---------------------------------------------------------------------- pass 2
  const float lse_s = stats[0], lse_t = stats[1];
  const float scale = valid ? grad_scale * temp : 0.0f;
  T* gr = grad + row * vocab;
  for (int64_t j = threadIdx.x; j < vocab; j += kKdThreads) {
    const float xs = ld1(sr + j) * inv_temp;
    const float xt = ld1(tr + j) * inv_temp;
    VecTraits<T>::store1(gr + j, (__expf(xs - lse_s) - __expf(xt - lse_t)) * scale);
  }
}

}  // namespace
}  // namespace qatf

using namespace qatf;

extern "C" int qatf_kd_forward_kl(const void* student, const void* teacher, int dtype, int64_t rows, int64_t vocab,
                                  int64_t ld_s, int64_t ld_t, float temperature, const uint8_t* row_valid,
                                  float* row_loss, void* grad, float grad_scale, void* stream) {
  if (rows < 0 || vocab < 0 || ld_s < vocab || ld_t < vocab || !(temperature > 0.0f)) return QATF_ERR_INVALID;
  if (rows == 0 || vocab == 0) return QATF_OK;
  if (student == nullptr || teacher == nullptr || row_loss == nullptr) return QATF_ERR_INVALID;
  if (rows > 0x7FFFFFFF) return QATF_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float inv = 1.0f / temperature;
  auto run = [&](auto tag) -> int {
    using T = decltype(tag);
    kd_forward_kl_kernel<T><<<(unsigned)rows, kKdThreads, 0, s>>>(
        static_cast<const T*>(student), static_cast<const T*>(teacher), vocab, ld_s, ld_t, inv, temperature,
        row_valid, row_loss, static_cast<T*>(grad), grad_scale);
    return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH);
  };
  switch (dtype) {
    case QATF_F32:
      return run(float{});
    case QATF_F16:
      return run(__half{});
    case QATF_BF16:
      return run(__nv_bfloat16{});
    default:
      return QATF_ERR_DTYPE;
  }
}
