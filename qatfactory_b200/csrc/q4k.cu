// Q4_K (GGUF block_q4_K) super-block encoder and decoder for sm_100a.
//
// A super-block is 256 consecutive weights of one row: 8 sub-blocks of 32, each with an
// affine (scale, min) fit whose 6-bit codes ls/lm are quantized against two FP16
// super-block scales d/dmin (qatfactory/quant/formats/q4_k.py:1-17).  The encoder writes
// any of: the reconstruction d*ls*q - dmin*lm in the input dtype, the STE bit mask and the
// 144-byte block [d f16][dmin f16][12 B packed 6-bit scales/mins][128 B nibbles].
//
// Two kernels share the level-2 code:
//   * minmax (the default "q4_k" format): one warp per super-block, 8 weights per lane,
//     one 16-byte load per lane; sub-block and super-block maxima by warp shuffles.  It is
//     HBM-bound.
//   * grid_search: one thread per sub-block, 8 lanes per super-block, the 21-step
//     weighted least-squares search of llama.cpp's make_qkx2_quants kept entirely in
//     registers.  It is FP32-ALU-bound.
// Every float operation repeats the reference's torch CPU expression in the same order:
// `c / t` is t.reciprocal() * c, 32-element sums use torch-CPU's 8-lane vector order
// t[k] = ((v[k] + v[k+8]) + v[k+16]) + v[k+24] followed by a sequential sum of t[0..7],
// and the per-weight division (x + dm) / deff is an exact Markstein quotient.
#include "qatf.h"
#include "qatf_common.cuh"

namespace qatf {

constexpr int kQK = 256;
constexpr int kQ4Threads = 256;

// (_RMIN + _RDELTA * step + nmax) evaluated in double by Python, then cast to float by
// torch when it multiplies a float tensor (q4_k.py:92-93).
#define QATF_TRIAL(s) ((float)(-1.0 + 0.1 * (double)(s) + 15.0))
__constant__ float c_trial[21] = {QATF_TRIAL(0),  QATF_TRIAL(1),  QATF_TRIAL(2),  QATF_TRIAL(3),  QATF_TRIAL(4),
                                  QATF_TRIAL(5),  QATF_TRIAL(6),  QATF_TRIAL(7),  QATF_TRIAL(8),  QATF_TRIAL(9),
                                  QATF_TRIAL(10), QATF_TRIAL(11), QATF_TRIAL(12), QATF_TRIAL(13), QATF_TRIAL(14),
                                  QATF_TRIAL(15), QATF_TRIAL(16), QATF_TRIAL(17), QATF_TRIAL(18), QATF_TRIAL(19),
                                  QATF_TRIAL(20)};
#undef QATF_TRIAL

__device__ __forceinline__ float clamp15(float v) { return fminf(fmaxf(v, 0.0f), 15.0f); }

// Level 2 (q4_k.py:173-183) from this lane's sub-block fit and the super-block maxima.
struct Level2 {
  float deff, dm;
  uint32_t ls, lm;
  uint16_t d_h, dmin_h;
};

__device__ __forceinline__ Level2 level2(float scale, float the_min, float max_scale, float max_min) {
  Level2 L;
  const float inv_scale = max_scale > 0.0f ? __fmul_rn(__frcp_rn(max_scale), 63.0f) : 0.0f;  // 63.0 / t
  const float inv_min = max_min > 0.0f ? __fmul_rn(__frcp_rn(max_min), 63.0f) : 0.0f;
  const float ls = fminf(fmaxf(rintf(__fmul_rn(inv_scale, scale)), 0.0f), 63.0f);
  const float lm = fminf(fmaxf(rintf(__fmul_rn(inv_min, the_min)), 0.0f), 63.0f);
  const __half dh = __float2half_rn(__fdiv_rn(max_scale, 63.0f));
  const __half dmh = __float2half_rn(__fdiv_rn(max_min, 63.0f));
  L.d_h = __half_as_ushort(dh);
  L.dmin_h = __half_as_ushort(dmh);
  L.deff = __fmul_rn(__half2float(dh), ls);
  L.dm = __fmul_rn(__half2float(dmh), lm);
  L.ls = (uint32_t)ls;
  L.lm = (uint32_t)lm;
  return L;
}

// Re-encode one weight against fp16 d/dmin (q4_k.py:185-189): returns the reconstruction,
// the code and the in-range bit.
struct Q4Elem {
  float recon;
  uint32_t code;
  uint32_t in_range;
};

__device__ __forceinline__ Q4Elem encode_elem(const Level2& L, const BlockDivisor& div, float x) {
  Q4Elem r;
  if (L.deff != 0.0f) {
    const float raw = divide(div, __fadd_rn(x, L.dm));
    const float q = clamp15(rintf(raw));
    r.recon = __fsub_rn(__fmul_rn(L.deff, q), L.dm);
    r.code = (uint32_t)q;
    r.in_range = (raw >= 0.0f && raw <= 15.0f) ? 1u : 0u;
  } else {
    r.recon = __fsub_rn(__fmul_rn(L.deff, 0.0f), L.dm);
    r.code = 0u;
    r.in_range = 1u;
  }
  return r;
}

// Divisor state for (x + dm) / deff over one sub-block whose |x| <= xabs.
__device__ __forceinline__ BlockDivisor q4_divisor(const Level2& L, float xabs) {
  const float bound = __fadd_ru(xabs, L.dm);
  return make_divisor(L.deff, __float_as_uint(bound));
}

// The 12-byte packed 6-bit scales/mins (q4_k.py:286-301) as three little-endian words,
// from ls/lm of the 8 sub-blocks.
__device__ __forceinline__ void pack_scales(const uint32_t* ls, const uint32_t* lm, uint32_t* w) {
  uint8_t s[12];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    s[j] = (uint8_t)((ls[j] & 0x3Fu) | ((ls[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)((lm[j] & 0x3Fu) | ((lm[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((ls[j + 4] & 0xFu) | ((lm[j + 4] & 0xFu) << 4));
  }
#pragma unroll
  for (int k = 0; k < 3; ++k)
    w[k] = (uint32_t)s[4 * k] | ((uint32_t)s[4 * k + 1] << 8) | ((uint32_t)s[4 * k + 2] << 16) |
           ((uint32_t)s[4 * k + 3] << 24);
}

// Spread the 8 nibbles of w into the low halves of 8 bytes (nibble t -> byte t).
__device__ __forceinline__ uint64_t spread_nibbles(uint32_t w) {
  uint64_t x = w;
  x = (x | (x << 16)) & 0x0000FFFF0000FFFFull;
  x = (x | (x << 8)) & 0x00FF00FF00FF00FFull;
  x = (x | (x << 4)) & 0x0F0F0F0F0F0F0F0Full;
  return x;
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, bool vec, float* f) {
  using VT = VecTraits<T>;
  if constexpr (VT::kVec == 8) {
    if (vec) {
      VT::to_float(ld_stream(p), f);
      return;
    }
  } else {
    if (vec) {
      VT::to_float(ld_stream(p), f);
      VT::to_float(ld_stream(p + 4), f + 4);
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = VT::load1(p + i);
}

template <typename T>
__device__ __forceinline__ void store8(T* p, bool vec, const float* f) {
  using VT = VecTraits<T>;
  if constexpr (VT::kVec == 8) {
    if (vec) {
      st_v4(p, VT::from_float(f));
      return;
    }
  } else {
    if (vec) {
      st_v4(p, VT::from_float(f));
      st_v4(p + 4, VT::from_float(f + 4));
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) VT::store1(p + i, f[i]);
}

// ---------------------------------------------------------------- minmax: warp / SB
template <typename T>
__global__ void __launch_bounds__(kQ4Threads) q4k_minmax_kernel(const T* __restrict__ x, int64_t n_sb,
                                                                int64_t sb_per_row, int64_t ld, bool vec,
                                                                T* __restrict__ recon, uint8_t* __restrict__ mask,
                                                                uint8_t* __restrict__ blocks) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t sb = warp; sb < n_sb; sb += n_warps) {
    const int64_t row = sb / sb_per_row, kb = sb - row * sb_per_row;
    const T* src = x + row * ld + kb * kQK + lane * 8;
    float f[8];
    load8(src, vec, f);
    // level 1, minmax (q4_k.py:159-163): per sub-block of 4 lanes
    float mx = f[0], mn = f[0], ab = fabsf(f[0]);
#pragma unroll
    for (int i = 1; i < 8; ++i) {
      mx = fmaxf(mx, f[i]);
      mn = fminf(mn, f[i]);
      ab = fmaxf(ab, fabsf(f[i]));
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      ab = fmaxf(ab, __shfl_xor_sync(0xffffffffu, ab, o));
    }
    const float vmin = fminf(mn, 0.0f);
    const float scale = __fdiv_rn(__fsub_rn(mx, vmin), 15.0f);
    const float the_min = -vmin;
    float max_scale = scale, max_min = the_min;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      max_scale = fmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, o));
      max_min = fmaxf(max_min, __shfl_xor_sync(0xffffffffu, max_min, o));
    }
    const Level2 L = level2(scale, the_min, max_scale, max_min);
    const BlockDivisor div = q4_divisor(L, ab);
    float rc[8];
    uint32_t bits = 0u, codes = 0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const Q4Elem e = encode_elem(L, div, f[i]);
      rc[i] = e.recon;
      bits |= e.in_range << i;
      codes |= e.code << (4 * i);
    }
    if (recon != nullptr) store8(recon + sb * kQK + lane * 8, vec, rc);
    if (mask != nullptr) mask[sb * 32 + lane] = (uint8_t)bits;
    if (blocks != nullptr) {
      uint8_t* blk = blocks + sb * 144;
      // qs[g*32 + i] = c[g*64 + i] | c[g*64 + 32 + i] << 4 (q4_k.py:304-315): lane l with
      // l % 8 < 4 holds the low nibbles and lane l + 4 the high nibbles of 8 bytes.
      const uint32_t hi = __shfl_down_sync(0xffffffffu, codes, 4);
      const uint32_t lsm = L.ls | (L.lm << 8);
      uint32_t ls_all[8], lm_all[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t v = __shfl_sync(0xffffffffu, lsm, j * 4);
        ls_all[j] = v & 0xFFu;
        lm_all[j] = v >> 8;
      }
      if ((lane & 7) < 4) {
        const uint64_t bytes = spread_nibbles(codes) | (spread_nibbles(hi) << 4);
        const int g = lane >> 3;
        uint2* dst = reinterpret_cast<uint2*>(blk + 16 + g * 32 + (lane & 7) * 8);
        *dst = make_uint2((uint32_t)bytes, (uint32_t)(bytes >> 32));
      }
      if (lane == 0) {
        uint32_t w[3];
        pack_scales(ls_all, lm_all, w);
        st_v4(blk, make_uint4((uint32_t)L.d_h | ((uint32_t)L.dmin_h << 16), w[0], w[1], w[2]));
      }
    }
  }
}

// ------------------------------------------------------------ grid search: thread / sub-block

// torch-CPU float32 sum of the 32 values f(0..31) (see the file comment).
template <typename F>
__device__ __forceinline__ float torch_sum32(F f) {
  float acc = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float t = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, f(k)), f(k + 8)), f(k + 16)), f(k + 24));
    acc = __fadd_rn(acc, t);
  }
  return acc;
}

// _make_qkx2 (q4_k.py:68-119) for one sub-block; returns (scale, the_min).
__device__ __forceinline__ void make_qkx2(const float* x, const float* w, float* scale_out, float* min_out) {
  float xmax = x[0], xmin = x[0];
#pragma unroll
  for (int i = 1; i < 32; ++i) {
    xmax = fmaxf(xmax, x[i]);
    xmin = fminf(xmin, x[i]);
  }
  const float vmin = fminf(xmin, 0.0f);
  const bool degenerate = xmax == vmin;
  const float denom = degenerate ? 1.0f : __fsub_rn(xmax, vmin);
  const float rden = __frcp_rn(denom);          // denom.reciprocal()
  const float iscale = __fmul_rn(rden, 15.0f);  // nmax / denom
  float scale = __frcp_rn(iscale);              // 1.0 / iscale
  float best_error = torch_sum32([&](int i) {
    const float code = clamp15(rintf(__fmul_rn(iscale, __fsub_rn(x[i], vmin))));
    const float diff = __fsub_rn(__fadd_rn(__fmul_rn(scale, code), vmin), x[i]);
    return __fmul_rn(__fmul_rn(w[i], diff), diff);
  });
  const float sum_w = torch_sum32([&](int i) { return w[i]; });
  const float sum_x = torch_sum32([&](int i) { return __fmul_rn(w[i], x[i]); });
  float cur_min = vmin;
#pragma unroll 1
  for (int step = 0; step <= 20; ++step) {
    const float trial = __fmul_rn(rden, c_trial[step]);
    float aux[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) aux[i] = clamp15(rintf(__fmul_rn(trial, __fsub_rn(x[i], vmin))));
    const float sum_l = torch_sum32([&](int i) { return __fmul_rn(w[i], aux[i]); });
    const float sum_l2 = torch_sum32([&](int i) { return __fmul_rn(__fmul_rn(w[i], aux[i]), aux[i]); });
    const float sum_xl = torch_sum32([&](int i) { return __fmul_rn(__fmul_rn(w[i], aux[i]), x[i]); });
    const float det = __fsub_rn(__fmul_rn(sum_w, sum_l2), __fmul_rn(sum_l, sum_l));
    const float safe_det = det > 0.0f ? det : 1.0f;
    float this_scale = __fdiv_rn(__fsub_rn(__fmul_rn(sum_w, sum_xl), __fmul_rn(sum_x, sum_l)), safe_det);
    float this_min = __fdiv_rn(__fsub_rn(__fmul_rn(sum_l2, sum_x), __fmul_rn(sum_l, sum_xl)), safe_det);
    if (this_min > 0.0f) {
      this_scale = __fdiv_rn(sum_xl, sum_l2 > 0.0f ? sum_l2 : 1.0f);
      this_min = 0.0f;
    }
    const float cur_error = torch_sum32([&](int i) {
      const float d = __fsub_rn(__fadd_rn(__fmul_rn(this_scale, aux[i]), this_min), x[i]);
      return __fmul_rn(__fmul_rn(w[i], d), d);
    });
    if (det > 0.0f && cur_error < best_error) {
      best_error = cur_error;
      scale = this_scale;
      cur_min = this_min;
    }
  }
  if (degenerate) {
    scale = 0.0f;
    cur_min = vmin;
  }
  *scale_out = scale;
  *min_out = -cur_min;
}

template <typename T>
__global__ void __launch_bounds__(128) q4k_grid_kernel(const T* __restrict__ x, int64_t n_sb, int64_t sb_per_row,
                                                       int64_t ld, T* __restrict__ recon, uint8_t* __restrict__ mask,
                                                       uint8_t* __restrict__ blocks) {
  using VT = VecTraits<T>;
  const int lane = threadIdx.x & 31;
  const int j = lane & 7;  // sub-block within the super-block
  const int64_t gthread = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n_threads = (int64_t)gridDim.x * blockDim.x;
  // 8 lanes per super-block; iterate whole warps so shuffles stay converged
  for (int64_t base = (gthread & ~31ll); base / 8 < n_sb; base += n_threads) {
    const int64_t sb = (base + lane) / 8;
    const bool live = sb < n_sb;
    float xs[32];
    if (live) {
      const int64_t row = sb / sb_per_row, kb = sb - row * sb_per_row;
      const T* src = x + row * ld + kb * kQK + j * 32;
#pragma unroll
      for (int i = 0; i < 32; ++i) xs[i] = VT::load1(src + i);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) xs[i] = 0.0f;
    }
    // _level1_grid_search_torch (q4_k.py:139-147)
    float w[32];
    const float av_x = __fsqrt_rn(__fmul_rn(torch_sum32([&](int i) { return __fmul_rn(xs[i], xs[i]); }), 0.03125f));
    float ab = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      w[i] = __fadd_rn(av_x, fabsf(xs[i]));
      ab = fmaxf(ab, fabsf(xs[i]));
    }
    float scale, the_min;
    make_qkx2(xs, w, &scale, &the_min);
    float max_scale = scale, max_min = the_min;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      max_scale = fmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, o));
      max_min = fmaxf(max_min, __shfl_xor_sync(0xffffffffu, max_min, o));
    }
    const Level2 L = level2(scale, the_min, max_scale, max_min);
    const BlockDivisor div = q4_divisor(L, ab);
    uint32_t bits = 0u, cw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const Q4Elem e = encode_elem(L, div, xs[i]);
      xs[i] = e.recon;
      bits |= e.in_range << i;
      cw[i >> 3] |= e.code << (4 * (i & 7));
    }
    uint32_t hw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) hw[k] = __shfl_down_sync(0xffffffffu, cw[k], 1);
    const uint32_t lsm = L.ls | (L.lm << 8);
    uint32_t ls_all[8], lm_all[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t v = __shfl_sync(0xffffffffu, lsm, (lane & ~7) + k);
      ls_all[k] = v & 0xFFu;
      lm_all[k] = v >> 8;
    }
    if (!live) continue;
    const int64_t e0 = sb * kQK + j * 32;
    if (recon != nullptr) {
#pragma unroll
      for (int i = 0; i < 32; ++i) VT::store1(recon + e0 + i, xs[i]);
    }
    if (mask != nullptr) reinterpret_cast<uint32_t*>(mask)[e0 >> 5] = bits;
    if (blocks != nullptr) {
      uint8_t* blk = blocks + sb * 144;
      if ((j & 1) == 0) {
        // sub-block j = 2g supplies the low nibbles, j + 1 the high nibbles of qs[g*32 .. +32)
        uint32_t out[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t b = spread_nibbles(cw[k]) | (spread_nibbles(hw[k]) << 4);
          out[2 * k] = (uint32_t)b;
          out[2 * k + 1] = (uint32_t)(b >> 32);
        }
        uint4* dst = reinterpret_cast<uint4*>(blk + 16 + (j >> 1) * 32);
        dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
        dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
      }
      if (j == 0) {
        uint32_t w3[3];
        pack_scales(ls_all, lm_all, w3);
        st_v4(blk, make_uint4((uint32_t)L.d_h | ((uint32_t)L.dmin_h << 16), w3[0], w3[1], w3[2]));
      }
    }
  }
}

// ------------------------------------------------------------------------ dequant
// dequantize_q4_k (q4_k.py:359-385): one warp per super-block, 8 outputs per lane.
__global__ void __launch_bounds__(kQ4Threads) q4k_dequant_kernel(const uint8_t* __restrict__ blocks, int64_t n_sb,
                                                                 float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t sb = warp; sb < n_sb; sb += n_warps) {
    const uint8_t* b = blocks + sb * 144;
    const float d = __half2float(__ushort_as_half((uint16_t)(b[0] | (b[1] << 8))));
    const float dmin = __half2float(__ushort_as_half((uint16_t)(b[2] | (b[3] << 8))));
    const int j = lane >> 2;  // sub-block of this lane's 8 weights
    const uint8_t* s = b + 4;
    uint32_t ls, lm;
    if (j < 4) {
      ls = s[j] & 0x3Fu;
      lm = s[j + 4] & 0x3Fu;
    } else {
      ls = (s[j + 4] & 0xFu) | (((uint32_t)(s[j - 4] >> 6) & 3u) << 4);
      lm = (uint32_t)(s[j + 4] >> 4) | (((uint32_t)(s[j] >> 6) & 3u) << 4);
    }
    const float deff = __fmul_rn(d, (float)ls), dm = __fmul_rn(dmin, (float)lm);
    const int e0 = lane * 8;
    const int g = e0 / 64, o = e0 % 64;
    const uint8_t* q = b + 16 + g * 32 + (o % 32);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t code = o < 32 ? (q[i] & 0xFu) : (q[i] >> 4);
      v[i] = __fsub_rn(__fmul_rn(deff, (float)code), dm);
    }
    float4* dst = reinterpret_cast<float4*>(out + sb * kQK + e0);
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

template <typename F>
int q4_dispatch(int dtype, F&& f) {
  switch (dtype) {
    case kF32:
      return f(float{});
    case kF16:
      return f(__half{});
    case kBF16:
      return f(__nv_bfloat16{});
    default:
      return QATF_ERR_DTYPE;
  }
}

inline int64_t q4_grid(int64_t threads_needed, const void* kernel, int block) {
  return persistent_grid(threads_needed, kernel, block);
}

}  // namespace qatf

using namespace qatf;

extern "C" int qatf_q4k_encode(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, int method, void* recon,
                               uint8_t* mask_bits, uint8_t* blocks, void* stream) {
  if (rows < 0 || cols < 0 || cols % kQK != 0 || ld < cols) return QATF_ERR_INVALID;
  if (method != QATF_Q4K_GRID_SEARCH && method != QATF_Q4K_MINMAX) return QATF_ERR_INVALID;
  if (rows == 0 || cols == 0) return QATF_OK;
  if (x == nullptr) return QATF_ERR_INVALID;
  if (blocks != nullptr && (reinterpret_cast<uintptr_t>(blocks) & 15u) != 0) return QATF_ERR_INVALID;
  if (mask_bits != nullptr && method == QATF_Q4K_GRID_SEARCH && (reinterpret_cast<uintptr_t>(mask_bits) & 3u) != 0)
    return QATF_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t sb_per_row = cols / kQK;
  const int64_t n_sb = rows * sb_per_row;
  return q4_dispatch(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    const T* xt = static_cast<const T*>(x);
    T* rt = static_cast<T*>(recon);
    if (method == QATF_Q4K_MINMAX) {
      const bool vec = aligned16(x) && ((ld * (int64_t)sizeof(T)) % 16 == 0) && (recon == nullptr || aligned16(recon));
      auto k = q4k_minmax_kernel<T>;
      q4k_minmax_kernel<T><<<q4_grid(n_sb * 32, (const void*)k, kQ4Threads), kQ4Threads, 0, s>>>(
          xt, n_sb, sb_per_row, ld, vec, rt, mask_bits, blocks);
    } else {
      auto k = q4k_grid_kernel<T>;
      q4k_grid_kernel<T><<<q4_grid(n_sb * 8, (const void*)k, 128), 128, 0, s>>>(xt, n_sb, sb_per_row, ld, rt,
                                                                               mask_bits, blocks);
    }
    return cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH;
  });
}

extern "C" int qatf_q4k_dequant(const uint8_t* blocks, int64_t rows, int64_t cols, float* out, void* stream) {
  if (rows < 0 || cols < 0 || cols % kQK != 0) return QATF_ERR_INVALID;
  if (rows == 0 || cols == 0) return QATF_OK;
  if (blocks == nullptr || out == nullptr || !aligned16(out)) return QATF_ERR_INVALID;
  const int64_t n_sb = rows * (cols / kQK);
  auto k = q4k_dequant_kernel;
  q4k_dequant_kernel<<<q4_grid(n_sb * 32, (const void*)k, kQ4Threads), kQ4Threads, 0, static_cast<cudaStream_t>(stream)>>>(
      blocks, n_sb, out);
  return cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH;
}
